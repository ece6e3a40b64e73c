// prefill.cu -- causal prefill attention (tcgen05/TMEM kernel: in progress).
#include "../../include/mslim_cuda.h"
#include "prefill.cuh"

namespace mslim {

bool prefill_supported(unsigned, unsigned) { return false; }

int launch_prefill(unsigned, unsigned, unsigned, const uint16_t *, const uint16_t *,
                   const uint16_t *, uint16_t *, unsigned, unsigned, float, int *, cudaStream_t,
                   std::string *err) {
    *err = "the tcgen05 prefill kernel is not built";
    return MSLIM_ERR_INVALID_GEOMETRY;
}

}  // namespace mslim
