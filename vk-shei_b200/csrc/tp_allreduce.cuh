// tp_allreduce.cuh -- the tensor-parallel decode collective fused with the
// residual add and RMSNorm that follow it, over NVLink peer memory.
#pragma once

#include "mslim_common.cuh"

namespace mslim {

constexpr int kTpMaxWorld = 8;

// Device view of one rank's communicator: every rank's data and flag regions
// mapped into this rank's address space (its own included).
//   data[r]:  bf16 [2 slots][max_rows][hidden]   rank r's row-parallel partials
//   flags[r]: uint32 [max_rows][kTpMaxWorld]      ready counters written by peers
//   epoch:    uint32 [max_rows]                   this rank's call count per row
struct TpCommDev {
    uint32_t world, rank, max_rows, hidden;
    const uint16_t *data[kTpMaxWorld];
    uint32_t *flags[kTpMaxWorld];
    uint32_t *epoch;
};

// x[row] = bf16(x[row] + bf16(sum over ranks of data[r][slot][row])), then
// y[row] = RMSNorm(x[row], w), for rows [0, rows).  The caller has written this
// rank's partial into data[rank][slot] (stream-ordered before the launch).
cudaError_t launch_tp_allreduce_rmsnorm(const TpCommDev &comm, uint32_t slot, uint16_t *x,
                                        const uint16_t *w, uint16_t *y, uint32_t rows, float eps,
                                        int *status, cudaStream_t stream);

}  // namespace mslim
