// prefill.cuh -- launcher of the tcgen05/TMEM causal prefill kernel.
#pragma once

#include <string>

#include "mslim_common.cuh"

namespace mslim {

// Query rows from which TiledAttention-style runs use the prefill kernel
// rather than the multi-query split-KV decode kernel.
constexpr unsigned kPrefillMinQueries = 64;

bool prefill_supported(unsigned head_dim, unsigned group);

// Enqueues causal attention of `queries` rows at positions prior.. over keys
// 0..=prior+row.  Returns an MSLIM_* status; *err receives the message.
int launch_prefill(unsigned qheads, unsigned kvheads, unsigned head_dim, const uint16_t *q,
                   const uint16_t *k, const uint16_t *v, uint16_t *out, unsigned queries,
                   unsigned prior, float scale_log2, int *status, cudaStream_t stream,
                   std::string *err);

}  // namespace mslim
