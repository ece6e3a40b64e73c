// prefill.cuh -- parameters and launcher of the tcgen05/TMEM causal prefill.
#pragma once

#include "mslim_common.cuh"

namespace mslim {

// Query rows from which TiledAttention-style runs use the prefill kernel
// rather than the multi-query split-KV decode kernel.
constexpr unsigned kPrefillMinQueries = 64;

struct PrefillParams {
    uint16_t *out;      // bf16 [queries][QH][D]
    int *status;        // device status word
    int qheads, kvheads, group;
    int queries, prior; // rows prior..prior+queries-1 attend to keys 0..=row
    int n_qtiles;       // ceil(queries / 128)
    int head_dim;       // the caller's head_dim, 64..128 (a multiple of 8); the
                        // kernel runs at 64 (even groups, head_dim 64) or 128
    float scale_log2;   // log2(e) / sqrt(D)
};

bool prefill_supported(unsigned head_dim, unsigned group);

// Even groups run two query heads per CTA (ping-pong kernel).
bool prefill_pairs_heads(unsigned group);

// q/k/v/out maps: bf16, dims (D, heads, rows), box (64, 1, 128), 128-byte
// swizzle; the out map (same shape as q) is written by bulk tensor stores.
cudaError_t launch_prefill(const CUtensorMap &qmap, const CUtensorMap &kmap,
                           const CUtensorMap &vmap, const CUtensorMap &omap,
                           const PrefillParams &p, cudaStream_t stream);

}  // namespace mslim
