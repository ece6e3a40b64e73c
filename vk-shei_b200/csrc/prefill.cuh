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
    int head_dim;       // the caller's head_dim, 64..256 (a multiple of 8); the
                        // kernel runs at 64 (even groups, head_dim 64), 128 or 256
    float scale_log2;   // log2(e) / sqrt(D)
};

bool prefill_supported(unsigned head_dim, unsigned group);

// Even groups up to head_dim 128 run two query heads per CTA (ping-pong
// kernel); the rest one head per CTA.
bool prefill_pairs_heads(unsigned group, unsigned head_dim);

// Rows of the k/v maps' boxes: 128 (one key tile), 64 above head_dim 128.
unsigned prefill_kv_box_rows(unsigned head_dim);

// q/k/v/out maps: bf16, dims (head_dim, heads, rows), 128-byte swizzle; q box
// (64, 1, 128), k and v boxes (64, 1, prefill_kv_box_rows); the out map (same
// shape as q, box (64, 1, 32): one warp's rows) is written by bulk tensor stores.
cudaError_t launch_prefill(const CUtensorMap &qmap, const CUtensorMap &kmap,
                           const CUtensorMap &vmap, const CUtensorMap &omap,
                           const PrefillParams &p, cudaStream_t stream);

}  // namespace mslim
