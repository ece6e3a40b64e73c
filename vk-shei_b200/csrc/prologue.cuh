// prologue.cuh -- launchers of the RMSNorm / RoPE / RoPE+append kernels.
#pragma once

#include <algorithm>

#include "mslim_common.cuh"

namespace mslim {

// Per-dimension RoPE frequency table, built on the host once per call.
// multiply == 0: angle = position / freq[i]  (CPU formula, freq = theta^(2i/D))
// multiply != 0: angle = position * freq[i]  (inverse frequency, optionally
//                Llama-3 scaled, src/gpu_llm/kernels.rs:50-67)
struct RopeTable {
    float freq[128];
    int multiply;
};

// The RoPE arithmetic, shared by every kernel that rotates (the RoPE and
// RoPE + append kernels, and the q|k|v projection that applies them in its
// epilogue), so all of them return the same bits.
__device__ __forceinline__ float rope_angle(const RopeTable &t, int i, uint32_t position) {
    const float pos = (float)position;
    return t.multiply ? pos * t.freq[i] : __fdiv_rn(pos, t.freq[i]);
}

// (cos, sin) of one angle, each rounded to bf16.
__device__ __forceinline__ float2 rope_cs(float angle) {
    double sd, cd;
    sincos((double)angle, &sd, &cd);
    return make_float2(bf16_round((float)cd), bf16_round((float)sd));
}

__device__ __forceinline__ void rope_rotate(float a, float b, float2 cs, float &out_a, float &out_b) {
    out_a = bf16_round(bf16_round(a * cs.x) - bf16_round(b * cs.y));
    out_b = bf16_round(bf16_round(b * cs.x) + bf16_round(a * cs.y));
}

cudaError_t launch_rmsnorm(const uint16_t *x, const uint16_t *w, uint16_t *y, uint32_t tokens,
                           uint32_t hidden, float eps, cudaStream_t stream);
// x = bf16(x + delta) in place, then y = RMSNorm(x): one pass per row.
cudaError_t launch_residual_rmsnorm(uint16_t *x, const uint16_t *delta, const uint16_t *w, uint16_t *y,
                                    uint32_t tokens, uint32_t hidden, float eps, cudaStream_t stream);
cudaError_t launch_rope(const uint16_t *in, uint16_t *out, uint32_t tokens, uint32_t heads,
                        uint32_t dim, uint32_t start_position, const RopeTable &table,
                        cudaStream_t stream);
cudaError_t launch_rope_append_paged(const uint16_t *q_in, uint16_t *q_out, const uint16_t *k_in,
                                     const uint16_t *v_in, uint32_t tokens, uint32_t qheads,
                                     uint32_t kvheads, uint32_t dim, uint32_t start_position,
                                     const int32_t *positions, uint16_t *k_pool,
                                     uint16_t *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                     const int32_t *page_table, uint32_t max_pages,
                                     const RopeTable &table, int *status, cudaStream_t stream,
                                     uint32_t q_stride = 0, uint32_t kv_stride = 0);
// q_stride / kv_stride: elements between consecutive tokens' q / k, v rows
// (0: the rows are packed, QH*D / KVH*D).
cudaError_t launch_rope_append_dense(const uint16_t *q_in, uint16_t *q_out, const uint16_t *k_in,
                                     const uint16_t *v_in, uint32_t n_seq, uint32_t qheads,
                                     uint32_t kvheads, uint32_t dim, const int32_t *positions,
                                     uint16_t *k_cache, uint16_t *v_cache, uint32_t max_tokens,
                                     const RopeTable &table, int *status, cudaStream_t stream,
                                     uint32_t q_stride = 0, uint32_t kv_stride = 0);

}  // namespace mslim
