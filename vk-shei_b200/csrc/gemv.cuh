// gemv.cuh -- the decode-step projections on the 5th-generation tensor cores.
#pragma once

#include "mslim_common.cuh"
#include "prologue.cuh"

namespace mslim {

// How one projection is cut into CTAs: 128 output features (weight rows) per
// tile, the K dimension in `splits` (<= 8, one cluster) chunks of `k_tiles`
// 64-wide steps.
struct GemvPlan {
    uint32_t n_tiles;  // ceil(n / 128)
    uint32_t k_steps;  // ceil(k / 64)
    uint32_t k_tiles;  // 64-wide K steps per split
    uint32_t splits;   // K chunks = CTAs per cluster
};

GemvPlan gemv_plan(uint32_t m, uint32_t n, uint32_t k);

// Y[m][n] (row stride ldy elements) = bf16(sum_k X[m][k] * W[n][k]), fp32
// accumulation in TMEM, the splits combined in order over distributed shared
// memory.  xmap: 2-D bf16 map over X (K, m) with a 64 x 16 box; wmap: over W
// (K, n) with a 64 x 128 box; both 128-byte swizzle.  swiglu: W's rows are
// gate and up interleaved in blocks of 64 (n = 2 x width, width % 64 == 0) and
// Y[m][width] = bf16(bf16(silu(bf16(gate))) * bf16(up)).
cudaError_t launch_gemv_tc(const CUtensorMap &xmap, const CUtensorMap &wmap, const GemvPlan &plan, uint32_t m,
                           uint32_t n, uint16_t *y, uint32_t ldy, int *status, cudaStream_t stream,
                           bool swiglu = false);

// Where the q|k|v projection's epilogue puts one decode token per row r:
// RoPE of its q heads into q_out [m][qheads * 128], RoPE of its k heads and a
// copy of its v heads into the K/V store at position positions[r] -- dense
// caches [m][max_tokens][kvheads][128] (page_table null) or ColdStore-exact
// pages [n_pages][kvheads][page_tokens][128] through page_table
// [m][max_pages].  A position or page id outside the store writes nothing for
// that row and is recorded in the status word.
struct GemvRopeAppend {
    const int32_t *positions;
    uint16_t *q_out, *k_dst, *v_dst;
    const int32_t *page_table;
    uint32_t qheads, kvheads, max_tokens, n_pages, page_tokens, max_pages;
    RopeTable table;
};

// The projection of x [m][k] on w_qkv [(qheads + 2 kvheads) * 128][k] with
// the RoPE + K/V append of mslim_rope_append_{dense,paged} in its epilogue
// (head_dim 128: one head per tile).
cudaError_t launch_gemv_qkv_rope_append(const CUtensorMap &xmap, const CUtensorMap &wmap, const GemvPlan &plan,
                                        uint32_t m, uint32_t n, const GemvRopeAppend &e, int *status,
                                        cudaStream_t stream);

}  // namespace mslim
