// decode.cu -- split-KV flash-decoding over dense or ColdStore-paged bf16 K/V.
//
// Replaces the reference decode attention (QK / softmax / PV of
// assets/gpu_llm.cl:150-212, the fused kernel of gpu_llm.cl:975-1026, the
// tiled split-KV kernel + merge of assets/tiled_attention.cl:9-155 and the
// ColdStore-staged PV of gpu_llm.cl:280-323) with one B200 kernel pair:
//
//   mslim_decode_split  one CTA per (split, KV-head chunk, sequence x query
//                       block); a sequence's keys are cut into
//                       ceil(L / split_tokens) splits of equal length.  A producer warp streams 64-token K and V
//                       tiles with TMA (128-byte swizzle, this GPU's HBM, no
//                       multicast) through an mbarrier ring; four consumer
//                       warps each own 16 tokens of every tile.  Rows of the
//                       MMA are the (query, head) pairs that share the KV
//                       head, so K/V bytes are read once per group.
//   mslim_decode_merge_row / mslim_decode_merge  fixed split-order combine of
//                       {m, l, acc[D]} partials (one CTA per row with every
//                       partial requested at once, up to 64 splits; one warp
//                       per row in batches of eight splits beyond that).
//
// Numeric contract (same code for dense and paged K/V, so the two layouts are
// bit-identical by construction, and run-to-run deterministic):
//   s = (q . k) * (log2(e)/sqrt(D))          fp32 accumulate (mma.sync bf16)
//   p = exp2(s - m_running)                   online softmax, fp32
//   acc += p_hi * v + p_lo * v                p split into two bf16 terms, so
//                                             the PV product keeps ~16 bits of p
//   out = bf16(sum_s w_s acc_s / sum_s w_s l_s)   fixed split order.
#include <algorithm>

#include "decode.cuh"

namespace mslim {

namespace {

constexpr int kTileT = 64;       // tokens per pipeline stage
// A split partial in global memory is {acc[D], m, l} and two pad floats:
// D + 4 floats, a multiple of 16 bytes, so any run of partials is one bulk copy.
constexpr int kPartPad = 4;
constexpr int kWarpTokens = 16;  // tokens per consumer warp per stage
constexpr int kConsumerWarps = kTileT / kWarpTokens;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kBoxBytes = kTileT * 128;  // one 64-column (128 B) swizzled box

template <int D>
struct Shape {
    static constexpr int kBoxes = D / 64;
    static constexpr int kTensorBytes = kBoxes * kBoxBytes;
    static constexpr int kStageBytes = 2 * kTensorBytes;
    static constexpr int kKSteps = D / 16;
    static constexpr int kNTiles = D / 8;
};

__device__ __forceinline__ uint32_t ld_u32(const uint16_t *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}

// Byte offset of the 16-byte chunk `chunk` (along D) of tile row `row` inside a
// stage tensor laid out as kBoxes boxes of [kTileT rows][128 B] with the TMA
// 128-byte swizzle (chunk index XOR row % 8).
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return (uint32_t)((chunk >> 3) * kBoxBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// Tokens per split of a run of `tokens` keys: the run is cut into
// ceil(tokens / split_tokens) splits of equal length (rounded up to the
// 64-token stage), so no split is a short remainder and the CTAs of a decode
// take about the same time.  The last split may be shorter by < 64 tokens
// per split.  0 for an empty run.
__device__ __forceinline__ int split_len(int tokens, int split_tokens) {
    if (tokens <= 0) return 0;
    const int n = (tokens + split_tokens - 1) / split_tokens;
    return ((tokens + n - 1) / n + kTileT - 1) / kTileT * kTileT;
}

// Loads the K and V tile at token t0 of (seq, kvh) into stage buffers kdst /
// vdst, completing on `bar`.  Paged: a page-table entry outside the pool is
// reported and nothing is loaded; the stage completes without bytes so the
// consumers do not wait (that session's output is then undefined and the
// status word says so).
template <int D, bool PAGED>
__device__ __forceinline__ void issue_tile(const CUtensorMap *kmap, const CUtensorMap *vmap, const DecodeParams &p,
                                           uint64_t *bar, uint8_t *kdst, uint8_t *vdst, int seq, int kvh, int t0) {
    using S = Shape<D>;
    if constexpr (PAGED) {
        const int lp = t0 / p.page_tokens;
        const int off = t0 - lp * p.page_tokens;
        const int phys = p.page_table[(size_t)seq * p.max_pages + lp];
        if (phys < 0 || phys >= p.n_pages) {
            if (p.status) atomicExch(p.status, MSLIM_DEVICE_BAD_PAGE_CODE);
            mbar_arrive(bar);
            return;
        }
        mbar_arrive_expect_tx(bar, S::kStageBytes);
        const int z = phys * p.kvheads + kvh;
#pragma unroll
        for (int b = 0; b < S::kBoxes; ++b) {
            tma_load_3d(kdst + b * kBoxBytes, kmap, bar, b * 64, off, z);
            tma_load_3d(vdst + b * kBoxBytes, vmap, bar, b * 64, off, z);
        }
    } else {
        mbar_arrive_expect_tx(bar, S::kStageBytes);
#pragma unroll
        for (int b = 0; b < S::kBoxes; ++b) {
            tma_load_4d(kdst + b * kBoxBytes, kmap, bar, b * 64, kvh, t0, seq);
            tma_load_4d(vdst + b * kBoxBytes, vmap, bar, b * 64, kvh, t0, seq);
        }
    }
}

// The (query, head) rows of one CTA's work item and where they sit: rows
// r = query (qg_first + r / hc) x head (kvh * group + hchunk * hc + r % hc).
struct DecodeItem {
    int seq, kvh, hchunk, qg_first, qg_last, prior, split;
};

// One consumer warp's share of a work item: MMA rows are the item's (query,
// head) rows, the warp owns 16 tokens of every 64-token tile, keeps its own
// online-softmax state, and the four warps are combined in warp order at the
// end of the item.
template <int D, bool QSPLIT>
struct DecodeConsumer {
    using S = Shape<D>;
    uint32_t qa[S::kKSteps][4];
    uint32_t qb[QSPLIT ? S::kKSteps : 1][4];
    int row_limit[2];
    bool row_ok[2];
    int row_q[2];
    float o[S::kNTiles][4];
    float m_run[2], l_run[2];

    // A fragments of Q (16 rows x 16 dims per k-step) and a fresh state.
    // With QSPLIT the query arrives as f32 and is carried as qa (bf16 of q) +
    // qb (bf16 of the remainder), two MMAs per k-step.
    // q_smem: the item's rows (r = query x head, head_dim elements each) staged
    // in shared memory, or null to read them from global memory.
    __device__ __forceinline__ void begin(const DecodeParams &p, const DecodeItem &it, int lane,
                                          const uint16_t *q_smem = nullptr) {
        const int g = lane >> 2, c = lane & 3;
        const int hc = p.heads_per_cta;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = g + 8 * h;
            row_q[h] = it.qg_first + r / hc;
            row_ok[h] = (r < p.q_per_cta * hc) && (row_q[h] <= it.qg_last);
            row_limit[h] = row_ok[h] ? it.prior + row_q[h] : -1;  // last visible token
        }
#pragma unroll
        for (int ks = 0; ks < S::kKSteps; ++ks) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = g + 8 * h;
                uint32_t k0 = 0, k8 = 0, k0r = 0, k8r = 0;
                if (row_ok[h]) {
                    const int qh = it.kvh * p.group + it.hchunk * hc + r % hc;
                    const int d0 = ks * 16 + 2 * c;  // dims d0, d0+1 and d0+8, d0+9
                    const size_t off = (((size_t)it.seq * p.nq + row_q[h]) * p.qheads + qh) * p.head_dim + d0;
                    if constexpr (QSPLIT) {
                        const float2 f0 = d0 < p.head_dim ? *reinterpret_cast<const float2 *>(p.q_f32 + off)
                                                          : make_float2(0.f, 0.f);
                        const float2 f8 = d0 + 8 < p.head_dim ? *reinterpret_cast<const float2 *>(p.q_f32 + off + 8)
                                                              : make_float2(0.f, 0.f);
                        k0 = pack_bf16x2(f0.x, f0.y);
                        k8 = pack_bf16x2(f8.x, f8.y);
                        k0r = pack_bf16x2(f0.x - bf16lo_f32(k0), f0.y - bf16hi_f32(k0));
                        k8r = pack_bf16x2(f8.x - bf16lo_f32(k8), f8.y - bf16hi_f32(k8));
                    } else if (q_smem) {
                        const uint16_t *row = q_smem + r * p.head_dim + d0;
                        k0 = d0 < p.head_dim ? *reinterpret_cast<const uint32_t *>(row) : 0u;
                        k8 = d0 + 8 < p.head_dim ? *reinterpret_cast<const uint32_t *>(row + 8) : 0u;
                    } else {
                        k0 = d0 < p.head_dim ? ld_u32(p.q + off) : 0u;
                        k8 = d0 + 8 < p.head_dim ? ld_u32(p.q + off + 8) : 0u;
                    }
                }
                qa[ks][h] = k0;      // a0 (row g) / a1 (row g+8): k = 2c, 2c+1
                qa[ks][2 + h] = k8;  // a2 / a3: k = 2c+8, 2c+9
                if constexpr (QSPLIT) {
                    qb[ks][h] = k0r;
                    qb[ks][2 + h] = k8r;
                }
            }
        }
#pragma unroll
        for (int n = 0; n < S::kNTiles; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        m_run[0] = m_run[1] = -INFINITY;
        l_run[0] = l_run[1] = 0.f;
    }

    // This warp's 16 tokens of the 64-token tile at token tile_t0 (stage s),
    // keys below t_end.
    __device__ __forceinline__ void tile(uint8_t *stage, int tile_t0, int t_end, float scale, int warp, int lane) {
        const int c = lane & 3;
        const int row0 = warp * kWarpTokens;
        const int t0 = tile_t0 + row0;
        const int valid = min(kWarpTokens, t_end - t0);
        if (valid <= 0) return;
        const uint32_t kt = smem_u32(stage);
        const uint32_t vt = kt + S::kTensorBytes;
        if (valid < kWarpTokens) {
            // Rows past the sequence end hold whatever the page or cache held;
            // zero their V so p == 0 cannot meet a NaN/Inf payload.
            uint8_t *vrow = stage + S::kTensorBytes;
            for (int x = lane; x < (kWarpTokens - valid) * S::kBoxes * 8; x += 32) {
                const int r = row0 + valid + x / (S::kBoxes * 8);
                const int ch = x % (S::kBoxes * 8);
                *reinterpret_cast<uint4 *>(vrow + swz(r, ch)) = make_uint4(0, 0, 0, 0);
            }
            fence_proxy_async_smem();
            __syncwarp();
        }
        // ---- S = Q K^T for this warp's 16 tokens (two n-tiles of 8) ----
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int j = 0; j < D / 32; ++j) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                const int r = row0 + nt * 8 + (lane & 7);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kt + swz(r, 4 * j + (lane >> 3)), b0, b1, b2, b3);
                mma_bf16_16816(sc[nt], qa[2 * j], b0, b1);
                mma_bf16_16816(sc[nt], qa[2 * j + 1], b2, b3);
                if constexpr (QSPLIT) {
                    mma_bf16_16816(sc[nt], qb[2 * j], b0, b1);
                    mma_bf16_16816(sc[nt], qb[2 * j + 1], b2, b3);
                }
            }
        }
        // ---- online softmax over the 16 tokens (rows g, g+8) ----
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e >> 1;
                const int tok = t0 + nt * 8 + 2 * c + (e & 1);
                const float v = (tok <= row_limit[h]) ? sc[nt][e] * scale : -INFINITY;
                sc[nt][e] = v;
                mx[h] = fmaxf(mx[h], v);
            }
        float alpha[2], base[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
            const float m_new = fmaxf(m_run[h], mx[h]);
            base[h] = (m_new == -INFINITY) ? 0.f : m_new;
            alpha[h] = fast_exp2(m_run[h] - base[h]);
            m_run[h] = m_new;
        }
        float ps[2] = {0.f, 0.f};
        uint32_t phi[4], plo[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float p0 = fast_exp2(sc[nt][2 * h] - base[h]);
                const float p1 = fast_exp2(sc[nt][2 * h + 1] - base[h]);
                ps[h] += p0 + p1;
                const uint32_t hi = pack_bf16x2(p0, p1);
                const uint32_t lo = pack_bf16x2(p0 - bf16lo_f32(hi), p1 - bf16hi_f32(hi));
                // A fragment of P (16 rows x 16 tokens): a0 = (g, 2c..), a1 = (g+8, 2c..),
                // a2 = (g, 2c+8..), a3 = (g+8, 2c+8..).
                phi[nt * 2 + h] = hi;
                plo[nt * 2 + h] = lo;
            }
#pragma unroll
        for (int h = 0; h < 2; ++h) l_run[h] = l_run[h] * alpha[h] + ps[h];
#pragma unroll
        for (int n = 0; n < S::kNTiles; ++n) {
            o[n][0] *= alpha[0];
            o[n][1] *= alpha[0];
            o[n][2] *= alpha[1];
            o[n][3] *= alpha[1];
        }
        // ---- O += P V (V^T fragments via transposed ldmatrix) ----
        const uint32_t pa_hi[4] = {phi[0], phi[1], phi[2], phi[3]};
        const uint32_t pa_lo[4] = {plo[0], plo[1], plo[2], plo[3]};
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
            const int mtx = lane >> 3;
            const int r = row0 + (mtx & 1) * 8 + (lane & 7);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_trans(vt + swz(r, 2 * j + (mtx >> 1)), b0, b1, b2, b3);
            mma_bf16_16816(o[2 * j], pa_hi, b0, b1);
            mma_bf16_16816(o[2 * j], pa_lo, b0, b1);
            mma_bf16_16816(o[2 * j + 1], pa_hi, b2, b3);
            mma_bf16_16816(o[2 * j + 1], pa_lo, b2, b3);
        }
    }

    // Drops the state of a finished split (the next stage always opens a new
    // split, whose begin() sets all of it): constants are not held in
    // registers across the code that runs between splits.
    __device__ __forceinline__ void clear() {
#pragma unroll
        for (int ks = 0; ks < S::kKSteps; ++ks)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                qa[ks][e] = 0u;
                if constexpr (QSPLIT) qb[ks][e] = 0u;
            }
#pragma unroll
        for (int n = 0; n < S::kNTiles; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        m_run[0] = m_run[1] = -INFINITY;
        l_run[0] = l_run[1] = 0.f;
        row_limit[0] = row_limit[1] = -1;
        row_ok[0] = row_ok[1] = false;
        row_q[0] = row_q[1] = 0;
    }

    // The four warps' states combined in warp order into the item's split
    // partial {acc[D], m, l}.  Warps 1-3 hand their states over through
    // `scratch` ([3][16 rows][D + 2] floats, a stage buffer every consumer is
    // done with); warp 0 combines them with its own, which it keeps in
    // registers.  Same arithmetic and order for every row and dim, whatever
    // kernel runs the item.
    __device__ __forceinline__ void finish(const DecodeParams &p, const DecodeItem &it, float *scratch, int warp,
                                           int lane) {
        constexpr int kRowF = D + 2;
        const int g = lane >> 2, c = lane & 3;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
            l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");  // the stage is read
        if (warp > 0) {
            float *mine = scratch + (warp - 1) * 16 * kRowF;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = g + 8 * h;
                if (c == 0) {
                    mine[r * kRowF + D] = m_run[h];
                    mine[r * kRowF + D + 1] = l_run[h];
                }
#pragma unroll
                for (int n = 0; n < S::kNTiles; ++n) {
                    mine[r * kRowF + n * 8 + 2 * c] = o[n][2 * h];
                    mine[r * kRowF + n * 8 + 2 * c + 1] = o[n][2 * h + 1];
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        if (warp == 0) {
            const int hc = p.heads_per_cta;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (!row_ok[h]) continue;
                const int r = g + 8 * h;
                float mw[kConsumerWarps], lw[kConsumerWarps], wgt[kConsumerWarps];
                mw[0] = m_run[h];
                lw[0] = l_run[h];
#pragma unroll
                for (int w = 1; w < kConsumerWarps; ++w) {
                    mw[w] = scratch[((w - 1) * 16 + r) * kRowF + D];
                    lw[w] = scratch[((w - 1) * 16 + r) * kRowF + D + 1];
                }
                float m = -INFINITY;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) m = fmaxf(m, mw[w]);
                const float mb = (m == -INFINITY) ? 0.f : m;
                float l = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) {
                    wgt[w] = fast_exp2(mw[w] - mb);
                    l += wgt[w] * lw[w];
                }
                const int qh = it.kvh * p.group + it.hchunk * hc + r % hc;
                float *dst = p.partials + ((((size_t)it.seq * p.nq + row_q[h]) * p.qheads + qh) * p.max_splits +
                                           it.split) * (D + kPartPad);
#pragma unroll
                for (int n = 0; n < S::kNTiles; ++n) {
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int d = n * 8 + 2 * c + e;
                        float a = 0.f;
                        a += wgt[0] * o[n][2 * h + e];
#pragma unroll
                        for (int w = 1; w < kConsumerWarps; ++w) a += wgt[w] * scratch[((w - 1) * 16 + r) * kRowF + d];
                        dst[d] = a;
                    }
                }
                if (c == 0) {
                    dst[D] = m;
                    dst[D + 1] = l;
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");  // scratch is free again
    }
};

// Causal extent of the query block `qblock` of sequence `seq`: query row qg
// (0-based among the nq new rows) sees tokens [0, prior + qg]; cta_end is the
// exclusive token bound of the block; 0 splits for an empty block.
struct UnitExtent {
    int ntok, prior, qg_first, qg_last, cta_end, slen, splits;
};
// The session's token count as the caller gave it (before the cap).
__device__ __forceinline__ int unit_tokens(const DecodeParams &p, int seq) {
    return p.fixed_tokens >= 0 ? p.fixed_tokens : p.seq_tokens[seq];
}
// Extent of query block `qblock` of a session holding `tokens` tokens.
__device__ __forceinline__ UnitExtent unit_extent_of(const DecodeParams &p, int tokens, int qblock) {
    UnitExtent u;
    u.ntok = min(p.token_cap, tokens);
    u.prior = u.ntok - p.nq;
    u.qg_first = qblock * p.q_per_cta;
    u.qg_last = min(p.nq, u.qg_first + p.q_per_cta) - 1;
    u.cta_end = u.prior + u.qg_last + 1;
    const bool empty = u.ntok <= 0 || u.cta_end <= 0;
    u.slen = empty ? 0 : split_len(u.cta_end, p.split_tokens);
    u.splits = empty ? 0 : min((int)p.max_splits, (u.cta_end + u.slen - 1) / u.slen);
    return u;
}
__device__ __forceinline__ UnitExtent unit_extent(const DecodeParams &p, int seq, int qblock) {
    return unit_extent_of(p, unit_tokens(p, seq), qblock);
}

// One CTA per (split, KV-head chunk, sequence x query block).
template <int D, int STAGES, bool PAGED, bool QSPLIT>
__global__ void __launch_bounds__(kThreads)
    mslim_decode_split(const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, const DecodeParams p) {
    using S = Shape<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * S::kStageBytes);
    uint64_t *empty = full + STAGES;

    // launched with programmatic dependent launch: inputs (and the partials a
    // previous merge may still read) are touched only after the predecessor
    griddep_launch_dependents();
    griddep_wait();
    DecodeItem it;
    it.split = blockIdx.x;
    it.kvh = blockIdx.y / p.head_chunks;
    it.hchunk = blockIdx.y % p.head_chunks;
    it.seq = blockIdx.z / p.q_blocks;
    const UnitExtent u = unit_extent(p, it.seq, blockIdx.z % p.q_blocks);
    it.prior = u.prior;
    it.qg_first = u.qg_first;
    it.qg_last = u.qg_last;
    if (it.split >= u.splits) return;  // CTA-uniform
    const int t_begin = it.split * u.slen;
    const int t_end = min(u.cta_end, t_begin + u.slen);
    const int ntiles = (t_end - t_begin + kTileT - 1) / kTileT;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbarrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer --
        if (lane == 0) {
            prefetch_tmap(&kmap);
            prefetch_tmap(&vmap);
            int issued = 0;
            for (int i = 0; i < ntiles; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1, p.status, 1)) break;
                uint8_t *kdst = smem + s * S::kStageBytes;
                issue_tile<D, PAGED>(&kmap, &vmap, p, &full[s], kdst, kdst + S::kTensorBytes, it.seq, it.kvh,
                                     t_begin + i * kTileT);
                issued = i + 1;
            }
            // Do not retire while our copies may still be landing in this CTA's
            // shared memory: wait (bounded) for the last stages issued.
            for (int i = max(0, issued - STAGES); i < issued; ++i)
                mbar_wait(&full[i % STAGES], (i / STAGES) & 1, p.status, 2);
        }
        return;
    }

    // ----------------------------------------------------------- consumers --
    DecodeConsumer<D, QSPLIT> cs;
    cs.begin(p, it, lane);
    for (int i = 0; i < ntiles; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1, p.status, 3)) break;
        cs.tile(smem + s * S::kStageBytes, t_begin + i * kTileT, t_end, p.scale_log2, warp, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    // All consumers are done with the ring (the producer has issued nothing
    // further), so its first stage is the combine's scratch.
    cs.finish(p, it, reinterpret_cast<float *>(smem), warp, lane);
}

// What the producer of the persistent kernel tells the consumers about each
// stage it fills: the work item, the tile and whether it opens or closes the
// item's split (or ends the CTA's work).
struct StageMeta {
    int seq, kvh, hchunk, split, prior, qg_first, qg_last;
    int t0, t_end, flags;
    int item, nsplits;  // the (unit, KV-head chunk) item and its split count
};
constexpr int kMaxFusedSplits = 64;  // splits per item the in-kernel merge takes

// The last CTA to finish a split of an item merges the item's partials (the
// other splits' from global memory) in split order -- the arithmetic and
// order of mslim_decode_merge_row, so the output bits are the same -- and
// writes its bf16 rows.  Run by the four consumer warps; `scratch` holds the
// split maxima and sums ([16 rows][kMaxFusedSplits] each).
template <int D>
__device__ __forceinline__ void merge_item(const DecodeParams &p, const DecodeItem &it, int nsplits,
                                           float *scratch) {
    constexpr int kRowF = D + kPartPad;
    constexpr int kThr = kConsumerWarps * 32;
    const int hc = p.heads_per_cta;
    const int rows = p.q_per_cta * hc;
    float *ms = scratch, *ls = scratch + 16 * kMaxFusedSplits;
    auto part = [&](int r, int s) -> const float * {
        const int qg = it.qg_first + r / hc;
        const int qh = it.kvh * p.group + it.hchunk * hc + r % hc;
        return p.partials + ((((size_t)it.seq * p.nq + qg) * p.qheads + qh) * p.max_splits + s) * kRowF;
    };
    for (int x = threadIdx.x; x < rows * nsplits; x += kThr) {
        const int r = x / nsplits, s = x % nsplits;
        if (it.qg_first + r / hc > it.qg_last) continue;
        const float *src = part(r, s);
        ms[r * kMaxFusedSplits + s] = __ldcg(src + D);
        ls[r * kMaxFusedSplits + s] = __ldcg(src + D + 1);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kThr) : "memory");
    // A thread takes one row's two adjacent dims at a time (the partial rows
    // are 8-byte aligned) with the loads of kBatch splits in flight, so an
    // item of <= kBatch splits costs one round trip per pair; the sums run in
    // split order, one split at a time (the arithmetic of
    // mslim_decode_merge_row, so the bits are the same).
    constexpr int kBatch = D >= 256 ? 4 : 8;  // (more would cost registers: at head_dim 128 the second CTA per SM)
    constexpr int kPairs = D / 2;
#pragma unroll 1
    for (int x = threadIdx.x; x < rows * kPairs; x += kThr) {
        const int r = x / kPairs, d = 2 * (x % kPairs);
        const int qg = it.qg_first + r / hc;
        if (qg > it.qg_last || d >= p.head_dim) continue;
        const float *mr = ms + r * kMaxFusedSplits, *lr = ls + r * kMaxFusedSplits;
        float m = -INFINITY;
        for (int s = 0; s < nsplits; ++s) m = fmaxf(m, mr[s]);
        const float mb = (m == -INFINITY) ? 0.f : m;
        float l = 0.f, acc0 = 0.f, acc1 = 0.f;
        const float *src = part(r, 0) + d;
#pragma unroll 1
        for (int s0 = 0; s0 < nsplits; s0 += kBatch) {
            float2 av[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
                if (s0 + u < nsplits) av[u] = __ldcg(reinterpret_cast<const float2 *>(src + (size_t)(s0 + u) * kRowF));
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                if (s0 + u < nsplits) {
                    const float w = fast_exp2(mr[s0 + u] - mb);
                    l += w * lr[s0 + u];
                    acc0 += w * av[u].x;
                    acc1 += w * av[u].y;
                }
            }
        }
        const float inv = (l > 0.f) ? 1.0f / l : 0.f;
        const int qh = it.kvh * p.group + it.hchunk * hc + r % hc;
        *reinterpret_cast<uint32_t *>(p.out + (((size_t)it.seq * p.nq + qg) * p.qheads + qh) * p.head_dim + d) =
            (uint32_t)bf16_bits_rn(acc0 * inv) | ((uint32_t)bf16_bits_rn(acc1 * inv) << 16);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kThr) : "memory");  // scratch is free again
}
// merge_item from shared memory: every valid row's first `nsplits` partials
// (contiguous 16-byte records) come in by one bulk copy per row, completing on
// `bar`, so the merge costs one round trip instead of a few dependent ones;
// `scratch` (free shared memory) holds them.  Same arithmetic and order as
// merge_item, so the bits are the same.
template <int D>
__device__ __forceinline__ void merge_item_bulk(const DecodeParams &p, const DecodeItem &it, int nsplits,
                                                float *scratch, uint64_t *bar, uint32_t parity) {
    constexpr int kRowF = D + kPartPad;
    constexpr int kThr = kConsumerWarps * 32;
    const int hc = p.heads_per_cta;
    const int nrows = (it.qg_last - it.qg_first + 1) * hc;  // row r: query r / hc, head r % hc
    // the stage's generic-proxy accesses are ordered before the copies' writes
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, %0;" ::"n"(kThr) : "memory");
    if (threadIdx.x == 0) {
        const uint32_t row_bytes = (uint32_t)(nsplits * kRowF * sizeof(float));
        mbar_arrive_expect_tx(bar, row_bytes * (uint32_t)nrows);
        for (int r = 0; r < nrows; ++r) {
            const int qg = it.qg_first + r / hc;
            const int qh = it.kvh * p.group + it.hchunk * hc + r % hc;
            bulk_load(scratch + (size_t)r * nsplits * kRowF,
                      p.partials + (((size_t)it.seq * p.nq + qg) * p.qheads + qh) * p.max_splits * kRowF, row_bytes,
                      bar);
        }
    }
    mbar_wait(bar, parity, p.status, 5);
    constexpr int kPairs = D / 2;
#pragma unroll 1
    for (int x = threadIdx.x; x < nrows * kPairs; x += kThr) {
        const int r = x / kPairs, d = 2 * (x % kPairs);
        if (d >= p.head_dim) continue;
        const float *rec = scratch + (size_t)r * nsplits * kRowF;
        float m = -INFINITY;
#pragma unroll 1
        for (int s = 0; s < nsplits; ++s) m = fmaxf(m, rec[s * kRowF + D]);
        const float mb = (m == -INFINITY) ? 0.f : m;
        float l = 0.f, acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1
        for (int s = 0; s < nsplits; ++s) {
            const float w = fast_exp2(rec[s * kRowF + D] - mb);
            l += w * rec[s * kRowF + D + 1];
            const float2 a = *reinterpret_cast<const float2 *>(rec + s * kRowF + d);
            acc0 += w * a.x;
            acc1 += w * a.y;
        }
        const float inv = (l > 0.f) ? 1.0f / l : 0.f;
        const int qg = it.qg_first + r / hc;
        const int qh = it.kvh * p.group + it.hchunk * hc + r % hc;
        *reinterpret_cast<uint32_t *>(p.out + (((size_t)it.seq * p.nq + qg) * p.qheads + qh) * p.head_dim + d) =
            (uint32_t)bf16_bits_rn(acc0 * inv) | ((uint32_t)bf16_bits_rn(acc1 * inv) << 16);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kThr) : "memory");  // scratch is free again
}

// kMetaLate: the split is among the launch's last two waves of work, where a
// merge would delay this CTA's remaining split past the others' (merges of
// such items wait until the CTA has no more work).
constexpr int kMetaFirst = 1, kMetaLast = 2, kMetaDone = 4, kMetaLate = 8;
constexpr int kMaxUnits = 256;  // (sequence, query block) pairs the persistent kernel takes
constexpr int kLenBuckets = 64;  // split-length buckets of the unit order (64 tokens each)
constexpr int kMaxPending = 16;  // merges a CTA defers to the end of its work
constexpr uint64_t kMaxDecodeItems = 16384;  // items whose counters the workspace head holds

// Persistent form: a fixed grid of resident CTAs takes (item, split) work
// units -- CTA b unit b first, then the next free unit from a counter in the
// workspace (the merge puts it back to zero) -- so fast SMs take more splits
// and no wave leaves SMs idle; each split is computed exactly as
// mslim_decode_split computes it (same tiles, same warp order), so the
// partials -- and the outputs -- are the same bits.  The producer numbers the
// work: the splits of every (sequence, query block) unit (a prefix sum over
// at most kMaxUnits units, kept in shared memory with each unit's extent, so
// a chunk boundary reads nothing from global memory) times the KV-head
// chunks.  A unit's query rows come into a per-stage shared-memory slot by a
// bulk copy that completes with the unit's first K/V stage, so the consumers
// never wait on global memory for Q.
template <int D, int STAGES, bool PAGED>
__global__ void __launch_bounds__(kThreads)
    mslim_decode_persist(const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap, const DecodeParams p) {
    using S = Shape<D>;
    constexpr int kQSlot = 16 * D * 2;  // up to 16 (query, head) rows
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint16_t *qslot = reinterpret_cast<uint16_t *>(smem + STAGES * S::kStageBytes);  // [STAGES][16 x D]
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * (S::kStageBytes + kQSlot));
    uint64_t *empty = full + STAGES;
    uint64_t *merge_bar = empty + STAGES;  // bulk copies of a merge's partials
    StageMeta *meta = reinterpret_cast<StageMeta *>(merge_bar + 1);
    int *prefix = reinterpret_cast<int *>(meta + STAGES);  // [kMaxUnits + 1] first split of each position
    int *utok = prefix + kMaxUnits + 1;                     // [kMaxUnits] token count of each unit
    int *order = utok + kMaxUnits;                          // [kMaxUnits] unit at each position
    int *hist = order + kMaxUnits;                          // [kLenBuckets] positions per split length
    volatile int *is_last = hist + kLenBuckets;             // consumers: merge the item now
    volatile int *pend_n = is_last + 1;                     // consumers: merges deferred so far
    volatile int *pend = pend_n + 1;                        // [kMaxPending] (item | nsplits << 16)

    griddep_launch_dependents();
    griddep_wait();  // inputs, and the counter the previous merge reset
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(merge_bar, 1);
        *pend_n = 0;
        fence_mbarrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer --
        // Units are taken longest split first (a counting sort on the split
        // length, 64-token buckets), so the last units of the launch are the
        // shortest and the CTAs finish close together; the order decides only
        // which CTA computes a split, never its arithmetic.
        const int units = p.n_seq * p.q_blocks;
        constexpr int kPer = kMaxUnits / 32;
        // Units go round-robin over the lanes (unit k * 32 + lane), so a batch
        // of up to 32 units is ranked in one round.  This lane's token counts
        // first, all loads in flight together (the shared-memory stores below
        // would otherwise order them one by one).
        const int rounds = (units + 31) / 32;
        int toks[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int uix = k * 32 + lane;
            toks[k] = (k < rounds && uix < units) ? unit_tokens(p, uix / p.q_blocks) : 0;
        }
        for (int b = lane; b < kLenBuckets; b += 32) hist[b] = 0;
        __syncwarp();
        int key[kPer], rank[kPer];  // split-length bucket (kLenBuckets: no unit), place in it
        int nspl[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            key[k] = kLenBuckets;  // no unit
            nspl[k] = 0;
            rank[k] = 0;
            if (k >= rounds) continue;  // warp-uniform
            const int uix = k * 32 + lane;
            if (uix < units) {
                utok[uix] = toks[k];
                const UnitExtent u = unit_extent_of(p, toks[k], uix % p.q_blocks);
                nspl[k] = u.splits;
                key[k] = u.splits ? kLenBuckets - 1 - min(kLenBuckets - 1, u.slen / kTileT) : kLenBuckets - 1;
            }
            // rank within the bucket: the lanes holding the same key this round
            // share one shared-memory atomic (most units of a batch fall in a
            // few buckets, and colliding atomics would serialise)
            const unsigned peers = __match_any_sync(0xffffffffu, key[k]);
            const int leader = __ffs(peers) - 1;
            int base = 0;
            if (lane == leader && key[k] < kLenBuckets) base = atomicAdd(&hist[key[k]], __popc(peers));
            base = __shfl_sync(0xffffffffu, base, leader);
            rank[k] = base + __popc(peers & ((1u << lane) - 1u));
        }
        __syncwarp();
        {
            // exclusive scan of the bucket counts, two buckets per lane
            static_assert(kLenBuckets == 64, "two buckets per lane");
            const int h0 = hist[2 * lane], h1 = hist[2 * lane + 1];
            int incl = h0 + h1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            __syncwarp();
            hist[2 * lane] = incl - h0 - h1;
            hist[2 * lane + 1] = incl - h1;
        }
        __syncwarp();
        // order entry: unit index (low 16 bits) and its split count
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            if (key[k] < kLenBuckets) order[hist[key[k]] + rank[k]] = (k * 32 + lane) | (nspl[k] << 16);
        __syncwarp();
        // splits per position, then a warp-wide prefix sum over positions
        int cnt[kPer];
        int local = 0;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int pk = lane * kPer + k;
            cnt[k] = pk < units ? (order[pk] >> 16) : 0;
            local += cnt[k];
        }
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            prefix[lane * kPer + k] = run;
            run += cnt[k];
        }
        if (lane == 31) prefix[kMaxUnits] = incl;
        __syncwarp();
        if (lane == 0) {
            prefetch_tmap(&kmap);
            prefetch_tmap(&vmap);
            const int H = p.kvheads * p.head_chunks;
            const long long total = (long long)prefix[kMaxUnits] * H;
            const int hc = p.heads_per_cta;
            int i = 0;  // stages filled so far
            bool ok = true;
            long long g = blockIdx.x;  // the first unit needs no counter
            while (ok && g < total) {
                const long long g_next = (long long)gridDim.x + atomicAdd(p.work_counter, 1u);
                const int w = (int)(g / H), hcid = (int)(g % H);
                int lo = 0, hi = units;  // the last position whose prefix is <= w
                while (hi - lo > 1) {
                    const int mid = (lo + hi) >> 1;
                    if (prefix[mid] <= w) lo = mid;
                    else hi = mid;
                }
                const int unit = order[lo] & 0xffff;
                const int seq = unit / p.q_blocks;
                const UnitExtent ue = unit_extent_of(p, utok[unit], unit % p.q_blocks);
                const int qg_first = ue.qg_first;
                const int qg_last = ue.qg_last;
                const int cta_end = ue.cta_end;
                const int slen = ue.slen;
                const int split = w - prefix[lo];
                const int t_begin = split * slen;
                const int t_end = min(cta_end, t_begin + slen);
                const int ntiles = (t_end - t_begin + kTileT - 1) / kTileT;
                const int kvh = hcid / p.head_chunks, hchunk = hcid % p.head_chunks;
                for (int t = 0; t < ntiles; ++t, ++i) {
                    const int s = i % STAGES;
                    if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1, p.status, 4)) {
                        ok = false;
                        break;
                    }
                    StageMeta &m = meta[s];
                    m.seq = seq;
                    m.kvh = kvh;
                    m.hchunk = hchunk;
                    m.split = split;
                    m.prior = ue.prior;
                    m.qg_first = qg_first;
                    m.qg_last = qg_last;
                    m.t0 = t_begin + t * kTileT;
                    m.t_end = t_end;
                    m.flags = (t == 0 ? kMetaFirst : 0) | (t == ntiles - 1 ? kMetaLast : 0) |
                              (g + 2LL * gridDim.x >= total ? kMetaLate : 0);
                    m.item = unit * H + hcid;
                    m.nsplits = prefix[lo + 1] - prefix[lo];
                    if (t == 0) {
                        // the unit's query rows, hc heads of each query row side by side
                        const uint32_t row_bytes = (uint32_t)(hc * p.head_dim * 2);
                        const int nrows = qg_last - qg_first + 1;
                        mbar_expect_tx(&full[s], row_bytes * nrows);
                        for (int qi = 0; qi < nrows; ++qi)
                            bulk_load(qslot + (size_t)s * (kQSlot / 2) + (size_t)qi * hc * p.head_dim,
                                      p.q + (((size_t)seq * p.nq + qg_first + qi) * p.qheads + kvh * p.group +
                                             hchunk * hc) * p.head_dim,
                                      row_bytes, &full[s]);
                    }
                    uint8_t *kdst = smem + s * S::kStageBytes;
                    issue_tile<D, PAGED>(&kmap, &vmap, p, &full[s], kdst, kdst + S::kTensorBytes, seq, kvh, m.t0);
                }
                g = g_next;
            }
            if (ok) {  // the end of this CTA's work: a stage with no bytes
                const int s = i % STAGES;
                if (mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1, p.status, 4)) {
                    meta[s].flags = kMetaDone;
                    mbar_arrive(&full[s]);
                    ++i;
                }
            }
            // this CTA takes no more work; the last CTA to get here puts the
            // counters back to zero for the next call
            __threadfence();
            if (atomicAdd(&p.work_counter[1], 1u) == gridDim.x - 1) {
                p.work_counter[0] = 0u;
                p.work_counter[1] = 0u;
            }
            // Do not retire while our copies may still be landing in this CTA's
            // shared memory: wait (bounded) for the last stages filled.
            for (int k = max(0, i - STAGES); k < i; ++k) mbar_wait(&full[k % STAGES], (k / STAGES) & 1, p.status, 2);
        }
        // units without keys (empty sessions) have no split to merge: their
        // rows are written as zeros by CTA u % grid
        for (int uix = 0; uix < units; ++uix) {
            if (uix % (int)gridDim.x != (int)blockIdx.x || unit_extent_of(p, utok[uix], uix % p.q_blocks).splits != 0)
                continue;
            const int seq = uix / p.q_blocks;
            const int qg_first = (uix % p.q_blocks) * p.q_per_cta;
            const int qg_last = min(p.nq, qg_first + p.q_per_cta) - 1;
            const size_t first = ((size_t)seq * p.nq + qg_first) * p.qheads * p.head_dim;
            const size_t n = (size_t)(qg_last - qg_first + 1) * p.qheads * p.head_dim;
            for (size_t x = lane; x < n; x += 32) p.out[first + x] = 0;
        }
        return;
    }

    // ----------------------------------------------------------- consumers --
    if constexpr (PAGED) {
        // While the producer numbers the units, the grid's consumer threads
        // pull the page table into L2 (one 128-byte line each, within the
        // table), so the first tiles' page lookups do not wait on DRAM.
        const size_t lines = ((size_t)p.n_seq * p.max_pages * sizeof(int32_t) + 127) / 128;
        const size_t line = (size_t)blockIdx.x * (kConsumerWarps * 32) + threadIdx.x;
        if (line < lines) prefetch_l2(reinterpret_cast<const uint8_t *>(p.page_table) + line * 128);
    }
    DecodeConsumer<D, false> cs;
    DecodeItem it{};
    bool streamed = false;  // the loop ended on the producer's end-of-work stage
    uint32_t merges = 0;    // merges this CTA ran from bulk copies (merge_bar's phase)
    // one item's partials: rows x splits records
    auto bulk_fits = [&](int nsplits, size_t bytes) {
        return (size_t)p.q_per_cta * p.heads_per_cta * nsplits * (D + kPartPad) * sizeof(float) <= bytes;
    };
    for (int i = 0;; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1, p.status, 3)) break;
        const StageMeta m = meta[s];
        if (m.flags & kMetaDone) {
            streamed = true;
            break;
        }
        uint8_t *stage = smem + s * S::kStageBytes;
        if (m.flags & kMetaFirst) {
            it.seq = m.seq;
            it.kvh = m.kvh;
            it.hchunk = m.hchunk;
            it.split = m.split;
            it.prior = m.prior;
            it.qg_first = m.qg_first;
            it.qg_last = m.qg_last;
            cs.begin(p, it, lane, qslot + (size_t)s * (kQSlot / 2));
        }
        cs.tile(stage, m.t0, m.t_end, p.scale_log2, warp, lane);
        if (m.flags & kMetaLast) {
            // the split's last stage is the combine's (and the merge's)
            // scratch before it is released
            cs.finish(p, it, reinterpret_cast<float *>(stage), warp, lane);
            cs.clear();
            // The partial is out (warp 0 wrote it).  The CTA whose split
            // completes the item merges it: at once while plenty of work is
            // left (other CTAs take up the slack), and in the launch's last
            // two waves after its own last split, from the queue of pending
            // merges (a merge under full HBM load costs several L2 round trips
            // and would make this CTA's remaining split finish last), or at
            // once when that queue is full.
            if (warp == 0) __threadfence();
            asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
            if (threadIdx.x == 0) {
                int now = 0;
                if (atomicAdd(&p.item_counters[m.item], 1u) + 1 == (unsigned)m.nsplits) {
                    if ((m.flags & kMetaLate) && *pend_n < kMaxPending) pend[(*pend_n)++] = m.item | (m.nsplits << 16);
                    else now = 1;
                }
                *is_last = now;
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
            if (*is_last) {
                __threadfence();
                if (bulk_fits(m.nsplits, S::kStageBytes))
                    merge_item_bulk<D>(p, it, m.nsplits, reinterpret_cast<float *>(stage), merge_bar, (merges++) & 1);
                else
                    merge_item<D>(p, it, m.nsplits, reinterpret_cast<float *>(stage));
                if (threadIdx.x == 0) p.item_counters[m.item] = 0u;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    // The deferred merges, once this CTA has no more splits to compute (every
    // stage is consumed, so stage 0 is the merge's scratch).  Skipped after a
    // wait that gave up: copies may still be landing in the stages.
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
    const int npend = streamed ? *pend_n : 0;
    if (npend > 0) {
        __threadfence();
        const int H = p.kvheads * p.head_chunks;
        for (int k = 0; k < npend; ++k) {
            const int e = pend[k];
            const int item = e & 0xffff, nsplits = e >> 16;
            const int unit = item / H, hcid = item % H;
            DecodeItem mi{};
            mi.seq = unit / p.q_blocks;
            mi.qg_first = (unit % p.q_blocks) * p.q_per_cta;
            mi.qg_last = min(p.nq, mi.qg_first + p.q_per_cta) - 1;
            mi.kvh = hcid / p.head_chunks;
            mi.hchunk = hcid % p.head_chunks;
            if (bulk_fits(nsplits, (size_t)STAGES * S::kStageBytes))
                merge_item_bulk<D>(p, mi, nsplits, reinterpret_cast<float *>(smem), merge_bar, (merges++) & 1);
            else
                merge_item<D>(p, mi, nsplits, reinterpret_cast<float *>(smem));
            if (threadIdx.x == 0) p.item_counters[item] = 0u;
        }
    }
}

// Splits whose partials feed (sequence, query row qg): the same count the
// split kernels produce for the row's query block.
__device__ __forceinline__ int merge_splits(const DecodeParams &p, int seq, int qg) {
    return unit_extent(p, seq, qg / p.q_per_cta).splits;
}

// One CTA per (sequence, query row, query head), thread d = output dim d, for
// rows of at most MAXS splits: every partial of the row is requested at once
// (the split maxima and sums through shared memory, thread d's acc[d] of
// every split in registers), so the combine costs one memory round trip
// instead of one per batch of splits.  Same arithmetic and order as
// mslim_decode_merge: m = max_s m_s, w_s = 2^(m_s - m), l and acc summed in
// split order, out = bf16(acc * (1 / l)).
template <int D, int MAXS>
__global__ void __launch_bounds__(D) mslim_decode_merge_row(const DecodeParams p, uint16_t *out) {
    griddep_launch_dependents();
    griddep_wait();  // the split kernel's partials
    if (blockIdx.x == 0 && threadIdx.x == 0 && p.work_counter) *p.work_counter = 0u;  // for the next call
    __shared__ float ms[MAXS], ls[MAXS];
    const size_t item = blockIdx.x;
    const size_t sq = item / p.qheads;  // seq * nq + qg
    const int qg = (int)(sq % p.nq);
    const int seq = (int)(sq / p.nq);
    constexpr int kRowF = D + kPartPad;
    const int splits = merge_splits(p, seq, qg);
    const float *src = p.partials + item * p.max_splits * kRowF;
    const int d = threadIdx.x;
    float av[MAXS];
#pragma unroll
    for (int s = 0; s < MAXS; ++s) av[s] = (s < splits) ? src[s * kRowF + d] : 0.f;
    for (int s = d; s < splits; s += D) {
        ms[s] = src[s * kRowF + D];
        ls[s] = src[s * kRowF + D + 1];
    }
    __syncthreads();
    float m = -INFINITY;
#pragma unroll
    for (int s = 0; s < MAXS; ++s)
        if (s < splits) m = fmaxf(m, ms[s]);
    const float mb = (m == -INFINITY) ? 0.f : m;
    float l = 0.f, acc = 0.f;
#pragma unroll
    for (int s = 0; s < MAXS; ++s) {
        if (s < splits) {
            const float w = fast_exp2(ms[s] - mb);
            l += w * ls[s];
            acc += w * av[s];
        }
    }
    const float inv = (l > 0.f) ? 1.0f / l : 0.f;
    if (d < p.head_dim) {
        if (p.out_f32)
            p.out_f32[item * p.head_dim + d] = acc * inv;
        else
            out[item * p.head_dim + d] = bf16_bits_rn(acc * inv);
    }
}

// One warp per (sequence, query row, query head): fixed split-order combine
// for rows of any number of splits.
template <int D>
__global__ void __launch_bounds__(128) mslim_decode_merge(const DecodeParams p, uint16_t *out) {
    griddep_launch_dependents();
    griddep_wait();  // the split kernel's partials
    if (blockIdx.x == 0 && threadIdx.x == 0 && p.work_counter) *p.work_counter = 0u;  // for the next call
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t item = (size_t)blockIdx.x * 4 + warp;
    const size_t items = (size_t)p.n_seq * p.nq * p.qheads;
    if (item >= items) return;
    const size_t sq = item / p.qheads;  // seq * nq + qg
    const int qg = (int)(sq % p.nq);
    const int seq = (int)(sq / p.nq);
    constexpr int kRowF = D + kPartPad;
    constexpr int kPer = D / 32;
    const int splits = merge_splits(p, seq, qg);
    const float *src = p.partials + item * p.max_splits * kRowF;
    // the maximum over the splits: lane s reads split s (32 per round), then a
    // warp max (exact, so the order does not matter)
    float m = -INFINITY;
    for (int s0 = 0; s0 < splits; s0 += 32)
        if (s0 + lane < splits) m = fmaxf(m, src[(s0 + lane) * kRowF + D]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float mb = (m == -INFINITY) ? 0.f : m;
    float l = 0.f;
    float acc[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) acc[k] = 0.f;
    // splits accumulated in order; eight at a time have their loads in flight
    constexpr int kBatch = 8;
    int s = 0;
    for (; s + kBatch <= splits; s += kBatch) {
        float mv[kBatch], lv[kBatch], pv[kBatch][kPer];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const float *part = src + (s + u) * kRowF;
            mv[u] = part[D];
            lv[u] = part[D + 1];
#pragma unroll
            for (int k = 0; k < kPer; ++k) pv[u][k] = part[lane + 32 * k];
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const float w = fast_exp2(mv[u] - mb);
            l += w * lv[u];
#pragma unroll
            for (int k = 0; k < kPer; ++k) acc[k] += w * pv[u][k];
        }
    }
    for (; s < splits; ++s) {
        const float *part = src + s * kRowF;
        const float w = fast_exp2(part[D] - mb);
        l += w * part[D + 1];
#pragma unroll
        for (int k = 0; k < kPer; ++k) acc[k] += w * part[lane + 32 * k];
    }
    const float inv = (l > 0.f) ? 1.0f / l : 0.f;
    const size_t obase = item * p.head_dim;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int d = lane + 32 * k;
        if (d >= p.head_dim) continue;
        if (p.out_f32)
            p.out_f32[obase + d] = acc[k] * inv;
        else
            out[obase + d] = bf16_bits_rn(acc[k] * inv);
    }
}

template <int D, int STAGES, bool PAGED, bool QSPLIT>
cudaError_t launch_impl(const CUtensorMap &kmap, const CUtensorMap &vmap, const DecodeParams &p,
                        uint16_t *out, cudaStream_t stream) {
    using S = Shape<D>;
    cudaError_t err;
    const uint64_t units = (uint64_t)p.n_seq * p.q_blocks;
    if (p.persistent && !QSPLIT && p.work_counter && p.item_counters && !p.out_f32 && units <= (uint64_t)kMaxUnits &&
        units * p.kvheads * p.head_chunks <= (uint64_t)kMaxDecodeItems && p.max_splits <= kMaxFusedSplits &&
        (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0) {
        // persistent: as many CTAs as stay resident, at most one per work unit
        const size_t smem = (size_t)STAGES * (S::kStageBytes + 16 * D * 2) + (2 * STAGES + 1) * sizeof(uint64_t) +
                            STAGES * sizeof(StageMeta) + (3 * kMaxUnits + 1 + kLenBuckets + 2 + kMaxPending) * sizeof(int) +
                            1024;
        auto kernel = mslim_decode_persist<D, STAGES, PAGED>;
        static int per_sm = 0, sms = 0;  // resident CTAs of this form (same on every B200)
        if (!per_sm) {
            err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (err != cudaSuccess) return err;
            int dev = 0, n = 0, b = 0;
            if ((err = cudaGetDevice(&dev)) != cudaSuccess) return err;
            if ((err = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return err;
            if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kThreads, smem)) != cudaSuccess)
                return err;
            sms = n;
            per_sm = b > 0 ? b : 1;
        } else if ((err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
                   cudaSuccess) {
            return err;
        }
        const uint64_t work = units * p.kvheads * p.head_chunks * p.max_splits;
        const unsigned ctas = (unsigned)std::min<uint64_t>(work, (uint64_t)per_sm * sms);
        return launch_pdl(kernel, dim3(ctas), dim3(kThreads), smem, stream, kmap, vmap, p);  // merges in-kernel
    } else {
        const size_t smem = (size_t)STAGES * S::kStageBytes + 2 * STAGES * sizeof(uint64_t) + 1024;
        auto kernel = mslim_decode_split<D, STAGES, PAGED, QSPLIT>;
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err != cudaSuccess) return err;
        dim3 grid(p.max_splits, p.kvheads * p.head_chunks, p.n_seq * p.q_blocks);
        err = launch_pdl(kernel, grid, dim3(kThreads), smem, stream, kmap, vmap, p);
    }
    if (err != cudaSuccess) return err;
    const size_t items = (size_t)p.n_seq * p.nq * p.qheads;
    if (items <= 0x7fffffffull) {
        const dim3 rows((unsigned)items);
        if (p.max_splits <= 8) return launch_pdl(mslim_decode_merge_row<D, 8>, rows, dim3(D), 0, stream, p, out);
        if (p.max_splits <= 16) return launch_pdl(mslim_decode_merge_row<D, 16>, rows, dim3(D), 0, stream, p, out);
        if (p.max_splits <= 32) return launch_pdl(mslim_decode_merge_row<D, 32>, rows, dim3(D), 0, stream, p, out);
        if (p.max_splits <= 64) return launch_pdl(mslim_decode_merge_row<D, 64>, rows, dim3(D), 0, stream, p, out);
    }
    return launch_pdl(mslim_decode_merge<D>, dim3((unsigned)((items + 3) / 4)), dim3(128), 0, stream, p, out);
}

}  // namespace

cudaError_t launch_decode(int head_dim, bool paged, const CUtensorMap &kmap,
                          const CUtensorMap &vmap, const DecodeParams &p, uint16_t *out,
                          cudaStream_t stream) {
    const bool qsplit = p.q_f32 != nullptr;
    if (qsplit && paged) return cudaErrorInvalidValue;
    switch (head_dim) {
        case 64:
            if (qsplit) return launch_impl<64, 4, false, true>(kmap, vmap, p, out, stream);
            return paged ? launch_impl<64, 4, true, false>(kmap, vmap, p, out, stream)
                         : launch_impl<64, 4, false, false>(kmap, vmap, p, out, stream);
        case 128:
            if (qsplit) return launch_impl<128, 3, false, true>(kmap, vmap, p, out, stream);
            return paged ? launch_impl<128, 3, true, false>(kmap, vmap, p, out, stream)
                         : launch_impl<128, 3, false, false>(kmap, vmap, p, out, stream);
        case 256:
            if (qsplit) return launch_impl<256, 2, false, true>(kmap, vmap, p, out, stream);
            return paged ? launch_impl<256, 2, true, false>(kmap, vmap, p, out, stream)
                         : launch_impl<256, 2, false, false>(kmap, vmap, p, out, stream);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace mslim
