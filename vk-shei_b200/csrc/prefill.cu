// prefill.cu -- chunked causal prefill attention on the 5th-generation tensor
// cores (tcgen05 + TMEM, TMA-fed).
//
// Replaces the reference prefill attention (assets/gpu_llm.cl:462-543, a
// materialised [B][QH][history] score matrix; and the tiled online kernel of
// assets/tiled_attention.cl:9-130 for queries > 1): query row i (absolute
// position prior + i) attends to keys 0..=prior+i.
//
// Two kernels share one numeric contract (S = Q K^T and O += P V as
// tcgen05.mma kind::f16, M 128 x N 128, fp32 accumulators in TMEM; an online
// softmax in exp2 whose running max moves only by more than 2^8; P written
// back into TMEM as bf16 and consumed by a TS-MMA, A from TMEM -- P never goes
// through shared memory), so for the same inputs they return the same bits:
//
//   mslim_prefill_pair    even GQA groups (C2: group 4).  Persistent: one CTA
//       per SM walks (128-row query tile, pair of query heads sharing a KV
//       head) items, heaviest first in snake order; every staged K/V byte
//       serves both heads.  TMEM: S_A, S_B, O_A, O_B (128 columns each).
//       Tensor-core order per key tile: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1),
//       so one head's MMAs run while the other head's softmax works.  Warps:
//       TMA K, MMA (one elected lane issues each group of MMAs), TMA V, TMA Q
//       (the next item's Q is prefetched as soon as the current item's last S
//       completes), then a softmax warpgroup per head, one thread per query
//       row, which also rescales O in TMEM and writes the output through a
//       swizzled staging buffer, each warp its own 32 rows with its own bulk
//       tensor stores.
//   mslim_prefill_causal  odd groups, and head_dim 256: one head per CTA, S
//       double-buffered in TMEM (S(j+1) issued before PV(j)), eight softmax
//       warps taking half a key tile each and exchanging row maxima through
//       shared memory; 128-key tiles, or 64-key tiles at head_dim 256 (O then
//       takes 256 TMEM columns).
//
// head_dim: the kernels run at 64, 128 or 256; a smaller multiple of 8 (from
// 64) runs zero-padded by the TMA (columns past head_dim read as zeros, the
// stores stop at head_dim).
//
// TMA loads read this GPU's HBM only (128-byte swizzle, no multicast); K and
// V have separate rings, a K slot is released once S_j is computed, a V slot
// after PV_j.  Consecutive calls overlap through programmatic dependent
// launch: a call waits for its predecessor's memory before reading an input.
// Every mbarrier wait is bounded; the CTA always frees its TMEM.
#include <atomic>
#include <mutex>

#include "../../include/mslim_cuda.h"
#include "prefill.cuh"

namespace mslim {

namespace {

constexpr int kRows = 128;                 // query rows per CTA = TMEM lanes
constexpr int kKeys = 128;                 // keys per tile
constexpr int kBox = kRows * 128;          // one [128 rows][64 bf16] swizzled box: 16 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;     // S[2] at 0/128, O (accumulating) at 256
// A row's running max is only moved (and O rescaled in TMEM) when a tile's
// max exceeds it by more than 2^8; until then P uses the stale max, which is
// exact arithmetic (numerator and denominator share it) with P <= 256.
constexpr float kRescaleLog2 = 8.0f;

// Instruction descriptors (kind::f16): D f32, A/B bf16, M=128, N=128;
// S: A and B K-major; PV: B (V) MN-major.
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((kKeys >> 3) << 17) | ((kRows >> 4) << 24);
constexpr uint32_t kIdescPV = kIdescS | (1u << 16);

// One head per CTA, S double-buffered in TMEM (any GQA group; head_dim 128,
// or 256 with 64-key tiles).
//   TMEM: S[0], S[1] (kKeys columns each), then O (head_dim columns,
//         accumulating).  P(j) is written as bf16 pairs over the first
//         kKeys / 2 columns of S[j & 1] once S(j) sits in registers, and
//         O += P V is a TS-MMA (A from TMEM).
//   Tensor-core order: S(0), then per tile j: S(j+1), PV(j).  S(j+1) goes to
//         the other buffer, so the softmax of tile j+1 overlaps PV(j) and
//         S(j+2); S(j+2) reuses buffer j & 1 only after PV(j) (in-order pipe).
//   smem: Q (128 rows x head_dim), K ring 2 x 32 KB, V ring 2 x 32 KB
//         (160 KB at head_dim 128, 192 KB at 256).
//   Warps: 0 TMA Q+K, 1 MMA, 2 TMA V, 3 idle; 4-11 softmax, a warp pair
//         (w, w+4) per 32 TMEM lanes (rows): warps 4-7 the first half of a
//         tile's keys (and of the output dims), warps 8-11 the second half;
//         the pair exchanges row maxima through shared memory.
template <int D>
struct SingleShape {
    static_assert(D == 128 || D == 256, "single-head prefill head_dim");
    static constexpr int kKeysT = D == 256 ? 64 : 128;  // keys per tile
    static constexpr int kBoxes = D / 64;               // 64-column boxes per row
    static constexpr int kQBytes = kBoxes * kBox;       // Q: 128 rows
    static constexpr int kKVBox = kKeysT * 128;         // one [kKeysT rows][64 bf16] box
    static constexpr int kTileBytes = kBoxes * kKVBox;  // one K or V tile (32 KB)
    static constexpr int kHalfKeys = kKeysT / 2;        // keys of one softmax half
    static constexpr int kHalfDims = D / 2;             // output dims of one softmax half
    static constexpr uint32_t kColO = 2 * kKeysT;       // O after S[0], S[1]
    static constexpr int kOffK = kQBytes;
    static constexpr int kOffV = kOffK + 2 * kTileBytes;
    static constexpr int kOffX = kOffV + 2 * kTileBytes;  // row-max / row-sum exchange
    static constexpr int kOffBar = kOffX + 6 * kRows * 4;
    static constexpr int kSmemBytes = kOffBar + 512 + 1024;
    // S: M 128, N kKeysT, A and B K-major; PV: N = D, B (V) MN-major
    static constexpr uint32_t kIdescS =
        (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kKeysT >> 3) << 17) | ((kRows >> 4) << 24);
    static constexpr uint32_t kIdescPV =
        (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(D >> 3) << 17) | ((kRows >> 4) << 24);
    static_assert(kColO + D <= kTmemCols, "TMEM columns");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory per block");
};
static_assert(SingleShape<128>::kColO == kColO && SingleShape<128>::kIdescS == kIdescS &&
                  SingleShape<128>::kIdescPV == kIdescPV,
              "head_dim 128 keeps the single-head layout");
constexpr int kSThreads = 12 * 32;
// One pair of P columns in eight goes through the FMA-pipe exp2, the rest
// through MUFU (the measured best split); both prefill kernels use the same
// pairs, so for the same inputs they return the same bits.
#define MSLIM_EXP_ON_FMA(i) (((i) & 7) == 7)

struct SingleBars {
    uint64_t q_full;
    uint64_t k_full[2], k_empty[2];
    uint64_t v_full[2], v_empty[2];
    uint64_t s_full[2];   // [buffer]
    uint64_t p_full[2];   // [buffer], 8 warps per tile: a phase per two tiles, so the
                          // MMA warp can never fall two phases behind
    uint64_t o_full;      // once per PV (waited only for PV(j-1) while S(j) is held)
    uint64_t o_done;      // once, after the last PV
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ void pair_sync(int quarter) {
    // the two softmax warps that own the same 32 TMEM lanes (rows)
    asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kSThreads, 1)
    mslim_prefill_causal(const __grid_constant__ CUtensorMap qmap,
                         const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    using SS = SingleShape<D>;
    constexpr int kKeysT = SS::kKeysT;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    SingleBars *bars = reinterpret_cast<SingleBars *>(smem + SS::kOffBar);
    volatile int *abort_flag = &bars->abort;

    const int bid = blockIdx.x;
    const int qt = p.n_qtiles - 1 - bid / p.qheads;  // heavy (late) tiles first
    const int qh = bid % p.qheads;
    const int kvh = qh / p.group;
    const int q0 = qt * kRows;
    const int last_row = min(q0 + kRows, p.queries) - 1;
    const int n_kv = (p.prior + last_row) / kKeysT + 1;  // key tiles this CTA needs
    const int first_pos = p.prior + q0;                 // smallest query position here

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->k_full[b], 1);
            mbar_init(&bars->k_empty[b], 1);
            mbar_init(&bars->v_full[b], 1);
            mbar_init(&bars->v_empty[b], 1);
            mbar_init(&bars->s_full[b], 1);
            mbar_init(&bars->p_full[b], 8);
        }
        mbar_init(&bars->o_full, 1);
        mbar_init(&bars->o_done, 1);
        bars->abort = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const uint32_t sbase = smem_u32(smem);

    if (warp < 4) {
        if ((warp == 0 || warp == 2) && lane == 0) {
            // ------------------------------------------------------ TMA --
            const bool is_k = warp == 0;
            const CUtensorMap *map = is_k ? &kmap : &vmap;
            uint64_t *full = is_k ? bars->k_full : bars->v_full;
            uint64_t *empty = is_k ? bars->k_empty : bars->v_empty;
            uint8_t *ring = smem + (is_k ? SS::kOffK : SS::kOffV);
            prefetch_tmap(map);
            if (is_k) {
                prefetch_tmap(&qmap);
                mbar_arrive_expect_tx(&bars->q_full, SS::kQBytes);
#pragma unroll
                for (int bx = 0; bx < SS::kBoxes; ++bx)
                    tma_load_3d(smem + bx * kBox, &qmap, &bars->q_full, bx * 64, qh, q0);
            }
            int issued = 0;
            for (int j = 0; j < n_kv && !*abort_flag; ++j) {
                const int st = j & 1;
                if (!mbar_wait(&empty[st], ((j >> 1) & 1) ^ 1, p.status, is_k ? 11 : 14)) {
                    *abort_flag = 1;
                    break;
                }
                uint8_t *dst = ring + st * SS::kTileBytes;
                mbar_arrive_expect_tx(&full[st], SS::kTileBytes);
#pragma unroll
                for (int bx = 0; bx < SS::kBoxes; ++bx)
                    tma_load_3d(dst + bx * SS::kKVBox, map, &full[st], bx * 64, kvh, j * kKeysT);
                issued = j + 1;
            }
            // Our copies must land before the CTA can retire.
            if (is_k) mbar_wait(&bars->q_full, 0, p.status, 12);
            for (int j = max(0, issued - 2); j < issued; ++j)
                mbar_wait(&full[j & 1], (j >> 1) & 1, p.status, 13);
        } else if (warp == 1) {
            // ------------------------------------------------------ MMA --
            // the whole warp runs the loop; umma_* elect the issuing lane
            auto wait_all = [&](uint64_t *bar, uint32_t parity, int where) -> bool {
                return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.status, where));
            };
            auto issue_s = [&](int j) -> bool {
                if (!wait_all(&bars->k_full[j & 1], (j >> 1) & 1, 22)) return false;
                tc_fence_after();
                const uint32_t kaddr = sbase + SS::kOffK + (j & 1) * SS::kTileBytes;
                const uint32_t sdst = tmem + kColS + (j & 1) * kKeysT;
                if constexpr (D == 128) {
                    umma_bf16_ss_k128(sdst, umma_desc_sw128(sbase, 16, 1024), umma_desc_sw128(kaddr, 16, 1024),
                                      SS::kIdescS, 0u, kBox >> 4);
                } else {
                    // one group of four K=16 steps per 64-column box (Q and K
                    // boxes have different row counts, so different strides)
#pragma unroll
                    for (int bx = 0; bx < SS::kBoxes; ++bx)
                        umma_bf16_ss_k64(sdst, umma_desc_sw128(sbase + bx * kBox, 16, 1024),
                                         umma_desc_sw128(kaddr + bx * SS::kKVBox, 16, 1024), SS::kIdescS,
                                         bx > 0 ? 1u : 0u);
                }
                umma_commit(&bars->s_full[j & 1]);
                umma_commit(&bars->k_empty[j & 1]);
                return true;
            };
            bool ok = wait_all(&bars->q_full, 0, 21) && issue_s(0);
            for (int j = 0; ok && j < n_kv; ++j) {
                if (__any_sync(0xffffffffu, *abort_flag != 0)) {
                    ok = false;
                    break;
                }
                if (j + 1 < n_kv) ok = issue_s(j + 1);
                ok = ok && wait_all(&bars->v_full[j & 1], (j >> 1) & 1, 26) &&
                     wait_all(&bars->p_full[j & 1], (j >> 1) & 1, 24);
                if (!ok) break;
                tc_fence_after();
                const uint32_t vaddr = sbase + SS::kOffV + (j & 1) * SS::kTileBytes;
                // 64 keys (four K=16 steps) per call: P columns advance 32 per
                // 64 keys, V rows 64 per 64 keys; V's 64-column boxes are
                // kKVBox bytes apart along N
#pragma unroll
                for (int kc = 0; kc < kKeysT / 64; ++kc)
                    umma_bf16_ts_k64(tmem + SS::kColO, tmem + kColS + (j & 1) * kKeysT + kc * 32,
                                     umma_desc_sw128(vaddr + kc * 4 * 16 * 128, SS::kKVBox, 1024), SS::kIdescPV,
                                     (j > 0 || kc > 0) ? 1u : 0u, (16 * 128) >> 4);
                umma_commit(j + 1 < n_kv ? &bars->o_full : &bars->o_done);
                umma_commit(&bars->v_empty[j & 1]);
            }
            if (!ok && lane == 0) *abort_flag = 1;
        }
    } else {
        // ---------------------------------------------------------- softmax --
        const int quarter = warp & 3;
        constexpr int kHK = SS::kHalfKeys, kHD = SS::kHalfDims;
        const int half = (warp >> 2) - 1;  // keys kHK*half..+kHK-1 of a tile, output dims kHD*half..
        const int row = quarter * 32 + lane;
        const int col0 = half * kHK;       // this half's first S column (key)
        const int dim0 = half * kHD;       // this half's first output dim
        const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
        const uint32_t ocol = lane_addr + SS::kColO + dim0;
        const int qpos = p.prior + q0 + row;
        const float scale = p.scale_log2;
        float *xmax = reinterpret_cast<float *>(smem + SS::kOffX);  // [2 parity][2 half][128]
        float *xsum = xmax + 4 * kRows;                           // [2 half][128]
        float m_used = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int b = j & 1;
            const bool got = mbar_wait(&bars->s_full[b], (j >> 1) & 1, p.status, 31);
            if (!__all_sync(0xffffffffu, got) || __any_sync(0xffffffffu, *abort_flag != 0)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t scol = lane_addr + kColS + b * kKeysT;
            float v[kHK];
            if constexpr (kHK == 64) tmem_ld64(scol + col0, v);
            else tmem_ld32(scol + col0, v);
            const int k0 = j * kKeysT + col0;
            if (j * kKeysT + kKeysT - 1 > first_pos) {
#pragma unroll
                for (int i = 0; i < kHK; ++i)
                    if (k0 + i > qpos) v[i] = -INFINITY;
            }
            float m8[8];
#pragma unroll
            for (int a = 0; a < 8; ++a) m8[a] = fmaxf(v[a], v[a + 8]);
#pragma unroll
            for (int i = 16; i < kHK; ++i) m8[i & 7] = fmaxf(m8[i & 7], v[i]);
            float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
            xmax[(b * 2 + half) * kRows + row] = mx;
            // after this barrier both halves hold their S values in registers,
            // so P may overwrite the S columns below
            pair_sync(quarter);
            mx = fmaxf(mx, xmax[(b * 2 + (half ^ 1)) * kRows + row]) * scale;
            const bool move = mx > m_used + kRescaleLog2;
            const float m_new = move ? mx : m_used;
            const float base = (m_new == -INFINITY) ? 0.f : m_new;
            const float alpha = move ? fast_exp2(m_used - base) : 1.f;
            if (j > 0 && __any_sync(0xffffffffu, move)) {
                // O must hold PV(j-1) before it is rescaled
                const bool gotc = mbar_wait(&bars->o_full, (j - 1) & 1, p.status, 32);
                if (!__all_sync(0xffffffffu, gotc)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < kHD / 32; ++c) {
                    float o[32];
                    tmem_ld32(ocol + c * 32, o);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= alpha;
                    tmem_st32(ocol + c * 32, o);
                }
            }
            const uint64_t scale2 = f2_pack(scale, scale);
            const uint64_t nbase2 = f2_pack(-base, -base);
            uint64_t sum2[4] = {0, 0, 0, 0};
            uint32_t w[kHK / 2];
#pragma unroll
            for (int i = 0; i < kHK / 2; ++i) {
                float x0, x1;
                f2_unpack(f2_fma(f2_pack(v[2 * i], v[2 * i + 1]), scale2, nbase2), x0, x1);
                const float p0 = MSLIM_EXP_ON_FMA(i) ? exp2_fma(x0) : fast_exp2(x0);
                const float p1 = MSLIM_EXP_ON_FMA(i) ? exp2_fma(x1) : fast_exp2(x1);
                sum2[i & 3] = f2_add(sum2[i & 3], f2_pack(p0, p1));
                w[i] = pack_bf16x2(p0, p1);
            }
            // this half's keys -> P columns (kHK/2)*half.. of S[b]
            if constexpr (kHK == 64) tmem_st32u_nowait(scol + half * 32, w);
            else tmem_st16u_nowait(scol + half * 16, w);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->p_full[b]);
            float s8[8];
#pragma unroll
            for (int a = 0; a < 4; ++a) f2_unpack(sum2[a], s8[2 * a], s8[2 * a + 1]);
            const float ps = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
            l_run = l_run * alpha + ps;
            m_used = m_new;
        }
        const bool last = ok && mbar_wait(&bars->o_done, 0, p.status, 33);
        if (__all_sync(0xffffffffu, last)) {
            tc_fence_after();
            xsum[half * kRows + row] = l_run;
            pair_sync(quarter);
            const float inv = 1.0f / (l_run + xsum[(half ^ 1) * kRows + row]);
            const int qrow = q0 + row;
            // rows are head_dim elements apart; columns past head_dim (zero
            // padding of a head_dim below the kernel's) are not written
            uint16_t *dst = p.out + ((size_t)qrow * p.qheads + qh) * p.head_dim + dim0;
#pragma unroll
            for (int c = 0; c < kHD / 32; ++c) {
                float o[32];
                tmem_ld32(ocol + c * 32, o);
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(o[2 * i] * inv, o[2 * i + 1] * inv);
                if (qrow < p.queries) {
#pragma unroll
                    for (int t = 0; t < 4; ++t)
                        if (dim0 + c * 32 + t * 8 < p.head_dim)
                            reinterpret_cast<uint4 *>(dst + c * 32)[t] =
                                make_uint4(w[4 * t], w[4 * t + 1], w[4 * t + 2], w[4 * t + 3]);
                }
            }
        } else {
            *abort_flag = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Two heads per CTA (ping-pong), P kept in tensor memory, persistent CTAs.  A
// work item is one 128-row query tile of two query heads that share a KV head:
// every K/V byte loaded serves both, both heads have the same causal extent,
// and while one head's softmax warpgroup works, the tensor core runs the other
// head's MMAs.  One CTA per SM walks the items heaviest first (late query tiles
// see the most keys) in snake order -- CTA b of G takes ranks b, 2G-1-b,
// 2G+b, ... -- which pairs heavy items with light ones.
//   smem: Q_A, Q_B (32 KB each), K ring 2 x 32 KB, V ring 2 x 32 KB, output
//         staging 16 KB per head (224 KB);
//   TMEM: S_A (0), S_B (128), O_A (256), O_B (384); P_h is written as bf16
//         pairs over the first 64 columns of S_h once S_h has been read, and
//         O_h += P_h V is a TS-MMA (A from TMEM), so P never touches shared
//         memory.
//   Tensor-core order per item: S_A(0), S_B(0), then per key tile j:
//         PV_A(j), S_A(j+1), PV_B(j), S_B(j+1).  S_h(j+1) overwrites P_h(j)
//         only after PV_h(j), which precedes it in the (in-order) tcgen05
//         pipe, and S_h(j) done implies PV_h(j-1) done.
//   Across items the K/V rings and the per-tile barriers keep counting; Q of
//   the next item is loaded as soon as the current item's last S MMAs have
//   completed, so the next item's S(0) overlaps the current output write.
//   Warps: 0 TMA K, 1 MMA, 2 TMA V, 3 TMA Q; 4-7 softmax head A, 8-11
//          softmax head B.  ptxas compiles every path within the registers the
//          launch allows (__launch_bounds__(384, 1): 168 per thread), and one CTA
//          fills the SM, so the kernel moves no registers between warpgroups.
//   head_dim: 128 (two 64-column boxes per Q/K/V/O row) or 64 (one box; the S
//   product then has four K=16 steps and O_h uses 64 of its 128 columns).
template <int D>
struct PairShape {
    static_assert(D == 64 || D == 128, "pair prefill head_dim");
    static constexpr int kBoxes = D / 64;                // 64-column boxes per row
    static constexpr int kQBytes = kBoxes * kBox;        // one head's Q tile
    static constexpr int kTileBytes = kBoxes * kBox;     // one K or V tile
    static constexpr int kOffQ = 0;                      // Q_h at h * kQBytes
    static constexpr int kOffK = 2 * kQBytes;            // K slot s at kOffK + s * kTileBytes
    static constexpr int kOffV = kOffK + 2 * kTileBytes;
    static constexpr int kOffStage = kOffV + 2 * kTileBytes;  // head h's 16 KB output box at + h * kBox
    static constexpr int kOffBar = kOffStage + 2 * kBox;
    static constexpr int kSmemBytes = kOffBar + 512 + 1024;
    // PV: M 128 query rows, N = head_dim, B (V) MN-major
    static constexpr uint32_t kIdescPV =
        (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(D >> 3) << 17) | ((kRows >> 4) << 24);
    static_assert(kSmemBytes <= 227 * 1024, "shared memory per block");
};
static_assert(PairShape<128>::kIdescPV == kIdescPV, "head_dim 128 keeps the single-head kernel's PV shape");
constexpr int kPThreads = 12 * 32;

struct PairBars {
    uint64_t q_full, q_empty;  // once per item
    uint64_t k_full[2], k_empty[2];
    uint64_t v_full[2], v_empty[2];
    uint64_t s_full[2];        // [head], once per key tile
    uint64_t p_full[2][2];     // [head][half]: P of keys 64*half..+63 written (4 warps)
    uint64_t o_done[2];        // [head], once per item, after the head's last PV
    uint32_t tmem_base;
    int abort;
};

// The item of this CTA's round `round` (false once the CTA is done).
struct PairItem {
    int qh0;        // heads qh0, qh0 + 1 share KV head qh0 / group
    int q0;         // first query row of the tile
    int n_kv;       // key tiles the tile attends to
    int first_pos;  // position of the tile's first query row
};
__device__ __forceinline__ bool pair_item(const PrefillParams &p, int round, PairItem &it) {
    const int grid = (int)gridDim.x, b = (int)blockIdx.x;
    const int pairs = p.qheads / 2;
    const long long r = (long long)round * grid + ((round & 1) ? (grid - 1 - b) : b);
    if (r >= (long long)p.n_qtiles * pairs) return false;
    const int qt = p.n_qtiles - 1 - (int)(r / pairs);
    it.qh0 = 2 * (int)(r % pairs);
    it.q0 = qt * kRows;
    const int last_row = min(it.q0 + kRows, p.queries) - 1;
    it.n_kv = (p.prior + last_row) / kKeys + 1;
    it.first_pos = p.prior + it.q0;
    return true;
}

template <int D>
__global__ void __launch_bounds__(kPThreads, 1)
    mslim_prefill_pair(const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap,
                       const __grid_constant__ CUtensorMap omap, const PrefillParams p) {
    using PS = PairShape<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    PairBars *bars = reinterpret_cast<PairBars *>(smem + PS::kOffBar);
    volatile int *abort_flag = &bars->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        mbar_init(&bars->q_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->k_full[b], 1);
            mbar_init(&bars->k_empty[b], 1);
            mbar_init(&bars->v_full[b], 1);
            mbar_init(&bars->v_empty[b], 1);
            mbar_init(&bars->s_full[b], 1);
            mbar_init(&bars->p_full[b][0], 4);
            mbar_init(&bars->p_full[b][1], 4);
            mbar_init(&bars->o_done[b], 1);
        }
        bars->abort = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const uint32_t sbase = smem_u32(smem);
    // Programmatic dependent launch: the next kernel of the stream may begin
    // launching (its CTAs take SMs as ours retire), and nothing below reads an
    // input or writes the output before the previous kernel's memory is visible.
    griddep_launch_dependents();
    griddep_wait();

    if (warp < 4) {
        if ((warp == 0 || warp == 2) && lane == 0) {
            // -------------------------------------------------- TMA K / V --
            const bool is_k = warp == 0;
            const CUtensorMap *map = is_k ? &kmap : &vmap;
            uint64_t *full = is_k ? bars->k_full : bars->v_full;
            uint64_t *empty = is_k ? bars->k_empty : bars->v_empty;
            uint8_t *ring = smem + (is_k ? PS::kOffK : PS::kOffV);
            prefetch_tmap(map);
            int g = 0;  // key tiles loaded so far, over all items
            bool run = true;
            PairItem it;
            for (int round = 0; run && pair_item(p, round, it); ++round) {
                const int kvh = it.qh0 / p.group;
                for (int j = 0; j < it.n_kv; ++j) {
                    const int st = g & 1;
                    if (*abort_flag ||
                        !mbar_wait(&empty[st], ((g >> 1) & 1) ^ 1, p.status, is_k ? 41 : 42)) {
                        *abort_flag = 1;
                        run = false;
                        break;
                    }
                    uint8_t *dst = ring + st * PS::kTileBytes;
                    mbar_arrive_expect_tx(&full[st], PS::kTileBytes);
#pragma unroll
                    for (int b = 0; b < PS::kBoxes; ++b)
                        tma_load_3d(dst + b * kBox, map, &full[st], b * 64, kvh, j * kKeys);
                    ++g;
                }
            }
            // our copies must land before the CTA can retire
            for (int t = max(0, g - 2); t < g; ++t) mbar_wait(&full[t & 1], (t >> 1) & 1, p.status, 44);
        } else if (warp == 3 && lane == 0) {
            // ------------------------------------------------------ TMA Q --
            prefetch_tmap(&qmap);
            int loaded = 0;
            PairItem it;
            for (int round = 0; pair_item(p, round, it); ++round) {
                // Q of the previous item is free once its last S MMAs completed
                if (*abort_flag ||
                    (round > 0 && !mbar_wait(&bars->q_empty, (round - 1) & 1, p.status, 43))) {
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&bars->q_full, 2 * PS::kQBytes);
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int b = 0; b < PS::kBoxes; ++b)
                        tma_load_3d(smem + PS::kOffQ + h * PS::kQBytes + b * kBox, &qmap, &bars->q_full, b * 64,
                                    it.qh0 + h, it.q0);
                ++loaded;
            }
            if (loaded > 0) mbar_wait(&bars->q_full, (loaded - 1) & 1, p.status, 45);
        } else if (warp == 1) {
            // ------------------------------------------------------ MMA --
            // the whole warp runs the loop; umma_* elect the issuing lane
            auto wait_all = [&](uint64_t *bar, uint32_t parity, int where) -> bool {
                return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.status, where));
            };
            auto issue_s = [&](int h, int slot) {
                const uint32_t qaddr = sbase + PS::kOffQ + h * PS::kQBytes;
                const uint32_t kaddr = sbase + PS::kOffK + slot * PS::kTileBytes;
                // the eight K=16 steps from one elect (see umma_bf16_ss_k128)
                if constexpr (D == 128)
                    umma_bf16_ss_k128(tmem + h * 128, umma_desc_sw128(qaddr, 16, 1024),
                                      umma_desc_sw128(kaddr, 16, 1024), kIdescS, 0u, kBox >> 4);
                else
                    umma_bf16_ss_k64(tmem + h * 128, umma_desc_sw128(qaddr, 16, 1024),
                                     umma_desc_sw128(kaddr, 16, 1024), kIdescS, 0u);
                umma_commit(&bars->s_full[h]);
            };
            int g = 0;  // key tiles consumed so far, over all items
            bool ok = true;
            PairItem it;
            for (int round = 0; ok && pair_item(p, round, it); ++round) {
                ok = wait_all(&bars->q_full, round & 1, 51) && wait_all(&bars->k_full[g & 1], (g >> 1) & 1, 52);
                if (!ok) break;
                tc_fence_after();
                issue_s(0, g & 1);
                issue_s(1, g & 1);
                umma_commit(&bars->k_empty[g & 1]);
                if (it.n_kv == 1) umma_commit(&bars->q_empty);
                for (int j = 0; ok && j < it.n_kv; ++j, ++g) {
                    if (__any_sync(0xffffffffu, *abort_flag != 0)) {
                        ok = false;
                        break;
                    }
                    const bool next = j + 1 < it.n_kv;
                    ok = wait_all(&bars->v_full[g & 1], (g >> 1) & 1, 54);
                    if (ok && next) ok = wait_all(&bars->k_full[(g + 1) & 1], ((g + 1) >> 1) & 1, 52);
                    const uint32_t vaddr = sbase + PS::kOffV + (g & 1) * PS::kTileBytes;
                    for (int h = 0; ok && h < 2; ++h) {
                        // PV over keys 0..63 starts while the softmax still
                        // writes P for keys 64..127
                        for (int half = 0; ok && half < 2; ++half) {
                            ok = wait_all(&bars->p_full[h][half], g & 1, 55);
                            if (!ok) break;
                            tc_fence_after();
                            // keys 64*half .. +63: four K=16 steps from one elect
                            umma_bf16_ts_k64(tmem + kColO + h * 128, tmem + h * 128 + half * 32,
                                             umma_desc_sw128(vaddr + half * 4 * 16 * 128, kBox, 1024),
                                             PS::kIdescPV, (j > 0 || half > 0) ? 1u : 0u, (16 * 128) >> 4);
                        }
                        if (!ok) break;
                        if (next) issue_s(h, (g + 1) & 1);
                        else umma_commit(&bars->o_done[h]);
                    }
                    if (ok) {
                        umma_commit(&bars->v_empty[g & 1]);
                        if (next) {
                            umma_commit(&bars->k_empty[(g + 1) & 1]);
                            if (j + 2 == it.n_kv) umma_commit(&bars->q_empty);
                        }
                    }
                }
            }
            if (!ok && lane == 0) *abort_flag = 1;
        }
    } else {
        // ---------------------------------------------------------- softmax --
        // warpgroup 1 (warps 4-7) owns head qh0, warpgroup 2 (8-11) head qh0 + 1;
        // one thread per query row, all 128 keys of a tile
        const int h = (warp >> 2) - 1;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
        const uint32_t scol = lane_addr + h * 128;
        const uint32_t ocol = lane_addr + kColO + h * 128;
        const float scale = p.scale_log2;
        uint8_t *stage = smem + PS::kOffStage + h * kBox;
        int g = 0;  // key tiles seen so far, over all items
        bool ok = true;
        PairItem it;
        for (int round = 0; ok && pair_item(p, round, it); ++round) {
            const int qpos = p.prior + it.q0 + row;
            float m_used = -INFINITY, l_run = 0.f;
            for (int j = 0; j < it.n_kv; ++j, ++g) {
                const bool got = mbar_wait(&bars->s_full[h], g & 1, p.status, 61);
                if (!__all_sync(0xffffffffu, got) || __any_sync(0xffffffffu, *abort_flag != 0)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int k0 = j * kKeys;
                // the whole 128-key row of S in registers (one load, one wait)
                float v[128];
                tmem_ld128(scol, v);
                if (k0 + kKeys - 1 > it.first_pos) {
#pragma unroll
                    for (int i = 0; i < 128; ++i)
                        if (k0 + i > qpos) v[i] = -INFINITY;
                }
                // row max of the raw scores (the scale is positive, so it is
                // applied to the max only); four independent three-input chains
                float m4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
                for (int i = 4; i + 8 <= 128; i += 8)
#pragma unroll
                    for (int a = 0; a < 4; ++a) m4[a] = fmax3(m4[a], v[i + a], v[i + 4 + a]);
#pragma unroll
                for (int a = 0; a < 4; ++a) m4[a] = fmaxf(m4[a], v[124 + a]);
                const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale;
                const bool move = mx > m_used + kRescaleLog2;
                const float m_new = move ? mx : m_used;
                const float base = (m_new == -INFINITY) ? 0.f : m_new;
                const float alpha = move ? fast_exp2(m_used - base) : 1.f;
                // P = 2^(s*scale - base); keys 64c..64c+63 go to columns
                // 32c..32c+31, whose S values are already in registers.  Each
                // half is announced on its own barrier; O is rescaled before
                // the first.
                const uint64_t scale2 = f2_pack(scale, scale);
                const uint64_t nbase2 = f2_pack(-base, -base);
                uint64_t sum2[4] = {0, 0, 0, 0};
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t w[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int e = c * 64 + 2 * i;
                        float x0, x1;
                        f2_unpack(f2_fma(f2_pack(v[e], v[e + 1]), scale2, nbase2), x0, x1);
                        const bool poly = MSLIM_EXP_ON_FMA(i);
                        const float p0 = poly ? exp2_fma(x0) : fast_exp2(x0);
                        const float p1 = poly ? exp2_fma(x1) : fast_exp2(x1);
                        sum2[i & 3] = f2_add(sum2[i & 3], f2_pack(p0, p1));
                        w[i] = pack_bf16x2(p0, p1);
                    }
                    tmem_st32u_nowait(scol + c * 32, w);
                    if (c == 0 && j > 0 && __any_sync(0xffffffffu, move)) {
                        // S_h(j) done implies PV_h(j-1) done: O_h is final for
                        // j-1, and PV_h(j) waits for the arrive below
#pragma unroll
                        for (int oc = 0; oc < D / 32; ++oc) {
                            float o[32];
                            tmem_ld32(ocol + oc * 32, o);
#pragma unroll
                            for (int i = 0; i < 32; ++i) o[i] *= alpha;
                            tmem_st32(ocol + oc * 32, o);
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->p_full[h][c]);
                }
                float s8[8];
#pragma unroll
                for (int a = 0; a < 4; ++a) f2_unpack(sum2[a], s8[2 * a], s8[2 * a + 1]);
                const float ps = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
                l_run = l_run * alpha + ps;
                m_used = m_new;
            }
            // ---- output of this item: O_h / l -> bf16, one 64-column box at a
            // time.  Each warp stages its own 32 rows (a 4 KB slice of the head's
            // 16 KB staging buffer, TMA 128-byte swizzled layout) and stores them
            // with its own bulk tensor store (32-row box), so no warp waits for
            // another's rows or for another's store to release the buffer; rows
            // past the last query are clipped by the store.
            const bool good = ok && __all_sync(0xffffffffu, mbar_wait(&bars->o_done[h], round & 1, p.status, 64));
            if (!good) *abort_flag = 1;
            tc_fence_after();
            const float inv = 1.0f / l_run;
            uint8_t *wstage = stage + quarter * 32 * 128;
            for (int box = 0; box < PS::kBoxes; ++box) {
                if (lane == 0) bulk_wait_read_all();  // this warp's previous store has read its slice
                __syncwarp();
                if (good) {
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        float o[32];
                        tmem_ld32(ocol + box * 64 + c * 32, o);
                        uint32_t w[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(o[2 * i] * inv, o[2 * i + 1] * inv);
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const int chunk = (c * 4 + t) ^ (lane & 7);
                            *reinterpret_cast<uint4 *>(wstage + lane * 128 + chunk * 16) =
                                make_uint4(w[4 * t], w[4 * t + 1], w[4 * t + 2], w[4 * t + 3]);
                        }
                    }
                    fence_proxy_async_smem();
                }
                __syncwarp();
                if (lane == 0 && good && *abort_flag == 0) {
                    tma_store_3d(&omap, wstage, box * 64, it.qh0 + h, it.q0 + quarter * 32);
                    bulk_commit_group();
                }
            }
            // the head's four warps continue or stop together
            if (named_bar_or(1 + h, 128, !good || *abort_flag != 0)) ok = false;
        }
        if (lane == 0) bulk_wait_all();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

bool prefill_supported(unsigned head_dim, unsigned group) {
    // The kernels run at head_dim 64 (two-head kernel), 128 (both) or 256
    // (single-head kernel, 64-key tiles); a smaller multiple of 8 runs
    // zero-padded: the tensor maps describe the caller's head_dim, the TMA
    // fills the columns past it with zeros (they add nothing to S, and their
    // O columns are zero), and the output stores stop at head_dim.
    return group >= 1 && head_dim >= 64 && head_dim <= 256 && head_dim % 8 == 0;
}

bool prefill_pairs_heads(unsigned group, unsigned head_dim) { return group % 2 == 0 && head_dim <= 128; }

unsigned prefill_kv_box_rows(unsigned head_dim) { return head_dim > 128 ? 64 : 128; }

namespace {

// Per-device launch setup, done once: shared-memory opt-in for both kernels,
// and the SM count.
struct PrefillDeviceSetup {
    std::atomic<int> state{0};  // 0 not yet, 1 ready, 2 failed
    cudaError_t err = cudaSuccess;
    int sms = 0;
};
constexpr int kMaxDevices = 64;
PrefillDeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mutex;

cudaError_t prefill_setup(int dev, int *sms) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    PrefillDeviceSetup &d = g_setup[dev];
    if (d.state.load(std::memory_order_acquire) == 0) {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (d.state.load(std::memory_order_relaxed) == 0) {
            cudaError_t err = cudaFuncSetAttribute(mslim_prefill_pair<128>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   PairShape<128>::kSmemBytes);
            if (err == cudaSuccess)
                err = cudaFuncSetAttribute(mslim_prefill_pair<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           PairShape<64>::kSmemBytes);
            if (err == cudaSuccess)
                err = cudaFuncSetAttribute(mslim_prefill_causal<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           SingleShape<128>::kSmemBytes);
            if (err == cudaSuccess)
                err = cudaFuncSetAttribute(mslim_prefill_causal<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           SingleShape<256>::kSmemBytes);
            if (err == cudaSuccess) err = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
            d.err = err;
            d.state.store(err == cudaSuccess ? 1 : 2, std::memory_order_release);
        }
    }
    if (d.state.load(std::memory_order_acquire) != 1) return d.err;
    *sms = d.sms;
    return cudaSuccess;
}

}  // namespace

cudaError_t launch_prefill(const CUtensorMap &qmap, const CUtensorMap &kmap,
                           const CUtensorMap &vmap, const CUtensorMap &omap,
                           const PrefillParams &p, cudaStream_t stream) {
    int dev = 0, sms = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    err = prefill_setup(dev, &sms);
    if (err != cudaSuccess) return err;
    if (prefill_pairs_heads((unsigned)p.group, (unsigned)p.head_dim)) {
        // persistent: one CTA per SM (at most one per item)
        const long long items = (long long)p.n_qtiles * (p.qheads / 2);
        const unsigned grid = (unsigned)(items < sms ? items : sms);
        if (p.head_dim <= 64)
            return launch_pdl(mslim_prefill_pair<64>, dim3(grid), dim3(kPThreads), PairShape<64>::kSmemBytes,
                              stream, qmap, kmap, vmap, omap, p);
        return launch_pdl(mslim_prefill_pair<128>, dim3(grid), dim3(kPThreads), PairShape<128>::kSmemBytes,
                          stream, qmap, kmap, vmap, omap, p);
    }
    const unsigned grid = (unsigned)(p.n_qtiles * p.qheads);
    if (p.head_dim > 128)
        mslim_prefill_causal<256><<<grid, kSThreads, SingleShape<256>::kSmemBytes, stream>>>(qmap, kmap, vmap, p);
    else
        mslim_prefill_causal<128><<<grid, kSThreads, SingleShape<128>::kSmemBytes, stream>>>(qmap, kmap, vmap, p);
    return counted(cudaGetLastError());
}

}  // namespace mslim
