// gemv.cu -- the decode step's projections (a few rows against a weight
// matrix) on the tcgen05 tensor cores.
//
// Replaces the reference's decode GEMVs (llm_gemv_bf16*, assets/gpu_llm.cl:
// 38-68, and the prefill-reuse forms of :553-733) for 1..16 activation rows:
// Y[m][n] = bf16(sum_k X[m][k] * W[n][k]), W in the [out][in] layout.
//
// The weight matrix is the A operand ("swap AB"): a CTA owns 128 output
// features, which are the 128 rows of one tcgen05.mma (kind::f16, M 128), and
// the activation rows are its N = 16 columns (rows past m are TMA zero fill).
// Every weight byte is read from HBM exactly once; the few activation rows
// are re-read per CTA from L2.  Warp roles, 128 threads:
//   warp 0  one lane issues TMA loads of [128 x 64] weight boxes and [16 x 64]
//           activation boxes (128-byte swizzle, this GPU's HBM, no multicast)
//           into a four-stage mbarrier ring.  The weights do not depend on
//           the preceding kernel, so the first four weight boxes are issued
//           before griddepcontrol.wait (programmatic dependent launch) and
//           stream while the predecessor finishes; the activations follow it;
//   warp 1  allocates 32 TMEM columns and, from one elected lane, issues four
//           K=16 MMAs per stage into the 128 x 16 fp32 accumulator, each
//           stage's commit releasing its ring slot;
//   all     read the accumulator with tcgen05.ld (thread t = output feature
//           t of the tile) and write bf16 rows.
// Long K is cut into up to eight splits so that the CTAs of a projection fill
// the GPU in one wave (three per SM).  The splits of one tile form a
// thread-block cluster: once the first CTA's own MMAs are done its ring is
// free, it signals its partners, they store their fp32 partials straight
// into its shared memory (distributed shared memory, no round trip) and
// arrive on its barrier, and it adds them in split order and rounds once, so
// the result does not depend on which CTA finished first, and nothing goes
// through global memory (no workspace).
//
// SwiGLU form (kSwiGLU): the weight rows are the gate and up projections
// interleaved in blocks of 64 (a tile's rows 0..63 are gate features
// 64t..64t+63, rows 64..127 the up features of the same block), so the tile
// that finishes a block's gate sums also holds its up sums: the epilogue rounds
// both to bf16 (as the plain form writes them), meets them in shared memory and
// writes bf16(bf16(silu(g)) * u) for 64 features (gpu_llm.cl
// llm_prefill_fused_swiglu_reuse8, one launch instead of a projection and an
// elementwise pass).
//
// RoPE + append form (head_dim 128): every tile of the q|k|v projection is one
// head; the epilogue rounds the tile to bf16 (as the plain form writes it),
// pairs features i and i + 64 through shared memory, rotates q and k heads
// with the shared RoPE arithmetic and writes q to q_out and k / v into the
// decode token's K/V row -- the work of mslim_rope_append_{dense,paged} on
// the projection's output, without writing or re-reading that output.
#include "gemv.cuh"

namespace mslim {

namespace {

constexpr int kEpiPlain = 0, kEpiSwiGLU = 1, kEpiRope = 2;
constexpr int kStages = 4;
constexpr int kWBytes = 128 * 128;              // [128 rows][64 bf16] swizzled: 16 KB
constexpr int kXBytes = 16 * 128;               // [16 rows][64 bf16]: 2 KB
constexpr int kStageBytes = kWBytes + kXBytes;  // 18 KB, a multiple of 1024
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 32;
constexpr uint32_t kCtasPerSm = 3;
constexpr uint32_t kMinKTiles = 4;  // 64-wide K steps per CTA at least
constexpr uint32_t kMaxSplits = 8;  // portable cluster size
// kind::f16 instruction descriptor: D f32, A = W and B = X bf16, both
// K-major, N = 16, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

struct GemvParams {
    uint32_t m, n, ldy;
    uint32_t k_steps, k_tiles, splits;
    uint16_t *y;
    int *status;
};

struct Bars {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc;
    uint64_t go;        // rank > 0: rank 0's ring is free for this CTA's partial
    uint64_t red_full;  // rank 0: every partner's partial has landed (S - 1 arrivals)
    uint32_t tmem_base;
};

// Remote (distributed shared memory) access within the cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(saddr), "r"(rank));
    return remote;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Arrives (release, cluster scope) on the mbarrier at `bar` of CTA `rank`.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t *bar, uint32_t rank) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(mapa(smem_u32(bar), rank))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait (acquire at cluster scope) for a phase completed by another
// CTA's remote arrival.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, int *status, int where) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t start = globaltimer();
    uint32_t spins = 0;
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (++spins >= 64) {
            spins = 0;
            if (globaltimer() - start > kWaitBoundNs) {
                record_timeout(status, where);
                return false;
            }
        }
    }
    return true;
}

// Split cluster barrier: every thread arrives once right after set-up and
// waits once before its first remote access, so the barrier's latency hides
// behind the K stream.
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int32_t x,
                                            int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (wait in the same
// asm block, so no use of the registers is scheduled before the load lands).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int kEpi>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    mslim_gemv_tc(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                  const GemvParams p, const __grid_constant__ GemvRopeAppend e) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars *bars = reinterpret_cast<Bars *>(smem + kStages * kStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t tile = blockIdx.x, split = blockIdx.y;
    const uint32_t ks0 = split * p.k_tiles;
    const int nk = (int)min(p.k_tiles, p.k_steps - ks0);  // >= 1 by the plan

    griddep_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        mbar_init(&bars->acc, 1);
        mbar_init(&bars->go, 1);
        mbar_init(&bars->red_full, p.splits > 1 ? p.splits - 1 : 1);
        fence_mbarrier_init();
    }
    if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    cluster_arrive();  // this CTA's barriers exist; partners may signal them after the wait
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&wmap);
            prefetch_tmap(&xmap);
            const int pre = min(kStages, nk);
            const int32_t n0 = (int32_t)(tile * 128);
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&bars->full[i], kStageBytes);
                tma_load_2d(smem + i * kStageBytes, &wmap, &bars->full[i], (int32_t)((ks0 + i) * 64), n0);
            }
            griddep_wait();  // the activation rows come from the preceding kernel
            for (int i = 0; i < pre; ++i)
                tma_load_2d(smem + i * kStageBytes + kWBytes, &xmap, &bars->full[i], (int32_t)((ks0 + i) * 64), 0);
            int issued = pre;
            for (int i = pre; i < nk; ++i) {
                const int s = i % kStages;
                if (!mbar_wait(&bars->empty[s], ((i / kStages) & 1) ^ 1, p.status, 21)) break;
                uint8_t *dst = smem + s * kStageBytes;
                const int32_t kx = (int32_t)((ks0 + i) * 64);
                mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
                tma_load_2d(dst, &wmap, &bars->full[s], kx, n0);
                tma_load_2d(dst + kWBytes, &xmap, &bars->full[s], kx, 0);
                issued = i + 1;
            }
            // the copies still in flight land before the CTA may retire
            for (int i = max(0, issued - kStages); i < issued; ++i)
                mbar_wait(&bars->full[i % kStages], (i / kStages) & 1, p.status, 22);
        }
    } else if (warp == 1) {
        for (int i = 0; i < nk; ++i) {
            const int s = i % kStages;
            if (!mbar_wait(&bars->full[s], (i / kStages) & 1, p.status, 23)) break;
            tc_fence_after();
            const uint32_t wa = smem_u32(smem + s * kStageBytes);
            umma_bf16_ss_k64(tmem, umma_desc_sw128(wa, 16, 1024), umma_desc_sw128(wa + kWBytes, 16, 1024),
                             kIdesc, i > 0 ? 1u : 0u);
            umma_commit(&bars->empty[s]);
        }
        umma_commit(&bars->acc);
    }

    // ---- epilogue: thread t holds output feature tile*128 + t, rows 0..15 ----
    __syncwarp();  // warp 0's producer lane rejoins before the warp-wide loads
    mbar_wait(&bars->acc, 0, p.status, 24);
    tc_fence_after();
    float acc[16];
    tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16), acc);
    griddep_wait();  // outputs are written only once the predecessor is done
    const uint32_t n = tile * 128 + threadIdx.x;
    const uint32_t M = p.m;
    // The tile's finished sums -> outputs (every thread of the CTA calls it).
    auto write_rows = [&](const float (&v)[16]) {
        if constexpr (kEpi == kEpiPlain) {
            if (n < p.n) {
#pragma unroll
                for (uint32_t r = 0; r < 16; ++r)
                    if (r < M) p.y[(size_t)r * p.ldy + n] = bf16_bits_rn(v[r]);
            }
        } else if constexpr (kEpi == kEpiSwiGLU) {
            // the ring is idle (every stage consumed, every partial added)
            float *up = reinterpret_cast<float *>(smem);  // [16 rows][64 features]
            __syncthreads();
            if (threadIdx.x >= 64) {
#pragma unroll
                for (uint32_t r = 0; r < 16; ++r)
                    if (r < M) up[r * 64 + (threadIdx.x - 64)] = bf16_round(v[r]);
            }
            __syncthreads();
            const uint32_t i = tile * 64 + threadIdx.x;  // output feature
            if (threadIdx.x < 64 && i < p.n / 2) {
#pragma unroll
                for (uint32_t r = 0; r < 16; ++r)
                    if (r < M)
                        p.y[(size_t)r * p.ldy + i] = bf16_bits_rn(silu_mul(bf16_round(v[r]), up[r * 64 + threadIdx.x]));
            }
        } else {
            // the ring is idle: the tile's bf16 values, [16 rows][128 features]
            float *xs = reinterpret_cast<float *>(smem);
            __syncthreads();
#pragma unroll
            for (uint32_t r = 0; r < 16; ++r)
                if (r < M) xs[r * 128 + threadIdx.x] = bf16_round(v[r]);
            __syncthreads();
            const uint32_t head = tile, t = threadIdx.x, i = t & 63;
            const bool is_q = head < e.qheads, is_k = !is_q && head < e.qheads + e.kvheads;
            // KV head of a k or v tile (0 for q tiles, whose rows go to q_out)
            const uint32_t kh = is_q ? 0 : is_k ? head - e.qheads : head - e.qheads - e.kvheads;
            // Each row's destination once, by thread r, in parallel: its
            // position and (paged) physical page, or -1 where the checks of
            // mslim_rope_append_{dense,paged} reject the row (nothing is
            // written for it and the status word records it).  [16] int pairs
            // after the tile's values.
            int32_t *row_pos = reinterpret_cast<int32_t *>(xs + 16 * 128);
            int32_t *row_phys = row_pos + 16;
            if (t < M) {
                const int32_t pp = e.positions[t];
                int32_t phys = 0;
                bool bad;
                if (e.page_table) {
                    bad = pp < 0 || (uint64_t)pp >= (uint64_t)e.max_pages * e.page_tokens;
                    if (!bad) phys = e.page_table[(size_t)t * e.max_pages + (uint32_t)pp / e.page_tokens];
                    bad = bad || phys < 0 || (uint32_t)phys >= e.n_pages;
                } else {
                    bad = pp < 0 || (uint32_t)pp >= e.max_tokens;
                }
                if (bad && p.status) atomicExch(p.status, MSLIM_DEVICE_BAD_PAGE_CODE);
                row_pos[t] = bad ? -1 : pp;
                row_phys[t] = phys;
            }
            __syncthreads();
            // the (cos, sin) of every (row, pair) once, shared by the tile's
            // threads: [16 rows][64 pairs]
            float2 *cs = reinterpret_cast<float2 *>(row_pos + 32);
            if (is_q || is_k) {
                for (uint32_t j = t; j < M * 64; j += kThreads) {
                    const int32_t pj = row_pos[j >> 6];
                    cs[j] = pj >= 0 ? rope_cs(rope_angle(e.table, (int)(j & 63), (uint32_t)pj)) : make_float2(0.f, 0.f);
                }
            }
            __syncthreads();
            for (uint32_t r = 0; r < M; ++r) {
                const int32_t pp = row_pos[r];
                if (pp < 0) continue;
                float out;
                if (is_q || is_k) {
                    float oa, ob;
                    rope_rotate(xs[r * 128 + i], xs[r * 128 + i + 64], cs[r * 64 + i], oa, ob);
                    out = t < 64 ? oa : ob;
                } else {
                    out = xs[r * 128 + t];
                }
                uint16_t *dst;
                if (is_q) {
                    dst = e.q_out + ((size_t)r * e.qheads + head) * 128;
                } else {
                    uint16_t *base = is_k ? e.k_dst : e.v_dst;
                    dst = e.page_table
                              ? base + (((size_t)row_phys[r] * e.kvheads + kh) * e.page_tokens +
                                        (uint32_t)pp % e.page_tokens) * 128
                              : base + (((size_t)r * e.max_tokens + (uint32_t)pp) * e.kvheads + kh) * 128;
                }
                dst[t] = bf16_bits_rn(out);
            }
        }
    };
    cluster_wait();  // every CTA of the cluster has its barriers initialised
    if (p.splits == 1) {
        write_rows(acc);
    } else {
        // Partners push their fp32 partials into rank 0's ring, which is idle
        // once rank 0's own MMAs completed (every stage was consumed):
        // partner r's rows at red[r - 1][row][feature].  Rank 0 says "go"
        // when its ring is free, adds the partials in rank order when all
        // have landed, and writes the row.  Partners leave after their push;
        // rank 0, whose memory they write, leaves last.
        const uint32_t rank = cluster_ctarank();
        float *red = reinterpret_cast<float *>(smem);
        if (rank == 0) {
            if (threadIdx.x >= 1 && threadIdx.x < p.splits) mbar_arrive_remote(&bars->go, threadIdx.x);
            mbar_wait_cluster(&bars->red_full, 0, p.status, 26);
            float sum[16];
#pragma unroll
            for (uint32_t r = 0; r < 16; ++r) sum[r] = acc[r];
            for (uint32_t s = 1; s < p.splits; ++s) {
#pragma unroll
                for (uint32_t r = 0; r < 16; ++r)
                    if (r < M) sum[r] += red[((s - 1) * 16 + r) * 128 + threadIdx.x];
            }
            write_rows(sum);
        } else {
            mbar_wait_cluster(&bars->go, 0, p.status, 25);
            const uint32_t dst = mapa(smem_u32(red + ((rank - 1) * 16) * 128 + threadIdx.x), 0);
#pragma unroll
            for (uint32_t r = 0; r < 16; ++r)
                if (r < M) st_cluster_f32(dst + r * 512, acc[r]);
            asm volatile("fence.acq_rel.cluster;" ::: "memory");
            __syncthreads();
            if (threadIdx.x == 0) mbar_arrive_remote(&bars->red_full, 0);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

GemvPlan gemv_plan(uint32_t m, uint32_t n, uint32_t k) {
    (void)m;
    GemvPlan pl{};
    pl.n_tiles = (n + 127) / 128;
    pl.k_steps = (k + 63) / 64;
    // One wave of CTAs (kCtasPerSm per SM) when the tiles allow: the largest
    // split count (at most eight, at least kMinKTiles K steps per CTA) whose
    // CTAs all fit at once, so they start together and finish together; a
    // second, nearly empty wave would stream its few CTAs with the HBM idle.
    // Tiles beyond one wave already fill the GPU unsplit.
    const uint32_t slots = 148u * kCtasPerSm;
    pl.splits = 1;
    for (uint32_t s = 2; s <= kMaxSplits; ++s) {
        const uint32_t kt = (pl.k_steps + s - 1) / s;
        const uint32_t splits = (pl.k_steps + kt - 1) / kt;  // no empty split
        if (kt < kMinKTiles || (uint64_t)pl.n_tiles * splits > slots) break;
        pl.splits = splits;
    }
    pl.k_tiles = (pl.k_steps + pl.splits - 1) / pl.splits;
    pl.splits = (pl.k_steps + pl.k_tiles - 1) / pl.k_tiles;
    return pl;
}

namespace {

cudaError_t launch_gemv_any(const CUtensorMap &xmap, const CUtensorMap &wmap, const GemvPlan &plan,
                            const GemvParams &p, const GemvRopeAppend &e, int epi, cudaStream_t stream) {
    const size_t smem = (size_t)kStages * kStageBytes + sizeof(Bars) + 1024;
    auto kernel = epi == kEpiSwiGLU ? mslim_gemv_tc<kEpiSwiGLU>
                                    : epi == kEpiRope ? mslim_gemv_tc<kEpiRope> : mslim_gemv_tc<kEpiPlain>;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.n_tiles, plan.splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = plan.splits;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return counted(cudaLaunchKernelEx(&cfg, kernel, xmap, wmap, p, e));
}

}  // namespace

cudaError_t launch_gemv_tc(const CUtensorMap &xmap, const CUtensorMap &wmap, const GemvPlan &plan, uint32_t m,
                           uint32_t n, uint16_t *y, uint32_t ldy, int *status, cudaStream_t stream, bool swiglu) {
    GemvParams p{};
    p.m = m;
    p.n = n;
    p.ldy = ldy;
    p.k_steps = plan.k_steps;
    p.k_tiles = plan.k_tiles;
    p.splits = plan.splits;
    p.y = y;
    p.status = status;
    return launch_gemv_any(xmap, wmap, plan, p, GemvRopeAppend{}, swiglu ? kEpiSwiGLU : kEpiPlain, stream);
}

cudaError_t launch_gemv_qkv_rope_append(const CUtensorMap &xmap, const CUtensorMap &wmap, const GemvPlan &plan,
                                        uint32_t m, uint32_t n, const GemvRopeAppend &e, int *status,
                                        cudaStream_t stream) {
    GemvParams p{};
    p.m = m;
    p.n = n;
    p.ldy = n;
    p.k_steps = plan.k_steps;
    p.k_tiles = plan.k_tiles;
    p.splits = plan.splits;
    p.y = nullptr;
    p.status = status;
    return launch_gemv_any(xmap, wmap, plan, p, e, kEpiRope, stream);
}


}  // namespace mslim
