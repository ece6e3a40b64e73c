// tp_allreduce.cu -- row-parallel partial sums of the tensor-parallel decode
// step (the o-projection and the MLP down projection, src/gpu_llm/mod.rs
// run_layer split over KV-head groups) reduced over NVLink peer memory inside
// the kernel that applies the residual add and the next RMSNorm.
//
// One CTA per row (decode: one row per session).  Lane r of warp 0 makes this
// rank's partial visible at system scope, publishes the row's call number into
// rank r's flag slot for this rank, and waits (bounded by %globaltimer) until
// rank r's number has arrived in this rank's flags.  Then the CTA reads the row
// from every rank with plain 16-byte loads that fetch afresh (ld.cv: the slot
// addresses repeat every second call), sums in fp32 in rank
// order (so every rank computes identical bits), rounds once to bf16, adds the
// residual and normalises as mslim_rmsnorm does.
//
// The partials are double-buffered by the caller (slot = call index & 1): a
// rank can be at most one call ahead of a peer (it waits for the peer's
// number), so the buffer it overwrites two calls later has been read.
#include "tp_allreduce.cuh"

namespace mslim {

namespace {

constexpr int kTpThreads = 256;
constexpr uint64_t kTpWaitBoundNs = 2000000000ull;  // error path only

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void nano_sleep(uint32_t ns) { asm volatile("nanosleep.u32 %0;" ::"r"(ns)); }

__device__ __forceinline__ void st_relaxed_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One 16-byte chunk of the row: every rank's partial summed in rank order in
// fp32, rounded once, added to the residual; returns the new x chunk and adds
// its squares to `sum` (element order fixed, so every rank gets the same bits).
template <int W>
__device__ __forceinline__ uint4 tp_reduce_chunk(const TpCommDev &c, size_t off, uint32_t i, uint4 xv,
                                                 float &sum) {
    uint4 p[W];
#pragma unroll
    for (int r = 0; r < W; ++r) p[r] = __ldcv(reinterpret_cast<const uint4 *>(c.data[r] + off + i));
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < W; ++r) {
        const uint32_t pv[4] = {p[r].x, p[r].y, p[r].z, p[r].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc[2 * k] += bf16lo_f32(pv[k]);
            acc[2 * k + 1] += bf16hi_f32(pv[k]);
        }
    }
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t nw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float a = bf16lo_f32(xw[k]) + bf16_round(acc[2 * k]);
        const float b = bf16hi_f32(xw[k]) + bf16_round(acc[2 * k + 1]);
        nw[k] = pack_bf16x2(a, b);
        const float na = bf16lo_f32(nw[k]), nb = bf16hi_f32(nw[k]);
        sum += na * na;
        sum += nb * nb;
    }
    return make_uint4(nw[0], nw[1], nw[2], nw[3]);
}

__device__ __forceinline__ uint4 tp_norm_chunk(uint4 v, uint4 wt, float scale) {
    const uint32_t xv[4] = {v.x, v.y, v.z, v.w};
    const uint32_t wv[4] = {wt.x, wt.y, wt.z, wt.w};
    uint32_t ov[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        ov[k] = pack_bf16x2(bf16_round(bf16lo_f32(xv[k]) * scale) * bf16lo_f32(wv[k]),
                            bf16_round(bf16hi_f32(xv[k]) * scale) * bf16hi_f32(wv[k]));
    return make_uint4(ov[0], ov[1], ov[2], ov[3]);
}

// Rows up to kTpThreads * 8 * kTpRegIters elements are held in registers: this
// rank's x and the norm weights are loaded before the wait for the peers (they
// do not depend on them) and x is not read back for the second pass.
constexpr int kTpRegIters = 4;

template <int W, bool kReg>
__global__ void __launch_bounds__(kTpThreads)
    mslim_tp_allreduce_rmsnorm(const TpCommDev c, uint32_t slot, uint16_t *__restrict__ x,
                               const uint16_t *__restrict__ w, uint16_t *__restrict__ y, float eps,
                               int *status) {
    // programmatic dependent launch: the partials, x and the flags are touched
    // only after the preceding projection has completed
    griddep_launch_dependents();
    griddep_wait();
    const uint32_t row = blockIdx.x;
    const uint32_t hidden = c.hidden;
    uint16_t *xr = x + (size_t)row * hidden;
    uint16_t *yr = y + (size_t)row * hidden;
    uint4 xv[kReg ? kTpRegIters : 1], wt[kReg ? kTpRegIters : 1];
    if constexpr (kReg) {
#pragma unroll
        for (int it = 0; it < kTpRegIters; ++it) {
            const uint32_t i = (threadIdx.x + it * kTpThreads) * 8;
            if (i < hidden) {
                xv[it] = *reinterpret_cast<const uint4 *>(xr + i);
                wt[it] = *reinterpret_cast<const uint4 *>(w + i);
            }
        }
    }
    __shared__ int s_ok;
    // warp 0: lane r (< W) publishes this rank's call number into rank r's
    // flags, then waits for rank r's number in this rank's flags; the lanes
    // work in parallel, each behind its own system-scope fence
    if (threadIdx.x < 32) {
        const uint32_t lane = threadIdx.x;
        // Call numbers wrap after 2^32 calls of a row (hours of serving at
        // batch-8 decode rates): they are compared as serial numbers, and 0 --
        // the value of a flag no peer has written -- is never used.
        uint32_t e = c.epoch[row] + 1;
        if (e == 0) e = 1;
        int ok = 1;
        if (lane < W) {
            fence_sys();   // this rank's partial (written by earlier kernels) before its number
            st_relaxed_sys(c.flags[lane] + row * kTpMaxWorld + c.rank, e);
            const uint32_t *f = c.flags[c.rank] + row * kTpMaxWorld + lane;
            const uint64_t start = globaltimer();
            // a peer may be one call ahead (its number e + 1)
            while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
                if (globaltimer() - start > kTpWaitBoundNs) {
                    record_timeout(status, 80 + (int)lane);
                    ok = 0;
                    break;
                }
                nano_sleep(20);
            }
        }
        ok = __all_sync(0xffffffffu, ok);
        if (lane == 0) {
            c.epoch[row] = e;
            s_ok = ok;
        }
    }
    __syncthreads();
    if (!s_ok) return;   // reported through the status word; x and y untouched
    fence_sys();
    const size_t off = ((size_t)slot * c.max_rows + row) * hidden;
    float sum = 0.f;
    if constexpr (kReg) {
#pragma unroll
        for (int it = 0; it < kTpRegIters; ++it) {
            const uint32_t i = (threadIdx.x + it * kTpThreads) * 8;
            if (i < hidden) {
                xv[it] = tp_reduce_chunk<W>(c, off, i, xv[it], sum);
                *reinterpret_cast<uint4 *>(xr + i) = xv[it];
            }
        }
    } else {
        for (uint32_t i = threadIdx.x * 8; i < hidden; i += kTpThreads * 8) {
            const uint4 nv = tp_reduce_chunk<W>(c, off, i, *reinterpret_cast<const uint4 *>(xr + i), sum);
            *reinterpret_cast<uint4 *>(xr + i) = nv;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __shared__ float part[kTpThreads / 32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int k = 0; k < kTpThreads / 32; ++k) total += part[k];
    const float mean = __fdiv_rn(total, (float)hidden);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(mean + eps));
    if constexpr (kReg) {
#pragma unroll
        for (int it = 0; it < kTpRegIters; ++it) {
            const uint32_t i = (threadIdx.x + it * kTpThreads) * 8;
            if (i < hidden) *reinterpret_cast<uint4 *>(yr + i) = tp_norm_chunk(xv[it], wt[it], scale);
        }
    } else {
        // reads back only the elements this thread wrote above
        for (uint32_t i = threadIdx.x * 8; i < hidden; i += kTpThreads * 8)
            *reinterpret_cast<uint4 *>(yr + i) = tp_norm_chunk(*reinterpret_cast<const uint4 *>(xr + i),
                                                               *reinterpret_cast<const uint4 *>(w + i), scale);
    }
}

template <int W>
cudaError_t launch_w(const TpCommDev &comm, uint32_t slot, uint16_t *x, const uint16_t *w, uint16_t *y,
                     uint32_t rows, float eps, int *status, cudaStream_t stream) {
    if (comm.hidden <= (uint32_t)kTpThreads * 8 * kTpRegIters)
        return launch_pdl(mslim_tp_allreduce_rmsnorm<W, true>, dim3(rows), dim3(kTpThreads), 0, stream, comm, slot,
                          x, w, y, eps, status);
    return launch_pdl(mslim_tp_allreduce_rmsnorm<W, false>, dim3(rows), dim3(kTpThreads), 0, stream, comm, slot, x,
                      w, y, eps, status);
}

}  // namespace

cudaError_t launch_tp_allreduce_rmsnorm(const TpCommDev &comm, uint32_t slot, uint16_t *x,
                                        const uint16_t *w, uint16_t *y, uint32_t rows, float eps,
                                        int *status, cudaStream_t stream) {
    switch (comm.world) {
    case 1: return launch_w<1>(comm, slot, x, w, y, rows, eps, status, stream);
    case 2: return launch_w<2>(comm, slot, x, w, y, rows, eps, status, stream);
    case 3: return launch_w<3>(comm, slot, x, w, y, rows, eps, status, stream);
    case 4: return launch_w<4>(comm, slot, x, w, y, rows, eps, status, stream);
    case 5: return launch_w<5>(comm, slot, x, w, y, rows, eps, status, stream);
    case 6: return launch_w<6>(comm, slot, x, w, y, rows, eps, status, stream);
    case 7: return launch_w<7>(comm, slot, x, w, y, rows, eps, status, stream);
    case 8: return launch_w<8>(comm, slot, x, w, y, rows, eps, status, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace mslim
