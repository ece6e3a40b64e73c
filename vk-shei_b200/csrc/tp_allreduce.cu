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

template <int W>
__global__ void __launch_bounds__(kTpThreads)
    mslim_tp_allreduce_rmsnorm(const TpCommDev c, uint32_t slot, uint16_t *__restrict__ x,
                               const uint16_t *__restrict__ w, uint16_t *__restrict__ y, float eps,
                               int *status) {
    const uint32_t row = blockIdx.x;
    const uint32_t hidden = c.hidden;
    __shared__ int s_ok;
    // warp 0: lane r (< W) publishes this rank's call number into rank r's
    // flags, then waits for rank r's number in this rank's flags; the lanes
    // work in parallel, each behind its own system-scope fence
    if (threadIdx.x < 32) {
        const uint32_t lane = threadIdx.x;
        const uint32_t e = c.epoch[row] + 1;
        int ok = 1;
        if (lane < W) {
            fence_sys();   // this rank's partial (written by earlier kernels) before its number
            st_relaxed_sys(c.flags[lane] + row * kTpMaxWorld + c.rank, e);
            const uint32_t *f = c.flags[c.rank] + row * kTpMaxWorld + lane;
            const uint64_t start = globaltimer();
            while (ld_acquire_sys(f) < e) {   // counters only grow; a peer may be one call ahead
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
    uint16_t *xr = x + (size_t)row * hidden;
    uint16_t *yr = y + (size_t)row * hidden;
    float sum = 0.f;
    for (uint32_t i = threadIdx.x * 8; i < hidden; i += kTpThreads * 8) {
        // every rank's chunk in flight at once, summed in rank order
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
        const uint4 xv = *reinterpret_cast<const uint4 *>(xr + i);
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
        *reinterpret_cast<uint4 *>(xr + i) = make_uint4(nw[0], nw[1], nw[2], nw[3]);
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
    // reads back only the elements this thread wrote above
    for (uint32_t i = threadIdx.x * 8; i < hidden; i += kTpThreads * 8) {
        const uint4 v = *reinterpret_cast<const uint4 *>(xr + i);
        const uint4 wt = *reinterpret_cast<const uint4 *>(w + i);
        const uint32_t xv[4] = {v.x, v.y, v.z, v.w};
        const uint32_t wv[4] = {wt.x, wt.y, wt.z, wt.w};
        uint32_t ov[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            ov[k] = pack_bf16x2(bf16_round(bf16lo_f32(xv[k]) * scale) * bf16lo_f32(wv[k]),
                                bf16_round(bf16hi_f32(xv[k]) * scale) * bf16hi_f32(wv[k]));
        *reinterpret_cast<uint4 *>(yr + i) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
    }
}

}  // namespace

cudaError_t launch_tp_allreduce_rmsnorm(const TpCommDev &comm, uint32_t slot, uint16_t *x,
                                        const uint16_t *w, uint16_t *y, uint32_t rows, float eps,
                                        int *status, cudaStream_t stream) {
    switch (comm.world) {
    case 1: mslim_tp_allreduce_rmsnorm<1><<<rows, kTpThreads, 0, stream>>>(comm, slot, x, w, y, eps, status); break;
    case 2: mslim_tp_allreduce_rmsnorm<2><<<rows, kTpThreads, 0, stream>>>(comm, slot, x, w, y, eps, status); break;
    case 3: mslim_tp_allreduce_rmsnorm<3><<<rows, kTpThreads, 0, stream>>>(comm, slot, x, w, y, eps, status); break;
    case 4: mslim_tp_allreduce_rmsnorm<4><<<rows, kTpThreads, 0, stream>>>(comm, slot, x, w, y, eps, status); break;
    case 5: mslim_tp_allreduce_rmsnorm<5><<<rows, kTpThreads, 0, stream>>>(comm, slot, x, w, y, eps, status); break;
    case 6: mslim_tp_allreduce_rmsnorm<6><<<rows, kTpThreads, 0, stream>>>(comm, slot, x, w, y, eps, status); break;
    case 7: mslim_tp_allreduce_rmsnorm<7><<<rows, kTpThreads, 0, stream>>>(comm, slot, x, w, y, eps, status); break;
    case 8: mslim_tp_allreduce_rmsnorm<8><<<rows, kTpThreads, 0, stream>>>(comm, slot, x, w, y, eps, status); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace mslim
