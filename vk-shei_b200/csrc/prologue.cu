// prologue.cu -- RMSNorm, RoPE and RoPE fused with the K/V page append.
//
// Numerics follow the reference CPU decoder (native_cpu_adapter.rs:194-221):
//   RMSNorm: s = 1 / sqrt(sum(x^2) / n + eps); y = bf16(bf16(x * s) * w)
//            (the sum is a tree here; the CPU sums sequentially, the OpenCL
//            kernel with a 128-lane tree, assets/gpu_llm.cl:72-98);
//   RoPE:    x' = bf16(bf16(x_i c) - bf16(x_{i+h} s)),
//            x'_{i+h} = bf16(bf16(x_{i+h} c) + bf16(x_i s)),
//            c, s = bf16(cos(angle)), bf16(sin(angle)), with the angle built
//            from a per-dimension frequency table computed on the host
//            (CPU formula position / theta^(2i/D), or the Llama-3 scaled
//            inverse frequency of src/gpu_llm/kernels.rs:50-67 times the
//            position, as assets/gpu_llm.cl:102-146 does).  cos/sin are
//            evaluated in double and rounded once, so they are the correctly
//            rounded f32 values.
#include "prologue.cuh"

namespace mslim {

namespace {

__device__ __forceinline__ float rope_angle(const RopeTable &t, int i, uint32_t position) {
    const float pos = (float)position;
    return t.multiply ? pos * t.freq[i] : __fdiv_rn(pos, t.freq[i]);
}

__device__ __forceinline__ void rope_pair(float a, float b, float angle, float &out_a,
                                          float &out_b) {
    double sd, cd;
    sincos((double)angle, &sd, &cd);
    const float s = bf16_round((float)sd);
    const float c = bf16_round((float)cd);
    out_a = bf16_round(bf16_round(a * c) - bf16_round(b * s));
    out_b = bf16_round(bf16_round(b * c) + bf16_round(a * s));
}

// One 128-thread CTA per token row; 16-byte vector loads.
__global__ void __launch_bounds__(128)
    mslim_rmsnorm(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                  uint16_t *__restrict__ y, uint32_t hidden, float eps) {
    const size_t row = blockIdx.x;
    const uint16_t *xr = x + row * hidden;
    uint16_t *yr = y + row * hidden;
    const bool vec = (hidden % 8 == 0);
    float sum = 0.f;
    if (vec) {
        for (uint32_t i = threadIdx.x * 8; i < hidden; i += 128 * 8) {
            const uint4 v = *reinterpret_cast<const uint4 *>(xr + i);
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float a = bf16lo_f32(wv[k]), b = bf16hi_f32(wv[k]);
                sum += a * a;
                sum += b * b;
            }
        }
    } else {
        for (uint32_t i = threadIdx.x; i < hidden; i += 128) {
            const float a = bf16_bits_to_f32(xr[i]);
            sum += a * a;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __shared__ float part[4];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
    __syncthreads();
    const float total = (part[0] + part[1]) + (part[2] + part[3]);
    const float mean = __fdiv_rn(total, (float)hidden);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(mean + eps));
    if (vec) {
        for (uint32_t i = threadIdx.x * 8; i < hidden; i += 128 * 8) {
            const uint4 v = *reinterpret_cast<const uint4 *>(xr + i);
            const uint4 wt = *reinterpret_cast<const uint4 *>(w + i);
            const uint32_t xv[4] = {v.x, v.y, v.z, v.w};
            const uint32_t wv[4] = {wt.x, wt.y, wt.z, wt.w};
            uint32_t ov[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float a = bf16_round(bf16lo_f32(xv[k]) * scale) * bf16lo_f32(wv[k]);
                const float b = bf16_round(bf16hi_f32(xv[k]) * scale) * bf16hi_f32(wv[k]);
                ov[k] = pack_bf16x2(a, b);
            }
            *reinterpret_cast<uint4 *>(yr + i) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
        }
    } else {
        for (uint32_t i = threadIdx.x; i < hidden; i += 128) {
            const float a = bf16_round(bf16_bits_to_f32(xr[i]) * scale) * bf16_bits_to_f32(w[i]);
            yr[i] = bf16_bits_rn(a);
        }
    }
}

// One thread per rotated pair (token, head, i < D/2).
__global__ void mslim_rope(const uint16_t *__restrict__ in, uint16_t *__restrict__ out,
                           uint32_t tokens, uint32_t heads, uint32_t dim, uint32_t start_position,
                           const RopeTable table) {
    const uint32_t half = dim / 2;
    const size_t pairs = (size_t)tokens * heads * half;
    for (size_t x = (size_t)blockIdx.x * blockDim.x + threadIdx.x; x < pairs;
         x += (size_t)gridDim.x * blockDim.x) {
        const uint32_t i = (uint32_t)(x % half);
        const size_t rowi = x / half;  // token * heads + head
        const uint32_t token = (uint32_t)(rowi / heads);
        const size_t base = rowi * dim;
        float oa, ob;
        rope_pair(bf16_bits_to_f32(in[base + i]), bf16_bits_to_f32(in[base + i + half]),
                  rope_angle(table, (int)i, start_position + token), oa, ob);
        out[base + i] = bf16_bits_rn(oa);
        out[base + i + half] = bf16_bits_rn(ob);
    }
}

// One CTA per new token: RoPE of its q heads into q_out, RoPE of its k heads
// and a copy of its v heads into the ColdStore-exact page that holds the
// token (head-major [KVH][page_tokens][D] inside the page).
//   prefill form (positions == null): CTA t is token t of one sequence at
//     position start_position + t, pages page_table[0..max_pages);
//   decode form (positions != null): CTA s is the new token of session s at
//     position positions[s], pages page_table[s * max_pages ..].
__global__ void __launch_bounds__(256)
    mslim_rope_append_paged(const uint16_t *__restrict__ q_in, uint16_t *__restrict__ q_out,
                            const uint16_t *__restrict__ k_in, const uint16_t *__restrict__ v_in,
                            uint32_t qheads, uint32_t kvheads, uint32_t dim,
                            uint32_t start_position, const int32_t *__restrict__ positions,
                            uint16_t *__restrict__ k_pool, uint16_t *__restrict__ v_pool,
                            uint32_t n_pages, uint32_t page_tokens,
                            const int32_t *__restrict__ page_table, uint32_t max_pages,
                            const RopeTable table, int *status) {
    const uint32_t token = blockIdx.x;
    uint32_t pos;
    const int32_t *row = page_table;
    if (positions) {
        const int32_t p = positions[token];
        if (p < 0 || (uint64_t)p >= (uint64_t)max_pages * page_tokens) {
            if (threadIdx.x == 0 && status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
            return;
        }
        pos = (uint32_t)p;
        row = page_table + (size_t)token * max_pages;
    } else {
        pos = start_position + token;
    }
    const uint32_t half = dim / 2;
    const int32_t phys = row[pos / page_tokens];
    if (phys < 0 || (uint32_t)phys >= n_pages) {
        // A page id outside the pool: write nothing, record it for the host.
        if (threadIdx.x == 0 && status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
        return;
    }
    const uint32_t slot = pos % page_tokens;
    const uint32_t q_pairs = qheads * half, k_pairs = kvheads * half;
    for (uint32_t x = threadIdx.x; x < q_pairs + k_pairs; x += blockDim.x) {
        const bool is_q = x < q_pairs;
        const uint32_t y = is_q ? x : x - q_pairs;
        const uint32_t head = y / half, i = y % half;
        const uint16_t *src = is_q ? q_in + ((size_t)token * qheads + head) * dim
                                   : k_in + ((size_t)token * kvheads + head) * dim;
        float oa, ob;
        rope_pair(bf16_bits_to_f32(src[i]), bf16_bits_to_f32(src[i + half]),
                  rope_angle(table, (int)i, pos), oa, ob);
        uint16_t *dst = is_q ? q_out + ((size_t)token * qheads + head) * dim
                             : k_pool + (((size_t)phys * kvheads + head) * page_tokens + slot) * dim;
        dst[i] = bf16_bits_rn(oa);
        dst[i + half] = bf16_bits_rn(ob);
    }
    for (uint32_t x = threadIdx.x; x < kvheads * dim; x += blockDim.x) {
        const uint32_t head = x / dim, d = x % dim;
        v_pool[(((size_t)phys * kvheads + head) * page_tokens + slot) * dim + d] =
            v_in[((size_t)token * kvheads + head) * dim + d];
    }
}

}  // namespace

cudaError_t launch_rmsnorm(const uint16_t *x, const uint16_t *w, uint16_t *y, uint32_t tokens,
                           uint32_t hidden, float eps, cudaStream_t stream) {
    mslim_rmsnorm<<<tokens, 128, 0, stream>>>(x, w, y, hidden, eps);
    return cudaGetLastError();
}

cudaError_t launch_rope(const uint16_t *in, uint16_t *out, uint32_t tokens, uint32_t heads,
                        uint32_t dim, uint32_t start_position, const RopeTable &table,
                        cudaStream_t stream) {
    const size_t pairs = (size_t)tokens * heads * (dim / 2);
    const unsigned blocks = (unsigned)std::min<size_t>((pairs + 255) / 256, 148 * 16);
    mslim_rope<<<blocks, 256, 0, stream>>>(in, out, tokens, heads, dim, start_position, table);
    return cudaGetLastError();
}

cudaError_t launch_rope_append_paged(const uint16_t *q_in, uint16_t *q_out, const uint16_t *k_in,
                                     const uint16_t *v_in, uint32_t tokens, uint32_t qheads,
                                     uint32_t kvheads, uint32_t dim, uint32_t start_position,
                                     const int32_t *positions, uint16_t *k_pool,
                                     uint16_t *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                     const int32_t *page_table, uint32_t max_pages,
                                     const RopeTable &table, int *status, cudaStream_t stream) {
    mslim_rope_append_paged<<<tokens, 256, 0, stream>>>(
        q_in, q_out, k_in, v_in, qheads, kvheads, dim, start_position, positions, k_pool, v_pool,
        n_pages, page_tokens, page_table, max_pages, table, status);
    return cudaGetLastError();
}

}  // namespace mslim
