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

// The angle depends on (position, i) only, so a CTA that rotates every head
// of one token evaluates its D/2 (cos, sin) pairs once, into shared memory.
constexpr int kRopeMaxHalf = 128;
__device__ __forceinline__ void rope_fill(const RopeTable &t, uint32_t position, uint32_t half,
                                          float2 *cs) {
    for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) cs[i] = rope_cs(rope_angle(t, (int)i, position));
    __syncthreads();
}

// One 128-thread CTA per token row; 16-byte vector loads.  With kResidual the
// row is first updated in place, x = bf16(x + delta) (the residual add of the
// layer, native_cpu_adapter.rs:186-191), and normalised from the updated
// values with the same reduction order, so the fused form returns the same
// bits as a residual add followed by RMSNorm.
// 1 / sqrt(mean(x^2) + eps) from each thread's partial sum of squares: warp
// xor-tree, then the four warps' sums in a fixed order.
__device__ __forceinline__ float rms_scale(float sum, uint32_t hidden, float eps) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __shared__ float part[4];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
    __syncthreads();
    const float total = (part[0] + part[1]) + (part[2] + part[3]);
    const float mean = __fdiv_rn(total, (float)hidden);
    return __fdiv_rn(1.0f, __fsqrt_rn(mean + eps));
}

// Rows up to 128 * 8 * kNormRegIters elements stay in registers.
constexpr int kNormRegIters = 8;

template <bool kResidual>
__global__ void __launch_bounds__(128)
    mslim_rmsnorm(uint16_t *__restrict__ x, const uint16_t *__restrict__ delta,
                  const uint16_t *__restrict__ w, uint16_t *__restrict__ y, uint32_t hidden, float eps) {
    griddep_launch_dependents();
    griddep_wait();  // programmatic dependent launch: inputs after the predecessor
    const size_t row = blockIdx.x;
    uint16_t *xr = x + row * hidden;
    const uint16_t *dr = kResidual ? delta + row * hidden : nullptr;
    uint16_t *yr = y + row * hidden;
    const bool vec = (hidden % 8 == 0);
    float sum = 0.f;
    if (vec && hidden <= 128 * 8 * kNormRegIters) {
        // The whole row in registers: every load (x, delta, w) is issued before
        // the first use, and the second pass does not read x back.  Same
        // element order and sums as the loops below, so the same bits.
        uint4 xv[kNormRegIters], wt[kNormRegIters];
#pragma unroll
        for (int it = 0; it < kNormRegIters; ++it) {
            const uint32_t i = (threadIdx.x + it * 128) * 8;
            if (i < hidden) {
                xv[it] = *reinterpret_cast<const uint4 *>(xr + i);
                wt[it] = *reinterpret_cast<const uint4 *>(w + i);
                if (kResidual) {
                    const uint4 v = xv[it];
                    const uint4 d = *reinterpret_cast<const uint4 *>(dr + i);
                    xv[it] = make_uint4(
                        pack_bf16x2(bf16lo_f32(v.x) + bf16lo_f32(d.x), bf16hi_f32(v.x) + bf16hi_f32(d.x)),
                        pack_bf16x2(bf16lo_f32(v.y) + bf16lo_f32(d.y), bf16hi_f32(v.y) + bf16hi_f32(d.y)),
                        pack_bf16x2(bf16lo_f32(v.z) + bf16lo_f32(d.z), bf16hi_f32(v.z) + bf16hi_f32(d.z)),
                        pack_bf16x2(bf16lo_f32(v.w) + bf16lo_f32(d.w), bf16hi_f32(v.w) + bf16hi_f32(d.w)));
                }
            }
        }
#pragma unroll
        for (int it = 0; it < kNormRegIters; ++it) {
            const uint32_t i = (threadIdx.x + it * 128) * 8;
            if (i < hidden) {
                if (kResidual) *reinterpret_cast<uint4 *>(xr + i) = xv[it];
                const uint32_t v4[4] = {xv[it].x, xv[it].y, xv[it].z, xv[it].w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float a = bf16lo_f32(v4[k]), b = bf16hi_f32(v4[k]);
                    sum += a * a;
                    sum += b * b;
                }
            }
        }
        const float scale = rms_scale(sum, hidden, eps);
#pragma unroll
        for (int it = 0; it < kNormRegIters; ++it) {
            const uint32_t i = (threadIdx.x + it * 128) * 8;
            if (i < hidden) {
                const uint32_t v4[4] = {xv[it].x, xv[it].y, xv[it].z, xv[it].w};
                const uint32_t w4[4] = {wt[it].x, wt[it].y, wt[it].z, wt[it].w};
                uint32_t ov[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float a = bf16_round(bf16lo_f32(v4[k]) * scale) * bf16lo_f32(w4[k]);
                    const float b = bf16_round(bf16hi_f32(v4[k]) * scale) * bf16hi_f32(w4[k]);
                    ov[k] = pack_bf16x2(a, b);
                }
                *reinterpret_cast<uint4 *>(yr + i) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
            }
        }
        return;
    }
    if (vec) {
        for (uint32_t i = threadIdx.x * 8; i < hidden; i += 128 * 8) {
            uint4 v = *reinterpret_cast<const uint4 *>(xr + i);
            if (kResidual) {
                const uint4 d = *reinterpret_cast<const uint4 *>(dr + i);
                v = make_uint4(pack_bf16x2(bf16lo_f32(v.x) + bf16lo_f32(d.x), bf16hi_f32(v.x) + bf16hi_f32(d.x)),
                               pack_bf16x2(bf16lo_f32(v.y) + bf16lo_f32(d.y), bf16hi_f32(v.y) + bf16hi_f32(d.y)),
                               pack_bf16x2(bf16lo_f32(v.z) + bf16lo_f32(d.z), bf16hi_f32(v.z) + bf16hi_f32(d.z)),
                               pack_bf16x2(bf16lo_f32(v.w) + bf16lo_f32(d.w), bf16hi_f32(v.w) + bf16hi_f32(d.w)));
                *reinterpret_cast<uint4 *>(xr + i) = v;
            }
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
            float a = bf16_bits_to_f32(xr[i]);
            if (kResidual) {
                const uint16_t nb = bf16_bits_rn(a + bf16_bits_to_f32(dr[i]));
                xr[i] = nb;
                a = bf16_bits_to_f32(nb);
            }
            sum += a * a;
        }
    }
    const float scale = rms_scale(sum, hidden, eps);
    // the second pass reads back only elements this thread itself wrote above
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

// One CTA per token: the token's (cos, sin) table, then every (head, i) pair.
__global__ void __launch_bounds__(128)
    mslim_rope(const uint16_t *__restrict__ in, uint16_t *__restrict__ out, uint32_t heads,
               uint32_t dim, uint32_t start_position, const RopeTable table) {
    __shared__ float2 cs[kRopeMaxHalf];
    const uint32_t token = blockIdx.x;
    const uint32_t half = dim / 2;
    rope_fill(table, start_position + token, half, cs);
    const size_t base = (size_t)token * heads * dim;
    for (uint32_t x = threadIdx.x; x < heads * half; x += blockDim.x) {
        const uint32_t head = x / half, i = x % half;
        const size_t o = base + (size_t)head * dim;
        float oa, ob;
        rope_rotate(bf16_bits_to_f32(in[o + i]), bf16_bits_to_f32(in[o + i + half]), cs[i], oa, ob);
        out[o + i] = bf16_bits_rn(oa);
        out[o + i + half] = bf16_bits_rn(ob);
    }
}

// Input rows of the fused appends: q of token t at q_in + t * q_stride, its k
// and v at k_in / v_in + t * kv_stride (q_stride = QH*D, kv_stride = KVH*D for
// separate buffers; both (QH+2KVH)*D for one fused q|k|v projection output).
struct QkvRows {
    const uint16_t *q, *k, *v;
    uint32_t q_stride, kv_stride;
};

// RoPE of one token's q heads into q_out ([token][QH][D]) and of its k heads
// into k_dst(head) rows, v copied into v_dst(head) rows; (cos, sin) in cs.
template <typename KDst, typename VDst>
__device__ __forceinline__ void rope_append_token(const QkvRows &in, uint16_t *q_out, uint32_t token,
                                                  uint32_t qheads, uint32_t kvheads, uint32_t dim,
                                                  const float2 *cs, KDst k_dst, VDst v_dst) {
    const uint32_t half = dim / 2;
    const uint32_t q_pairs = qheads * half, k_pairs = kvheads * half;
    const uint16_t *qr = in.q + (size_t)token * in.q_stride;
    const uint16_t *kr = in.k + (size_t)token * in.kv_stride;
    const uint16_t *vr = in.v + (size_t)token * in.kv_stride;
    for (uint32_t x = threadIdx.x; x < q_pairs + k_pairs; x += blockDim.x) {
        const bool is_q = x < q_pairs;
        const uint32_t y = is_q ? x : x - q_pairs;
        const uint32_t head = y / half, i = y % half;
        const uint16_t *src = (is_q ? qr : kr) + (size_t)head * dim;
        float oa, ob;
        rope_rotate(bf16_bits_to_f32(src[i]), bf16_bits_to_f32(src[i + half]), cs[i], oa, ob);
        uint16_t *dst = is_q ? q_out + ((size_t)token * qheads + head) * dim : k_dst(head);
        dst[i] = bf16_bits_rn(oa);
        dst[i + half] = bf16_bits_rn(ob);
    }
    for (uint32_t x = threadIdx.x; x < kvheads * dim; x += blockDim.x) {
        const uint32_t head = x / dim, d = x % dim;
        v_dst(head)[d] = vr[(size_t)head * dim + d];
    }
}

// The same work in 16-byte groups, spread over gridDim.y CTAs per token: item
// x < (QH + KVH) * D/16 rotates eight consecutive pairs (i0..i0+7 with
// i0+D/2..i0+D/2+7) of one q or k head; the remaining items copy one 16-byte
// chunk of a v head.  Every load of a thread is independent of its stores, so
// the loads of all items are in flight together.  Needs D % 16 == 0 and 16-byte
// aligned rows (checked by the launcher); same arithmetic, same bits.
template <typename KDst, typename VDst>
__device__ __forceinline__ void rope_append_token_vec(const QkvRows &in, uint16_t *q_out, uint32_t token,
                                                      uint32_t qheads, uint32_t kvheads, uint32_t dim,
                                                      const float2 *cs, KDst k_dst, VDst v_dst) {
    const uint32_t half = dim / 2, groups = half / 8;
    const uint32_t rot = (qheads + kvheads) * groups, total = rot + kvheads * (dim / 8);
    const uint16_t *qr = in.q + (size_t)token * in.q_stride;
    const uint16_t *kr = in.k + (size_t)token * in.kv_stride;
    const uint16_t *vr = in.v + (size_t)token * in.kv_stride;
    for (uint32_t x = blockIdx.y * blockDim.x + threadIdx.x; x < total; x += gridDim.y * blockDim.x) {
        if (x < rot) {
            const bool is_q = x < qheads * groups;
            const uint32_t y = is_q ? x : x - qheads * groups;
            const uint32_t head = y / groups, i0 = (y % groups) * 8;
            const uint16_t *src = (is_q ? qr : kr) + (size_t)head * dim;
            const uint4 a4 = *reinterpret_cast<const uint4 *>(src + i0);
            const uint4 b4 = *reinterpret_cast<const uint4 *>(src + i0 + half);
            const uint32_t a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
            uint32_t oa[4], ob[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                float r0, r1, s0, s1;
                rope_rotate(bf16_bits_to_f32((uint16_t)(a[w] & 0xffffu)), bf16_bits_to_f32((uint16_t)(b[w] & 0xffffu)),
                            cs[i0 + 2 * w], r0, s0);
                rope_rotate(bf16_bits_to_f32((uint16_t)(a[w] >> 16)), bf16_bits_to_f32((uint16_t)(b[w] >> 16)),
                            cs[i0 + 2 * w + 1], r1, s1);
                oa[w] = (uint32_t)bf16_bits_rn(r0) | ((uint32_t)bf16_bits_rn(r1) << 16);
                ob[w] = (uint32_t)bf16_bits_rn(s0) | ((uint32_t)bf16_bits_rn(s1) << 16);
            }
            uint16_t *dst = is_q ? q_out + ((size_t)token * qheads + head) * dim : k_dst(head);
            *reinterpret_cast<uint4 *>(dst + i0) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
            *reinterpret_cast<uint4 *>(dst + i0 + half) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
        } else {
            const uint32_t c = x - rot, head = c / (dim / 8), d0 = (c % (dim / 8)) * 8;
            *reinterpret_cast<uint4 *>(v_dst(head) + d0) =
                *reinterpret_cast<const uint4 *>(vr + (size_t)head * dim + d0);
        }
    }
}

// Per new token (blockIdx.x; with kVec its work spread over gridDim.y CTAs):
// RoPE of its q heads into q_out, RoPE of its k heads and a copy of its v
// heads into the ColdStore-exact page that holds the token (head-major
// [KVH][page_tokens][D] inside the page).
//   prefill form (positions == null): token t of one sequence at position
//     start_position + t, pages page_table[0..max_pages);
//   decode form (positions != null): the new token of session s at position
//     positions[s], pages page_table[s * max_pages ..].
template <bool kVec>
__global__ void __launch_bounds__(256)
    mslim_rope_append_paged(const QkvRows in, uint16_t *__restrict__ q_out, uint32_t qheads,
                            uint32_t kvheads, uint32_t dim, uint32_t start_position,
                            const int32_t *__restrict__ positions, uint16_t *__restrict__ k_pool,
                            uint16_t *__restrict__ v_pool, uint32_t n_pages, uint32_t page_tokens,
                            const int32_t *__restrict__ page_table, uint32_t max_pages,
                            const RopeTable table, int *status) {
    griddep_launch_dependents();
    griddep_wait();  // programmatic dependent launch: the predecessor's writes are visible
    __shared__ float2 cs[kRopeMaxHalf];
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
    const int32_t phys = row[pos / page_tokens];
    if (phys < 0 || (uint32_t)phys >= n_pages) {
        // A page id outside the pool: write nothing, record it for the host.
        if (threadIdx.x == 0 && status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
        return;
    }
    rope_fill(table, pos, dim / 2, cs);
    const uint32_t slot = pos % page_tokens;
    auto k_dst = [&](uint32_t head) {
        return k_pool + (((size_t)phys * kvheads + head) * page_tokens + slot) * dim;
    };
    auto v_dst = [&](uint32_t head) {
        return v_pool + (((size_t)phys * kvheads + head) * page_tokens + slot) * dim;
    };
    if constexpr (kVec) rope_append_token_vec(in, q_out, token, qheads, kvheads, dim, cs, k_dst, v_dst);
    else rope_append_token(in, q_out, token, qheads, kvheads, dim, cs, k_dst, v_dst);
}

// Dense-cache twin of the decode form above: blockIdx.x = s is the new token
// of session s at position positions[s]; q -> RoPE -> q_out, k -> RoPE and
// v -> copy into the token-major caches [n_seq][max_tokens][KVH][D] at row
// positions[s].
template <bool kVec>
__global__ void __launch_bounds__(256)
    mslim_rope_append_dense(const QkvRows in, uint16_t *__restrict__ q_out, uint32_t qheads,
                            uint32_t kvheads, uint32_t dim, const int32_t *__restrict__ positions,
                            uint16_t *__restrict__ k_cache, uint16_t *__restrict__ v_cache,
                            uint32_t max_tokens, const RopeTable table, int *status) {
    griddep_launch_dependents();
    griddep_wait();  // programmatic dependent launch: the predecessor's writes are visible
    __shared__ float2 cs[kRopeMaxHalf];
    const uint32_t token = blockIdx.x;
    const int32_t p = positions[token];
    if (p < 0 || (uint32_t)p >= max_tokens) {
        if (threadIdx.x == 0 && status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
        return;
    }
    const uint32_t pos = (uint32_t)p;
    rope_fill(table, pos, dim / 2, cs);
    const size_t row = ((size_t)token * max_tokens + pos) * kvheads;  // cache row of this token
    auto k_dst = [&](uint32_t head) { return k_cache + (row + head) * dim; };
    auto v_dst = [&](uint32_t head) { return v_cache + (row + head) * dim; };
    if constexpr (kVec) rope_append_token_vec(in, q_out, token, qheads, kvheads, dim, cs, k_dst, v_dst);
    else rope_append_token(in, q_out, token, qheads, kvheads, dim, cs, k_dst, v_dst);
}

// The 16-byte form: head_dim a multiple of 16 and every row start 16-byte
// aligned (bases, and the q / kv row strides in elements a multiple of 8).
bool rope_vec_ok(const QkvRows &in, const void *q_out, const void *k_dst, const void *v_dst, uint32_t dim) {
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return dim % 16 == 0 && al(in.q) && al(in.k) && al(in.v) && al(q_out) && al(k_dst) && al(v_dst) &&
           in.q_stride % 8 == 0 && in.kv_stride % 8 == 0;
}

// CTAs per token for the 16-byte form: about one 16-byte item per thread of a
// 128-thread CTA, at most eight CTAs.
unsigned rope_vec_ctas(uint32_t qheads, uint32_t kvheads, uint32_t dim) {
    const uint64_t items = (uint64_t)(qheads + kvheads) * (dim / 16) + (uint64_t)kvheads * (dim / 8);
    return (unsigned)std::min<uint64_t>(8, std::max<uint64_t>(1, (items + 127) / 128));
}

}  // namespace

cudaError_t launch_rmsnorm(const uint16_t *x, const uint16_t *w, uint16_t *y, uint32_t tokens,
                           uint32_t hidden, float eps, cudaStream_t stream) {
    return launch_pdl(mslim_rmsnorm<false>, dim3(tokens), dim3(128), 0, stream, const_cast<uint16_t *>(x),
                      static_cast<const uint16_t *>(nullptr), w, y, hidden, eps);
}

cudaError_t launch_residual_rmsnorm(uint16_t *x, const uint16_t *delta, const uint16_t *w, uint16_t *y,
                                    uint32_t tokens, uint32_t hidden, float eps, cudaStream_t stream) {
    return launch_pdl(mslim_rmsnorm<true>, dim3(tokens), dim3(128), 0, stream, x, delta, w, y, hidden, eps);
}

cudaError_t launch_rope(const uint16_t *in, uint16_t *out, uint32_t tokens, uint32_t heads,
                        uint32_t dim, uint32_t start_position, const RopeTable &table,
                        cudaStream_t stream) {
    mslim_rope<<<tokens, 128, 0, stream>>>(in, out, heads, dim, start_position, table);
    return counted(cudaGetLastError());
}

cudaError_t launch_rope_append_paged(const uint16_t *q_in, uint16_t *q_out, const uint16_t *k_in,
                                     const uint16_t *v_in, uint32_t tokens, uint32_t qheads,
                                     uint32_t kvheads, uint32_t dim, uint32_t start_position,
                                     const int32_t *positions, uint16_t *k_pool,
                                     uint16_t *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                     const int32_t *page_table, uint32_t max_pages,
                                     const RopeTable &table, int *status, cudaStream_t stream,
                                     uint32_t q_stride, uint32_t kv_stride) {
    const QkvRows in{q_in, k_in, v_in, q_stride ? q_stride : qheads * dim,
                     kv_stride ? kv_stride : kvheads * dim};
    if (rope_vec_ok(in, q_out, k_pool, v_pool, dim)) {
        return launch_pdl(mslim_rope_append_paged<true>, dim3(tokens, rope_vec_ctas(qheads, kvheads, dim)),
                          dim3(128), 0, stream, in, q_out, qheads, kvheads, dim, start_position, positions, k_pool,
                          v_pool, n_pages, page_tokens, page_table, max_pages, table, status);
    }
    return launch_pdl(mslim_rope_append_paged<false>, dim3(tokens), dim3(256), 0, stream, in, q_out, qheads,
                      kvheads, dim, start_position, positions, k_pool, v_pool, n_pages, page_tokens, page_table,
                      max_pages, table, status);
}

cudaError_t launch_rope_append_dense(const uint16_t *q_in, uint16_t *q_out, const uint16_t *k_in,
                                     const uint16_t *v_in, uint32_t n_seq, uint32_t qheads,
                                     uint32_t kvheads, uint32_t dim, const int32_t *positions,
                                     uint16_t *k_cache, uint16_t *v_cache, uint32_t max_tokens,
                                     const RopeTable &table, int *status, cudaStream_t stream,
                                     uint32_t q_stride, uint32_t kv_stride) {
    const QkvRows in{q_in, k_in, v_in, q_stride ? q_stride : qheads * dim,
                     kv_stride ? kv_stride : kvheads * dim};
    if (rope_vec_ok(in, q_out, k_cache, v_cache, dim)) {
        return launch_pdl(mslim_rope_append_dense<true>, dim3(n_seq, rope_vec_ctas(qheads, kvheads, dim)),
                          dim3(128), 0, stream, in, q_out, qheads, kvheads, dim, positions, k_cache, v_cache,
                          max_tokens, table, status);
    }
    return launch_pdl(mslim_rope_append_dense<false>, dim3(n_seq), dim3(256), 0, stream, in, q_out, qheads,
                      kvheads, dim, positions, k_cache, v_cache, max_tokens, table, status);
}

}  // namespace mslim
