// layer_ops.cu -- elementwise decoder-layer kernels around attention.
//
//   mslim_residual_add   out = bf16(a + b)                 native_cpu_adapter.rs:186-191,
//                                                          gpu_llm.cl llm_add
//   mslim_swiglu         out = bf16(bf16(g / (1 + exp(-g))) * u)
//                                                          native_cpu_adapter.rs:553-560,
//                                                          gpu_llm.cl llm_swiglu
//   mslim_argmax         greedy token per row of logits    native_cpu_adapter.rs:582-587,
//                                                          gpu_llm.cl llm_argmax
//
// All three are HBM-bound streams: 16-byte vector loads, grids of a few waves
// of 148 SMs, grid-stride loops.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdint>

#include "layer_ops.cuh"

namespace mslim {

namespace {

constexpr int kEltThreads = 256;

__device__ __forceinline__ uint32_t add_pair(uint32_t a, uint32_t b) {
    return pack_bf16x2(bf16lo_f32(a) + bf16lo_f32(b), bf16hi_f32(a) + bf16hi_f32(b));
}

__device__ __forceinline__ uint32_t swiglu_pair(uint32_t g, uint32_t u) {
    return pack_bf16x2(silu_mul(bf16lo_f32(g), bf16lo_f32(u)), silu_mul(bf16hi_f32(g), bf16hi_f32(u)));
}

// n8 = number of whole 8-element vectors; the tail (< 8) is done by thread 0.
__global__ void __launch_bounds__(kEltThreads)
    mslim_residual_add(const uint16_t *__restrict__ a, const uint16_t *__restrict__ b,
                       uint16_t *__restrict__ out, uint64_t n) {
    griddep_launch_dependents();
    griddep_wait();  // programmatic dependent launch: inputs after the predecessor
    const uint64_t n8 = n / 8;
    const uint4 *a4 = reinterpret_cast<const uint4 *>(a);
    const uint4 *b4 = reinterpret_cast<const uint4 *>(b);
    uint4 *o4 = reinterpret_cast<uint4 *>(out);
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n8;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint4 x = a4[i], y = b4[i];
        o4[i] = make_uint4(add_pair(x.x, y.x), add_pair(x.y, y.y), add_pair(x.z, y.z), add_pair(x.w, y.w));
    }
    if (blockIdx.x == 0 && threadIdx.x == 0)
        for (uint64_t i = n8 * 8; i < n; ++i)
            out[i] = bf16_bits_rn(bf16_bits_to_f32(a[i]) + bf16_bits_to_f32(b[i]));
}

__global__ void __launch_bounds__(kEltThreads)
    mslim_swiglu(const uint16_t *__restrict__ gate, const uint16_t *__restrict__ up,
                 uint16_t *__restrict__ out, uint64_t n) {
    griddep_launch_dependents();
    griddep_wait();
    const uint64_t n8 = n / 8;
    const uint4 *g4 = reinterpret_cast<const uint4 *>(gate);
    const uint4 *u4 = reinterpret_cast<const uint4 *>(up);
    uint4 *o4 = reinterpret_cast<uint4 *>(out);
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n8;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint4 g = g4[i], u = u4[i];
        o4[i] = make_uint4(swiglu_pair(g.x, u.x), swiglu_pair(g.y, u.y), swiglu_pair(g.z, u.z),
                           swiglu_pair(g.w, u.w));
    }
    if (blockIdx.x == 0 && threadIdx.x == 0)
        for (uint64_t i = n8 * 8; i < n; ++i)
            out[i] = bf16_bits_rn(silu_mul(bf16_bits_to_f32(gate[i]), bf16_bits_to_f32(up[i])));
}

// SwiGLU over rows of a fused gate|up projection: row r of gate_up holds
// [gate (width) | up (width)]; out is [rows][width].  width % 8 == 0.
__global__ void __launch_bounds__(kEltThreads)
    mslim_swiglu_rows(const uint16_t *__restrict__ gate_up, uint16_t *__restrict__ out, uint32_t rows,
                      uint32_t width) {
    griddep_launch_dependents();
    griddep_wait();
    const uint32_t w8 = width / 8;
    const uint64_t n8 = (uint64_t)rows * w8;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n8;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / w8, c = i % w8;
        const uint4 *row = reinterpret_cast<const uint4 *>(gate_up + r * 2ull * width);
        const uint4 g = row[c], u = row[w8 + c];
        reinterpret_cast<uint4 *>(out + r * (uint64_t)width)[c] =
            make_uint4(swiglu_pair(g.x, u.x), swiglu_pair(g.y, u.y), swiglu_pair(g.z, u.z),
                       swiglu_pair(g.w, u.w));
    }
}

// ------------------------------------------------------------ page seal --
// Per-token FNV-1a 64 of ColdStore pages straight from the device page pool
// (src/cold_store.rs:725-742 token_hashes over a record payload): token t's
// hash runs over the D*2 bytes of token t of head 0, then head 1, ... in
// memory order.  One thread per token; the hash only depends on each token's
// bytes, so a partly filled page hashes like its compact record payload.
__global__ void __launch_bounds__(128)
    mslim_page_token_hashes(const uint16_t *__restrict__ pool, uint32_t n_pool_pages, uint32_t kv_heads,
                            uint32_t page_tokens, uint32_t head_dim, const int32_t *__restrict__ page_ids,
                            uint32_t tokens, uint64_t *__restrict__ hashes, int *status) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t pi = blockIdx.y;
    if (t >= tokens) return;
    const int32_t page = page_ids[pi];
    uint64_t *out = hashes + (size_t)pi * tokens + t;
    if (page < 0 || (uint32_t)page >= n_pool_pages) {
        if (t == 0 && status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
        *out = 0;
        return;
    }
    uint64_t state = 0xcbf29ce484222325ull;
    for (uint32_t h = 0; h < kv_heads; ++h) {
        const uint4 *row =
            reinterpret_cast<const uint4 *>(pool + (((size_t)page * kv_heads + h) * page_tokens + t) * head_dim);
        for (uint32_t c = 0; c < head_dim / 8; ++c) {
            const uint4 v = __ldg(row + c);
            const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int wd = 0; wd < 4; ++wd)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    state ^= (words[wd] >> (8 * b)) & 0xffu;
                    state *= 0x100000001b3ull;
                }
        }
    }
    *out = state;
}

// ---------------------------------------------------------------- argmax --

constexpr int kArgThreads = 1024;

// Order key of a bf16 value.  total_cmp: signed-magnitude order of the bits
// (f32::total_cmp on the widened value orders identically).  Float order:
// NaN ranks below everything, -0 == +0.
__device__ __forceinline__ int32_t order_key(uint16_t b, bool total) {
    if (total) {
        const int32_t s = (int32_t)(int16_t)b;
        return s ^ (int32_t)((uint32_t)(s >> 31) >> 17);
    }
    const uint32_t mag = b & 0x7fffu;
    if (mag > 0x7f80u) return INT_MIN;        // NaN
    if (mag == 0) return 0;                   // +-0 compare equal
    return (b & 0x8000u) ? -(int32_t)mag : (int32_t)mag;
}

// (key, index) is better than (k2, i2)
__device__ __forceinline__ bool better(int32_t k, int32_t i, int32_t k2, int32_t i2, bool last) {
    return k > k2 || (k == k2 && (last ? i > i2 : i < i2));
}

// One CTA per row.
__global__ void __launch_bounds__(kArgThreads)
    mslim_argmax(const uint16_t *__restrict__ logits, uint32_t n, int ties_to_last,
                 int32_t *__restrict__ out) {
    griddep_launch_dependents();
    griddep_wait();
    const bool last = ties_to_last != 0;
    const uint16_t *row = logits + (uint64_t)blockIdx.x * n;
    int32_t best_k = INT_MIN, best_i = -1;
    for (uint32_t i = threadIdx.x; i < n; i += kArgThreads) {
        const int32_t k = order_key(row[i], last);
        if (best_i < 0 || better(k, (int32_t)i, best_k, best_i, last)) {
            best_k = k;
            best_i = (int32_t)i;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const int32_t k2 = __shfl_xor_sync(0xffffffffu, best_k, off);
        const int32_t i2 = __shfl_xor_sync(0xffffffffu, best_i, off);
        if (i2 >= 0 && (best_i < 0 || better(k2, i2, best_k, best_i, last))) {
            best_k = k2;
            best_i = i2;
        }
    }
    __shared__ int32_t sk[kArgThreads / 32], si[kArgThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sk[warp] = best_k;
        si[warp] = best_i;
    }
    __syncthreads();
    if (warp == 0) {
        best_k = sk[lane];
        best_i = si[lane];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const int32_t k2 = __shfl_xor_sync(0xffffffffu, best_k, off);
            const int32_t i2 = __shfl_xor_sync(0xffffffffu, best_i, off);
            if (i2 >= 0 && (best_i < 0 || better(k2, i2, best_k, best_i, last))) {
                best_k = k2;
                best_i = i2;
            }
        }
        if (lane == 0) out[blockIdx.x] = best_i;
    }
}

unsigned elt_grid(uint64_t n) {
    const uint64_t vec = (n / 8 + kEltThreads - 1) / kEltThreads;
    const uint64_t cap = 148ull * 8;  // a few waves; the loop strides the rest
    return (unsigned)(vec == 0 ? 1 : (vec < cap ? vec : cap));
}

// Canonical logical K (or V) rows of one session and layer: out[h][t][0..D)
// for h < kv_heads, t < tokens, the per-tensor byte order of the logical KV
// digest (K then V, layer-major, each [kv_heads][tokens][head_dim]).  Source
// rows: a token-major dense cache (page_row == null: row (t, h) at
// src + (t * kv_heads + h) * D) or ColdStore-exact pool pages (logical page
// t / page_tokens -> physical page page_row[..], head-major inside the page).
// One thread per eight-element chunk (D % 8 == 0, 16-byte aligned) or per
// element otherwise.  A page id outside the pool writes nothing for that row
// and is recorded in the status word.
template <bool kVec>
__global__ void __launch_bounds__(256)
    mslim_kv_canonical(const uint16_t *__restrict__ src, uint16_t *__restrict__ out, uint32_t kv_heads,
                       uint32_t tokens, uint32_t dim, const int32_t *__restrict__ page_row,
                       uint32_t page_tokens, uint32_t n_pages, int *status) {
    constexpr uint32_t kW = kVec ? 8 : 1;
    const uint32_t per_row = dim / kW;
    const uint64_t total = (uint64_t)kv_heads * tokens * per_row;
    for (uint64_t x = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; x < total;
         x += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t c = (uint32_t)(x % per_row);
        const uint64_t ht = x / per_row;
        const uint32_t t = (uint32_t)(ht % tokens), h = (uint32_t)(ht / tokens);
        const uint16_t *row;
        if (page_row) {
            const int32_t phys = page_row[t / page_tokens];
            if (phys < 0 || (uint32_t)phys >= n_pages) {
                if (status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
                continue;
            }
            row = src + (((size_t)phys * kv_heads + h) * page_tokens + t % page_tokens) * dim;
        } else {
            row = src + ((size_t)t * kv_heads + h) * dim;
        }
        uint16_t *dst = out + ((size_t)h * tokens + t) * dim;
        if constexpr (kVec)
            *reinterpret_cast<uint4 *>(dst + c * 8) = *reinterpret_cast<const uint4 *>(row + c * 8);
        else
            dst[c] = row[c];
    }
}

// Certified-selection gather: for session s, the count[s] token positions
// selected[s][0..count) (strictly increasing, each below the session's
// committed length seq_tokens[s]) have their K and V rows copied to rows
// 0..count of gk/gv [n_seq][max_selected][kv_heads][dim], so a dense decode
// over count tokens attends to exactly the selected set.  The source is the
// token-major dense caches [n_seq][max_tokens][kv_heads][dim] or, with a page
// table, ColdStore-exact pool pages [n_pages][kv_heads][page_tokens][dim]
// (position t of session s is token t % page_tokens of page
// page_table[s][t / page_tokens]; head h's row of it is contiguous).  A count
// above max_selected or above the committed length, a position out of range
// or not above its predecessor, or a page id outside the pool is recorded in
// the status word and its row is not copied.  One thread per 16-byte chunk
// (dim % 8 == 0) or per element.
struct GatherSrc {
    const uint16_t *k, *v;
    uint32_t max_tokens;        // dense: rows per session; paged: max_pages * page_tokens
    const int32_t *page_table;  // null: dense
    uint32_t max_pages, page_tokens, n_pages;
};

template <bool kVec>
__global__ void __launch_bounds__(256)
    mslim_gather_selected(const GatherSrc src, uint32_t kv_heads, uint32_t dim,
                          const int32_t *__restrict__ seq_tokens, const int32_t *__restrict__ selected,
                          const int32_t *__restrict__ counts, uint32_t max_selected, uint16_t *__restrict__ gk,
                          uint16_t *__restrict__ gv, int *status) {
    constexpr uint32_t kW = kVec ? 8 : 1;
    const uint32_t s = blockIdx.x;
    const int32_t committed = seq_tokens[s];
    int32_t count = counts[s];
    if (count < 0 || (uint32_t)count > max_selected || count > committed) {
        if (threadIdx.x == 0 && blockIdx.y == 0 && status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
        return;
    }
    const int32_t *sel = selected + (size_t)s * max_selected;
    const uint32_t row_elems = kv_heads * dim;
    const uint32_t per_head = dim / kW;
    const uint32_t per_row = row_elems / kW;
    const uint64_t total = (uint64_t)count * per_row;
    for (uint64_t x = (uint64_t)blockIdx.y * blockDim.x + threadIdx.x; x < total;
         x += (uint64_t)gridDim.y * blockDim.x) {
        const uint32_t e = (uint32_t)(x / per_row), c = (uint32_t)(x % per_row);
        const int32_t pos = sel[e];
        if (pos < 0 || pos >= committed || (uint32_t)pos >= src.max_tokens || (e > 0 && sel[e - 1] >= pos)) {
            if (c == 0 && status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
            continue;
        }
        size_t from;
        if (src.page_table) {
            const int32_t phys = src.page_table[(size_t)s * src.max_pages + (uint32_t)pos / src.page_tokens];
            if (phys < 0 || (uint32_t)phys >= src.n_pages) {
                if (c == 0 && status) atomicExch(status, MSLIM_DEVICE_BAD_PAGE_CODE);
                continue;
            }
            const uint32_t h = c / per_head, within = c % per_head;
            from = (((size_t)phys * kv_heads + h) * src.page_tokens + (uint32_t)pos % src.page_tokens) * dim +
                   (size_t)within * kW;
        } else {
            from = ((size_t)s * src.max_tokens + (uint32_t)pos) * row_elems + (size_t)c * kW;
        }
        const size_t dst = ((size_t)s * max_selected + e) * row_elems + (size_t)c * kW;
        if constexpr (kVec) {
            *reinterpret_cast<uint4 *>(gk + dst) = *reinterpret_cast<const uint4 *>(src.k + from);
            *reinterpret_cast<uint4 *>(gv + dst) = *reinterpret_cast<const uint4 *>(src.v + from);
        } else {
            gk[dst] = src.k[from];
            gv[dst] = src.v[from];
        }
    }
}

}  // namespace

cudaError_t launch_gather_selected(const uint16_t *k_src, const uint16_t *v_src, uint32_t max_tokens,
                                   const int32_t *page_table, uint32_t max_pages, uint32_t page_tokens,
                                   uint32_t n_pages, uint32_t kv_heads, uint32_t dim, const int32_t *seq_tokens,
                                   const int32_t *selected, const int32_t *counts, uint32_t max_selected,
                                   uint32_t n_seq, uint16_t *gk, uint16_t *gv, int *status, cudaStream_t stream) {
    auto al = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const uint32_t row_elems = kv_heads * dim;
    const bool vec = dim % 8 == 0 && al(k_src) && al(v_src) && al(gk) && al(gv);
    const uint64_t per_session = (uint64_t)max_selected * (vec ? row_elems / 8 : row_elems);
    const unsigned chunks = (unsigned)std::min<uint64_t>(std::max<uint64_t>(1, (per_session + 255) / 256), 64);
    const dim3 grid(n_seq, chunks);
    const GatherSrc src{k_src, v_src, max_tokens, page_table, max_pages, page_tokens, n_pages};
    if (vec)
        mslim_gather_selected<true><<<grid, 256, 0, stream>>>(src, kv_heads, dim, seq_tokens, selected, counts,
                                                               max_selected, gk, gv, status);
    else
        mslim_gather_selected<false><<<grid, 256, 0, stream>>>(src, kv_heads, dim, seq_tokens, selected, counts,
                                                                max_selected, gk, gv, status);
    return counted(cudaGetLastError());
}

cudaError_t launch_kv_canonical(const uint16_t *src, uint16_t *out, uint32_t kv_heads, uint32_t tokens,
                                uint32_t dim, const int32_t *page_row, uint32_t page_tokens, uint32_t n_pages,
                                int *status, cudaStream_t stream) {
    if (tokens == 0) return cudaSuccess;
    auto al = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const bool vec = dim % 8 == 0 && al(src) && al(out);
    const uint64_t total = (uint64_t)kv_heads * tokens * (vec ? dim / 8 : dim);
    const unsigned grid = (unsigned)std::min<uint64_t>((total + 255) / 256, 148ull * 16);
    if (vec)
        mslim_kv_canonical<true><<<grid, 256, 0, stream>>>(src, out, kv_heads, tokens, dim, page_row, page_tokens,
                                                            n_pages, status);
    else
        mslim_kv_canonical<false><<<grid, 256, 0, stream>>>(src, out, kv_heads, tokens, dim, page_row, page_tokens,
                                                             n_pages, status);
    return counted(cudaGetLastError());
}

cudaError_t launch_residual_add(const uint16_t *a, const uint16_t *b, uint16_t *out, uint64_t n,
                                cudaStream_t stream) {
    return launch_pdl(mslim_residual_add, dim3(elt_grid(n)), dim3(kEltThreads), 0, stream, a, b, out, n);
}

cudaError_t launch_swiglu(const uint16_t *gate, const uint16_t *up, uint16_t *out, uint64_t n,
                          cudaStream_t stream) {
    return launch_pdl(mslim_swiglu, dim3(elt_grid(n)), dim3(kEltThreads), 0, stream, gate, up, out, n);
}

cudaError_t launch_swiglu_rows(const uint16_t *gate_up, uint16_t *out, uint32_t rows, uint32_t width,
                               cudaStream_t stream) {
    return launch_pdl(mslim_swiglu_rows, dim3(elt_grid((uint64_t)rows * width)), dim3(kEltThreads), 0, stream,
                      gate_up, out, rows, width);
}

cudaError_t launch_page_token_hashes(const uint16_t *pool, uint32_t n_pool_pages, uint32_t kv_heads,
                                     uint32_t page_tokens, uint32_t head_dim, const int32_t *page_ids,
                                     uint32_t n_pages, uint32_t tokens, uint64_t *hashes, int *status,
                                     cudaStream_t stream) {
    dim3 grid((tokens + 127) / 128, n_pages);
    mslim_page_token_hashes<<<grid, 128, 0, stream>>>(pool, n_pool_pages, kv_heads, page_tokens, head_dim,
                                                      page_ids, tokens, hashes, status);
    return counted(cudaGetLastError());
}

cudaError_t launch_argmax(const uint16_t *logits, uint32_t rows, uint32_t n, int ties_to_last,
                          int32_t *out, cudaStream_t stream) {
    return launch_pdl(mslim_argmax, dim3(rows), dim3(kArgThreads), 0, stream, logits, n, ties_to_last, out);
}

// ------------------------------------------------------ exp2 diagnostic --

__global__ void mslim_exp2_eval(const float *x, float *y_poly, float *y_mufu, float *y_ref, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = x[i];
        y_poly[i] = exp2_fma(v);
        y_mufu[i] = fast_exp2(v);
        y_ref[i] = exp2f(v);
    }
}

cudaError_t launch_exp2_eval(const float *x, float *y_poly, float *y_mufu, float *y_ref, uint32_t n,
                             cudaStream_t stream) {
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, 148u * 8);
    mslim_exp2_eval<<<blocks, 256, 0, stream>>>(x, y_poly, y_mufu, y_ref, n);
    return counted(cudaGetLastError());
}

}  // namespace mslim
