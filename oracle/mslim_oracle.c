/*
 * mslim_oracle.c -- CPU restatement of the M-SLIM attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library: it is called from tests/, from __graft_entry__.smoke() and from the
 * cpu_baseline / --impl reference legs of bench.py, never from the product
 * path.  It restates, operation for operation, the reference's portable CPU
 * decoder ("CPU hot-dense", the parity reference named by the north star):
 *
 *   src/native_cpu_adapter.rs:179-237  round_bf16, round_vec, rms_norm,
 *                                       apply_rope, softmax, attention_scale
 *   src/native_cpu_adapter.rs:253-307  dense_attention_bf16 (primary oracle)
 *   src/native_cpu_adapter.rs:386-455  ColdStore-exact branch of attend()
 *   src/native_cpu_adapter.rs:717-784  prefill = forward_token per prompt row
 *   src/portable.rs:575-646            CpuReferenceBackend::decode (f64)
 *   src/gpu_llm/kernels.rs:50-67       RopeKernelConfig::inverse_frequency
 *   assets/gpu_llm.cl:72-146           GPU RMSNorm / RoPE formulas
 *   src/cold_store.rs:909-922,763-781  FNV-1a checksum and per-token hashes
 *   src/gpu_region_store.rs:470-483    token-major -> head-major page layout
 *   src/native_cpu_adapter.rs:129-148  matvec (rows of bf16 weights . f32 x)
 *   src/native_cpu_adapter.rs:486-591  forward_token: one decoder layer per
 *                                       token, SwiGLU, residuals, final norm,
 *                                       lm_head and the greedy argmax
 *
 * Numeric rules kept from the Rust source:
 *   - every f32 sum is a left-to-right fold (Rust `Iterator::sum::<f32>()`
 *     folds from -0.0), with no FMA contraction: build with
 *     -ffp-contract=off and without -ffast-math;
 *   - bf16 rounding is `half` 2.7.1 `bf16::from_f32`: round to nearest even,
 *     NaN kept NaN with the quiet bit forced (also assets/gpu_llm.cl:10-21);
 *   - bf16 decode is `half` `bf16::to_f32` (NaN quiet bit forced);
 *   - exp/powf/sinf/cosf/sqrtf are glibc libm, as Rust std lowers them.
 *
 * Parity pinning: the reference ships no stored attention-output vectors; its
 * parity tests compare two live implementations.  This restatement is pinned
 * against every known-answer test the reference holds for the path (see
 * tests/test_oracle_kat.py): the Llama-3 RoPE inverse-frequency table
 * (src/gpu_llm/mod.rs:2849-2878), the GQA/MQA head mapping and extreme-score
 * softmax cases (src/portable.rs:683-726), RoPE-at-zero identity, bf16
 * representable RMSNorm and normalised softmax (src/native_cpu_adapter.rs:
 * 990-1008), all 65 536 bf16 decodes (tests/fixed_width_decode.rs:11-21) and
 * ColdStore page byte preservation (src/gpu_region_store.rs:992-1042).
 * Transcendental bits (expf/powf/sinf/cosf) are not pinned by any reference
 * test; the attention tolerance (max-abs 2e-2) covers them.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__FP_FAST_FMAF) || defined(__FAST_MATH__)
#error "the oracle must be built without fast-math (Rust does not reassociate or contract)"
#endif

#define MO_OK 0
#define MO_ERR_GEOMETRY 1
#define MO_ERR_SHAPE 2
#define MO_ERR_NONFINITE 3

/* ---------------------------------------------------------------- bf16 -- */

static inline uint32_t f32_bits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float bits_f32(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* half 2.7.1 bf16::from_f32 (round-nearest-even; NaN keeps its upper payload
 * and gets the quiet bit).  Same algorithm as write_bf16, gpu_llm.cl:10-21. */
uint16_t mo_bf16_from_f32(float value) {
    uint32_t x = f32_bits(value);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x0040u);
    const uint32_t round_bit = 0x00008000u;
    if ((x & round_bit) != 0 && (x & (3u * round_bit - 1u)) != 0)
        return (uint16_t)((x >> 16) + 1u);
    return (uint16_t)(x >> 16);
}

/* half 2.7.1 bf16::to_f32: exact widening, NaN gets the quiet bit. */
float mo_bf16_to_f32(uint16_t bits) {
    if ((bits & 0x7fffu) > 0x7f80u) return bits_f32(((uint32_t)bits | 0x0040u) << 16);
    return bits_f32((uint32_t)bits << 16);
}

/* half 2.7.1 f16::to_f32 (used only by the f64 backend for F16 frames). */
float mo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    if (exp == 0x1fu) {
        if (man == 0) return bits_f32(sign | 0x7f800000u);
        return bits_f32(sign | 0x7fc00000u | (man << 13));
    }
    if (exp == 0) {
        if (man == 0) return bits_f32(sign);
        /* subnormal: value = man * 2^-24, exactly representable in f32 */
        int e = -1;
        uint32_t m = man;
        do { e++; m <<= 1; } while ((m & 0x400u) == 0);
        uint32_t f_exp = (uint32_t)(127 - 15 - e);
        uint32_t f_man = (m & 0x3ffu) << 13;
        return bits_f32(sign | (f_exp << 23) | f_man);
    }
    return bits_f32(sign | ((exp + 127u - 15u) << 23) | (man << 13));
}

/* native_cpu_adapter.rs:179 */
float mo_round_bf16(float value) { return mo_bf16_to_f32(mo_bf16_from_f32(value)); }

void mo_bf16_encode(const float *src, uint16_t *dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = mo_bf16_from_f32(src[i]);
}
void mo_bf16_decode(const uint16_t *src, float *dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = mo_bf16_to_f32(src[i]);
}

/* -------------------------------------------------------- CPU helpers -- */

/* native_cpu_adapter.rs:194-204: sequential f32 sum of squares, mean by
 * division, scale = 1 / sqrt(mean + eps), out = bf16(bf16(x*scale) * w). */
void mo_rms_norm(const float *x, const float *weight, size_t n, float eps, float *out) {
    float sum = -0.0f;
    for (size_t i = 0; i < n; ++i) sum = sum + x[i] * x[i];
    float mean = sum / (float)n;
    float scale = 1.0f / sqrtf(mean + eps);
    for (size_t i = 0; i < n; ++i) {
        float normalized = mo_round_bf16(x[i] * scale);
        out[i] = mo_round_bf16(normalized * weight[i]);
    }
}

/* Batched restatement over `tokens` rows of bf16 input, as the CPU path
 * applies rms_norm once per token. */
void mo_rms_norm_rows_bf16(const uint16_t *x, const uint16_t *w, uint16_t *y,
                           size_t tokens, size_t hidden, float eps) {
    float *xf = (float *)malloc(hidden * sizeof(float));
    float *wf = (float *)malloc(hidden * sizeof(float));
    float *of = (float *)malloc(hidden * sizeof(float));
    mo_bf16_decode(w, wf, hidden);
    for (size_t t = 0; t < tokens; ++t) {
        mo_bf16_decode(x + t * hidden, xf, hidden);
        mo_rms_norm(xf, wf, hidden, eps, of);
        mo_bf16_encode(of, y + t * hidden, hidden);
    }
    free(xf); free(wf); free(of);
}

/* native_cpu_adapter.rs:206-221: rotate_half RoPE with the CPU frequency
 * formula angle = position / theta^(2i/dim); cos/sin rounded to bf16 and every
 * product and sum rounded to bf16. */
void mo_apply_rope(float *values, size_t heads, size_t dim, size_t position, float theta) {
    size_t half = dim / 2;
    for (size_t head = 0; head < heads; ++head) {
        size_t base = head * dim;
        for (size_t i = 0; i < half; ++i) {
            float angle = (float)position / powf(theta, (float)(2 * i) / (float)dim);
            float s = mo_round_bf16(sinf(angle));
            float c = mo_round_bf16(cosf(angle));
            float a = values[base + i];
            float b = values[base + i + half];
            values[base + i] = mo_round_bf16(mo_round_bf16(a * c) - mo_round_bf16(b * s));
            values[base + i + half] = mo_round_bf16(mo_round_bf16(b * c) + mo_round_bf16(a * s));
        }
    }
}

/* RoPE over `tokens` rows [tokens][heads][dim] of bf16, row t at position
 * start_position + t (the CPU prefill runs forward_token per prompt row). */
void mo_apply_rope_rows_bf16(const uint16_t *in, uint16_t *out, size_t tokens, size_t heads,
                             size_t dim, size_t start_position, float theta) {
    size_t row = heads * dim;
    float *tmp = (float *)malloc(row * sizeof(float));
    for (size_t t = 0; t < tokens; ++t) {
        mo_bf16_decode(in + t * row, tmp, row);
        mo_apply_rope(tmp, heads, dim, start_position + t, theta);
        mo_bf16_encode(tmp, out + t * row, row);
    }
    free(tmp);
}

/* native_cpu_adapter.rs:223-233 */
void mo_softmax(float *values, size_t n) {
    float max = -INFINITY;
    for (size_t i = 0; i < n; ++i) max = fmaxf(max, values[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        values[i] = expf(values[i] - max);
        sum += values[i];
    }
    for (size_t i = 0; i < n; ++i) values[i] /= sum;
}

/* native_cpu_adapter.rs:235-237 */
float mo_attention_scale(size_t head_dim) { return 1.0f / sqrtf((float)head_dim); }

/* ----------------------------------------------- dense_attention_bf16 -- */

/* One query head of native_cpu_adapter.rs:253-307.  `key_rows`/`value_rows`
 * address token t's row for this KV head as base + t*token_stride. */
static void attend_one_head(const float *q, const uint16_t *keys, const uint16_t *values,
                            size_t tokens, size_t token_stride, size_t head_dim, float scale,
                            float *scores, float *out) {
    for (size_t t = 0; t < tokens; ++t) {
        const uint16_t *k = keys + t * token_stride;
        float dot = -0.0f;
        for (size_t d = 0; d < head_dim; ++d) dot = dot + q[d] * mo_bf16_to_f32(k[d]);
        scores[t] = dot * scale;
    }
    mo_softmax(scores, tokens);
    for (size_t d = 0; d < head_dim; ++d) out[d] = 0.0f;
    for (size_t t = 0; t < tokens; ++t) {
        const uint16_t *v = values + t * token_stride;
        float p = scores[t];
        for (size_t d = 0; d < head_dim; ++d) out[d] += p * mo_bf16_to_f32(v[d]);
    }
    for (size_t d = 0; d < head_dim; ++d) out[d] = mo_round_bf16(out[d]);
}

/* native_cpu_adapter.rs:253-307.  query: f32 [QH*D] holding the bf16-rounded
 * post-RoPE query; keys/values: bf16 token-major [tokens][KVH][D]; out: f32
 * [QH*D] holding bf16 values.  Parallel over query heads like the rayon
 * `par_chunks_mut(head_dim)` of the reference (no reduction order changes). */
int mo_dense_attention_bf16(size_t query_heads, size_t kv_heads, size_t head_dim,
                            const float *query, const uint16_t *keys, const uint16_t *values,
                            size_t tokens, float *output, int threads) {
    if (query_heads == 0 || kv_heads == 0 || head_dim == 0 || query_heads % kv_heads != 0)
        return MO_ERR_GEOMETRY;
    size_t group = query_heads / kv_heads;
    size_t token_stride = kv_heads * head_dim;
    float scale = mo_attention_scale(head_dim);
    long qh;
    (void)threads;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (qh = 0; qh < (long)query_heads; ++qh) {
        float *scores = (float *)malloc((tokens ? tokens : 1) * sizeof(float));
        size_t kh = (size_t)qh / group;
        attend_one_head(query + (size_t)qh * head_dim, keys + kh * head_dim,
                        values + kh * head_dim, tokens, token_stride, head_dim, scale, scores,
                        output + (size_t)qh * head_dim);
        free(scores);
    }
    return MO_OK;
}

/* Causal chunked prefill as the CPU path computes it: every prompt row runs
 * forward_token (native_cpu_adapter.rs:717-784), so query row i (absolute
 * position prior+i) attends over keys 0..=prior+i with dense_attention_bf16.
 * q: bf16 [queries][QH][D]; k/v: bf16 [prior+queries][KVH][D];
 * out: bf16 [queries][QH][D].  Parallel over (row, head). */
int mo_causal_prefill_bf16(size_t query_heads, size_t kv_heads, size_t head_dim,
                           const uint16_t *q, const uint16_t *keys, const uint16_t *values,
                           size_t queries, size_t prior, uint16_t *out, int threads) {
    if (query_heads == 0 || kv_heads == 0 || head_dim == 0 || query_heads % kv_heads != 0)
        return MO_ERR_GEOMETRY;
    size_t group = query_heads / kv_heads;
    size_t token_stride = kv_heads * head_dim;
    float scale = mo_attention_scale(head_dim);
    long item;
    long items = (long)(queries * query_heads);
    (void)threads;
#pragma omp parallel for schedule(dynamic, 4) num_threads(threads > 0 ? threads : 1)
    for (item = items - 1; item >= 0; --item) {
        size_t row = (size_t)item / query_heads;
        size_t qh = (size_t)item % query_heads;
        size_t history = prior + row + 1;
        float *scores = (float *)malloc(history * sizeof(float));
        float *qf = (float *)malloc(head_dim * sizeof(float));
        float *of = (float *)malloc(head_dim * sizeof(float));
        mo_bf16_decode(q + (row * query_heads + qh) * head_dim, qf, head_dim);
        size_t kh = qh / group;
        attend_one_head(qf, keys + kh * head_dim, values + kh * head_dim, history, token_stride,
                        head_dim, scale, scores, of);
        mo_bf16_encode(of, out + (row * query_heads + qh) * head_dim, head_dim);
        free(scores); free(qf); free(of);
    }
    return MO_OK;
}

/* ------------------------------------------ ColdStore-exact decode path -- */

/* native_cpu_adapter.rs:386-455 with epsilon 0: K and V are read back from
 * head-major pages [KVH][page_tokens][D] into token-major order (what
 * GpuRegionStore::read_keys/read_values return, gpu_region_store.rs:828-931),
 * then the same f32 scores / softmax / PV as dense_attention_bf16.
 * page_table: physical page index for each logical page of this session. */
int mo_paged_attention_bf16(size_t query_heads, size_t kv_heads, size_t head_dim,
                            const float *query, const uint16_t *k_pool, const uint16_t *v_pool,
                            const int32_t *page_table, size_t page_tokens, size_t tokens,
                            float *output, int threads) {
    size_t row = kv_heads * head_dim;
    uint16_t *k = (uint16_t *)malloc((tokens ? tokens : 1) * row * sizeof(uint16_t));
    uint16_t *v = (uint16_t *)malloc((tokens ? tokens : 1) * row * sizeof(uint16_t));
    size_t page_elems = kv_heads * page_tokens * head_dim;
    for (size_t t = 0; t < tokens; ++t) {
        size_t page = (size_t)page_table[t / page_tokens];
        size_t off = t % page_tokens;
        for (size_t h = 0; h < kv_heads; ++h) {
            size_t src = page * page_elems + (h * page_tokens + off) * head_dim;
            memcpy(k + t * row + h * head_dim, k_pool + src, head_dim * sizeof(uint16_t));
            memcpy(v + t * row + h * head_dim, v_pool + src, head_dim * sizeof(uint16_t));
        }
    }
    int rc = mo_dense_attention_bf16(query_heads, kv_heads, head_dim, query, k, v, tokens, output,
                                     threads);
    free(k); free(v);
    return rc;
}

/* ------------------------------------------------ f64 portable backend -- */

/* src/portable.rs:575-646: online log-sum-exp in f64 over frames
 * [t][KVH][D]; dtype 1 = bf16, 2 = f16, 3 = f32 (little-endian raw bits).
 * Returns MO_ERR_NONFINITE for the same conditions as PortableError. */
static double element_f64(const void *data, size_t index, int dtype) {
    if (dtype == 3) { float f; memcpy(&f, (const char *)data + index * 4, 4); return (double)f; }
    uint16_t h; memcpy(&h, (const char *)data + index * 2, 2);
    return (double)(dtype == 1 ? mo_bf16_to_f32(h) : mo_f16_to_f32(h));
}

int mo_cpu_reference_decode_f64(size_t query_heads, size_t kv_heads, size_t head_dim,
                                const float *query, const void *keys, const void *values,
                                int key_dtype, int value_dtype, size_t tokens, float *output) {
    if (query_heads == 0 || kv_heads == 0 || head_dim == 0 || query_heads % kv_heads != 0)
        return MO_ERR_GEOMETRY;
    for (size_t i = 0; i < query_heads * head_dim; ++i)
        if (!isfinite(query[i])) return MO_ERR_NONFINITE;
    if (tokens == 0) {
        for (size_t i = 0; i < query_heads * head_dim; ++i) output[i] = 0.0f;
        return MO_OK;
    }
    double scale = 1.0 / sqrt((double)head_dim);
    size_t group = query_heads / kv_heads;
    double *weighted = (double *)malloc(head_dim * sizeof(double));
    int rc = MO_OK;
    for (size_t qh = 0; qh < query_heads && rc == MO_OK; ++qh) {
        size_t kvh = qh / group;
        const float *q = query + qh * head_dim;
        double max_score = -INFINITY, denominator = 0.0;
        for (size_t i = 0; i < head_dim; ++i) weighted[i] = 0.0;
        for (size_t t = 0; t < tokens && rc == MO_OK; ++t) {
            size_t offset = (t * kv_heads + kvh) * head_dim;
            double dot = 0.0;
            for (size_t i = 0; i < head_dim; ++i) {
                double kvalue = element_f64(keys, offset + i, key_dtype);
                if (!isfinite(kvalue)) { rc = MO_ERR_NONFINITE; break; }
                dot += (double)q[i] * kvalue;
            }
            if (rc) break;
            double score = dot * scale;
            if (!isfinite(score)) { rc = MO_ERR_NONFINITE; break; }
            double next_max = fmax(max_score, score);
            double prior = exp(max_score - next_max);
            double current = exp(score - next_max);
            denominator = denominator * prior + current;
            for (size_t i = 0; i < head_dim; ++i) {
                double item = element_f64(values, offset + i, value_dtype);
                if (!isfinite(item)) { rc = MO_ERR_NONFINITE; break; }
                weighted[i] = weighted[i] * prior + current * item;
            }
            max_score = next_max;
        }
        if (rc) break;
        if (!isfinite(denominator) || denominator <= 0.0) { rc = MO_ERR_NONFINITE; break; }
        for (size_t i = 0; i < head_dim; ++i) {
            double value = weighted[i] / denominator;
            if (!isfinite(value) || fabs(value) > 3.4028234663852886e38) { rc = MO_ERR_NONFINITE; break; }
            output[qh * head_dim + i] = (float)value;
        }
    }
    free(weighted);
    return rc;
}

/* ----------------------------------------------- GPU prologue formulas -- */

/* src/gpu_llm/kernels.rs:50-67 (== assets/gpu_llm.cl:121-136): inverse RoPE
 * frequency exp(-fdim * ln(theta) / head_dim) with optional Llama-3 scaling.
 * TAU is std::f32::consts::TAU. */
float mo_rope_inverse_frequency(float theta, uint32_t llama3, float factor, float low_freq_factor,
                                float high_freq_factor, float original_max_position,
                                size_t frequency_dim, size_t head_dim) {
    float inverse = expf(-(float)frequency_dim * logf(theta) / (float)head_dim);
    if (llama3) {
        const float tau = 6.28318530717958647692f;
        float wavelength = tau / inverse;
        float low_wavelength = original_max_position / low_freq_factor;
        float high_wavelength = original_max_position / high_freq_factor;
        if (wavelength > low_wavelength) {
            inverse /= factor;
        } else if (wavelength >= high_wavelength) {
            float smooth = (original_max_position / wavelength - low_freq_factor) /
                           (high_freq_factor - low_freq_factor);
            inverse = (1.0f - smooth) * (inverse / factor) + smooth * inverse;
        }
    }
    return inverse;
}

/* assets/gpu_llm.cl:102-146 / 412-456 (llm_rope, llm_prefill_rope): the
 * reference GPU RoPE formula, element-wise over [tokens][heads][dim]. */
void mo_gpu_rope_rows_bf16(const uint16_t *in, uint16_t *out, size_t tokens, size_t heads,
                           size_t dim, size_t start_position, float theta, uint32_t llama3,
                           float factor, float low_freq_factor, float high_freq_factor,
                           float original_max_position) {
    size_t elements = heads * dim, half = dim / 2;
    for (size_t i = 0; i < tokens * elements; ++i) {
        size_t token = i / elements, in_token = i % elements;
        size_t head = in_token / dim, d = in_token % dim;
        size_t counterpart = token * elements + head * dim + (d < half ? d + half : d - half);
        float rotated = d < half ? -mo_bf16_to_f32(in[counterpart]) : mo_bf16_to_f32(in[counterpart]);
        size_t fdim = (d % half) * 2;
        float inv = mo_rope_inverse_frequency(theta, llama3, factor, low_freq_factor,
                                              high_freq_factor, original_max_position, fdim, dim);
        float angle = (float)(start_position + token) * inv;
        float c = mo_round_bf16(cosf(angle));
        float s = mo_round_bf16(sinf(angle));
        float left = mo_round_bf16(mo_bf16_to_f32(in[i]) * c);
        float right = mo_round_bf16(rotated * s);
        out[i] = mo_bf16_from_f32(left + right);
    }
}

/* ----------------------------------------------------------- ColdStore -- */

/* src/cold_store.rs:909-922 FNV-1a 64 over a byte string. */
uint64_t mo_fnv1a64(const uint8_t *bytes, size_t n) {
    uint64_t state = 0xcbf29ce484222325ull;
    for (size_t i = 0; i < n; ++i) {
        state ^= (uint64_t)bytes[i];
        state *= 0x100000001b3ull;
    }
    return state;
}

/* src/cold_store.rs:763-781 token_hashes: per token, FNV-1a over that token's
 * bytes in every head of a head-major payload [heads][tokens][per_head_token]. */
void mo_token_hashes(const uint8_t *payload, size_t heads, size_t tokens,
                     size_t per_head_token, uint64_t *hashes) {
    for (size_t token = 0; token < tokens; ++token) {
        uint64_t state = 0xcbf29ce484222325ull;
        for (size_t head = 0; head < heads; ++head) {
            const uint8_t *p = payload + (head * tokens + token) * per_head_token;
            for (size_t b = 0; b < per_head_token; ++b) {
                state ^= (uint64_t)p[b];
                state *= 0x100000001b3ull;
            }
        }
        hashes[token] = state;
    }
}

/* src/gpu_region_store.rs:470-483: one page of n tokens, token-major
 * [n][KVH][D] -> head-major [KVH][n][D]. */
void mo_page_from_token_major(const uint16_t *token_major, uint16_t *page, size_t n,
                              size_t kv_heads, size_t head_dim) {
    for (size_t h = 0; h < kv_heads; ++h)
        for (size_t t = 0; t < n; ++t)
            memcpy(page + (h * n + t) * head_dim, token_major + (t * kv_heads + h) * head_dim,
                   head_dim * sizeof(uint16_t));
}

int mo_openmp_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------- decoder layer -- */

/* native_cpu_adapter.rs:129-148: out[r] = round_bf16(sum_c bf16(w[r][c]) * x[c]),
 * the sum a left fold in column order.  Rows in parallel (rayon
 * par_chunks_exact over rows; no reduction order changes). */
void mo_matvec_bf16(const uint16_t *w, size_t rows, size_t cols, const float *x, float *out,
                    int threads) {
    long r;
    (void)threads;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (r = 0; r < (long)rows; ++r) {
        const uint16_t *row = w + (size_t)r * cols;
        float sum = -0.0f;
        for (size_t c = 0; c < cols; ++c) sum = sum + mo_bf16_to_f32(row[c]) * x[c];
        out[r] = mo_round_bf16(sum);
    }
}

/* native_cpu_adapter.rs:186-191 */
void mo_add_residual(const float *lhs, const float *rhs, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = mo_round_bf16(lhs[i] + rhs[i]);
}

/* native_cpu_adapter.rs:553-560: silu = bf16(g / (1 + exp(-g))), out = bf16(silu * u). */
void mo_swiglu(const float *gate, const float *up, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float g = gate[i];
        float silu = mo_round_bf16(g / (1.0f + expf(-g)));
        out[i] = mo_round_bf16(silu * up[i]);
    }
}

/* f32::total_cmp key: a signed-magnitude order over the bits
 * (-NaN < -inf < ... < -0 < +0 < ... < +inf < +NaN). */
static inline int32_t total_key(float v) {
    int32_t b = (int32_t)f32_bits(v);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

/* native_cpu_adapter.rs:582-587: logits.iter().enumerate().max_by(total_cmp);
 * Iterator::max_by returns the last of equally maximal elements. */
long mo_argmax_last(const float *x, size_t n) {
    if (n == 0) return -1;
    size_t best = 0;
    int32_t key = total_key(x[0]);
    for (size_t i = 1; i < n; ++i) {
        int32_t k = total_key(x[i]);
        if (k >= key) { key = k; best = i; }
    }
    return (long)best;
}

/* Weights of one decoder layer, bf16 row-major [out][in] (HF names). */
typedef struct {
    const uint16_t *input_norm;   /* [hidden] input_layernorm */
    const uint16_t *wq;           /* [QH*D][hidden] self_attn.q_proj */
    const uint16_t *wk;           /* [KVH*D][hidden] */
    const uint16_t *wv;           /* [KVH*D][hidden] */
    const uint16_t *wo;           /* [hidden][QH*D] self_attn.o_proj */
    const uint16_t *post_norm;    /* [hidden] post_attention_layernorm */
    const uint16_t *wg;           /* [intermediate][hidden] mlp.gate_proj */
    const uint16_t *wu;           /* [intermediate][hidden] mlp.up_proj */
    const uint16_t *wd;           /* [hidden][intermediate] mlp.down_proj */
} mo_layer_weights;

/* One layer of forward_token (native_cpu_adapter.rs:503-577) for the token at
 * `position`.  k_cache / v_cache: bf16 token-major [>= position+1][KVH][D]
 * holding positions 0..position-1; this token's K/V are written at
 * `position` (the hot-dense append, :457-481) and attention runs over
 * position+1 tokens (dense_attention_bf16).  state: f32 [hidden] holding bf16
 * values, updated in place.  Optional outputs (NULL skips): q_rope (QH*D),
 * k_rope (KVH*D), attn (QH*D): the post-RoPE query/key and the attention
 * output of this token. */
int mo_layer_forward_token(const mo_layer_weights *w, size_t hidden, size_t intermediate,
                           size_t query_heads, size_t kv_heads, size_t head_dim, float eps,
                           float theta, size_t position, uint16_t *k_cache, uint16_t *v_cache,
                           float *state, float *q_rope, float *k_rope, float *attn_out,
                           int threads) {
    if (query_heads == 0 || kv_heads == 0 || head_dim == 0 || query_heads % kv_heads != 0)
        return MO_ERR_GEOMETRY;
    const size_t qd = query_heads * head_dim, kd = kv_heads * head_dim;
    size_t big = hidden > intermediate ? hidden : intermediate;
    if (qd > big) big = qd;
    float *wf = (float *)malloc(hidden * sizeof(float));
    float *normed = (float *)malloc(hidden * sizeof(float));
    float *q = (float *)malloc(qd * sizeof(float));
    float *k = (float *)malloc(kd * sizeof(float));
    float *v = (float *)malloc(kd * sizeof(float));
    float *att = (float *)malloc(qd * sizeof(float));
    float *proj = (float *)malloc(big * sizeof(float));
    float *gate = (float *)malloc(intermediate * sizeof(float));
    float *up = (float *)malloc(intermediate * sizeof(float));
    int rc = MO_OK;

    mo_bf16_decode(w->input_norm, wf, hidden);
    mo_rms_norm(state, wf, hidden, eps, normed);
    mo_matvec_bf16(w->wq, qd, hidden, normed, q, threads);
    mo_matvec_bf16(w->wk, kd, hidden, normed, k, threads);
    mo_matvec_bf16(w->wv, kd, hidden, normed, v, threads);
    /* round_vec after matvec is the identity on already-rounded values */
    mo_apply_rope(q, query_heads, head_dim, position, theta);
    mo_apply_rope(k, kv_heads, head_dim, position, theta);
    mo_bf16_encode(k, k_cache + position * kd, kd);
    mo_bf16_encode(v, v_cache + position * kd, kd);
    rc = mo_dense_attention_bf16(query_heads, kv_heads, head_dim, q, k_cache, v_cache,
                                 position + 1, att, threads);
    if (rc == MO_OK) {
        if (q_rope) memcpy(q_rope, q, qd * sizeof(float));
        if (k_rope) memcpy(k_rope, k, kd * sizeof(float));
        if (attn_out) memcpy(attn_out, att, qd * sizeof(float));
        mo_matvec_bf16(w->wo, hidden, qd, att, proj, threads);
        mo_add_residual(state, proj, state, hidden);
        mo_bf16_decode(w->post_norm, wf, hidden);
        mo_rms_norm(state, wf, hidden, eps, normed);
        mo_matvec_bf16(w->wg, intermediate, hidden, normed, gate, threads);
        mo_matvec_bf16(w->wu, intermediate, hidden, normed, up, threads);
        mo_swiglu(gate, up, gate, intermediate);
        mo_matvec_bf16(w->wd, hidden, intermediate, gate, proj, threads);
        mo_add_residual(state, proj, state, hidden);
    }
    free(wf); free(normed); free(q); free(k); free(v); free(att); free(proj); free(gate); free(up);
    return rc;
}

/* native_cpu_adapter.rs:579-587: final RMSNorm, lm_head matvec and the greedy
 * token.  logits (optional): f32 [vocab] holding bf16 values. */
long mo_lm_head_argmax(const float *state, const uint16_t *final_norm, const uint16_t *lm_head,
                       size_t hidden, size_t vocab, float eps, float *logits, int threads) {
    float *wf = (float *)malloc(hidden * sizeof(float));
    float *normed = (float *)malloc(hidden * sizeof(float));
    float *lg = logits ? logits : (float *)malloc(vocab * sizeof(float));
    mo_bf16_decode(final_norm, wf, hidden);
    mo_rms_norm(state, wf, hidden, eps, normed);
    mo_matvec_bf16(lm_head, vocab, hidden, normed, lg, threads);
    long next = mo_argmax_last(lg, vocab);
    if (!logits) free(lg);
    free(wf); free(normed);
    return next;
}
