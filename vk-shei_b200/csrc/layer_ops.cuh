// layer_ops.cuh -- launchers of the decoder-layer elementwise kernels around
// attention: residual add, SwiGLU, and the greedy argmax over logits.
#pragma once

#include "mslim_common.cuh"

namespace mslim {

cudaError_t launch_residual_add(const uint16_t *a, const uint16_t *b, uint16_t *out, uint64_t n,
                                cudaStream_t stream);
cudaError_t launch_swiglu(const uint16_t *gate, const uint16_t *up, uint16_t *out, uint64_t n,
                          cudaStream_t stream);
// gate_up: [rows][gate (width) | up (width)] -> out [rows][width]; width % 8 == 0.
cudaError_t launch_swiglu_rows(const uint16_t *gate_up, uint16_t *out, uint32_t rows, uint32_t width,
                               cudaStream_t stream);
// hashes[p][t] = FNV-1a 64 of token t (t < tokens) of pool page page_ids[p]
// over its heads in order; pool: bf16 [n_pool_pages][kv_heads][page_tokens][head_dim].
cudaError_t launch_page_token_hashes(const uint16_t *pool, uint32_t n_pool_pages, uint32_t kv_heads,
                                     uint32_t page_tokens, uint32_t head_dim, const int32_t *page_ids,
                                     uint32_t n_pages, uint32_t tokens, uint64_t *hashes, int *status,
                                     cudaStream_t stream);
// rows x n bf16 logits -> int32 index per row.  ties_to_last != 0: the largest
// value under f32::total_cmp, last index among equals (the CPU path's
// Iterator::max_by); 0: the largest by float comparison, first index among
// equals, NaN never chosen unless every entry is NaN (the OpenCL llm_argmax).
cudaError_t launch_argmax(const uint16_t *logits, uint32_t rows, uint32_t n, int ties_to_last,
                          int32_t *out, cudaStream_t stream);
// Rows selected[s][0..counts[s]) of session s -> rows 0..counts[s] of gk/gv
// [n_seq][max_selected][kv_heads][dim] (positions strictly increasing and
// below seq_tokens[s]; violations go to the status word).  Source: dense
// caches [n_seq][max_tokens][kv_heads][dim] (page_table null) or pool pages
// [n_pages][kv_heads][page_tokens][dim] listed by page_table [n_seq][max_pages]
// (max_tokens = max_pages * page_tokens).
cudaError_t launch_gather_selected(const uint16_t *k_src, const uint16_t *v_src, uint32_t max_tokens,
                                   const int32_t *page_table, uint32_t max_pages, uint32_t page_tokens,
                                   uint32_t n_pages, uint32_t kv_heads, uint32_t dim, const int32_t *seq_tokens,
                                   const int32_t *selected, const int32_t *counts, uint32_t max_selected,
                                   uint32_t n_seq, uint16_t *gk, uint16_t *gv, int *status, cudaStream_t stream);
// out [kv_heads][tokens][dim] bf16: one session's K (or V) rows in the logical
// KV digest order, from a token-major dense cache (page_row == null) or from
// ColdStore-exact pool pages [n_pages][kv_heads][page_tokens][dim] listed by
// page_row (logical page -> physical page).
cudaError_t launch_kv_canonical(const uint16_t *src, uint16_t *out, uint32_t kv_heads, uint32_t tokens,
                                uint32_t dim, const int32_t *page_row, uint32_t page_tokens, uint32_t n_pages,
                                int *status, cudaStream_t stream);

// y_poly[i] = exp2_fma(x[i]), y_mufu[i] = fast_exp2(x[i]) (the two 2^x
// evaluations of the prefill softmax), y_ref[i] = exp2f(x[i]).
cudaError_t launch_exp2_eval(const float *x, float *y_poly, float *y_mufu, float *y_ref, uint32_t n,
                             cudaStream_t stream);

}  // namespace mslim
