// decode.cuh -- parameters and launcher of the split-KV decode kernels.
#pragma once

#include "mslim_common.cuh"

namespace mslim {

struct DecodeParams {
    const uint16_t *q;           // bf16 [n_seq][nq][QH][D]
    const float *q_f32;          // f32 query of the same shape (dense only), or null
    const int32_t *seq_tokens;   // [n_seq] tokens in each sequence's cache
    const int32_t *page_table;   // [n_seq][max_pages] physical page ids (paged only)
    float *partials;             // [n_seq][nq][QH][max_splits][D + 4] (kernel D): acc, m, l, 2 pad
    int persistent;              // 1: the persistent form where the shape allows (the decode schedule)
    unsigned *work_counter;      // [2]: work taken and CTAs done, zero on entry, left zero;
                                 // null: one CTA per split and a merge kernel instead of
                                 // the persistent form
    unsigned *item_counters;     // persistent form: splits finished per (unit, KV-head
                                 // chunk) item, zero on entry, left zero
    uint16_t *out;               // bf16 [n_seq][nq][QH][head_dim]
    int *status;                 // device status word
    int qheads, kvheads, group;  // group = QH / KVH
    int head_chunks;             // CTAs per KV head along the group
    int heads_per_cta;           // group / head_chunks (<= 16)
    int nq;                      // query rows per sequence (1 for decode)
    int q_per_cta;               // query rows per CTA (heads_per_cta * q_per_cta <= 16)
    int q_blocks;                // ceil(nq / q_per_cta)
    int split_tokens;            // multiple of 64
    int max_splits;
    int page_tokens;             // paged only, multiple of 64
    int max_pages;               // paged only
    int n_pages;                 // paged only: pool size; table entries outside
                                 // [0, n_pages) are reported, never loaded
    int n_seq;
    int head_dim;                // caller's head_dim (<= kernel D, multiple of 8); TMA
                                 // zero-fills K/V columns past it
    int token_cap;               // tokens addressable per sequence (dense max_tokens or
                                 // max_pages * page_tokens); longer lengths are clamped
    int fixed_tokens;            // >= 0: every sequence holds this many tokens
                                 // (seq_tokens unused); < 0: read seq_tokens
    float scale_log2;            // log2(e) / sqrt(head_dim of the caller)
    float *out_f32;              // if set, the merge writes f32 here instead of bf16
};

// Enqueues the split kernel and the merge kernel on `stream`.
cudaError_t launch_decode(int head_dim, bool paged, const CUtensorMap &kmap,
                          const CUtensorMap &vmap, const DecodeParams &p, uint16_t *out,
                          cudaStream_t stream);

}  // namespace mslim
