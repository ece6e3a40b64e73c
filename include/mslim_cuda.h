/*
 * mslim_cuda.h -- C ABI of the B200 (sm_100a) attention hot path for M-SLIM.
 *
 * The Rust host side of M-SLIM keeps its attention-kernel / backend API and
 * calls these functions through `extern "C"`; every entry point names the
 * reference interface it replaces (paths inside sheilyneural-afk/VK-SHEI).
 *
 * Conventions (modelled on native/hipblaslt_bridge.cpp:25-38,155-160):
 *   - every function returns an int status, MSLIM_OK (0) on success;
 *   - the message of the last failure on the calling thread is returned by
 *     mslim_cuda_last_error() (thread-local, valid until the next call);
 *   - device pointers are owned by the caller; no function allocates device
 *     memory per call.  Scratch is passed in (workspace) or owned by a plan
 *     created once, like TiledAttention::build owns its split partials
 *     (src/gpu_llm/tiled_attention.rs:127-129);
 *   - work is enqueued on the caller's stream (`stream` is a cudaStream_t,
 *     NULL = legacy default stream); no host synchronisation inside decode;
 *   - inputs are read-only and must not alias the output
 *     (src/gpu_llm/tiled_attention.rs:204-207);
 *   - the device addresses of the library's own device globals (the status
 *     word, the static decode scratch) are looked up once per device and
 *     kept for the life of the process: do not call the library on a device
 *     after cudaDeviceReset or any other teardown of its primary context.
 *
 * Data formats: "bf16" is raw little-endian uint16 bits.  K/V are either
 * token-major [tokens][kv_heads][head_dim] (the reference's dense GPU caches,
 * src/gpu_llm/mod.rs:2099-2116) or ColdStore-exact pages, head-major
 * [kv_heads][page_tokens][head_dim] per page (src/cold_store.rs:725-742,
 * src/gpu_region_store.rs:470-483), addressed through a device page table.
 */
#ifndef MSLIM_CUDA_H
#define MSLIM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  1..5 map one-to-one onto PortableError (src/portable.rs:39-59);
 * 6 is the anyhow error of AttentionKernelConfig::validate
 * (src/attention_kernel.rs:43-79); 7 is a device-side wait that hit its
 * bound (the kernel recorded it and returned; see mslim_cuda_device_status). */
#define MSLIM_OK 0
#define MSLIM_ERR_INVALID_GEOMETRY 1
#define MSLIM_ERR_SHAPE_MISMATCH 2
#define MSLIM_ERR_NON_FINITE 3
#define MSLIM_ERR_UNSUPPORTED_DEVICE 4
#define MSLIM_ERR_BACKEND_FAILURE 5
#define MSLIM_ERR_INVALID_CONFIG 6
#define MSLIM_ERR_DEVICE_TIMEOUT 7

/* AttentionGeometry, src/portable.rs:413-457. */
typedef struct {
    uint32_t query_heads;
    uint32_t kv_heads;
    uint32_t head_dim;
} mslim_geometry_t;

/* AttentionKernelMode, src/attention_kernel.rs:8-14 (serde snake_case names:
 * "reference", "strict_tiled", "online_experimental", "split_kv_experimental"). */
#define MSLIM_MODE_REFERENCE 0
#define MSLIM_MODE_STRICT_TILED 1
#define MSLIM_MODE_ONLINE_EXPERIMENTAL 2
#define MSLIM_MODE_SPLIT_KV_EXPERIMENTAL 3

/* AttentionKernelConfig, src/attention_kernel.rs:18-34 (same fields, same
 * defaults: mode reference, block_queries 1, block_keys 64, work_group 64,
 * splits 1). */
typedef struct {
    int32_t mode;
    uint32_t block_queries;
    uint32_t block_keys;
    uint32_t work_group;
    uint32_t splits;
} mslim_kernel_config_t;

/* RopeKernelConfig, src/gpu_llm/kernels.rs:16-47. */
typedef struct {
    float theta;
    uint32_t llama3_scaling;
    float factor;
    float low_freq_factor;
    float high_freq_factor;
    float original_max_position;
} mslim_rope_config_t;

/* ------------------------------------------------------------ errors -- */

/* Thread-local message of the last failure (hipblaslt_bridge.cpp:157-159). */
const char *mslim_cuda_last_error(void);

/* Reads (and with reset != 0 clears) the device status word that kernels set
 * when a bounded device-side wait gives up (*status = MSLIM_ERR_DEVICE_TIMEOUT,
 * same return code) or a page-table entry lies outside the page pool
 * (*status = MSLIM_ERR_SHAPE_MISMATCH, same return code; the pool is never
 * addressed through such an entry: appends and gathers write nothing for it,
 * a paged decode leaves that session's output undefined); synchronises
 * `device`.  No reference counterpart: the
 * reference relies on the OpenCL queue timeout (docs/validation/
 * tiled-attention.json:790-796). */
int mslim_cuda_device_status(int device, int reset, int *status);

/* Kernels this library has launched in the process so far (every device and
 * stream; a launch recorded into a stream capture counts once, at capture).
 * A host that replays a captured step K times ran K x the launches the
 * capture added.  No reference counterpart (an accounting aid). */
uint64_t mslim_cuda_kernel_launches(void);

/* ------------------------------------------- configuration contract -- */

/* AttentionGeometry::new (src/portable.rs:421-443). */
int mslim_cuda_geometry_validate(const mslim_geometry_t *geometry);

/* AttentionKernelConfig::default (src/attention_kernel.rs:25-35). */
mslim_kernel_config_t mslim_cuda_config_default(void);

/* AttentionKernelConfig::validate / validate_activation
 * (src/attention_kernel.rs:43-79,93-100).  allow_experimental < 0 runs
 * validate() only. */
int mslim_cuda_config_validate(const mslim_kernel_config_t *config, int allow_experimental);

/* AttentionKernelConfig::id (src/attention_kernel.rs:101-110); writes a NUL
 * terminated string of at most len bytes. */
int mslim_cuda_config_id(const mslim_kernel_config_t *config, char *out, size_t len);

/* AttentionKernelConfig::local_bytes / decode_scratch_bytes
 * (src/attention_kernel.rs:113-138). */
int mslim_cuda_config_local_bytes(const mslim_kernel_config_t *config, uint32_t head_dim,
                                  size_t *bytes);
int mslim_cuda_config_decode_scratch_bytes(const mslim_kernel_config_t *config, uint32_t heads,
                                           uint32_t head_dim, size_t *bytes);

/* ---------------------------------------------- attention plan (L3) -- */

typedef struct mslim_plan mslim_plan_t;

/* TiledAttention::build (src/gpu_llm/tiled_attention.rs:39-145): validates
 * config and geometry, checks the device is sm_100, and allocates the plan's
 * split scratch once on `device`.  Every mode runs the same B200 numeric
 * contract (split-KV online softmax with a fixed-order combine). */
int mslim_cuda_plan_build(const mslim_kernel_config_t *config, const mslim_geometry_t *geometry,
                          int device, mslim_plan_t **plan);
void mslim_cuda_plan_destroy(mslim_plan_t *plan);

/* TiledAttention::run (src/gpu_llm/tiled_attention.rs:161-293): `queries`
 * new query rows at positions prior..prior+queries attend causally to keys
 * 0..=prior+row.  q/out: bf16 [queries][QH][D]; k/v: bf16 token-major
 * [prior+queries][KVH][D].  The *_bytes arguments are the allocation sizes
 * (checked like Buffer::size() at tiled_attention.rs:198-203). */
int mslim_cuda_plan_run(mslim_plan_t *plan, const void *q, size_t q_bytes, const void *k,
                        size_t k_bytes, const void *v, size_t v_bytes, void *out,
                        size_t out_bytes, uint32_t queries, uint32_t prior, void *stream);

/* TiledAttention::diagnostics (src/gpu_llm/tiled_attention.rs:147-158):
 * JSON with the same keys. */
int mslim_cuda_plan_diagnostics(const mslim_plan_t *plan, char *out, size_t len);

/* ------------------------------------------------- decode attention -- */

/* Bytes of split scratch that mslim_cuda_decode_* need for n_seq sequences
 * of at most max_tokens tokens split every split_tokens tokens
 * (split_tokens 0 = library policy).  Counterpart of
 * AttentionKernelConfig::decode_scratch_bytes (src/attention_kernel.rs:124-138).
 * A decode workspace must be zero-filled once before its first use: its
 * head holds the counters from which the persistent schedule's resident CTAs
 * take their work and find the last split of each item (see
 * mslim_cuda_set_decode_schedule), and every call leaves them zero again.
 * One workspace serves any later calls that fit it, on one stream at a time. */
int mslim_cuda_decode_workspace_bytes(const mslim_geometry_t *geometry, uint32_t n_seq,
                                      uint32_t max_tokens, uint32_t split_tokens, size_t *bytes);

/* The split size (tokens, a multiple of 64) that split_tokens == 0 selects
 * for n_seq sequences of at most max_tokens tokens: the model of
 * mslim_cuda_decode_split_tokens_for_lengths with every sequence taken at
 * max_tokens, its constants fitted to sweeps of equal-length batches (256..3072
 * tokens; remembered per shape).  The number of splits
 * it gives is not monotone in max_tokens, so a workspace meant for every
 * history up to some capacity is sized with split_tokens = 256, the shortest
 * split it takes.  Outputs depend on the split size only through rounding; a
 * caller that needs the same bits from two calls passes the same explicit
 * value (or the same max_tokens).  Counterpart of the split count that
 * AttentionKernelConfig carries (src/attention_kernel.rs:6-42). */
int mslim_cuda_decode_split_tokens(const mslim_geometry_t *geometry, uint32_t n_seq,
                                   uint32_t max_tokens, uint32_t *split_tokens);

/* A split size for one batch whose token counts the host knows (host int32
 * lengths[n_seq], as the runtime tracks them): the split CTAs of a decode
 * run in waves of the GPU's resident CTAs, each paying a fixed start-up cost
 * besides its tokens, so every candidate size (3072, 2688, 2048, 1536, 1024,
 * 768, 512, 256 tokens; none needing more than 16 waves, except 3072) runs
 * through a model of those CTAs sharing HBM and the fastest is kept (at most
 * the longest sequence rounded up to 64, at least 256); pass it to the decode
 * calls of that batch (bits are identical for every call with the same split
 * size).  No reference counterpart: the reference's split-KV plan takes a
 * fixed split count. */
int mslim_cuda_decode_split_tokens_for_lengths(const mslim_geometry_t *geometry, uint32_t n_seq,
                                               const int32_t *lengths, uint32_t *split_tokens);

/* Decode schedule, process-wide: every decode entry point follows it.
 * MSLIM_DECODE_SPLIT_MERGE (the default): one CTA per (split, KV-head chunk,
 * sequence), then a merge kernel -- two launches per decode.
 * MSLIM_DECODE_PERSISTENT: resident CTAs take splits from a work counter in
 * the workspace head and merge each item in-kernel -- one launch -- where the
 * shape allows (up to 256 sequence x query blocks, 64 splits, 16384 items, a
 * 16-byte aligned bf16 query), the split + merge form otherwise.  Both return
 * the same bits.  Measured on B200 at the C4 shapes (the shares of 1, 2, 4
 * and 8 GPUs, splits from mslim_cuda_decode_split_tokens_for_lengths): split
 * + merge 5-7 % faster.  Returns MSLIM_ERR_SHAPE_MISMATCH for another value.
 * No reference counterpart. */
#define MSLIM_DECODE_SPLIT_MERGE 0
#define MSLIM_DECODE_PERSISTENT 1
int mslim_cuda_set_decode_schedule(int schedule);
int mslim_cuda_get_decode_schedule(void);

/* Dense decode: GpuEngine::attention / exact_hot_fused_attention
 * (src/gpu_llm/gpu_resources.rs:583-643,783-828) for a batch of sequences.
 * q: bf16 [n_seq][QH][D] (post-RoPE); k_cache/v_cache: bf16 token-major
 * [n_seq][max_tokens][KVH][D]; seq_tokens: device int32 [n_seq], each in
 * 0..=max_tokens; out: bf16 [n_seq][QH][D].  A sequence with 0 tokens gives
 * zeros.  workspace: >= mslim_cuda_decode_workspace_bytes, 16-byte aligned. */
int mslim_cuda_decode_dense(const mslim_geometry_t *geometry, const void *q, const void *k_cache,
                            const void *v_cache, const int32_t *seq_tokens, uint32_t n_seq,
                            uint32_t max_tokens, uint32_t split_tokens, void *workspace,
                            size_t workspace_bytes, void *out, void *stream);

/* Certified sparse decode (epsilon > 0): attention of one query per session
 * restricted to a certified set of token positions, the GPU side of the
 * micro-region path -- GpuEngine::micro_sparse_scores followed by the
 * ordinary softmax / PV (src/gpu_llm/gpu_resources.rs:656-729;
 * llm_micro_clear_scores + llm_micro_sparse_qk, assets/gpu_llm.cl:847-882:
 * every omitted score -inf) and GpuEngine::micro_hot_attention (:736-771,
 * llm_micro_hot_fused_attention, gpu_llm.cl:899-964: softmax over the
 * selected positions only).  The certificate that authorises the omission
 * (gpu_micro_regions.rs, attention_certificate.rs) stays with the host.
 * q: bf16 [n_seq][QH][D]; k_cache/v_cache: dense token-major
 * [n_seq][max_tokens][KVH][D]; seq_tokens: device int32 [n_seq] committed
 * lengths; selected: device int32 [n_seq][max_selected] positions, strictly
 * increasing, each below the session's committed length (the reference checks
 * this on the host before its upload, gpu_resources.rs:664-671,838-845; here a
 * violation is recorded in the device status word, reported as
 * MSLIM_ERR_SHAPE_MISMATCH by mslim_cuda_device_status, and that session's
 * output is unspecified); selected_counts: device int32 [n_seq], 0 gives zeros.
 * The selected K/V rows are gathered into the workspace and the split-KV
 * decode runs over them, so selecting every position gives the bits of
 * mslim_cuda_decode_dense with the same split_tokens.  workspace: 256-byte
 * aligned, >= mslim_cuda_decode_selected_workspace_bytes, zero-filled once
 * before its first use (calls leave its counter at zero). */
int mslim_cuda_decode_selected_workspace_bytes(const mslim_geometry_t *geometry, uint32_t n_seq,
                                               uint32_t max_selected, uint32_t split_tokens, size_t *bytes);
int mslim_cuda_decode_selected(const mslim_geometry_t *geometry, const void *q, const void *k_cache,
                               const void *v_cache, uint32_t max_tokens, const int32_t *seq_tokens,
                               const int32_t *selected, const int32_t *selected_counts, uint32_t max_selected,
                               uint32_t n_seq, uint32_t split_tokens, void *workspace, size_t workspace_bytes,
                               void *out, void *stream);

/* The same certified sparse decode over ColdStore-exact pages: the selected
 * rows are gathered straight out of the page pool (k_pool/v_pool bf16
 * [n_pages][KVH][page_tokens][D], page_table device int32
 * [n_seq][max_pages_per_seq]), so an epsilon > 0 decode needs no dense copy
 * of the cache (the reference's micro path reads its dense GPU caches,
 * src/gpu_llm/gpu_resources.rs:656-771).  Workspace and results as
 * mslim_cuda_decode_selected: selecting every position gives the bits of
 * mslim_cuda_decode_paged with the same split_tokens.  A page id outside the
 * pool is reported by mslim_cuda_device_status. */
int mslim_cuda_decode_selected_paged(const mslim_geometry_t *geometry, const void *q, const void *k_pool,
                                     const void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                     const int32_t *page_table, uint32_t max_pages_per_seq,
                                     const int32_t *seq_tokens, const int32_t *selected,
                                     const int32_t *selected_counts, uint32_t max_selected, uint32_t n_seq,
                                     uint32_t split_tokens, void *workspace, size_t workspace_bytes, void *out,
                                     void *stream);

/* Paged decode over ColdStore-exact pages: the device-resident replacement of
 * GpuEngine::attention_gpu_region (src/gpu_llm/gpu_resources.rs:883-1063),
 * which staged V from the ColdStore through the host.  k_pool/v_pool: bf16
 * [n_pages][KVH][page_tokens][D]; page_table: device int32
 * [n_seq][max_pages_per_seq] of physical page ids; seq_tokens: device int32
 * [n_seq].  page_tokens must be a multiple of 64.  A session of L tokens is
 * decoded as ceil(L / split_tokens) splits of equal length (rounded up to 64
 * tokens), whose partials are combined in order.  Results are bit-identical
 * to mslim_cuda_decode_dense on the same K/V bytes.  A table entry outside
 * [0, n_pages) is not loaded; it is reported by mslim_cuda_device_status and
 * the output rows of its session are undefined (other sessions are
 * unaffected). */
int mslim_cuda_decode_paged(const mslim_geometry_t *geometry, const void *q, const void *k_pool,
                            const void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                            const int32_t *page_table, uint32_t max_pages_per_seq,
                            const int32_t *seq_tokens, uint32_t n_seq, uint32_t split_tokens,
                            void *workspace, size_t workspace_bytes, void *out, void *stream);

/* Paged decode that allocates nothing and takes no workspace.  No counterpart
 * in the reference: it is for callers that cannot allocate device memory --
 * a serving loop that must never hit the implicit device synchronisation of
 * cudaMalloc/cudaFree, or a host (e.g. a Rust FFI caller) that holds only the
 * K/V, page-table and output pointers and has no device allocator bound.
 * Same arguments and results as mslim_cuda_decode_paged minus the workspace;
 * with the same split_tokens the output is bit-identical to it.
 * The split partials live in a library-owned static device array of
 * MSLIM_STATIC_SCRATCH_BYTES (16 MiB, a fixed limit of this library), held by
 * every GPU that loads the library until the process exits.  A request whose partials exceed it fails with
 * MSLIM_ERR_SHAPE_MISMATCH; split_tokens == 0 picks the library's split size
 * and, if needed, larger splits until the partials fit.  The first call on a
 * device looks up the array's device address (no allocation); make that first
 * call before any stream capture.  That address is kept for the life of the
 * process, so the library must not be used on a device after
 * cudaDeviceReset (or any other teardown of its primary context).  Every
 * call shares the one array and finds the previous call's contents there;
 * each call first clears the array's head of work counters on its stream
 * (a memset, no allocation).  Calls that can overlap on the GPU (different
 * streams, no ordering) race on it. */
#define MSLIM_STATIC_SCRATCH_BYTES (16u << 20)
int mslim_cuda_decode_paged_static_scratch(const mslim_geometry_t *geometry, const void *q,
                                           const void *k_pool, const void *v_pool,
                                           uint32_t n_pages, uint32_t page_tokens,
                                           const int32_t *page_table, uint32_t max_pages_per_seq,
                                           const int32_t *seq_tokens, uint32_t n_seq,
                                           uint32_t split_tokens, void *out, void *stream);

/* ------------------------------------------------ prefill attention -- */

/* BatchKernels::attention (src/gpu_llm/prefill.rs:363-435): chunked causal
 * prefill, tcgen05/TMEM tensor cores.  q/out: bf16 [queries][QH][D];
 * k/v: bf16 token-major [prior+queries][KVH][D].  head_dim 64..256, a
 * multiple of 8, any GQA group (the kernels run at 64, 128 or 256; a head_dim
 * between runs zero-padded on the chip); other shapes return
 * MSLIM_ERR_INVALID_GEOMETRY (mslim_cuda_plan_run serves them). */
int mslim_cuda_prefill_causal(const mslim_geometry_t *geometry, const void *q, const void *k,
                              const void *v, void *out, uint32_t queries, uint32_t prior,
                              void *stream);

/* Logical K/V serialisation of one session and layer, for the validation
 * digest `logical_kv_sha256` (GpuLlm::logical_kv_sha256,
 * src/gpu_llm/mod.rs:1981-2023, dense caches; GpuRegionStore::logical_kv_sha256,
 * src/gpu_region_store.rs:338-371, ColdStore pages; both hash
 * "mslim-dense-kv-state-v1", the token count as u64 LE, then per layer K and
 * V, each ordered [kv_heads][tokens][head_dim]).  These write one such
 * tensor, out: bf16 [kv_heads][tokens][head_dim] on the device, from
 *   dense: cache = one session's token-major rows [>= tokens][kv_heads][head_dim];
 *   paged: pool [n_pages][kv_heads][page_tokens][head_dim] (the ColdStore-exact
 *          page layout) and page_row = the session's device page table row
 *          (logical page -> physical page, max_pages entries), i.e. the
 *          GpuRegionStore::read_keys / read_values gather
 *          (src/gpu_region_store.rs:828-931) in head-major order.
 * The host hashes the stream (the reference does the same after its
 * read-back).  A page id outside the pool leaves its rows unwritten and is
 * reported by mslim_cuda_device_status. */
int mslim_cuda_kv_canonical_dense(const void *cache, uint32_t kv_heads, uint32_t head_dim, uint32_t tokens,
                                  void *out, void *stream);
int mslim_cuda_kv_canonical_paged(const void *pool, uint32_t n_pages, uint32_t kv_heads, uint32_t page_tokens,
                                  uint32_t head_dim, const int32_t *page_row, uint32_t max_pages,
                                  uint32_t tokens, void *out, void *stream);

/* ColdStore page sealing from device pages: the per-token FNV-1a 64 hashes of
 * a page record (src/cold_store.rs:725-742 token_hashes; computed by the
 * writer in GpuRegionStore::append_batch, src/gpu_region_store.rs:391-522)
 * taken directly from the device page pool that the appends fill, so the host
 * receives head-major pages and their hashes with no transpose.
 * pool: bf16 [n_pool_pages][kv_heads][page_tokens][head_dim] (K or V);
 * page_ids: device int32 [n_pages]; hashes: device uint64 [n_pages][tokens],
 * tokens <= page_tokens (a partly filled page hashes like its compact record).
 * A page id outside the pool yields 0 hashes and is reported by
 * mslim_cuda_device_status.  The record's whole-payload checksums are
 * sequential FNV over each payload and stay with the host writer. */
int mslim_cuda_page_token_hashes(const void *pool, uint32_t n_pool_pages, uint32_t kv_heads,
                                 uint32_t page_tokens, uint32_t head_dim, const int32_t *page_ids,
                                 uint32_t n_pages, uint32_t tokens, uint64_t *hashes, void *stream);

/* ------------------------------------------------- layer elementwise -- */

/* GpuEngine::add (src/gpu_llm/gpu_resources.rs:539-559, kernel llm_add) and the
 * CPU add_residual (src/native_cpu_adapter.rs:186-191): out = bf16(a + b),
 * n bf16 elements; out may alias a or b. */
int mslim_cuda_residual_add(const void *a, const void *b, void *out, uint64_t n, void *stream);

/* GpuEngine::swiglu (src/gpu_llm/gpu_resources.rs:561-581, kernel llm_swiglu)
 * and the CPU MLP (src/native_cpu_adapter.rs:553-560):
 * out = bf16(bf16(g / (1 + exp(-g))) * u); out may alias gate or up. */
int mslim_cuda_swiglu(const void *gate, const void *up, void *out, uint64_t n, void *stream);

/* A projection of the decode step (GpuEngine's GEMVs, llm_gemv_bf16*,
 * assets/gpu_llm.cl:38-68, for a few sessions at once) on the tcgen05 tensor
 * cores: y[r][n] = bf16(sum_k x[r][k] * w[n][k]) for r < m, fp32
 * accumulation, every weight byte read once.  x: bf16 [m][k], w: bf16 [n][k]
 * (the HF [out][in] layout), both 16-byte aligned; y: bf16 rows of ldy >= n
 * elements; 1 <= m <= 16, k a multiple of 8.  Long K is cut into up to eight
 * splits combined in a fixed order on the chip (no workspace), so repeated
 * calls return the same bits.  The kernel starts streaming w before the
 * preceding kernel in the stream has finished (programmatic dependent
 * launch): w must not be written by that kernel. */
int mslim_cuda_gemv(const void *x, const void *w, void *y, uint32_t m, uint32_t n, uint32_t k, uint32_t ldy,
                    void *stream);

/* A SwiGLU MLP's gate and up projections and the activation in one launch
 * (llm_prefill_fused_swiglu_reuse8, assets/gpu_llm.cl:1323-1337, which fuses
 * the gate/up GEMVs with llm_swiglu the same way):
 * out[r][i] = bf16(bf16(g / (1 + exp(-g))) * u), g and u the bf16-rounded
 * projections of x[r] on feature i's gate and up weight rows.  w_gu: bf16
 * [2 * width][k], gate and up rows interleaved in blocks of 64 -- rows
 * 128b .. 128b+63 are the gate rows of features 64b .. 64b+63, rows
 * 128b+64 .. 128b+127 their up rows; width a multiple of 64; out bf16 rows of
 * ldo >= width elements; x, m, k, alignment and streaming as mslim_cuda_gemv.
 * The same bits as mslim_cuda_gemv over w_gu into y [m][2 * width] followed by
 * mslim_cuda_swiglu_rows(y, out, m * width / 64, 64) (each 128-wide block of y
 * read as one [gate 64 | up 64] row), without writing y. */
int mslim_cuda_gemv_swiglu(const void *x, const void *w_gu, void *out, uint32_t m, uint32_t width, uint32_t k,
                           uint32_t ldo, void *stream);

/* SwiGLU over a fused gate|up projection (no reference counterpart: the
 * reference keeps gate and up in separate buffers, GpuEngine::swiglu):
 * gate_up bf16 [rows][gate (width) | up (width)], out bf16 [rows][width],
 * out = bf16(bf16(g / (1 + exp(-g))) * u); width a multiple of 8. */
int mslim_cuda_swiglu_rows(const void *gate_up, void *out, uint32_t rows, uint32_t width, void *stream);

/* GpuEngine::argmax (src/gpu_llm/gpu_resources.rs:1065, kernel llm_argmax) and
 * the CPU greedy step (src/native_cpu_adapter.rs:582-587): one int32 token id
 * per row of `rows` x `vocab` bf16 logits (device pointers).
 * ties_to_last = 1: f32::total_cmp order, last index among equal maxima (the
 * CPU path's Iterator::max_by, the parity reference); 0: float order, first
 * index among equals, NaN never preferred (the OpenCL kernel). */
int mslim_cuda_argmax(const void *logits, uint32_t rows, uint32_t vocab, int ties_to_last,
                      int32_t *token_ids, void *stream);

/* Diagnostic of the prefill softmax's exponentials, no reference counterpart:
 * for device f32 arrays of n values, y_poly = the FMA-pipe polynomial 2^x the
 * prefill kernels evaluate for one pair in eight, y_mufu = the MUFU ex2.approx
 * they use for the rest, y_ref = CUDA's exp2f.  Lets a test measure the
 * polynomial's stated error bound on the device. */
int mslim_cuda_exp2_eval(const float *x, float *y_poly, float *y_mufu, float *y_ref, uint32_t n,
                         void *stream);

/* ------------------------------------------- tensor-parallel decode -- */

/* Communicator of one rank of a tensor-parallel group (at most 8 ranks, one
 * GPU each), built once by the host: every rank allocates its regions with
 * mslim_cuda_tp_alloc, exports them with mslim_cuda_ipc_handle, and maps the
 * peers' with mslim_cuda_ipc_open (handles travel over any host channel).
 *   data[r]:  rank r's bf16 [2][max_rows][hidden] partial-sum slots;
 *   flags[r]: rank r's uint32 [max_rows][8] ready counters (zeroed);
 *   epoch:    this rank's uint32 [max_rows] call counters (zeroed).
 * No reference counterpart: the reference runs on one iGPU; the north star's
 * KV-head tensor parallelism needs the per-layer reduction. */
typedef struct {
    uint32_t world, rank, max_rows, hidden;
    void *data[8];
    void *flags[8];
    void *epoch;
} mslim_tp_comm_t;

int mslim_cuda_tp_alloc(size_t bytes, void **ptr);   /* zero-filled device memory */
int mslim_cuda_tp_free(void *ptr);
int mslim_cuda_ipc_handle(const void *ptr, void *handle /* 64 bytes */);
int mslim_cuda_ipc_open(const void *handle /* 64 bytes */, void **ptr);
int mslim_cuda_ipc_close(void *ptr);

/* The collective after a row-parallel projection of the decode step, fused
 * with what run_layer does next (residual add, RMSNorm): for rows [0, rows),
 * x = bf16(x + bf16(sum over ranks r of data[r][slot][row])) and
 * y = RMSNorm(x, w), every rank computing identical bits (fp32 sum in rank
 * order).  The caller writes its own partial into data[rank][slot] first and
 * alternates slot 0/1 from call to call.  Waits on peers are bounded; a rank
 * that never arrives is reported by mslim_cuda_device_status and leaves x, y
 * untouched. */
int mslim_cuda_tp_allreduce_rmsnorm(const mslim_tp_comm_t *comm, uint32_t slot, void *x, const void *w,
                                    void *y, uint32_t rows, float eps, void *stream);

/* ------------------------------------------------------ prologue -- */

/* GpuEngine::norm / BatchKernels::norm (src/gpu_llm/gpu_resources.rs:485-507,
 * src/gpu_llm/prefill.rs:292-320): per token y = bf16(bf16(x*s)*w),
 * s = 1/sqrt(mean(x^2)+eps).  x/y: bf16 [tokens][hidden]; w: bf16 [hidden]. */
int mslim_cuda_rmsnorm(const void *x, const void *w, void *y, uint32_t tokens, uint32_t hidden,
                       float eps, void *stream);

/* The layer's residual add followed by the next RMSNorm in one pass (the pair
 * GpuEngine::add + GpuEngine::norm of run_layer, src/gpu_llm/mod.rs:2118-2329):
 * x = bf16(x + delta) in place, then y = RMSNorm(x, w) exactly as
 * mslim_cuda_rmsnorm computes it.  y must not alias x or delta. */
int mslim_cuda_residual_rmsnorm(void *x, const void *delta, const void *w, void *y, uint32_t tokens,
                                uint32_t hidden, float eps, void *stream);

/* GpuEngine::rope / BatchKernels::rope (src/gpu_llm/gpu_resources.rs:509-537,
 * src/gpu_llm/prefill.rs:322-361): rotate_half RoPE of bf16
 * [tokens][heads][head_dim], row t at position start_position+t. */
int mslim_cuda_rope(const void *in, void *out, uint32_t tokens, uint32_t heads, uint32_t head_dim,
                    uint32_t start_position, const mslim_rope_config_t *rope, void *stream);

/* RoPE of new q/k rows fused with the K/V append into ColdStore-exact pages:
 * replaces rope(q), rope(k) + the K/V copies of run_layer
 * (src/gpu_llm/mod.rs:2099-2116) and the host transpose of
 * GpuRegionStore::append_batch (src/gpu_region_store.rs:470-483).
 * q_in/q_out: bf16 [tokens][QH][D]; k_in/v_in: bf16 [tokens][KVH][D]; row t is
 * token position start_position+t of one sequence whose page ids are
 * page_table[0..]. */
int mslim_cuda_rope_append_paged(const mslim_geometry_t *geometry, const void *q_in, void *q_out,
                                 const void *k_in, const void *v_in, uint32_t tokens,
                                 uint32_t start_position, const mslim_rope_config_t *rope,
                                 void *k_pool, void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                 const int32_t *page_table, uint32_t max_pages, void *stream);

/* Decode-step form of the fused append for a batch of sessions, one new token
 * each: session s appends its token at position positions[s] (device int32,
 * usually its current length) into the pages page_table[s][..].  Replaces, per
 * session, rope(q) + rope(k) + the K/V copies of run_layer
 * (src/gpu_llm/mod.rs:2099-2116).  q_in/q_out: bf16 [n_seq][QH][D];
 * k_in/v_in: bf16 [n_seq][KVH][D].  A position beyond the page table or a page
 * id outside the pool writes nothing and is reported by
 * mslim_cuda_device_status. */
int mslim_cuda_rope_append_decode_paged(const mslim_geometry_t *geometry, const void *q_in,
                                        void *q_out, const void *k_in, const void *v_in,
                                        const int32_t *positions, uint32_t n_seq,
                                        const mslim_rope_config_t *rope, void *k_pool,
                                        void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                        const int32_t *page_table, uint32_t max_pages,
                                        void *stream);

/* The same decode step for the dense token-major caches of the GPU runtime
 * (k_cache/v_cache: bf16 [n_seq][max_tokens][KVH][D]): rope(q), rope(k) and
 * the K/V copies of run_layer (src/gpu_llm/mod.rs:2099-2116) for a batch of
 * sessions, session s writing row positions[s].  Same RoPE arithmetic as every
 * other form, so a dense and a paged store hold identical K bits.  A position
 * outside [0, max_tokens) writes nothing and is reported by
 * mslim_cuda_device_status. */
int mslim_cuda_rope_append_decode_dense(const mslim_geometry_t *geometry, const void *q_in,
                                        void *q_out, const void *k_in, const void *v_in,
                                        const int32_t *positions, uint32_t n_seq,
                                        const mslim_rope_config_t *rope, void *k_cache,
                                        void *v_cache, uint32_t max_tokens, void *stream);

/* The two decode-step appends reading q, k and v straight out of one fused
 * projection output qkv: bf16 [n_seq][(QH + 2*KVH) * D] holding the q heads,
 * then the k heads, then the v heads of each session's new token (the
 * reference projects them into three buffers; the fused GEMM saves two
 * launches and the copies).  Otherwise as the forms above. */
int mslim_cuda_rope_append_decode_dense_qkv(const mslim_geometry_t *geometry, const void *qkv,
                                            void *q_out, const int32_t *positions, uint32_t n_seq,
                                            const mslim_rope_config_t *rope, void *k_cache,
                                            void *v_cache, uint32_t max_tokens, void *stream);
int mslim_cuda_rope_append_decode_paged_qkv(const mslim_geometry_t *geometry, const void *qkv,
                                            void *q_out, const int32_t *positions, uint32_t n_seq,
                                            const mslim_rope_config_t *rope, void *k_pool, void *v_pool,
                                            uint32_t n_pages, uint32_t page_tokens,
                                            const int32_t *page_table, uint32_t max_pages, void *stream);

/* The decode step's q|k|v projection with RoPE and the K/V append in its
 * epilogue (the reference's run_layer projects q, k and v, rotates q and k
 * and appends k and v, src/gpu_llm/mod.rs:2090-2125; its opt-in
 * llm_prefill_fused_qkv_reuse8, assets/gpu_llm.cl:1253, fuses the three
 * projections the same way, without the rotation): x bf16
 * [n_seq][k] (1 <= n_seq <= 16, k a multiple of 8, 16-byte aligned), w_qkv
 * bf16 [(query_heads + 2 kv_heads) * 128][k] (q, k, v weight rows, 16-byte
 * aligned); head_dim must be 128 (else MSLIM_ERR_INVALID_GEOMETRY).  The same
 * bits as mslim_cuda_gemv into qkv [n_seq][(QH + 2 KVH) * 128] followed by
 * mslim_cuda_rope_append_decode_{dense,paged}_qkv with the same arguments,
 * including their handling of a position or page id outside the store (that
 * row is not written; mslim_cuda_device_status reports it), without writing
 * or re-reading qkv.  Like mslim_cuda_gemv it starts streaming w_qkv before
 * the preceding kernel in the stream has finished. */
int mslim_cuda_gemv_qkv_rope_append_dense(const mslim_geometry_t *geometry, const void *x, const void *w_qkv,
                                          uint32_t k, const int32_t *positions, uint32_t n_seq,
                                          const mslim_rope_config_t *rope, void *q_out, void *k_cache,
                                          void *v_cache, uint32_t max_tokens, void *stream);
int mslim_cuda_gemv_qkv_rope_append_paged(const mslim_geometry_t *geometry, const void *x, const void *w_qkv,
                                          uint32_t k, const int32_t *positions, uint32_t n_seq,
                                          const mslim_rope_config_t *rope, void *q_out, void *k_pool,
                                          void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                          const int32_t *page_table, uint32_t max_pages, void *stream);

/* ------------------------------------------- isolated backend (L3) -- */

typedef struct mslim_backend mslim_backend_t;

/* GpuBackend::new (src/gpu_backend.rs:56-140): selects `device` (it must be
 * an sm_100 GPU, else MSLIM_ERR_UNSUPPORTED_DEVICE) and creates the backend's
 * stream.  Device buffers are grown on demand and reused across calls. */
int mslim_cuda_backend_create(int device, mslim_backend_t **backend);
void mslim_cuda_backend_destroy(mslim_backend_t *backend);

/* AttentionBackend::decode as GpuBackend implements it
 * (src/gpu_backend.rs:149-377): host query f32 [QH*D] (any finite f32; it is
 * carried as a bf16 hi + lo pair), host K/V frames concatenated token-major
 * [tokens][KVH][D] of dtype 1 = bf16, 2 = f16 or 3 = f32, host output
 * f32 [QH*D].  The kernels read bf16: f16/f32 frames whose values are all
 * exact bf16 values are carried bit for bit; otherwise each value becomes a
 * bf16 hi + lo pair laid side by side along the head dimension (kernel
 * head_dim 2*D, so D <= 128 there, else MSLIM_ERR_UNSUPPORTED_DEVICE) with
 * the query duplicated, and the two output halves are added on the host.
 * Uploads, runs the dense decode, reads back and synchronises, like the
 * reference's blocking dispatch.  tokens == 0 gives zeros; a non-finite
 * query, frame value or output gives MSLIM_ERR_NON_FINITE. */
int mslim_cuda_backend_decode(mslim_backend_t *backend, const mslim_geometry_t *geometry,
                              const float *query_host, const void *keys_host,
                              const void *values_host, int dtype, uint32_t tokens,
                              float *out_host);

/* GpuBackend::last_timings (src/gpu_backend.rs:142-147, GpuTimings :34-44)
 * as JSON: dispatch_ms, kernel_ms, input_kv_bytes, scratch_bytes,
 * output_bytes. */
int mslim_cuda_backend_last_timings(const mslim_backend_t *backend, char *out, size_t len);

/* Library version string (for diagnostics). */
const char *mslim_cuda_version(void);

/* Hex SHA-256 of the sources this library was built from (every CUDA source,
 * device header, this header and the build recipe, each hashed as its length
 * u64 LE then its bytes, then the target architecture flags).  The reference's
 * calibration profile identity, implementation_digest
 * (src/calibration_profile.rs:90-125), hashes its kernel sources
 * (assets/gpu_llm.cl, assets/tiled_attention.cl, src/gpu_llm/...) the same
 * way; with this library in their place it folds this string in instead, so a
 * profile recorded against one build of the kernels is not reused with
 * another.  "unknown" when built without the recipe. */
const char *mslim_cuda_implementation_digest(void);

#ifdef __cplusplus
}
#endif
#endif /* MSLIM_CUDA_H */
