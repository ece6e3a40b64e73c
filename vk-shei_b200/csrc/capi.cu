// capi.cu -- the extern "C" boundary (include/mslim_cuda.h).
//
// Host-side validation mirrors the reference's checks before every dispatch
// (src/portable.rs:421-443, src/attention_kernel.rs:43-138,
// src/gpu_llm/tiled_attention.rs:161-235, src/gpu_backend.rs:149-207); the
// error convention is an int status plus a thread-local message
// (native/hipblaslt_bridge.cpp:25-38,155-160).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <queue>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/mslim_cuda.h"
#include "decode.cuh"
#include "prefill.cuh"
#include "layer_ops.cuh"
#include "gemv.cuh"
#include "tp_allreduce.cuh"
#include "prologue.cuh"

// One status word per device; kernels record bounded-wait timeouts here.
__device__ int g_mslim_status_word;

// Split partials of mslim_cuda_decode_paged_static_scratch: a fixed device
// array, so that entry point never allocates.  Its contents persist between
// calls.  Every partial the merge reads is written by the split kernel of the
// same call first; only the head of work counters has to start at zero, and
// the entry point clears it on its stream before each call (so a call that
// gave up on a bounded wait cannot leave the next one a stale count).
static __device__ __align__(256) float g_static_decode_scratch[MSLIM_STATIC_SCRATCH_BYTES / sizeof(float)];

namespace {
std::atomic<uint64_t> g_kernel_launches{0};
std::atomic<int> g_decode_schedule{MSLIM_DECODE_SPLIT_MERGE};
}  // namespace

void mslim::note_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t err, const char *what) {
    return fail(MSLIM_ERR_BACKEND_FAILURE, "%s: %s", what, cudaGetErrorString(err));
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

constexpr int kMaxDevices = 64;
std::mutex g_dev_mutex;
int *g_status_ptr[kMaxDevices] = {};
int g_dev_checked[kMaxDevices] = {};  // 0 unknown, 1 sm_100, -1 other

// Current device, checked to be sm_100 (B200) once.
int current_device(int *dev) {
    cudaError_t err = cudaGetDevice(dev);
    if (err != cudaSuccess) return cuda_fail(err, "no CUDA device");
    if (*dev < 0 || *dev >= kMaxDevices) return fail(MSLIM_ERR_UNSUPPORTED_DEVICE, "device index %d", *dev);
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (g_dev_checked[*dev] == 0) {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, *dev);
        g_dev_checked[*dev] = (major == 10 && minor == 0) ? 1 : -1;
        if (g_dev_checked[*dev] < 0) {
            return fail(MSLIM_ERR_UNSUPPORTED_DEVICE,
                        "no native kernel registered for compute capability %d.%d (needs sm_100)",
                        major, minor);
        }
    }
    if (g_dev_checked[*dev] < 0)
        return fail(MSLIM_ERR_UNSUPPORTED_DEVICE, "no native kernel registered for this device");
    return MSLIM_OK;
}

int *status_ptr(int dev) {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (!g_status_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_mslim_status_word) == cudaSuccess)
            g_status_ptr[dev] = static_cast<int *>(p);
    }
    return g_status_ptr[dev];
}

// Device address of g_static_decode_scratch, looked up once per device with
// that device current (host code may not take the address of a __device__
// array directly: that would be a host-side stand-in, not device memory).
// Like g_status_ptr it is kept for the life of the process; the C ABI states
// that the library is not used on a device after a reset of its context.
void *g_static_scratch_ptr[kMaxDevices] = {};

int static_scratch_ptr(int dev, void **ptr) {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (!g_static_scratch_ptr[dev]) {
        void *p = nullptr;
        cudaError_t err = cudaGetSymbolAddress(&p, g_static_decode_scratch);
        if (err != cudaSuccess || !p)
            return fail(MSLIM_ERR_BACKEND_FAILURE, "static scratch address lookup failed: %s",
                        cudaGetErrorString(err));
        g_static_scratch_ptr[dev] = p;
    }
    *ptr = g_static_scratch_ptr[dev];
    return MSLIM_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// bf16 tensor map with 128-byte swizzle; dims[0] innermost.
int make_tmap(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
              const uint64_t *strides_bytes, const uint32_t *box) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(MSLIM_ERR_BACKEND_FAILURE, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t gdim[5], gstr[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        gdim[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) gstr[i] = strides_bytes[i];
    }
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void *>(base), gdim,
                    gstr, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MSLIM_ERR_BACKEND_FAILURE, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return MSLIM_OK;
}

int check_geometry(const mslim_geometry_t *g) {
    if (!g) return fail(MSLIM_ERR_INVALID_GEOMETRY, "geometry is null");
    const uint64_t qh = g->query_heads, kvh = g->kv_heads, d = g->head_dim;
    if (qh == 0 || kvh == 0 || d == 0 || qh % kvh != 0 || qh * d > 0xffffffffull ||
        kvh * d > 0xffffffffull)
        return fail(MSLIM_ERR_INVALID_GEOMETRY,
                    "heads and dimension must be positive, q_heads divisible by kv_heads, "
                    "products finite");
    return MSLIM_OK;
}

bool kernel_head_dim(uint32_t d) { return d >= 8 && d <= 256 && d % 8 == 0; }

// ------------------------------------------------------ decode plumbing --

struct DecodeShapeInfo {
    int group, head_chunks, heads_per_cta, q_per_cta, q_blocks;
};

int decode_shape(const mslim_geometry_t *g, uint32_t nq, DecodeShapeInfo *s) {
    s->group = (int)(g->query_heads / g->kv_heads);
    if (s->group <= 16) {
        s->heads_per_cta = s->group;
        s->head_chunks = 1;
    } else if (s->group % 16 == 0) {
        s->heads_per_cta = 16;
        s->head_chunks = s->group / 16;
    } else {
        return fail(MSLIM_ERR_INVALID_GEOMETRY,
                    "query heads per KV head above 16 must be a multiple of 16 (got %d)", s->group);
    }
    s->q_per_cta = std::max(1, std::min<int>((int)nq, 16 / s->heads_per_cta));
    s->q_blocks = (int)((nq + s->q_per_cta - 1) / s->q_per_cta);
    return MSLIM_OK;
}

// Step time of the split kernel with split size `st`, in token-times of one CTA
// streaming at its share of HBM under full load.  CTAs start in grid order
// (split fastest, then KV-head chunk, then session) as the `slots` resident
// places free up.  While n CTAs run, each streams at min(cap, slots / n)
// times its full-load rate: HBM is shared, and a CTA is also limited by its
// own pipeline.  `cap` is fitted to measured split sweeps of the kernel on
// B200 (see the two policies below).  A CTA costs its tokens plus kFixed
// (filling its pipeline, combining its warps); a CTA past its session's splits
// exits at once (kExit).  Every running CTA receives the same service, so the
// next one to finish is the one with the least service left: a heap of
// completion levels, O(CTAs log slots).
double fluid_step_time(const int32_t *lengths, uint32_t n_seq, uint64_t per_seq, uint64_t slots, uint32_t st,
                       double cap) {
    constexpr double kFixed = 300.0, kExit = 8.0;
    const double kCap = cap;
    uint64_t max_splits = 1;
    for (uint32_t i = 0; i < n_seq; ++i)
        if (lengths[i] > 0) max_splits = std::max<uint64_t>(max_splits, ((uint64_t)lengths[i] + st - 1) / st);
    std::priority_queue<double, std::vector<double>, std::greater<double>> running;  // completion levels
    double level = 0.0, t = 0.0;
    auto finish = [&]() {  // advance to the next completion
        const double n = (double)running.size();
        const double rate = std::min(kCap, (double)slots / n);
        t += (running.top() - level) / rate;
        level = running.top();
        running.pop();
    };
    for (uint32_t i = 0; i < n_seq; ++i) {
        const uint64_t L = lengths[i] > 0 ? (uint64_t)lengths[i] : 0;
        const uint64_t n = L ? (L + st - 1) / st : 0;
        const uint64_t slen = n ? ((L + n - 1) / n + 63) / 64 * 64 : 0;
        for (uint64_t h = 0; h < per_seq; ++h)
            for (uint64_t k = 0; k < max_splits; ++k) {
                const double work = k < n ? (double)std::min<uint64_t>(slen, L - k * slen) + kFixed : kExit;
                if (running.size() == slots) finish();
                running.push(level + work);
            }
    }
    while (!running.empty()) finish();
    return t;
}

// Resident split CTAs per GPU: shared memory allows three per SM at head_dim
// 64, two at 128 and one at 256 (the kernel's stage rings).
uint64_t decode_slots(uint32_t kernel_dim) { return 148ull * (kernel_dim <= 64 ? 3 : kernel_dim <= 128 ? 2 : 1); }

// Split sizes the policies choose from, longest first: the sizes the model was
// checked against on the C4 shards of 1, 2, 4 and 8 GPUs (its choice within
// 2 % of the best measured; sizes in between can land the last wave badly),
// then shorter ones for small batches, where more CTAs than items pay.
constexpr uint32_t kSplitCandidates[] = {3072, 2688, 2048, 1536, 1024, 768, 512, 256};
// A split that needs more than this many waves of CTAs is not modelled: its
// per-CTA costs outweigh any tail it could balance (and the model's heap would
// grow with the CTA count).  The longest candidate is always modelled.
constexpr uint64_t kPolicyMaxWaves = 16;

// Per-CTA speed-up cap of the model, fitted per policy to sweeps of every
// candidate split on one B200 (the policy's pick against the fastest measured):
// sessions of varied lengths (the C4 draw and its LPT shards of 2, 4 and 8
// GPUs; CTAs that finish early leave their HBM share to the long ones) fit
// 2.5, within 2.2 % of the fastest on every shard; equal lengths (the policy
// without host lengths assumes every session at max_tokens; every CTA of a
// wave starts and ends together, so a part-filled wave cannot speed up) fit
// 1.0, within 1.2 % of the fastest on 14 shapes from 1 session of 128 K
// tokens to 64 of 1 K, head_dim 64 to 256, GQA groups 4 to 32.
constexpr double kCapVariedLengths = 2.5;
constexpr double kCapEqualLengths = 1.0;

// The candidate with the shortest modelled step (the longer split when two are
// within 0.5 %), at most the longest sequence rounded up to the 64-token stage
// and at least 256 tokens.  `lengths` holds n_seq sequences, each with per_seq
// (KV-head chunk) items.
uint32_t choose_split(const int32_t *lengths, uint32_t n_seq, uint64_t per_seq, uint64_t slots, double cap) {
    uint64_t longest = 0;
    for (uint32_t i = 0; i < n_seq; ++i) longest = std::max<uint64_t>(longest, lengths[i] > 0 ? (uint64_t)lengths[i] : 0);
    const uint64_t limit = std::max<uint64_t>(256, (longest + 63) / 64 * 64);
    // Past kPolicyMaxWaves waves at the longest candidate every shorter one is
    // pruned too, so the model's answer is the longest: skip the simulation
    // (whose cost grows with the CTA count).
    const uint64_t longest_grid =
        (uint64_t)n_seq * per_seq * std::max<uint64_t>(1, (longest + kSplitCandidates[0] - 1) / kSplitCandidates[0]);
    if (longest_grid > kPolicyMaxWaves * slots) return (uint32_t)std::min<uint64_t>(kSplitCandidates[0], limit);
    double best = 0.0;
    uint32_t best_st = kSplitCandidates[0];
    for (uint32_t st : kSplitCandidates) {
        const uint64_t grid = (uint64_t)n_seq * per_seq * std::max<uint64_t>(1, (longest + st - 1) / st);
        if (st != kSplitCandidates[0] && grid > kPolicyMaxWaves * slots) continue;
        const double t = fluid_step_time(lengths, n_seq, per_seq, slots, st, cap);
        if (best == 0.0 || t < best * 0.995) {
            best = t;
            best_st = st;
        }
    }
    return (uint32_t)std::min<uint64_t>(best_st, limit);
}

// Split policy when only the longest sequence is known (lengths on the
// device): the same model with every one of the work_items (sequence x query
// block, KV-head chunk) items at max_tokens, and the equal-lengths cap.
// Remembered per shape, so a decode loop pays for the model once.
uint32_t policy_split_tokens(uint64_t work_items, uint64_t max_tokens, uint64_t slots) {
    static std::mutex mu;
    static std::map<std::tuple<uint64_t, uint64_t, uint64_t>, uint32_t> memo;
    const int32_t len = (int32_t)std::min<uint64_t>(max_tokens, 0x7fffffffu);
    const auto key = std::make_tuple(work_items, (uint64_t)len, slots);
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = memo.find(key);
        if (it != memo.end()) return it->second;
    }
    // uniform lengths: one sequence of work_items items walks the same CTAs
    const uint32_t st = choose_split(&len, 1, work_items, slots, kCapEqualLengths);
    std::lock_guard<std::mutex> lock(mu);
    if (memo.size() >= 4096) memo.clear();
    memo.emplace(key, st);
    return st;
}

// The kernel runs at the next head_dim in {64, 128, 256}; the caller's
// head_dim must be a multiple of 8 (16-byte TMA row strides) and at most 256.
uint32_t kernel_dim_for(uint32_t d) { return d <= 64 ? 64 : d <= 128 ? 128 : 256; }

// Decode workspace: a head of counters for the persistent split kernel (the
// work counter and its CTAs-done counter, then one arrival counter per
// (sequence x query block, KV-head chunk) item, at most kMaxDecodeItems;
// zero before the first call, left zero by every call), then the split
// partials.
constexpr uint64_t kMaxDecodeItems = 16384;
constexpr uint64_t kDecodeCounterBytes = 256 + 4 * kMaxDecodeItems;

uint64_t partial_bytes(const mslim_geometry_t *g, uint64_t n_seq, uint64_t nq, uint64_t splits) {
    // split partials {acc[D], m, l, 2 pad} (D + 4 floats: 16-byte records)
    return kDecodeCounterBytes + n_seq * nq * g->query_heads * splits * (kernel_dim_for(g->head_dim) + 4) * sizeof(float);
}

struct DecodeCall {
    const mslim_geometry_t *g;
    const void *q;
    const float *q_f32;
    const void *k;
    const void *v;
    bool paged;
    uint32_t n_pages, page_tokens;
    const int32_t *page_table;
    uint32_t max_pages;
    const int32_t *seq_tokens;
    int fixed_tokens;
    uint32_t n_seq, nq, max_tokens;
    uint32_t split_tokens;
    void *workspace;
    size_t workspace_bytes;
    void *out;
    float *out_f32;
    float scale_log2;
    uint32_t kernel_dim;  // head_dim the kernel runs at (>= g->head_dim)
    cudaStream_t stream;
};

int run_decode(const DecodeCall &c) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    const mslim_geometry_t *g = c.g;
    const uint32_t D = c.kernel_dim;
    DecodeShapeInfo sh;
    if (int rc = decode_shape(g, c.nq, &sh)) return rc;
    if (c.split_tokens == 0 || c.split_tokens % 64 != 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "split_tokens must be a positive multiple of 64");
    const uint64_t max_splits = (c.max_tokens + c.split_tokens - 1) / c.split_tokens;
    if (max_splits == 0 || max_splits > 0x7fffffff)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "split count out of range");
    const uint64_t need = partial_bytes(g, c.n_seq, c.nq, max_splits);
    if (c.workspace_bytes < need || !c.workspace)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "workspace holds %zu bytes, needs %llu",
                    c.workspace_bytes, (unsigned long long)need);
    if ((uint64_t)g->kv_heads * sh.head_chunks > 65535 || (uint64_t)c.n_seq * sh.q_blocks > 65535)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "launch grid exceeds 65535 along y or z");
    if (!aligned(c.k, 16) || !aligned(c.v, 16) || !aligned(c.workspace, 16) ||
        (c.q && !aligned(c.q, 4)) || (c.q_f32 && !aligned(c.q_f32, 8)) || !aligned(c.out, 4))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "K/V/workspace must be 16-byte aligned, Q/out 4-byte");
    if (c.out == c.q || c.out == c.k || c.out == c.v)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "output must not alias read-only Q/K/V");

    CUtensorMap kmap, vmap;
    // Tensor maps describe the caller's head_dim (GD); the kernel runs at D >= GD
    // and the TMA fills the columns past GD with zeros.
    const uint64_t GD = g->head_dim;
    if (c.paged) {
        const uint64_t dims[3] = {GD, c.page_tokens, (uint64_t)c.n_pages * g->kv_heads};
        const uint64_t str[2] = {GD * 2ull, (uint64_t)c.page_tokens * GD * 2};
        const uint32_t box[3] = {64, 64, 1};
        if (int rc = make_tmap(&kmap, c.k, 3, dims, str, box)) return rc;
        if (int rc = make_tmap(&vmap, c.v, 3, dims, str, box)) return rc;
    } else {
        const uint64_t dims[4] = {GD, g->kv_heads, c.max_tokens, c.n_seq};
        const uint64_t str[3] = {GD * 2ull, (uint64_t)g->kv_heads * GD * 2,
                                 (uint64_t)c.max_tokens * g->kv_heads * GD * 2};
        const uint32_t box[4] = {64, 1, 64, 1};
        if (int rc = make_tmap(&kmap, c.k, 4, dims, str, box)) return rc;
        if (int rc = make_tmap(&vmap, c.v, 4, dims, str, box)) return rc;
    }
    mslim::DecodeParams p{};
    p.q = static_cast<const uint16_t *>(c.q);
    p.q_f32 = c.q_f32;
    p.seq_tokens = c.seq_tokens;
    p.page_table = c.page_table;
    p.persistent = g_decode_schedule.load(std::memory_order_relaxed) == MSLIM_DECODE_PERSISTENT ? 1 : 0;
    p.work_counter = static_cast<unsigned *>(c.workspace);
    p.item_counters = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(c.workspace) + 256);
    p.out = static_cast<uint16_t *>(c.out);
    p.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(c.workspace) + kDecodeCounterBytes);
    p.status = status_ptr(dev);
    p.qheads = (int)g->query_heads;
    p.kvheads = (int)g->kv_heads;
    p.group = sh.group;
    p.head_chunks = sh.head_chunks;
    p.heads_per_cta = sh.heads_per_cta;
    p.nq = (int)c.nq;
    p.q_per_cta = sh.q_per_cta;
    p.q_blocks = sh.q_blocks;
    p.split_tokens = (int)c.split_tokens;
    p.max_splits = (int)max_splits;
    p.page_tokens = (int)c.page_tokens;
    p.max_pages = (int)c.max_pages;
    p.n_pages = (int)std::min<uint64_t>(c.n_pages, 0x7fffffff);
    p.n_seq = (int)c.n_seq;
    p.head_dim = (int)g->head_dim;
    p.token_cap = c.paged ? (int)std::min<uint64_t>((uint64_t)c.max_pages * c.page_tokens, 0x7fffffff)
                          : (int)c.max_tokens;
    p.fixed_tokens = c.fixed_tokens;
    p.scale_log2 = c.scale_log2;
    p.out_f32 = c.out_f32;
    cudaError_t err = mslim::launch_decode((int)D, c.paged, kmap, vmap, p,
                                           static_cast<uint16_t *>(c.out), c.stream);
    if (err != cudaSuccess) return cuda_fail(err, "decode launch");
    return MSLIM_OK;
}

float scale_log2_for(uint32_t head_dim) {
    return (float)(1.4426950408889634 / std::sqrt((double)head_dim));
}

// ------------------------------------------------------------- RoPE ----

int build_rope_table(const mslim_rope_config_t *rope, uint32_t dim, mslim::RopeTable *t) {
    if (!rope) return fail(MSLIM_ERR_INVALID_CONFIG, "rope config is null");
    if (!(std::isfinite(rope->theta) && rope->theta > 0.0f))
        return fail(MSLIM_ERR_INVALID_CONFIG, "invalid RoPE theta");
    if (dim == 0 || dim % 2 != 0 || dim > 256)
        return fail(MSLIM_ERR_INVALID_GEOMETRY, "RoPE head_dim must be even and at most 256");
    std::memset(t, 0, sizeof(*t));
    const uint32_t half = dim / 2;
    if (!rope->llama3_scaling) {
        // CPU decoder formula (native_cpu_adapter.rs:211): theta^(2i/dim) in f32.
        t->multiply = 0;
        for (uint32_t i = 0; i < half; ++i)
            t->freq[i] = powf(rope->theta, (float)(2 * i) / (float)dim);
    } else {
        // RopeKernelConfig::inverse_frequency (src/gpu_llm/kernels.rs:50-67).
        t->multiply = 1;
        for (uint32_t i = 0; i < half; ++i) {
            float inv = expf(-(float)(2 * i) * logf(rope->theta) / (float)dim);
            const float tau = 6.28318530717958647692f;
            const float wavelength = tau / inv;
            const float low_wavelength = rope->original_max_position / rope->low_freq_factor;
            const float high_wavelength = rope->original_max_position / rope->high_freq_factor;
            if (wavelength > low_wavelength) {
                inv /= rope->factor;
            } else if (wavelength >= high_wavelength) {
                const float smooth = (rope->original_max_position / wavelength - rope->low_freq_factor) /
                                     (rope->high_freq_factor - rope->low_freq_factor);
                inv = (1.0f - smooth) * (inv / rope->factor) + smooth * inv;
            }
            t->freq[i] = inv;
        }
    }
    return MSLIM_OK;
}

// binary32 -> bf16 bits, round to nearest even (finite inputs).
uint16_t bf16_bits_rne(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

// IEEE binary16 -> binary32 (exact).
float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
    if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

const char *mode_debug_name(int32_t mode) {
    switch (mode) {
        case MSLIM_MODE_REFERENCE: return "Reference";
        case MSLIM_MODE_STRICT_TILED: return "StrictTiled";
        case MSLIM_MODE_ONLINE_EXPERIMENTAL: return "OnlineExperimental";
        case MSLIM_MODE_SPLIT_KV_EXPERIMENTAL: return "SplitKvExperimental";
        default: return nullptr;
    }
}

const char *mode_serde_name(int32_t mode) {
    switch (mode) {
        case MSLIM_MODE_REFERENCE: return "reference";
        case MSLIM_MODE_STRICT_TILED: return "strict_tiled";
        case MSLIM_MODE_ONLINE_EXPERIMENTAL: return "online_experimental";
        case MSLIM_MODE_SPLIT_KV_EXPERIMENTAL: return "split_kv_experimental";
        default: return "invalid";
    }
}

bool is_experimental(const mslim_kernel_config_t &c) {
    return c.mode == MSLIM_MODE_ONLINE_EXPERIMENTAL || c.mode == MSLIM_MODE_SPLIT_KV_EXPERIMENTAL;
}

// Split scratch owned by a plan: the reference's split scratch bound.
constexpr size_t kPlanScratchBytes = 16u << 20;

}  // namespace

struct mslim_plan {
    mslim_kernel_config_t config;
    mslim_geometry_t geometry;
    int device;
    void *scratch;
    size_t scratch_bytes;
    std::atomic<uint64_t> calls{0};
    std::atomic<uint64_t> split_calls{0};
    std::atomic<uint64_t> prefill_calls{0};
};

struct mslim_backend {
    int device;
    cudaStream_t stream;
    void *buf;
    size_t buf_bytes;
    cudaEvent_t ev0, ev1;
    double dispatch_ms, kernel_ms;
    size_t input_kv_bytes, scratch_bytes, output_bytes;
    bool have_timings;
};

extern "C" {

const char *mslim_cuda_last_error(void) { return g_last_error.c_str(); }

const char *mslim_cuda_version(void) { return "mslim-cuda 0.1.0 (sm_100a)"; }

#ifndef MSLIM_SOURCE_DIGEST
#define MSLIM_SOURCE_DIGEST "unknown"  // built outside vk-shei_b200/build.py
#endif
const char *mslim_cuda_implementation_digest(void) { return MSLIM_SOURCE_DIGEST; }

uint64_t mslim_cuda_kernel_launches(void) { return g_kernel_launches.load(std::memory_order_relaxed); }

int mslim_cuda_set_decode_schedule(int schedule) {
    if (schedule != MSLIM_DECODE_SPLIT_MERGE && schedule != MSLIM_DECODE_PERSISTENT)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "unknown decode schedule %d", schedule);
    g_decode_schedule.store(schedule, std::memory_order_relaxed);
    return MSLIM_OK;
}

int mslim_cuda_get_decode_schedule(void) { return g_decode_schedule.load(std::memory_order_relaxed); }

int mslim_cuda_device_status(int device, int reset, int *status) {
    if (!status) return fail(MSLIM_ERR_SHAPE_MISMATCH, "status pointer is null");
    int prev;
    if (cudaGetDevice(&prev) != cudaSuccess) return fail(MSLIM_ERR_BACKEND_FAILURE, "no CUDA device");
    if (cudaSetDevice(device) != cudaSuccess) return fail(MSLIM_ERR_UNSUPPORTED_DEVICE, "bad device %d", device);
    int value = 0;
    cudaError_t err = cudaDeviceSynchronize();
    if (err == cudaSuccess) err = cudaMemcpyFromSymbol(&value, g_mslim_status_word, sizeof(int));
    if (err == cudaSuccess && reset) {
        const int zero = 0;
        err = cudaMemcpyToSymbol(g_mslim_status_word, &zero, sizeof(int));
    }
    cudaSetDevice(prev);
    if (err != cudaSuccess) return cuda_fail(err, "device status");
    *status = value & 0xff;
    if (*status == MSLIM_DEVICE_BAD_PAGE_CODE)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "a page table entry was outside the page pool");
    if (value) {
        return fail(MSLIM_ERR_DEVICE_TIMEOUT, "a device-side wait hit its bound (site %d)",
                    value >> 8);
    }
    return MSLIM_OK;
}

int mslim_cuda_geometry_validate(const mslim_geometry_t *geometry) { return check_geometry(geometry); }

mslim_kernel_config_t mslim_cuda_config_default(void) {
    mslim_kernel_config_t c;
    c.mode = MSLIM_MODE_REFERENCE;
    c.block_queries = 1;
    c.block_keys = 64;
    c.work_group = 64;
    c.splits = 1;
    return c;
}

int mslim_cuda_config_validate(const mslim_kernel_config_t *config, int allow_experimental) {
    if (!config) return fail(MSLIM_ERR_INVALID_CONFIG, "config is null");
    const mslim_kernel_config_t c = *config;
    if (!mode_debug_name(c.mode)) return fail(MSLIM_ERR_INVALID_CONFIG, "unknown attention mode %d", c.mode);
    if (!(c.block_queries == 1 || c.block_queries == 2 || c.block_queries == 4))
        return fail(MSLIM_ERR_INVALID_CONFIG, "attention block_queries must be 1,2,4");
    if (!(c.block_keys == 32 || c.block_keys == 64 || c.block_keys == 128))
        return fail(MSLIM_ERR_INVALID_CONFIG, "attention block_keys must be 32,64,128");
    if (!(c.work_group == 32 || c.work_group == 64 || c.work_group == 128))
        return fail(MSLIM_ERR_INVALID_CONFIG, "attention work_group must be 32,64,128");
    if (c.splits < 1 || c.splits > 64)
        return fail(MSLIM_ERR_INVALID_CONFIG, "attention splits must be 1..=64");
    if (c.mode == MSLIM_MODE_SPLIT_KV_EXPERIMENTAL) {
        if (!(c.block_queries == 1 && c.splits >= 2))
            return fail(MSLIM_ERR_INVALID_CONFIG,
                        "split-KV requires one query per group and at least two splits");
    } else if (c.splits != 1) {
        return fail(MSLIM_ERR_INVALID_CONFIG, "only explicit split-KV may request multiple splits");
    }
    if (c.mode == MSLIM_MODE_REFERENCE) {
        const mslim_kernel_config_t d = mslim_cuda_config_default();
        if (c.block_queries != d.block_queries || c.block_keys != d.block_keys ||
            c.work_group != d.work_group || c.splits != d.splits)
            return fail(MSLIM_ERR_INVALID_CONFIG, "reference attention cannot carry ignored tuning values");
    }
    if (allow_experimental >= 0 && is_experimental(c) && !allow_experimental)
        return fail(MSLIM_ERR_INVALID_CONFIG,
                    "experimental attention requires explicit numeric-contract opt-in");
    return MSLIM_OK;
}

int mslim_cuda_config_id(const mslim_kernel_config_t *config, char *out, size_t len) {
    if (int rc = mslim_cuda_config_validate(config, -1)) return rc;
    if (!out || len == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "output buffer is empty");
    std::string id;
    if (config->mode == MSLIM_MODE_REFERENCE) {
        id = "reference";
    } else {
        char buf[128];
        snprintf(buf, sizeof(buf), "%s-q%u-k%u-wg%u-s%u", mode_debug_name(config->mode),
                 config->block_queries, config->block_keys, config->work_group, config->splits);
        id = buf;
        for (auto &ch : id) ch = (char)tolower((unsigned char)ch);
    }
    if (id.size() + 1 > len) return fail(MSLIM_ERR_SHAPE_MISMATCH, "output buffer too small");
    memcpy(out, id.c_str(), id.size() + 1);
    return MSLIM_OK;
}

int mslim_cuda_config_local_bytes(const mslim_kernel_config_t *config, uint32_t head_dim,
                                  size_t *bytes) {
    if (int rc = mslim_cuda_config_validate(config, -1)) return rc;
    if (head_dim < 1 || head_dim > 256)
        return fail(MSLIM_ERR_INVALID_CONFIG, "tiled attention head dimension must be 1..=256");
    const size_t bk = config->block_keys, bq = config->block_queries;
    *bytes = 2 * bk * head_dim + 2 * bq * head_dim + 4 * bq * bk + 4 * bq * 4;
    return MSLIM_OK;
}

int mslim_cuda_config_decode_scratch_bytes(const mslim_kernel_config_t *config, uint32_t heads,
                                           uint32_t head_dim, size_t *bytes) {
    if (int rc = mslim_cuda_config_validate(config, -1)) return rc;
    if (config->mode != MSLIM_MODE_SPLIT_KV_EXPERIMENTAL) {
        *bytes = 0;
        return MSLIM_OK;
    }
    const unsigned __int128 n =
        (unsigned __int128)heads * config->splits * ((unsigned __int128)head_dim + 2) * 4;
    if (n == 0 || n > (16u << 20))
        return fail(MSLIM_ERR_INVALID_CONFIG, "split-KV scratch exceeds its 16 MiB bound or overflows");
    *bytes = (size_t)n;
    return MSLIM_OK;
}

// ------------------------------------------------------------ decode --

int mslim_cuda_decode_workspace_bytes(const mslim_geometry_t *geometry, uint32_t n_seq,
                                      uint32_t max_tokens, uint32_t split_tokens, size_t *bytes) {
    if (int rc = check_geometry(geometry)) return rc;
    if (!bytes) return fail(MSLIM_ERR_SHAPE_MISMATCH, "bytes pointer is null");
    if (n_seq == 0 || max_tokens == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty batch");
    DecodeShapeInfo sh;
    if (int rc = decode_shape(geometry, 1, &sh)) return rc;
    if (split_tokens == 0)
        split_tokens = policy_split_tokens((uint64_t)n_seq * geometry->kv_heads * sh.head_chunks,
                                           max_tokens, decode_slots(kernel_dim_for(geometry->head_dim)));
    if (split_tokens % 64 != 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "split_tokens must be a multiple of 64");
    const uint64_t splits = (max_tokens + split_tokens - 1) / split_tokens;
    *bytes = partial_bytes(geometry, n_seq, 1, splits);
    return MSLIM_OK;
}

int mslim_cuda_decode_split_tokens(const mslim_geometry_t *geometry, uint32_t n_seq,
                                   uint32_t max_tokens, uint32_t *split_tokens) {
    if (int rc = check_geometry(geometry)) return rc;
    if (!split_tokens) return fail(MSLIM_ERR_SHAPE_MISMATCH, "split_tokens pointer is null");
    if (n_seq == 0 || max_tokens == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty batch");
    DecodeShapeInfo sh;
    if (int rc = decode_shape(geometry, 1, &sh)) return rc;
    *split_tokens = policy_split_tokens((uint64_t)n_seq * geometry->kv_heads * sh.head_chunks, max_tokens,
                                        decode_slots(kernel_dim_for(geometry->head_dim)));
    return MSLIM_OK;
}

int mslim_cuda_decode_split_tokens_for_lengths(const mslim_geometry_t *geometry, uint32_t n_seq,
                                               const int32_t *lengths, uint32_t *split_tokens) {
    if (int rc = check_geometry(geometry)) return rc;
    if (!split_tokens || !lengths) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null pointer");
    if (n_seq == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty batch");
    DecodeShapeInfo sh;
    if (int rc = decode_shape(geometry, 1, &sh)) return rc;
    // every candidate split through the model of the split kernel's CTAs on
    // the GPU (fluid_step_time); choose_split keeps the fastest
    *split_tokens = choose_split(lengths, n_seq, (uint64_t)geometry->kv_heads * sh.head_chunks,
                                 decode_slots(kernel_dim_for(geometry->head_dim)), kCapVariedLengths);
    return MSLIM_OK;
}

static int decode_common_checks(const mslim_geometry_t *geometry, uint32_t n_seq,
                                uint32_t *split_tokens, uint32_t max_tokens) {
    if (int rc = check_geometry(geometry)) return rc;
    if (!kernel_head_dim(geometry->head_dim))
        return fail(MSLIM_ERR_INVALID_GEOMETRY,
                    "head_dim %u has no sm_100a decode kernel (multiples of 8 up to 256)",
                    geometry->head_dim);
    if (n_seq == 0 || max_tokens == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty batch");
    DecodeShapeInfo sh;
    if (int rc = decode_shape(geometry, 1, &sh)) return rc;
    if (*split_tokens == 0)
        *split_tokens = policy_split_tokens((uint64_t)n_seq * geometry->kv_heads * sh.head_chunks,
                                            max_tokens, decode_slots(kernel_dim_for(geometry->head_dim)));
    return MSLIM_OK;
}

int mslim_cuda_decode_dense(const mslim_geometry_t *geometry, const void *q, const void *k_cache,
                            const void *v_cache, const int32_t *seq_tokens, uint32_t n_seq,
                            uint32_t max_tokens, uint32_t split_tokens, void *workspace,
                            size_t workspace_bytes, void *out, void *stream) {
    if (int rc = decode_common_checks(geometry, n_seq, &split_tokens, max_tokens)) return rc;
    if (!q || !k_cache || !v_cache || !seq_tokens || !out)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    DecodeCall c{};
    c.g = geometry;
    c.q = q;
    c.k = k_cache;
    c.v = v_cache;
    c.seq_tokens = seq_tokens;
    c.fixed_tokens = -1;
    c.n_seq = n_seq;
    c.nq = 1;
    c.max_tokens = max_tokens;
    c.split_tokens = split_tokens;
    c.workspace = workspace;
    c.workspace_bytes = workspace_bytes;
    c.out = out;
    c.scale_log2 = scale_log2_for(geometry->head_dim);
    c.kernel_dim = kernel_dim_for(geometry->head_dim);
    c.stream = static_cast<cudaStream_t>(stream);
    return run_decode(c);
}

// Certified sparse decode: the gathered K and V rows, then the split partials,
// each section 256-byte aligned.
struct SelectedLayout {
    size_t kv_bytes, partial_bytes, total;
};
static int selected_layout(const mslim_geometry_t *geometry, uint32_t n_seq, uint32_t max_selected,
                           uint32_t split_tokens, SelectedLayout *l) {
    if (int rc = check_geometry(geometry)) return rc;
    // the gathered rows are indexed like a dense cache (i32 token counts)
    if ((uint64_t)n_seq * max_selected > 0x7fffffffull ||
        (uint64_t)n_seq * max_selected * geometry->kv_heads * geometry->head_dim > (1ull << 40))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "selection capacity too large");
    size_t part = 0;
    if (int rc = mslim_cuda_decode_workspace_bytes(geometry, n_seq, max_selected, split_tokens, &part)) return rc;
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    l->kv_bytes = up((size_t)n_seq * max_selected * geometry->kv_heads * geometry->head_dim * 2);
    l->partial_bytes = part;
    l->total = 2 * l->kv_bytes + up(part);
    return MSLIM_OK;
}

int mslim_cuda_decode_selected_workspace_bytes(const mslim_geometry_t *geometry, uint32_t n_seq,
                                               uint32_t max_selected, uint32_t split_tokens, size_t *bytes) {
    if (!bytes) return fail(MSLIM_ERR_SHAPE_MISMATCH, "bytes pointer is null");
    SelectedLayout l;
    if (int rc = selected_layout(geometry, n_seq, max_selected, split_tokens, &l)) return rc;
    *bytes = l.total;
    return MSLIM_OK;
}

// The gather into the workspace, then the dense split-KV decode over the
// gathered rows (shared by the dense-cache and the page-pool forms).
static int run_decode_selected(const mslim_geometry_t *geometry, const void *q, const void *k_src,
                               const void *v_src, uint32_t max_tokens, const int32_t *page_table,
                               uint32_t max_pages, uint32_t page_tokens, uint32_t n_pages,
                               const int32_t *seq_tokens, const int32_t *selected, const int32_t *selected_counts,
                               uint32_t max_selected, uint32_t n_seq, uint32_t split_tokens, void *workspace,
                               size_t workspace_bytes, void *out, void *stream) {
    if (max_tokens == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty cache");
    if (max_selected == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty selection capacity");
    uint32_t st = split_tokens;
    if (int rc = decode_common_checks(geometry, n_seq, &st, max_selected)) return rc;
    if (!q || !k_src || !v_src || !seq_tokens || !selected || !selected_counts || !out || !workspace)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    SelectedLayout l;
    if (int rc = selected_layout(geometry, n_seq, max_selected, st, &l)) return rc;
    if (workspace_bytes < l.total)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "workspace holds %zu bytes, needs %zu", workspace_bytes, l.total);
    if (!aligned(workspace, 256)) return fail(MSLIM_ERR_SHAPE_MISMATCH, "workspace must be 256-byte aligned");
    int dev;
    if (int rc = current_device(&dev)) return rc;
    uint8_t *base = static_cast<uint8_t *>(workspace);
    uint16_t *gk = reinterpret_cast<uint16_t *>(base);
    uint16_t *gv = reinterpret_cast<uint16_t *>(base + l.kv_bytes);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = mslim::launch_gather_selected(
        static_cast<const uint16_t *>(k_src), static_cast<const uint16_t *>(v_src), max_tokens, page_table,
        max_pages, page_tokens, n_pages, geometry->kv_heads, geometry->head_dim, seq_tokens, selected,
        selected_counts, max_selected, n_seq, gk, gv, status_ptr(dev), s);
    if (err != cudaSuccess) return cuda_fail(err, "selection gather launch");
    DecodeCall c{};
    c.g = geometry;
    c.q = q;
    c.k = gk;
    c.v = gv;
    c.seq_tokens = selected_counts;  // the gathered rows are the whole attended set
    c.fixed_tokens = -1;
    c.n_seq = n_seq;
    c.nq = 1;
    c.max_tokens = max_selected;
    c.split_tokens = st;
    c.workspace = base + 2 * l.kv_bytes;
    c.workspace_bytes = l.partial_bytes;
    c.out = out;
    c.scale_log2 = scale_log2_for(geometry->head_dim);
    c.kernel_dim = kernel_dim_for(geometry->head_dim);
    c.stream = s;
    return run_decode(c);
}

int mslim_cuda_decode_selected(const mslim_geometry_t *geometry, const void *q, const void *k_cache,
                               const void *v_cache, uint32_t max_tokens, const int32_t *seq_tokens,
                               const int32_t *selected, const int32_t *selected_counts, uint32_t max_selected,
                               uint32_t n_seq, uint32_t split_tokens, void *workspace, size_t workspace_bytes,
                               void *out, void *stream) {
    return run_decode_selected(geometry, q, k_cache, v_cache, max_tokens, nullptr, 0, 0, 0, seq_tokens, selected,
                               selected_counts, max_selected, n_seq, split_tokens, workspace, workspace_bytes, out,
                               stream);
}

int mslim_cuda_decode_selected_paged(const mslim_geometry_t *geometry, const void *q, const void *k_pool,
                                     const void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                     const int32_t *page_table, uint32_t max_pages_per_seq,
                                     const int32_t *seq_tokens, const int32_t *selected,
                                     const int32_t *selected_counts, uint32_t max_selected, uint32_t n_seq,
                                     uint32_t split_tokens, void *workspace, size_t workspace_bytes, void *out,
                                     void *stream) {
    if (page_tokens == 0 || n_pages == 0 || max_pages_per_seq == 0 || !page_table)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty page pool or page table");
    const uint64_t reach = (uint64_t)max_pages_per_seq * page_tokens;
    if (reach > 0x7fffffffull) return fail(MSLIM_ERR_SHAPE_MISMATCH, "page table spans too many tokens");
    return run_decode_selected(geometry, q, k_pool, v_pool, (uint32_t)reach, page_table, max_pages_per_seq,
                               page_tokens, n_pages, seq_tokens, selected, selected_counts, max_selected, n_seq,
                               split_tokens, workspace, workspace_bytes, out, stream);
}

int mslim_cuda_decode_paged(const mslim_geometry_t *geometry, const void *q, const void *k_pool,
                            const void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                            const int32_t *page_table, uint32_t max_pages_per_seq,
                            const int32_t *seq_tokens, uint32_t n_seq, uint32_t split_tokens,
                            void *workspace, size_t workspace_bytes, void *out, void *stream) {
    if (page_tokens == 0 || page_tokens % 64 != 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "page_tokens must be a positive multiple of 64");
    if (n_pages == 0 || max_pages_per_seq == 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty page pool or page table");
    const uint64_t max_tokens64 = (uint64_t)max_pages_per_seq * page_tokens;
    if (max_tokens64 > 0x7fffffffull) return fail(MSLIM_ERR_SHAPE_MISMATCH, "page table spans too many tokens");
    const uint32_t max_tokens = (uint32_t)max_tokens64;
    if (int rc = decode_common_checks(geometry, n_seq, &split_tokens, max_tokens)) return rc;
    if (!q || !k_pool || !v_pool || !page_table || !seq_tokens || !out)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if ((uint64_t)n_pages * geometry->kv_heads > 0xffffffffull)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "page pool too large for a tensor map");
    DecodeCall c{};
    c.g = geometry;
    c.q = q;
    c.k = k_pool;
    c.v = v_pool;
    c.paged = true;
    c.n_pages = n_pages;
    c.page_tokens = page_tokens;
    c.page_table = page_table;
    c.max_pages = max_pages_per_seq;
    c.seq_tokens = seq_tokens;
    c.fixed_tokens = -1;
    c.n_seq = n_seq;
    c.nq = 1;
    c.max_tokens = max_tokens;
    c.split_tokens = split_tokens;
    c.workspace = workspace;
    c.workspace_bytes = workspace_bytes;
    c.out = out;
    c.scale_log2 = scale_log2_for(geometry->head_dim);
    c.kernel_dim = kernel_dim_for(geometry->head_dim);
    c.stream = static_cast<cudaStream_t>(stream);
    return run_decode(c);
}

int mslim_cuda_decode_paged_static_scratch(const mslim_geometry_t *geometry, const void *q,
                                           const void *k_pool, const void *v_pool,
                                           uint32_t n_pages, uint32_t page_tokens,
                                           const int32_t *page_table, uint32_t max_pages_per_seq,
                                           const int32_t *seq_tokens, uint32_t n_seq,
                                           uint32_t split_tokens, void *out, void *stream) {
    if (int rc = check_geometry(geometry)) return rc;
    if (page_tokens == 0 || page_tokens % 64 != 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "page_tokens must be a positive multiple of 64");
    if (n_pages == 0 || max_pages_per_seq == 0 || n_seq == 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty page pool, page table or batch");
    const uint64_t max_tokens = (uint64_t)max_pages_per_seq * page_tokens;
    if (max_tokens > 0x7fffffffull) return fail(MSLIM_ERR_SHAPE_MISMATCH, "page table spans too many tokens");
    if (split_tokens % 64 != 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "split_tokens must be a multiple of 64");
    uint32_t st = split_tokens;
    if (st == 0) {
        if (int rc = decode_common_checks(geometry, n_seq, &st, (uint32_t)max_tokens)) return rc;
        // Larger splits until the partials fit the static array.
        while (partial_bytes(geometry, n_seq, 1, (max_tokens + st - 1) / st) > MSLIM_STATIC_SCRATCH_BYTES &&
               st < max_tokens)
            st *= 2;
    }
    const uint64_t need = partial_bytes(geometry, n_seq, 1, (max_tokens + st - 1) / st);
    if (need > MSLIM_STATIC_SCRATCH_BYTES)
        return fail(MSLIM_ERR_SHAPE_MISMATCH,
                    "split partials need %llu bytes; the static scratch holds %u bytes "
                    "(use fewer sessions, larger split_tokens or mslim_cuda_decode_paged)",
                    (unsigned long long)need, (unsigned)MSLIM_STATIC_SCRATCH_BYTES);
    int dev;
    if (int rc = current_device(&dev)) return rc;
    void *scratch = nullptr;
    if (int rc = static_scratch_ptr(dev, &scratch)) return rc;
    cudaError_t err = cudaMemsetAsync(scratch, 0, kDecodeCounterBytes, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "clearing the static scratch counters");
    return mslim_cuda_decode_paged(geometry, q, k_pool, v_pool, n_pages, page_tokens, page_table,
                                   max_pages_per_seq, seq_tokens, n_seq, st, scratch,
                                   MSLIM_STATIC_SCRATCH_BYTES, out, stream);
}

// ----------------------------------------------------------- prefill --

int mslim_cuda_prefill_causal(const mslim_geometry_t *geometry, const void *q, const void *k,
                              const void *v, void *out, uint32_t queries, uint32_t prior,
                              void *stream) {
    if (int rc = check_geometry(geometry)) return rc;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!q || !k || !v || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (queries == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "prefill needs at least one query");
    const uint64_t history = (uint64_t)prior + queries;
    if (history > 0x7fffffffull) return fail(MSLIM_ERR_SHAPE_MISMATCH, "history exceeds indexing bound");
    if (out == q || out == k || out == v)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "output must not alias read-only Q/K/V");
    if (!mslim::prefill_supported(geometry->head_dim, geometry->query_heads / geometry->kv_heads))
        return fail(MSLIM_ERR_INVALID_GEOMETRY,
                    "head_dim %u with %u query heads per KV head has no sm_100a prefill kernel "
                    "(head_dim 64..256, a multiple of 8)",
                    geometry->head_dim, geometry->query_heads / geometry->kv_heads);
    if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "prefill buffers must be 16-byte aligned");
    const uint64_t D = geometry->head_dim;
    CUtensorMap qmap, kmap, vmap, omap;
    {
        const uint64_t qd[3] = {D, geometry->query_heads, queries};
        const uint64_t qs[2] = {D * 2, (uint64_t)geometry->query_heads * D * 2};
        const uint64_t kd[3] = {D, geometry->kv_heads, history};
        const uint64_t ks[2] = {D * 2, (uint64_t)geometry->kv_heads * D * 2};
        const uint32_t box[3] = {64, 1, 128};
        const uint32_t kvbox[3] = {64, 1, mslim::prefill_kv_box_rows(geometry->head_dim)};
        if (int rc = make_tmap(&qmap, q, 3, qd, qs, box)) return rc;
        const uint32_t obox[3] = {64, 1, 32};  // the pair kernel stores 32 rows per warp
        if (int rc = make_tmap(&omap, out, 3, qd, qs, obox)) return rc;
        if (int rc = make_tmap(&kmap, k, 3, kd, ks, kvbox)) return rc;
        if (int rc = make_tmap(&vmap, v, 3, kd, ks, kvbox)) return rc;
    }
    mslim::PrefillParams p{};
    p.out = static_cast<uint16_t *>(out);
    p.status = status_ptr(dev);
    p.qheads = (int)geometry->query_heads;
    p.kvheads = (int)geometry->kv_heads;
    p.group = (int)(geometry->query_heads / geometry->kv_heads);
    p.queries = (int)queries;
    p.prior = (int)prior;
    p.n_qtiles = (int)((queries + 127) / 128);
    p.head_dim = (int)geometry->head_dim;
    p.scale_log2 = scale_log2_for(geometry->head_dim);
    if ((uint64_t)p.n_qtiles * p.qheads > 0x7fffffffull)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "prefill grid too large");
    cudaError_t err = mslim::launch_prefill(qmap, kmap, vmap, omap, p, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "prefill launch");
    return MSLIM_OK;
}

// -------------------------------------------------- layer elementwise --

int mslim_cuda_residual_add(const void *a, const void *b, void *out, uint64_t n, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!a || !b || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (n == 0) return MSLIM_OK;
    if (!aligned(a, 16) || !aligned(b, 16) || !aligned(out, 16))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "residual buffers must be 16-byte aligned");
    cudaError_t err = mslim::launch_residual_add(static_cast<const uint16_t *>(a),
                                                 static_cast<const uint16_t *>(b),
                                                 static_cast<uint16_t *>(out), n,
                                                 static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "residual add launch");
}

int mslim_cuda_swiglu(const void *gate, const void *up, void *out, uint64_t n, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!gate || !up || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (n == 0) return MSLIM_OK;
    if (!aligned(gate, 16) || !aligned(up, 16) || !aligned(out, 16))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "SwiGLU buffers must be 16-byte aligned");
    cudaError_t err = mslim::launch_swiglu(static_cast<const uint16_t *>(gate),
                                           static_cast<const uint16_t *>(up),
                                           static_cast<uint16_t *>(out), n,
                                           static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "SwiGLU launch");
}

int mslim_cuda_page_token_hashes(const void *pool, uint32_t n_pool_pages, uint32_t kv_heads,
                                 uint32_t page_tokens, uint32_t head_dim, const int32_t *page_ids,
                                 uint32_t n_pages, uint32_t tokens, uint64_t *hashes, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!pool || !page_ids || !hashes) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (n_pages == 0 || tokens == 0) return MSLIM_OK;
    if (kv_heads == 0 || head_dim == 0 || head_dim % 8 != 0 || page_tokens == 0 || n_pool_pages == 0)
        return fail(MSLIM_ERR_INVALID_GEOMETRY, "page geometry (head_dim a multiple of 8)");
    if (tokens > page_tokens) return fail(MSLIM_ERR_SHAPE_MISMATCH, "more tokens than a page holds");
    if (n_pages > 65535) return fail(MSLIM_ERR_SHAPE_MISMATCH, "at most 65535 pages per call");
    if (!aligned(pool, 16) || !aligned(hashes, 8)) return fail(MSLIM_ERR_SHAPE_MISMATCH, "misaligned buffer");
    cudaError_t err = mslim::launch_page_token_hashes(static_cast<const uint16_t *>(pool), n_pool_pages, kv_heads,
                                                      page_tokens, head_dim, page_ids, n_pages, tokens, hashes,
                                                      status_ptr(dev), static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "page hash launch");
}

int mslim_cuda_kv_canonical_dense(const void *cache, uint32_t kv_heads, uint32_t head_dim, uint32_t tokens,
                                  void *out, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!cache || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (kv_heads == 0 || head_dim == 0) return fail(MSLIM_ERR_INVALID_GEOMETRY, "empty KV geometry");
    if (tokens == 0) return MSLIM_OK;
    if (out == cache) return fail(MSLIM_ERR_SHAPE_MISMATCH, "output must not alias the cache");
    cudaError_t err = mslim::launch_kv_canonical(static_cast<const uint16_t *>(cache), static_cast<uint16_t *>(out),
                                                 kv_heads, tokens, head_dim, nullptr, 0, 0, status_ptr(dev),
                                                 static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "canonical KV launch");
}

int mslim_cuda_kv_canonical_paged(const void *pool, uint32_t n_pages, uint32_t kv_heads, uint32_t page_tokens,
                                  uint32_t head_dim, const int32_t *page_row, uint32_t max_pages, uint32_t tokens,
                                  void *out, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!pool || !page_row || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (kv_heads == 0 || head_dim == 0 || page_tokens == 0 || n_pages == 0)
        return fail(MSLIM_ERR_INVALID_GEOMETRY, "empty page geometry");
    if (tokens == 0) return MSLIM_OK;
    if ((uint64_t)tokens > (uint64_t)max_pages * page_tokens)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "more tokens than the session's pages hold");
    if (out == pool) return fail(MSLIM_ERR_SHAPE_MISMATCH, "output must not alias the pool");
    cudaError_t err = mslim::launch_kv_canonical(static_cast<const uint16_t *>(pool), static_cast<uint16_t *>(out),
                                                 kv_heads, tokens, head_dim, page_row, page_tokens, n_pages,
                                                 status_ptr(dev), static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "canonical KV launch");
}

int mslim_cuda_gemv(const void *x, const void *w, void *y, uint32_t m, uint32_t n, uint32_t k, uint32_t ldy,
                    void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!x || !w || !y) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (m == 0 || m > 16) return fail(MSLIM_ERR_SHAPE_MISMATCH, "the decode projection takes 1..16 rows");
    if (n == 0 || k == 0 || k % 8 != 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "n must be positive and k a positive multiple of 8");
    if (n > 0x7fffff80u || k > 0x7fffffc0u) return fail(MSLIM_ERR_SHAPE_MISMATCH, "projection too large");
    if (ldy < n) return fail(MSLIM_ERR_SHAPE_MISMATCH, "ldy must be at least n");
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 2))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "x and w must be 16-byte aligned");
    if (y == x || y == w) return fail(MSLIM_ERR_SHAPE_MISMATCH, "the output must not alias an input");
    const mslim::GemvPlan plan = mslim::gemv_plan(m, n, k);
    CUtensorMap xmap, wmap;
    {
        const uint64_t xd[2] = {k, m}, xs[1] = {(uint64_t)k * 2};
        const uint32_t xbox[2] = {64, 16};
        const uint64_t wd[2] = {k, n}, ws[1] = {(uint64_t)k * 2};
        const uint32_t wbox[2] = {64, 128};
        if (int rc = make_tmap(&xmap, x, 2, xd, xs, xbox)) return rc;
        if (int rc = make_tmap(&wmap, w, 2, wd, ws, wbox)) return rc;
    }
    cudaError_t err = mslim::launch_gemv_tc(xmap, wmap, plan, m, n, static_cast<uint16_t *>(y), ldy,
                                            status_ptr(dev), static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "projection launch");
}

int mslim_cuda_gemv_swiglu(const void *x, const void *w_gu, void *out, uint32_t m, uint32_t width, uint32_t k,
                           uint32_t ldo, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!x || !w_gu || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (m == 0 || m > 16) return fail(MSLIM_ERR_SHAPE_MISMATCH, "the decode projection takes 1..16 rows");
    if (width == 0 || width % 64 != 0 || k == 0 || k % 8 != 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "width must be a positive multiple of 64 and k of 8");
    if (width > 0x3fffffc0u || k > 0x7fffffc0u) return fail(MSLIM_ERR_SHAPE_MISMATCH, "projection too large");
    if (ldo < width) return fail(MSLIM_ERR_SHAPE_MISMATCH, "ldo must be at least width");
    if (!aligned(x, 16) || !aligned(w_gu, 16) || !aligned(out, 2))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "x and w_gu must be 16-byte aligned");
    if (out == x || out == w_gu) return fail(MSLIM_ERR_SHAPE_MISMATCH, "the output must not alias an input");
    const uint32_t n = 2 * width;
    const mslim::GemvPlan plan = mslim::gemv_plan(m, n, k);
    CUtensorMap xmap, wmap;
    {
        const uint64_t xd[2] = {k, m}, xs[1] = {(uint64_t)k * 2};
        const uint32_t xbox[2] = {64, 16};
        const uint64_t wd[2] = {k, n}, ws[1] = {(uint64_t)k * 2};
        const uint32_t wbox[2] = {64, 128};
        if (int rc = make_tmap(&xmap, x, 2, xd, xs, xbox)) return rc;
        if (int rc = make_tmap(&wmap, w_gu, 2, wd, ws, wbox)) return rc;
    }
    cudaError_t err = mslim::launch_gemv_tc(xmap, wmap, plan, m, n, static_cast<uint16_t *>(out), ldo,
                                            status_ptr(dev), static_cast<cudaStream_t>(stream), true);
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "gate|up projection launch");
}

int mslim_cuda_swiglu_rows(const void *gate_up, void *out, uint32_t rows, uint32_t width, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!gate_up || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (rows == 0) return MSLIM_OK;
    if (width == 0 || width % 8 != 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "SwiGLU width must be a positive multiple of 8");
    if (!aligned(gate_up, 16) || !aligned(out, 16))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "SwiGLU buffers must be 16-byte aligned");
    cudaError_t err = mslim::launch_swiglu_rows(static_cast<const uint16_t *>(gate_up),
                                                static_cast<uint16_t *>(out), rows, width,
                                                static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "SwiGLU launch");
}

int mslim_cuda_argmax(const void *logits, uint32_t rows, uint32_t vocab, int ties_to_last,
                      int32_t *token_ids, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!logits || !token_ids) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (rows == 0) return MSLIM_OK;
    if (vocab == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty vocabulary");
    if (vocab > 0x7fffffffu || rows > 0x7fffffffu) return fail(MSLIM_ERR_SHAPE_MISMATCH, "argmax too large");
    cudaError_t err = mslim::launch_argmax(static_cast<const uint16_t *>(logits), rows, vocab,
                                           ties_to_last, token_ids, static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "argmax launch");
}

int mslim_cuda_exp2_eval(const float *x, float *y_poly, float *y_mufu, float *y_ref, uint32_t n,
                         void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (n == 0) return MSLIM_OK;
    if (!x || !y_poly || !y_mufu || !y_ref) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    cudaError_t err = mslim::launch_exp2_eval(x, y_poly, y_mufu, y_ref, n, static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "exp2 evaluation launch");
}

// ------------------------------------------------ tensor-parallel decode --

int mslim_cuda_tp_alloc(size_t bytes, void **ptr) {
    if (!ptr) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null pointer slot");
    *ptr = nullptr;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (bytes == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty allocation");
    cudaError_t err = cudaMalloc(ptr, bytes);
    if (err != cudaSuccess) return cuda_fail(err, "tensor-parallel buffer allocation");
    err = cudaMemset(*ptr, 0, bytes);
    if (err != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return cuda_fail(err, "tensor-parallel buffer clear");
    }
    return MSLIM_OK;
}

int mslim_cuda_tp_free(void *ptr) {
    if (!ptr) return MSLIM_OK;
    cudaError_t err = cudaFree(ptr);
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "tensor-parallel buffer free");
}

int mslim_cuda_ipc_handle(const void *ptr, void *handle) {
    if (!ptr || !handle) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaIpcMemHandle_t h;
    cudaError_t err = cudaIpcGetMemHandle(&h, const_cast<void *>(ptr));
    if (err != cudaSuccess) return cuda_fail(err, "IPC handle export");
    std::memcpy(handle, &h, sizeof(h));
    return MSLIM_OK;
}

int mslim_cuda_ipc_open(const void *handle, void **ptr) {
    if (!handle || !ptr) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "IPC handle open");
}

int mslim_cuda_ipc_close(void *ptr) {
    if (!ptr) return MSLIM_OK;
    cudaError_t err = cudaIpcCloseMemHandle(ptr);
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "IPC handle close");
}

int mslim_cuda_tp_allreduce_rmsnorm(const mslim_tp_comm_t *comm, uint32_t slot, void *x, const void *w,
                                    void *y, uint32_t rows, float eps, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!comm || !x || !w || !y) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (comm->world == 0 || comm->world > (uint32_t)mslim::kTpMaxWorld || comm->rank >= comm->world)
        return fail(MSLIM_ERR_INVALID_CONFIG, "tensor-parallel world of 1..8 ranks");
    if (slot > 1) return fail(MSLIM_ERR_SHAPE_MISMATCH, "slot is 0 or 1");
    if (rows == 0) return MSLIM_OK;
    if (rows > comm->max_rows) return fail(MSLIM_ERR_SHAPE_MISMATCH, "more rows than the communicator holds");
    if (comm->hidden == 0 || comm->hidden % 8 != 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "hidden size must be a positive multiple of 8");
    if (!std::isfinite(eps) || eps < 0.f) return fail(MSLIM_ERR_INVALID_CONFIG, "invalid epsilon");
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16) || !comm->epoch)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "buffers must be 16-byte aligned");
    mslim::TpCommDev d{};
    d.world = comm->world;
    d.rank = comm->rank;
    d.max_rows = comm->max_rows;
    d.hidden = comm->hidden;
    for (uint32_t r = 0; r < comm->world; ++r) {
        if (!comm->data[r] || !comm->flags[r] || !aligned(comm->data[r], 16))
            return fail(MSLIM_ERR_SHAPE_MISMATCH, "rank %u of the communicator is not mapped", r);
        d.data[r] = static_cast<const uint16_t *>(comm->data[r]);
        d.flags[r] = static_cast<uint32_t *>(comm->flags[r]);
    }
    d.epoch = static_cast<uint32_t *>(comm->epoch);
    cudaError_t err = mslim::launch_tp_allreduce_rmsnorm(d, slot, static_cast<uint16_t *>(x),
                                                         static_cast<const uint16_t *>(w),
                                                         static_cast<uint16_t *>(y), rows, eps, status_ptr(dev),
                                                         static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "tensor-parallel all-reduce launch");
}

// ---------------------------------------------------------- prologue --

int mslim_cuda_rmsnorm(const void *x, const void *w, void *y, uint32_t tokens, uint32_t hidden,
                       float eps, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!x || !w || !y) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (tokens == 0 || hidden == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty RMSNorm");
    if (!std::isfinite(eps) || eps < 0.f) return fail(MSLIM_ERR_INVALID_CONFIG, "invalid epsilon");
    if (hidden % 8 == 0 && (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16)))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "RMSNorm buffers must be 16-byte aligned");
    if (tokens > 0x7fffffffu) return fail(MSLIM_ERR_SHAPE_MISMATCH, "too many tokens");
    cudaError_t err = mslim::launch_rmsnorm(static_cast<const uint16_t *>(x),
                                            static_cast<const uint16_t *>(w),
                                            static_cast<uint16_t *>(y), tokens, hidden, eps,
                                            static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "RMSNorm launch");
}

int mslim_cuda_residual_rmsnorm(void *x, const void *delta, const void *w, void *y, uint32_t tokens,
                                uint32_t hidden, float eps, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!x || !delta || !w || !y) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (tokens == 0 || hidden == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty RMSNorm");
    if (!std::isfinite(eps) || eps < 0.f) return fail(MSLIM_ERR_INVALID_CONFIG, "invalid epsilon");
    if (hidden % 8 == 0 && (!aligned(x, 16) || !aligned(delta, 16) || !aligned(w, 16) || !aligned(y, 16)))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "RMSNorm buffers must be 16-byte aligned");
    if (y == x || y == delta) return fail(MSLIM_ERR_SHAPE_MISMATCH, "RMSNorm output must not alias its inputs");
    if (tokens > 0x7fffffffu) return fail(MSLIM_ERR_SHAPE_MISMATCH, "too many tokens");
    cudaError_t err = mslim::launch_residual_rmsnorm(static_cast<uint16_t *>(x), static_cast<const uint16_t *>(delta),
                                                     static_cast<const uint16_t *>(w), static_cast<uint16_t *>(y),
                                                     tokens, hidden, eps, static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "residual RMSNorm launch");
}

int mslim_cuda_rope(const void *in, void *out, uint32_t tokens, uint32_t heads, uint32_t head_dim,
                    uint32_t start_position, const mslim_rope_config_t *rope, void *stream) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!in || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (tokens == 0 || heads == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty RoPE");
    if ((uint64_t)start_position + tokens > 0xffffffffull)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "RoPE position overflow");
    mslim::RopeTable table;
    if (int rc = build_rope_table(rope, head_dim, &table)) return rc;
    cudaError_t err = mslim::launch_rope(static_cast<const uint16_t *>(in),
                                         static_cast<uint16_t *>(out), tokens, heads, head_dim,
                                         start_position, table, static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "RoPE launch");
}

int mslim_cuda_rope_append_paged(const mslim_geometry_t *geometry, const void *q_in, void *q_out,
                                 const void *k_in, const void *v_in, uint32_t tokens,
                                 uint32_t start_position, const mslim_rope_config_t *rope,
                                 void *k_pool, void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                 const int32_t *page_table, uint32_t max_pages, void *stream) {
    if (int rc = check_geometry(geometry)) return rc;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!q_in || !q_out || !k_in || !v_in || !k_pool || !v_pool || !page_table)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (tokens == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty append");
    if (page_tokens == 0 || n_pages == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty page pool");
    if ((uint64_t)start_position + tokens > (uint64_t)max_pages * page_tokens)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "append past the end of the page table");
    mslim::RopeTable table;
    if (int rc = build_rope_table(rope, geometry->head_dim, &table)) return rc;
    cudaError_t err = mslim::launch_rope_append_paged(
        static_cast<const uint16_t *>(q_in), static_cast<uint16_t *>(q_out),
        static_cast<const uint16_t *>(k_in), static_cast<const uint16_t *>(v_in), tokens,
        geometry->query_heads, geometry->kv_heads, geometry->head_dim, start_position, nullptr,
        static_cast<uint16_t *>(k_pool), static_cast<uint16_t *>(v_pool), n_pages, page_tokens,
        page_table, max_pages, table, status_ptr(dev), static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "RoPE append launch");
}

int mslim_cuda_rope_append_decode_paged(const mslim_geometry_t *geometry, const void *q_in,
                                        void *q_out, const void *k_in, const void *v_in,
                                        const int32_t *positions, uint32_t n_seq,
                                        const mslim_rope_config_t *rope, void *k_pool,
                                        void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                        const int32_t *page_table, uint32_t max_pages,
                                        void *stream) {
    if (int rc = check_geometry(geometry)) return rc;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!q_in || !q_out || !k_in || !v_in || !positions || !k_pool || !v_pool || !page_table)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (n_seq == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty batch");
    if (page_tokens == 0 || n_pages == 0 || max_pages == 0)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty page pool");
    if (n_seq > 0x7fffffffu) return fail(MSLIM_ERR_SHAPE_MISMATCH, "too many sessions");
    mslim::RopeTable table;
    if (int rc = build_rope_table(rope, geometry->head_dim, &table)) return rc;
    cudaError_t err = mslim::launch_rope_append_paged(
        static_cast<const uint16_t *>(q_in), static_cast<uint16_t *>(q_out),
        static_cast<const uint16_t *>(k_in), static_cast<const uint16_t *>(v_in), n_seq,
        geometry->query_heads, geometry->kv_heads, geometry->head_dim, 0, positions,
        static_cast<uint16_t *>(k_pool), static_cast<uint16_t *>(v_pool), n_pages, page_tokens,
        page_table, max_pages, table, status_ptr(dev), static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "RoPE decode append launch");
}

int mslim_cuda_rope_append_decode_dense(const mslim_geometry_t *geometry, const void *q_in,
                                        void *q_out, const void *k_in, const void *v_in,
                                        const int32_t *positions, uint32_t n_seq,
                                        const mslim_rope_config_t *rope, void *k_cache,
                                        void *v_cache, uint32_t max_tokens, void *stream) {
    if (int rc = check_geometry(geometry)) return rc;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!q_in || !q_out || !k_in || !v_in || !positions || !k_cache || !v_cache)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (n_seq == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty batch");
    if (max_tokens == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty cache");
    if (n_seq > 0x7fffffffu) return fail(MSLIM_ERR_SHAPE_MISMATCH, "too many sessions");
    mslim::RopeTable table;
    if (int rc = build_rope_table(rope, geometry->head_dim, &table)) return rc;
    cudaError_t err = mslim::launch_rope_append_dense(
        static_cast<const uint16_t *>(q_in), static_cast<uint16_t *>(q_out),
        static_cast<const uint16_t *>(k_in), static_cast<const uint16_t *>(v_in), n_seq,
        geometry->query_heads, geometry->kv_heads, geometry->head_dim, positions,
        static_cast<uint16_t *>(k_cache), static_cast<uint16_t *>(v_cache), max_tokens, table,
        status_ptr(dev), static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "RoPE dense append launch");
}

int mslim_cuda_rope_append_decode_dense_qkv(const mslim_geometry_t *geometry, const void *qkv,
                                            void *q_out, const int32_t *positions, uint32_t n_seq,
                                            const mslim_rope_config_t *rope, void *k_cache,
                                            void *v_cache, uint32_t max_tokens, void *stream) {
    if (int rc = check_geometry(geometry)) return rc;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!qkv || !q_out || !positions || !k_cache || !v_cache) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (n_seq == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty batch");
    if (max_tokens == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty cache");
    if (n_seq > 0x7fffffffu) return fail(MSLIM_ERR_SHAPE_MISMATCH, "too many sessions");
    mslim::RopeTable table;
    if (int rc = build_rope_table(rope, geometry->head_dim, &table)) return rc;
    const uint32_t D = geometry->head_dim, QH = geometry->query_heads, KVH = geometry->kv_heads;
    const uint16_t *base = static_cast<const uint16_t *>(qkv);
    const uint32_t stride = (QH + 2 * KVH) * D;
    cudaError_t err = mslim::launch_rope_append_dense(
        base, static_cast<uint16_t *>(q_out), base + (size_t)QH * D, base + (size_t)(QH + KVH) * D, n_seq,
        QH, KVH, D, positions, static_cast<uint16_t *>(k_cache), static_cast<uint16_t *>(v_cache), max_tokens,
        table, status_ptr(dev), static_cast<cudaStream_t>(stream), stride, stride);
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "RoPE dense append launch");
}

int mslim_cuda_rope_append_decode_paged_qkv(const mslim_geometry_t *geometry, const void *qkv,
                                            void *q_out, const int32_t *positions, uint32_t n_seq,
                                            const mslim_rope_config_t *rope, void *k_pool, void *v_pool,
                                            uint32_t n_pages, uint32_t page_tokens,
                                            const int32_t *page_table, uint32_t max_pages, void *stream) {
    if (int rc = check_geometry(geometry)) return rc;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!qkv || !q_out || !positions || !k_pool || !v_pool || !page_table)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (n_seq == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty batch");
    if (page_tokens == 0 || n_pages == 0 || max_pages == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty page pool");
    if (n_seq > 0x7fffffffu) return fail(MSLIM_ERR_SHAPE_MISMATCH, "too many sessions");
    mslim::RopeTable table;
    if (int rc = build_rope_table(rope, geometry->head_dim, &table)) return rc;
    const uint32_t D = geometry->head_dim, QH = geometry->query_heads, KVH = geometry->kv_heads;
    const uint16_t *base = static_cast<const uint16_t *>(qkv);
    const uint32_t stride = (QH + 2 * KVH) * D;
    cudaError_t err = mslim::launch_rope_append_paged(
        base, static_cast<uint16_t *>(q_out), base + (size_t)QH * D, base + (size_t)(QH + KVH) * D, n_seq, QH,
        KVH, D, 0, positions, static_cast<uint16_t *>(k_pool), static_cast<uint16_t *>(v_pool), n_pages,
        page_tokens, page_table, max_pages, table, status_ptr(dev), static_cast<cudaStream_t>(stream), stride,
        stride);
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "RoPE decode append launch");
}

// The decode q|k|v projection with RoPE + K/V append in its epilogue: the
// checks of mslim_cuda_gemv and of the q|k|v append entry points.
static int gemv_qkv_rope_append(const mslim_geometry_t *geometry, const void *x, const void *w_qkv, uint32_t k,
                                const int32_t *positions, uint32_t n_seq, const mslim_rope_config_t *rope,
                                void *q_out, mslim::GemvRopeAppend e, void *stream) {
    if (int rc = check_geometry(geometry)) return rc;
    if (geometry->head_dim != 128)
        return fail(MSLIM_ERR_INVALID_GEOMETRY,
                    "the fused q|k|v projection needs head_dim 128 (got %u); use mslim_cuda_gemv and "
                    "mslim_cuda_rope_append_decode_*_qkv", geometry->head_dim);
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!x || !w_qkv || !q_out || !positions || !e.k_dst || !e.v_dst) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (n_seq == 0 || n_seq > 16) return fail(MSLIM_ERR_SHAPE_MISMATCH, "the decode projection takes 1..16 rows");
    if (k == 0 || k % 8 != 0 || k > 0x7fffffc0u) return fail(MSLIM_ERR_SHAPE_MISMATCH, "k must be a positive multiple of 8");
    if (!aligned(x, 16) || !aligned(w_qkv, 16) || !aligned(q_out, 2))
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "x and w_qkv must be 16-byte aligned");
    const uint64_t n64 = ((uint64_t)geometry->query_heads + 2ull * geometry->kv_heads) * 128;
    if (n64 > 0x7fffff80u) return fail(MSLIM_ERR_SHAPE_MISMATCH, "projection too large");
    if (int rc = build_rope_table(rope, 128, &e.table)) return rc;
    e.positions = positions;
    e.q_out = static_cast<uint16_t *>(q_out);
    e.qheads = geometry->query_heads;
    e.kvheads = geometry->kv_heads;
    const uint32_t n = (uint32_t)n64;
    const mslim::GemvPlan plan = mslim::gemv_plan(n_seq, n, k);
    CUtensorMap xmap, wmap;
    {
        const uint64_t xd[2] = {k, n_seq}, xs[1] = {(uint64_t)k * 2};
        const uint32_t xbox[2] = {64, 16};
        const uint64_t wd[2] = {k, n}, ws[1] = {(uint64_t)k * 2};
        const uint32_t wbox[2] = {64, 128};
        if (int rc = make_tmap(&xmap, x, 2, xd, xs, xbox)) return rc;
        if (int rc = make_tmap(&wmap, w_qkv, 2, wd, ws, wbox)) return rc;
    }
    cudaError_t err = mslim::launch_gemv_qkv_rope_append(xmap, wmap, plan, n_seq, n, e, status_ptr(dev),
                                                         static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MSLIM_OK : cuda_fail(err, "q|k|v projection launch");
}

int mslim_cuda_gemv_qkv_rope_append_dense(const mslim_geometry_t *geometry, const void *x, const void *w_qkv,
                                          uint32_t k, const int32_t *positions, uint32_t n_seq,
                                          const mslim_rope_config_t *rope, void *q_out, void *k_cache,
                                          void *v_cache, uint32_t max_tokens, void *stream) {
    if (max_tokens == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty cache");
    mslim::GemvRopeAppend e{};
    e.k_dst = static_cast<uint16_t *>(k_cache);
    e.v_dst = static_cast<uint16_t *>(v_cache);
    e.page_table = nullptr;
    e.max_tokens = max_tokens;
    return gemv_qkv_rope_append(geometry, x, w_qkv, k, positions, n_seq, rope, q_out, e, stream);
}

int mslim_cuda_gemv_qkv_rope_append_paged(const mslim_geometry_t *geometry, const void *x, const void *w_qkv,
                                          uint32_t k, const int32_t *positions, uint32_t n_seq,
                                          const mslim_rope_config_t *rope, void *q_out, void *k_pool,
                                          void *v_pool, uint32_t n_pages, uint32_t page_tokens,
                                          const int32_t *page_table, uint32_t max_pages, void *stream) {
    if (!page_table) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null buffer");
    if (page_tokens == 0 || n_pages == 0 || max_pages == 0) return fail(MSLIM_ERR_SHAPE_MISMATCH, "empty page pool");
    mslim::GemvRopeAppend e{};
    e.k_dst = static_cast<uint16_t *>(k_pool);
    e.v_dst = static_cast<uint16_t *>(v_pool);
    e.page_table = page_table;
    e.n_pages = n_pages;
    e.page_tokens = page_tokens;
    e.max_pages = max_pages;
    return gemv_qkv_rope_append(geometry, x, w_qkv, k, positions, n_seq, rope, q_out, e, stream);
}

// -------------------------------------------------------------- plan --

int mslim_cuda_plan_build(const mslim_kernel_config_t *config, const mslim_geometry_t *geometry,
                          int device, mslim_plan_t **plan) {
    if (!plan) return fail(MSLIM_ERR_SHAPE_MISMATCH, "plan pointer is null");
    *plan = nullptr;
    if (int rc = mslim_cuda_config_validate(config, -1)) return rc;
    if (int rc = check_geometry(geometry)) return rc;
    if (config->mode == MSLIM_MODE_REFERENCE)
        return fail(MSLIM_ERR_INVALID_CONFIG, "reference does not compile tiled kernels");
    size_t local = 0;
    if (int rc = mslim_cuda_config_local_bytes(config, geometry->head_dim, &local)) return rc;
    if (!kernel_head_dim(geometry->head_dim))
        return fail(MSLIM_ERR_INVALID_GEOMETRY,
                    "head_dim %u has no sm_100a kernel (multiples of 8 up to 256)",
                    geometry->head_dim);
    DecodeShapeInfo sh;
    if (int rc = decode_shape(geometry, 1, &sh)) return rc;
    int prev;
    if (cudaGetDevice(&prev) != cudaSuccess) return fail(MSLIM_ERR_BACKEND_FAILURE, "no CUDA device");
    if (cudaSetDevice(device) != cudaSuccess) return fail(MSLIM_ERR_UNSUPPORTED_DEVICE, "bad device %d", device);
    int dev;
    int rc = current_device(&dev);
    void *scratch = nullptr;
    if (rc == MSLIM_OK) {
        cudaError_t err = cudaMalloc(&scratch, kPlanScratchBytes);
        if (err != cudaSuccess) rc = cuda_fail(err, "allocate plan split scratch");
        // the decode work counter at its head starts at zero (calls leave it there)
        else if ((err = cudaMemset(scratch, 0, kPlanScratchBytes)) != cudaSuccess)
            rc = cuda_fail(err, "clear plan split scratch");
    }
    cudaSetDevice(prev);
    if (rc) return rc;
    mslim_plan *p = new mslim_plan();
    p->config = *config;
    p->geometry = *geometry;
    p->device = device;
    p->scratch = scratch;
    p->scratch_bytes = kPlanScratchBytes;
    *plan = p;
    return MSLIM_OK;
}

void mslim_cuda_plan_destroy(mslim_plan_t *plan) {
    if (!plan) return;
    int prev;
    if (cudaGetDevice(&prev) == cudaSuccess) {
        cudaSetDevice(plan->device);
        cudaFree(plan->scratch);
        cudaSetDevice(prev);
    }
    delete plan;
}

int mslim_cuda_plan_run(mslim_plan_t *plan, const void *q, size_t q_bytes, const void *k,
                        size_t k_bytes, const void *v, size_t v_bytes, void *out,
                        size_t out_bytes, uint32_t queries, uint32_t prior, void *stream) {
    if (!plan) return fail(MSLIM_ERR_SHAPE_MISMATCH, "plan is null");
    const mslim_geometry_t *g = &plan->geometry;
    if (queries == 0 || queries > 512) return fail(MSLIM_ERR_SHAPE_MISMATCH, "attention query count must be 1..=512");
    const uint64_t history = (uint64_t)prior + queries;
    if (history > 0xffffffffull - 64 || history > 0x7fffffffull)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "attention history exceeds indexing bound");
    const uint64_t qbytes = (uint64_t)queries * g->query_heads * g->head_dim * 2;
    const uint64_t kvbytes = history * g->kv_heads * g->head_dim * 2;
    if (q_bytes < qbytes || out_bytes < qbytes || k_bytes < kvbytes || v_bytes < kvbytes)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "tiled attention buffer is smaller than its declared geometry");
    if (out == q || out == k || out == v)
        return fail(MSLIM_ERR_SHAPE_MISMATCH, "tiled attention output must not alias read-only Q/K/V");
    int prev;
    if (cudaGetDevice(&prev) != cudaSuccess) return fail(MSLIM_ERR_BACKEND_FAILURE, "no CUDA device");
    if (prev != plan->device) return fail(MSLIM_ERR_UNSUPPORTED_DEVICE, "plan belongs to device %d", plan->device);
    int rc;
    if (queries >= mslim::kPrefillMinQueries && mslim::prefill_supported(g->head_dim, g->query_heads / g->kv_heads)) {
        rc = mslim_cuda_prefill_causal(g, q, k, v, out, queries, prior, stream);
        if (rc == MSLIM_OK) plan->prefill_calls++;
    } else {
        DecodeShapeInfo sh;
        if ((rc = decode_shape(g, queries, &sh))) return rc;
        uint32_t st;
        if (plan->config.mode == MSLIM_MODE_SPLIT_KV_EXPERIMENTAL && queries == 1) {
            // tiled_attention.rs:208-213: splits = min(configured splits, history).
            const uint64_t splits = std::min<uint64_t>(plan->config.splits, history);
            st = (uint32_t)(((history + splits - 1) / splits + 63) / 64 * 64);
        } else {
            st = policy_split_tokens((uint64_t)sh.q_blocks * g->kv_heads * sh.head_chunks, history,
                                     decode_slots(kernel_dim_for(g->head_dim)));
        }
        // Keep the partials inside the plan's scratch.
        while (partial_bytes(g, 1, queries, (history + st - 1) / st) > plan->scratch_bytes) st *= 2;
        DecodeCall c{};
        c.g = g;
        c.q = q;
        c.k = k;
        c.v = v;
        c.fixed_tokens = (int)history;
        c.n_seq = 1;
        c.nq = queries;
        c.max_tokens = (uint32_t)history;
        c.split_tokens = st;
        c.workspace = plan->scratch;
        c.workspace_bytes = plan->scratch_bytes;
        c.out = out;
        c.scale_log2 = scale_log2_for(g->head_dim);
        c.kernel_dim = kernel_dim_for(g->head_dim);
        c.stream = static_cast<cudaStream_t>(stream);
        rc = run_decode(c);
        if (rc == MSLIM_OK && (history + st - 1) / st > 1) plan->split_calls++;
    }
    if (rc == MSLIM_OK) plan->calls++;
    return rc;
}

int mslim_cuda_plan_diagnostics(const mslim_plan_t *plan, char *out, size_t len) {
    if (!plan || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null argument");
    const mslim_kernel_config_t &c = plan->config;
    char id[128];
    mslim_cuda_config_id(&c, id, sizeof(id));
    std::string json;
    char buf[2048];
    snprintf(buf, sizeof(buf),
             "{\"settings\":{\"mode\":\"%s\",\"block_queries\":%u,\"block_keys\":%u,"
             "\"work_group\":%u,\"splits\":%u},"
             "\"program_key\":\"sm_100a-%s-d%u-qh%u-kvh%u\","
             "\"numeric_contract\":\"%s\","
             "\"local_bytes_per_group\":%d,\"local_memory_type\":1,"
             "\"preferred_work_group_multiple\":32,"
             "\"global_score_matrix_bytes\":0,\"split_scratch_bytes\":%zu,"
             "\"unused_memory_argument_bytes\":0,"
             "\"dispatches_since_configuration\":%llu,"
             "\"split_dispatches_since_configuration\":%llu,"
             "\"prefill_dispatches_since_configuration\":%llu,"
             "\"split_policy\":\"split-KV over 64-token stages for every query count; "
             "fixed split-order merge\","
             "\"fallback_policy\":\"none: ColdStore pages are read on the device through the "
             "page table\"}",
             mode_serde_name(c.mode), c.block_queries, c.block_keys, c.work_group, c.splits, id,
             plan->geometry.head_dim, plan->geometry.query_heads, plan->geometry.kv_heads,
             is_experimental(c) ? "experimental_online_not_bitwise"
                                : "b200_split_kv_online_fixed_order",
             (int)(3 * 2 * 64 * plan->geometry.head_dim * 2), plan->scratch_bytes,
             (unsigned long long)plan->calls.load(), (unsigned long long)plan->split_calls.load(),
             (unsigned long long)plan->prefill_calls.load());
    json = buf;
    if (json.size() + 1 > len) return fail(MSLIM_ERR_SHAPE_MISMATCH, "output buffer too small");
    memcpy(out, json.c_str(), json.size() + 1);
    return MSLIM_OK;
}

// ----------------------------------------------------------- backend --

int mslim_cuda_backend_create(int device, mslim_backend_t **backend) {
    if (!backend) return fail(MSLIM_ERR_SHAPE_MISMATCH, "backend pointer is null");
    *backend = nullptr;
    int prev;
    if (cudaGetDevice(&prev) != cudaSuccess) return fail(MSLIM_ERR_UNSUPPORTED_DEVICE, "no GPU matches device filter");
    if (cudaSetDevice(device) != cudaSuccess) return fail(MSLIM_ERR_UNSUPPORTED_DEVICE, "no GPU %d", device);
    int dev;
    int rc = current_device(&dev);
    mslim_backend *b = nullptr;
    if (rc == MSLIM_OK) {
        b = new mslim_backend();
        b->device = device;
        cudaError_t err = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
        if (err == cudaSuccess) err = cudaEventCreate(&b->ev0);
        if (err == cudaSuccess) err = cudaEventCreate(&b->ev1);
        if (err != cudaSuccess) {
            rc = cuda_fail(err, "create GPU command queue");
            delete b;
            b = nullptr;
        }
    }
    cudaSetDevice(prev);
    if (rc) return rc;
    *backend = b;
    return MSLIM_OK;
}

void mslim_cuda_backend_destroy(mslim_backend_t *b) {
    if (!b) return;
    int prev;
    if (cudaGetDevice(&prev) == cudaSuccess) {
        cudaSetDevice(b->device);
        cudaStreamSynchronize(b->stream);
        cudaFree(b->buf);
        cudaEventDestroy(b->ev0);
        cudaEventDestroy(b->ev1);
        cudaStreamDestroy(b->stream);
        cudaSetDevice(prev);
    }
    delete b;
}

int mslim_cuda_backend_decode(mslim_backend_t *b, const mslim_geometry_t *geometry,
                              const float *query_host, const void *keys_host,
                              const void *values_host, int dtype, uint32_t tokens,
                              float *out_host) {
    if (!b) return fail(MSLIM_ERR_BACKEND_FAILURE, "backend is null");
    if (int rc = check_geometry(geometry)) return rc;
    if (!query_host || !out_host) return fail(MSLIM_ERR_SHAPE_MISMATCH, "GPU Q shape");
    const uint32_t QH = geometry->query_heads, KVH = geometry->kv_heads, D = geometry->head_dim;
    const size_t qn = (size_t)QH * D;
    for (size_t i = 0; i < qn; ++i)
        if (!std::isfinite(query_host[i])) return fail(MSLIM_ERR_NON_FINITE, "non-finite computation: GPU Q");
    if (tokens == 0) {
        std::fill(out_host, out_host + qn, 0.0f);
        return MSLIM_OK;
    }
    if (dtype < 1 || dtype > 3) return fail(MSLIM_ERR_UNSUPPORTED_DEVICE, "unknown frame format %d", dtype);
    if (!keys_host || !values_host) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null KV frames");
    // The sm_100a kernels read bf16.  FP16/FP32 frames whose values are all
    // exact bf16 values are carried bit for bit.  Otherwise every value is
    // split into two bf16 terms, hi = bf16(f), lo = bf16(f - hi) (exact for
    // FP16, 16 significant bits for FP32), laid side by side along the head
    // dimension ([k_hi | k_lo], [v_hi | v_lo]) with the query duplicated
    // ([q | q]): q'.k' = q.k_hi + q.k_lo, and the two output halves add up to
    // the attention output.  The scale stays 1/sqrt(D) of the caller.
    std::vector<uint16_t> conv_k, conv_v;
    uint32_t DE = D;          // head dimension the kernel sees
    bool split = false;
    if (dtype != 1) {
        const size_t n = (size_t)tokens * KVH * D;
        auto value = [&](const void *src, size_t i) {
            float f;
            if (dtype == 3) {
                memcpy(&f, static_cast<const uint8_t *>(src) + 4 * i, 4);
            } else {
                uint16_t h;
                memcpy(&h, static_cast<const uint8_t *>(src) + 2 * i, 2);
                f = half_bits_to_float(h);
            }
            return f;
        };
        for (int which = 0; which < 2 && !split; ++which) {
            const void *src = which ? values_host : keys_host;
            for (size_t i = 0; i < n; ++i) {
                const float f = value(src, i);
                if (!std::isfinite(f)) return fail(MSLIM_ERR_NON_FINITE, "non-finite computation: KV frame");
                uint32_t bits;
                memcpy(&bits, &f, 4);
                if ((bits & 0xffffu) != 0) {
                    split = true;
                    break;
                }
            }
        }
        if (split && 2 * D > 256)
            return fail(MSLIM_ERR_UNSUPPORTED_DEVICE,
                        "%s frames with values that are not exact bf16 values need head_dim <= 128",
                        dtype == 2 ? "FP16" : "FP32");
        DE = split ? 2 * D : D;
        conv_k.resize((size_t)tokens * KVH * DE);
        conv_v.resize((size_t)tokens * KVH * DE);
        for (int which = 0; which < 2; ++which) {
            const void *src = which ? values_host : keys_host;
            uint16_t *dst = which ? conv_v.data() : conv_k.data();
            for (size_t row = 0; row < (size_t)tokens * KVH; ++row) {
                for (uint32_t d = 0; d < D; ++d) {
                    const float f = value(src, row * D + d);
                    if (!std::isfinite(f)) return fail(MSLIM_ERR_NON_FINITE, "non-finite computation: KV frame");
                    const uint16_t hi = bf16_bits_rne(f);
                    dst[row * DE + d] = hi;
                    if (split) {
                        uint32_t hb = (uint32_t)hi << 16;
                        float hf;
                        memcpy(&hf, &hb, 4);
                        dst[row * DE + D + d] = bf16_bits_rne(f - hf);
                    }
                }
            }
        }
        keys_host = conv_k.data();
        values_host = conv_v.data();
    }
    if (D > 256) return fail(MSLIM_ERR_INVALID_GEOMETRY, "head_dim above 256");
    if (tokens > 0x7fffffffu) return fail(MSLIM_ERR_INVALID_GEOMETRY, "GPU token count > i32");
    // The kernel runs at the next supported head_dim; pad with zeros (zero
    // query/key lanes add nothing to q.k and padded value lanes are dropped).
    const uint32_t KD = DE <= 64 ? 64 : DE <= 128 ? 128 : 256;
    DecodeShapeInfo sh;
    if (int rc = decode_shape(geometry, 1, &sh)) return rc;
    const uint32_t st = policy_split_tokens((uint64_t)KVH * sh.head_chunks, tokens, decode_slots(KD));
    const uint64_t splits = (tokens + st - 1) / st;
    mslim_geometry_t kg = {QH, KVH, KD};
    const size_t q_bytes = (size_t)QH * KD * 4;
    const size_t kv_bytes = (size_t)tokens * KVH * KD * 2;
    const size_t out_bytes = (size_t)QH * KD * 4;
    const size_t ws_bytes = partial_bytes(&kg, 1, 1, splits);
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t total = up(q_bytes) + 2 * up(kv_bytes) + up(out_bytes) + up(ws_bytes);
    int prev;
    if (cudaGetDevice(&prev) != cudaSuccess) return fail(MSLIM_ERR_BACKEND_FAILURE, "no CUDA device");
    cudaSetDevice(b->device);
    auto done = [&](int rc) {
        cudaSetDevice(prev);
        return rc;
    };
    cudaError_t err;
    if (total > b->buf_bytes) {
        cudaFree(b->buf);
        b->buf = nullptr;
        b->buf_bytes = 0;
        err = cudaMalloc(&b->buf, total);
        if (err != cudaSuccess) return done(cuda_fail(err, "allocate KV"));
        b->buf_bytes = total;
    }
    uint8_t *base = static_cast<uint8_t *>(b->buf);
    float *dq = reinterpret_cast<float *>(base);
    uint16_t *dk = reinterpret_cast<uint16_t *>(base + up(q_bytes));
    uint16_t *dv = reinterpret_cast<uint16_t *>(base + up(q_bytes) + up(kv_bytes));
    float *dout = reinterpret_cast<float *>(base + up(q_bytes) + 2 * up(kv_bytes));
    void *dws = base + up(q_bytes) + 2 * up(kv_bytes) + up(out_bytes);
    // the buffer is re-cut per call: the decode workspace's counter head is
    // cleared each time
    err = cudaMemsetAsync(dws, 0, 256, b->stream);
    if (err != cudaSuccess) return done(cuda_fail(err, "clear decode workspace"));
    const auto t0 = std::chrono::steady_clock::now();
    // Host staging with zero padding of the head dimension.
    std::vector<float> qpad((size_t)QH * KD, 0.0f);
    for (uint32_t h = 0; h < QH; ++h) {
        memcpy(&qpad[(size_t)h * KD], query_host + (size_t)h * D, D * 4);
        if (split) memcpy(&qpad[(size_t)h * KD + D], query_host + (size_t)h * D, D * 4);
    }
    err = cudaMemcpyAsync(dq, qpad.data(), q_bytes, cudaMemcpyHostToDevice, b->stream);
    if (err == cudaSuccess && KD == DE) {
        err = cudaMemcpyAsync(dk, keys_host, kv_bytes, cudaMemcpyHostToDevice, b->stream);
        if (err == cudaSuccess) err = cudaMemcpyAsync(dv, values_host, kv_bytes, cudaMemcpyHostToDevice, b->stream);
    } else if (err == cudaSuccess) {
        err = cudaMemcpy2DAsync(dk, KD * 2, keys_host, DE * 2, DE * 2, (size_t)tokens * KVH,
                                cudaMemcpyHostToDevice, b->stream);
        if (err == cudaSuccess)
            err = cudaMemcpy2DAsync(dv, KD * 2, values_host, DE * 2, DE * 2, (size_t)tokens * KVH,
                                    cudaMemcpyHostToDevice, b->stream);
        if (err == cudaSuccess)
            err = cudaMemset2DAsync(dk + DE, KD * 2, 0, (KD - DE) * 2, (size_t)tokens * KVH, b->stream);
        if (err == cudaSuccess)
            err = cudaMemset2DAsync(dv + DE, KD * 2, 0, (KD - DE) * 2, (size_t)tokens * KVH, b->stream);
    }
    if (err != cudaSuccess) return done(cuda_fail(err, "write KV"));
    DecodeCall c{};
    c.g = &kg;
    c.q_f32 = dq;
    c.k = dk;
    c.v = dv;
    c.fixed_tokens = (int)tokens;
    c.n_seq = 1;
    c.nq = 1;
    c.max_tokens = tokens;
    c.split_tokens = st;
    c.workspace = dws;
    c.workspace_bytes = ws_bytes;
    c.out = dout;
    c.out_f32 = dout;
    c.scale_log2 = scale_log2_for(D);
    c.kernel_dim = KD;
    c.stream = b->stream;
    cudaEventRecord(b->ev0, b->stream);
    int rc = run_decode(c);
    if (rc) return done(rc);
    cudaEventRecord(b->ev1, b->stream);
    std::vector<float> opad((size_t)QH * KD);
    err = cudaMemcpyAsync(opad.data(), dout, out_bytes, cudaMemcpyDeviceToHost, b->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(b->stream);
    if (err != cudaSuccess) return done(cuda_fail(err, "GPU output readback"));
    int status = 0;
    mslim_cuda_device_status(b->device, 1, &status);
    if (status) return done(fail(MSLIM_ERR_DEVICE_TIMEOUT, "device wait bound hit during decode"));
    float kernel_ms = 0.f;
    cudaEventElapsedTime(&kernel_ms, b->ev0, b->ev1);
    for (uint32_t h = 0; h < QH; ++h) {
        const float *o = &opad[(size_t)h * KD];
        for (uint32_t d = 0; d < D; ++d) out_host[(size_t)h * D + d] = split ? o[d] + o[D + d] : o[d];
    }
    b->dispatch_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    b->kernel_ms = kernel_ms;
    b->input_kv_bytes = 2 * (size_t)tokens * KVH * D * (dtype == 3 ? 4 : 2);
    b->scratch_bytes = ws_bytes;
    b->output_bytes = qn * 4;
    b->have_timings = true;
    for (size_t i = 0; i < qn; ++i)
        if (!std::isfinite(out_host[i])) return done(fail(MSLIM_ERR_NON_FINITE, "non-finite computation: GPU output"));
    return done(MSLIM_OK);
}

int mslim_cuda_backend_last_timings(const mslim_backend_t *b, char *out, size_t len) {
    if (!b || !out) return fail(MSLIM_ERR_SHAPE_MISMATCH, "null argument");
    if (!b->have_timings) return fail(MSLIM_ERR_BACKEND_FAILURE, "no dispatch yet");
    char buf[512];
    snprintf(buf, sizeof(buf),
             "{\"dispatch_ms\":%.6f,\"kernel_ms\":%.6f,\"input_kv_bytes\":%zu,"
             "\"scratch_bytes\":%zu,\"output_bytes\":%zu}",
             b->dispatch_ms, b->kernel_ms, b->input_kv_bytes, b->scratch_bytes, b->output_bytes);
    if (strlen(buf) + 1 > len) return fail(MSLIM_ERR_SHAPE_MISMATCH, "output buffer too small");
    memcpy(out, buf, strlen(buf) + 1);
    return MSLIM_OK;
}

}  // extern "C"
