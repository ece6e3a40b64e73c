"""ctypes view of the CPU restatement in ``mslim_oracle.c``.

TEST INFRASTRUCTURE ONLY.  Imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU legs of ``bench.py`` (``cpu_baseline`` and ``--impl reference``)
as the checker / timed CPU reference.  The product library never imports it.

Every function documents the reference source it restates; the C file holds
the operation-by-operation restatement and its citations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "libmslim_oracle.so")
_lock = threading.Lock()
_lib = None

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t

OK, ERR_GEOMETRY, ERR_SHAPE, ERR_NONFINITE = 0, 1, 2, 3


def build() -> str:
    """Compile the restatement with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        src = os.path.join(_HERE, "mslim_oracle.c")
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.mo_bf16_from_f32.argtypes = [ctypes.c_float]
        L.mo_bf16_from_f32.restype = ctypes.c_uint16
        L.mo_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.mo_bf16_to_f32.restype = ctypes.c_float
        L.mo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.mo_f16_to_f32.restype = ctypes.c_float
        L.mo_round_bf16.argtypes = [ctypes.c_float]
        L.mo_round_bf16.restype = ctypes.c_float
        L.mo_bf16_encode.argtypes = [_f32p, _u16p, _sz]
        L.mo_bf16_decode.argtypes = [_u16p, _f32p, _sz]
        L.mo_rms_norm.argtypes = [_f32p, _f32p, _sz, ctypes.c_float, _f32p]
        L.mo_rms_norm_rows_bf16.argtypes = [_u16p, _u16p, _u16p, _sz, _sz, ctypes.c_float]
        L.mo_apply_rope.argtypes = [_f32p, _sz, _sz, _sz, ctypes.c_float]
        L.mo_apply_rope_rows_bf16.argtypes = [_u16p, _u16p, _sz, _sz, _sz, _sz, ctypes.c_float]
        L.mo_softmax.argtypes = [_f32p, _sz]
        L.mo_attention_scale.argtypes = [_sz]
        L.mo_attention_scale.restype = ctypes.c_float
        L.mo_dense_attention_bf16.argtypes = [_sz, _sz, _sz, _f32p, _u16p, _u16p, _sz, _f32p, ctypes.c_int]
        L.mo_dense_attention_bf16.restype = ctypes.c_int
        L.mo_causal_prefill_bf16.argtypes = [_sz, _sz, _sz, _u16p, _u16p, _u16p, _sz, _sz, _u16p, ctypes.c_int]
        L.mo_causal_prefill_bf16.restype = ctypes.c_int
        L.mo_paged_attention_bf16.argtypes = [_sz, _sz, _sz, _f32p, _u16p, _u16p, _i32p, _sz, _sz, _f32p, ctypes.c_int]
        L.mo_paged_attention_bf16.restype = ctypes.c_int
        L.mo_cpu_reference_decode_f64.argtypes = [_sz, _sz, _sz, _f32p, ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.c_int, ctypes.c_int, _sz, _f32p]
        L.mo_cpu_reference_decode_f64.restype = ctypes.c_int
        L.mo_rope_inverse_frequency.argtypes = [ctypes.c_float, ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                                ctypes.c_float, ctypes.c_float, _sz, _sz]
        L.mo_rope_inverse_frequency.restype = ctypes.c_float
        L.mo_gpu_rope_rows_bf16.argtypes = [_u16p, _u16p, _sz, _sz, _sz, _sz, ctypes.c_float, ctypes.c_uint32,
                                            ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float]
        L.mo_fnv1a64.argtypes = [_u8p, _sz]
        L.mo_fnv1a64.restype = ctypes.c_uint64
        L.mo_token_hashes.argtypes = [_u8p, _sz, _sz, _sz, _u64p]
        L.mo_page_from_token_major.argtypes = [_u16p, _u16p, _sz, _sz, _sz]
        L.mo_openmp_max_threads.restype = ctypes.c_int
        L.mo_matvec_bf16.argtypes = [_u16p, _sz, _sz, _f32p, _f32p, ctypes.c_int]
        L.mo_add_residual.argtypes = [_f32p, _f32p, _f32p, _sz]
        L.mo_swiglu.argtypes = [_f32p, _f32p, _f32p, _sz]
        L.mo_argmax_last.argtypes = [_f32p, _sz]
        L.mo_argmax_last.restype = ctypes.c_long
        L.mo_layer_forward_token.argtypes = [ctypes.POINTER(LayerWeightsC), _sz, _sz, _sz, _sz, _sz,
                                             ctypes.c_float, ctypes.c_float, _sz, _u16p, _u16p, _f32p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.mo_layer_forward_token.restype = ctypes.c_int
        L.mo_lm_head_argmax.argtypes = [_f32p, _u16p, _u16p, _sz, _sz, ctypes.c_float, ctypes.c_void_p,
                                        ctypes.c_int]
        L.mo_lm_head_argmax.restype = ctypes.c_long
        _lib = L
        return L


class LayerWeightsC(ctypes.Structure):
    """mo_layer_weights: pointers to one layer's bf16 weights."""
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("input_norm", "wq", "wk", "wv", "wo", "post_norm", "wg", "wu", "wd")]


def max_threads() -> int:
    return int(lib().mo_openmp_max_threads())


# ------------------------------------------------------------------ bf16 --

def bf16_from_f32(x: np.ndarray) -> np.ndarray:
    """half 2.7.1 ``bf16::from_f32`` on every element (native_cpu_adapter.rs:179)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.shape, np.uint16)
    lib().mo_bf16_encode(x, out, x.size)
    return out


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16).reshape(-1)
    out = np.empty(b.shape, np.float32)
    lib().mo_bf16_decode(b, out, b.size)
    return out


# ------------------------------------------------------------- helpers --

def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """native_cpu_adapter.rs:194-204 on one f32 vector."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(weight, np.float32)
    out = np.empty_like(x)
    lib().mo_rms_norm(x, w, x.size, eps, out)
    return out


def rms_norm_rows_bf16(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rms_norm per token row of a bf16 [tokens][hidden] matrix."""
    x = np.ascontiguousarray(x, np.uint16)
    tokens, hidden = x.shape
    y = np.empty_like(x)
    lib().mo_rms_norm_rows_bf16(x, np.ascontiguousarray(w, np.uint16), y, tokens, hidden, eps)
    return y


def apply_rope(values: np.ndarray, heads: int, dim: int, position: int, theta: float) -> np.ndarray:
    """native_cpu_adapter.rs:206-221 (in place on a copy)."""
    v = np.array(values, dtype=np.float32, copy=True).reshape(-1)
    lib().mo_apply_rope(v, heads, dim, position, theta)
    return v


def rope_rows_bf16(x: np.ndarray, start_position: int, theta: float) -> np.ndarray:
    """CPU RoPE on bf16 rows [tokens][heads][dim]; row t at start_position+t."""
    x = np.ascontiguousarray(x, np.uint16)
    tokens, heads, dim = x.shape
    out = np.empty_like(x)
    lib().mo_apply_rope_rows_bf16(x, out, tokens, heads, dim, start_position, theta)
    return out


def gpu_rope_rows_bf16(x: np.ndarray, start_position: int, theta: float, llama3: bool = False,
                       factor: float = 1.0, low: float = 1.0, high: float = 2.0,
                       original_max_position: float = 1.0) -> np.ndarray:
    """assets/gpu_llm.cl:412-456 formula on bf16 rows [tokens][heads][dim]."""
    x = np.ascontiguousarray(x, np.uint16)
    tokens, heads, dim = x.shape
    out = np.empty_like(x)
    lib().mo_gpu_rope_rows_bf16(x, out, tokens, heads, dim, start_position, theta, int(llama3), factor,
                                low, high, original_max_position)
    return out


def rope_inverse_frequency(theta: float, frequency_dim: int, head_dim: int, llama3: bool = False,
                           factor: float = 1.0, low: float = 1.0, high: float = 2.0,
                           original_max_position: float = 1.0) -> float:
    """src/gpu_llm/kernels.rs:50-67."""
    return float(lib().mo_rope_inverse_frequency(theta, int(llama3), factor, low, high,
                                                  original_max_position, frequency_dim, head_dim))


def softmax(values: np.ndarray) -> np.ndarray:
    v = np.array(values, dtype=np.float32, copy=True).reshape(-1)
    lib().mo_softmax(v, v.size)
    return v


# ----------------------------------------------------------- attention --

def dense_attention_bf16(query_heads: int, kv_heads: int, head_dim: int, query_f32: np.ndarray,
                         keys: np.ndarray, values: np.ndarray, threads: int = 0) -> np.ndarray:
    """native_cpu_adapter.rs:253-307.  keys/values bf16 [T][KVH][D]."""
    q = np.ascontiguousarray(query_f32, np.float32).reshape(-1)
    k = np.ascontiguousarray(keys, np.uint16).reshape(-1)
    v = np.ascontiguousarray(values, np.uint16).reshape(-1)
    row = kv_heads * head_dim
    tokens = k.size // row
    if q.size != query_heads * head_dim or k.size != tokens * row or v.size != k.size:
        raise ValueError("geometría KV caliente incompatible")
    out = np.empty(query_heads * head_dim, np.float32)
    rc = lib().mo_dense_attention_bf16(query_heads, kv_heads, head_dim, q, k, v, tokens, out,
                                       threads or max_threads())
    if rc:
        raise ValueError(f"oracle dense attention error {rc}")
    return out


def paged_attention_bf16(query_heads: int, kv_heads: int, head_dim: int, query_f32: np.ndarray,
                         k_pool: np.ndarray, v_pool: np.ndarray, page_table: np.ndarray,
                         page_tokens: int, tokens: int, threads: int = 0) -> np.ndarray:
    """ColdStore-exact branch (native_cpu_adapter.rs:386-455, epsilon 0)."""
    q = np.ascontiguousarray(query_f32, np.float32).reshape(-1)
    out = np.empty(query_heads * head_dim, np.float32)
    rc = lib().mo_paged_attention_bf16(query_heads, kv_heads, head_dim, q,
                                       np.ascontiguousarray(k_pool, np.uint16).reshape(-1),
                                       np.ascontiguousarray(v_pool, np.uint16).reshape(-1),
                                       np.ascontiguousarray(page_table, np.int32).reshape(-1),
                                       page_tokens, tokens, out, threads or max_threads())
    if rc:
        raise ValueError(f"oracle paged attention error {rc}")
    return out


def causal_prefill_bf16(query_heads: int, kv_heads: int, head_dim: int, q: np.ndarray,
                        keys: np.ndarray, values: np.ndarray, queries: int, prior: int,
                        threads: int = 0) -> np.ndarray:
    """Per-row dense attention = CPU prefill (native_cpu_adapter.rs:717-784).
    q bf16 [queries][QH][D]; keys/values bf16 [prior+queries][KVH][D]."""
    qa = np.ascontiguousarray(q, np.uint16).reshape(-1)
    out = np.empty(queries * query_heads * head_dim, np.uint16)
    rc = lib().mo_causal_prefill_bf16(query_heads, kv_heads, head_dim, qa,
                                      np.ascontiguousarray(keys, np.uint16).reshape(-1),
                                      np.ascontiguousarray(values, np.uint16).reshape(-1),
                                      queries, prior, out, threads or max_threads())
    if rc:
        raise ValueError(f"oracle prefill error {rc}")
    return out.reshape(queries, query_heads, head_dim)


DTYPE_CODES = {"bf16": 1, "f16": 2, "f32": 3}


def cpu_reference_decode_f64(query_heads: int, kv_heads: int, head_dim: int, query: np.ndarray,
                             keys: np.ndarray, values: np.ndarray, key_dtype: str = "bf16",
                             value_dtype: str = "bf16") -> np.ndarray:
    """src/portable.rs:575-646 (f64 online softmax).  Raises ArithmeticError
    for the PortableError::NonFinite conditions."""
    q = np.ascontiguousarray(query, np.float32).reshape(-1)
    k = np.ascontiguousarray(keys)
    v = np.ascontiguousarray(values)
    ebytes = {"bf16": 2, "f16": 2, "f32": 4}
    tokens = k.nbytes // (kv_heads * head_dim * ebytes[key_dtype])
    out = np.zeros(query_heads * head_dim, np.float32)
    rc = lib().mo_cpu_reference_decode_f64(query_heads, kv_heads, head_dim, q,
                                           k.ctypes.data_as(ctypes.c_void_p),
                                           v.ctypes.data_as(ctypes.c_void_p),
                                           DTYPE_CODES[key_dtype], DTYPE_CODES[value_dtype], tokens, out)
    if rc == ERR_NONFINITE:
        raise ArithmeticError("non-finite computation")
    if rc:
        raise ValueError(f"invalid geometry ({rc})")
    return out


# ----------------------------------------------------------- ColdStore --

def fnv1a64(data: bytes | np.ndarray) -> int:
    """src/cold_store.rs:909-922."""
    a = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    return int(lib().mo_fnv1a64(np.ascontiguousarray(a), a.size))


def token_hashes(page_payload: np.ndarray, heads: int, tokens: int) -> np.ndarray:
    """src/cold_store.rs:763-781 over a head-major page payload."""
    p = np.ascontiguousarray(page_payload).view(np.uint8).reshape(-1)
    per = p.size // (heads * tokens)
    out = np.empty(tokens, np.uint64)
    lib().mo_token_hashes(p, heads, tokens, per, out)
    return out


def selected_attention_bf16(query_heads: int, kv_heads: int, head_dim: int, q: np.ndarray,
                            k: np.ndarray, v: np.ndarray, positions) -> np.ndarray:
    """Certified sparse decode (epsilon > 0): llm_micro_clear_scores +
    llm_micro_sparse_qk (assets/gpu_llm.cl:847-882) leave every omitted score
    at -inf, so the softmax and PV that follow weigh only the selected
    positions; llm_micro_hot_fused_attention (gpu_llm.cl:899-964) computes the
    same over the selected list directly.  Restated as the CPU hot-dense
    attention over the selected token-major rows, in increasing position
    order (positions must be strictly increasing)."""
    pos = np.asarray(positions, np.int64)
    if pos.size and (np.any(np.diff(pos) <= 0) or pos[0] < 0):
        raise ValueError("selected positions must be strictly increasing")
    if pos.size == 0:
        return np.zeros(query_heads * head_dim, np.float32)
    kk = np.ascontiguousarray(np.asarray(k, np.uint16).reshape(-1, kv_heads, head_dim)[pos])
    vv = np.ascontiguousarray(np.asarray(v, np.uint16).reshape(-1, kv_heads, head_dim)[pos])
    return dense_attention_bf16(query_heads, kv_heads, head_dim, q, kk, vv)


def logical_kv_sha256(tokens: int, layers, kv_heads: int, head_dim: int) -> str:
    """The validation digest of the logical K/V state, restated row by row
    from GpuLlm::logical_kv_sha256 (src/gpu_llm/mod.rs:1981-2023) and
    GpuRegionStore::logical_kv_sha256 (src/gpu_region_store.rs:338-371):
    "mslim-dense-kv-state-v1", tokens as u64 LE, then for each layer (K, V)
    its token-major rows [tokens][kv_heads][head_dim] visited head-major
    (for head: for token: the head_dim bf16 values of that row).
    layers: list of (k, v) uint16 arrays shaped [>= tokens][kv_heads][head_dim].
    SHA-256 is Python's hashlib (FIPS 180-4), as the reference uses the sha2
    crate."""
    import hashlib
    import struct
    h = hashlib.sha256()
    h.update(b"mslim-dense-kv-state-v1")
    h.update(struct.pack("<Q", int(tokens)))
    for k, v in layers:
        for tm in (k, v):
            a = np.ascontiguousarray(tm, np.uint16).reshape(-1, kv_heads, head_dim)[:tokens]
            for head in range(kv_heads):
                for token in range(tokens):
                    h.update(a[token, head].tobytes())
    return h.hexdigest()


def logical_kv_sha256_fast(tokens: int, layers, kv_heads: int, head_dim: int) -> str:
    """logical_kv_sha256 with each tensor transposed to [kv_heads][tokens][head_dim]
    first (the same bytes in the same order; for large states)."""
    import hashlib
    import struct
    h = hashlib.sha256()
    h.update(b"mslim-dense-kv-state-v1")
    h.update(struct.pack("<Q", int(tokens)))
    for k, v in layers:
        for tm in (k, v):
            a = np.ascontiguousarray(tm, np.uint16).reshape(-1, kv_heads, head_dim)[:tokens]
            h.update(np.ascontiguousarray(a.transpose(1, 0, 2)).tobytes())
    return h.hexdigest()


def page_from_token_major(token_major: np.ndarray, kv_heads: int, head_dim: int) -> np.ndarray:
    """src/gpu_region_store.rs:470-483 for one page."""
    t = np.ascontiguousarray(token_major, np.uint16).reshape(-1)
    n = t.size // (kv_heads * head_dim)
    page = np.empty(kv_heads * n * head_dim, np.uint16)
    lib().mo_page_from_token_major(t, page, n, kv_heads, head_dim)
    return page.reshape(kv_heads, n, head_dim)


# ----------------------------------------------------------- decoder layer --

def matvec_bf16(w: np.ndarray, x: np.ndarray, threads: int = 0) -> np.ndarray:
    """native_cpu_adapter.rs:129-148: bf16-rounded rows of w (bf16 bits [rows][cols]) . x."""
    w = np.ascontiguousarray(w, np.uint16)
    rows, cols = w.shape
    out = np.empty(rows, np.float32)
    lib().mo_matvec_bf16(w, rows, cols, np.ascontiguousarray(x, np.float32), out, threads or max_threads())
    return out


def add_residual(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """native_cpu_adapter.rs:186-191."""
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty_like(a)
    lib().mo_add_residual(a, np.ascontiguousarray(b, np.float32), out, a.size)
    return out


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """native_cpu_adapter.rs:553-560."""
    g = np.ascontiguousarray(gate, np.float32)
    out = np.empty_like(g)
    lib().mo_swiglu(g, np.ascontiguousarray(up, np.float32), out, g.size)
    return out


def argmax_last(x: np.ndarray) -> int:
    """native_cpu_adapter.rs:582-587: max_by(total_cmp), last of equal maxima."""
    return int(lib().mo_argmax_last(np.ascontiguousarray(x, np.float32).reshape(-1), np.size(x)))


class LayerOracle:
    """One decoder layer run token by token as forward_token does
    (native_cpu_adapter.rs:486-577), with its hot-dense K/V cache.

    `weights` maps the HF-style names input_norm, wq, wk, wv, wo, post_norm,
    wg, wu, wd to bf16-bit arrays ([out][in] for matrices)."""

    def __init__(self, weights: dict, hidden: int, intermediate: int, query_heads: int, kv_heads: int,
                 head_dim: int, eps: float, theta: float, capacity: int, threads: int = 0):
        self.w = {k: np.ascontiguousarray(v, np.uint16) for k, v in weights.items()}
        self.c = LayerWeightsC(**{k: v.ctypes.data for k, v in self.w.items()})
        self.dims = (hidden, intermediate, query_heads, kv_heads, head_dim)
        self.eps, self.theta = float(eps), float(theta)
        self.k_cache = np.zeros((capacity, kv_heads, head_dim), np.uint16)
        self.v_cache = np.zeros_like(self.k_cache)
        self.position = 0
        self.threads = threads or max_threads()

    def forward(self, state: np.ndarray):
        """Runs the token whose layer input is `state` (f32, bf16 values) at the
        next position; returns (new state, post-RoPE q, post-RoPE k, attention)."""
        hidden, inter, qh, kvh, d = self.dims
        if self.position >= self.k_cache.shape[0]:
            raise ValueError("K/V cache capacity exceeded")
        st = np.array(state, np.float32, copy=True).reshape(-1)
        if st.size != hidden:
            raise ValueError(f"state has {st.size} values, the layer takes {hidden}")
        q = np.empty(qh * d, np.float32)
        k = np.empty(kvh * d, np.float32)
        att = np.empty(qh * d, np.float32)
        rc = lib().mo_layer_forward_token(ctypes.byref(self.c), hidden, inter, qh, kvh, d, self.eps,
                                          self.theta, self.position, self.k_cache, self.v_cache, st,
                                          q.ctypes.data, k.ctypes.data, att.ctypes.data, self.threads)
        if rc != OK:
            raise ValueError(f"layer oracle error {rc}")
        self.position += 1
        return st, q, k, att


def lm_head_argmax(state: np.ndarray, final_norm: np.ndarray, lm_head: np.ndarray, eps: float,
                   threads: int = 0):
    """native_cpu_adapter.rs:579-587: final norm, lm_head, greedy token; returns (token, logits)."""
    lm = np.ascontiguousarray(lm_head, np.uint16)
    vocab, hidden = lm.shape
    logits = np.empty(vocab, np.float32)
    tok = lib().mo_lm_head_argmax(np.ascontiguousarray(state, np.float32),
                                  np.ascontiguousarray(final_norm, np.uint16), lm, hidden, vocab,
                                  float(eps), logits.ctypes.data, threads or max_threads())
    return int(tok), logits
