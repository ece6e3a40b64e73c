"""Host-side mirror of M-SLIM's attention API over the sm_100a C ABI.

Names, argument meaning and error behaviour follow the reference's Rust
interfaces so its callers map one-to-one:

  AttentionGeometry        src/portable.rs:413-457
  AttentionKernelConfig    src/attention_kernel.rs:6-139
  TiledAttention           src/gpu_llm/tiled_attention.rs:22-293 (build/run/diagnostics)
  GpuEngine                src/gpu_llm/gpu_resources.rs (norm :485, rope :509,
                           attention :583, exact_hot_fused_attention :783) and
                           BatchKernels::{norm, rope, attention} (src/gpu_llm/prefill.rs:292-435)
  ExactKvFrames / GpuBackend   src/portable.rs:461-565, src/gpu_backend.rs:149-377
  PortableError variants   src/portable.rs:39-59

Device buffers are torch CUDA tensors (raw bf16 bits in any 16-bit dtype);
torch is only the allocator and stream source here.  Every compute call goes
to libmslim_cuda.so; nothing runs on the CPU.
"""
from __future__ import annotations

import ctypes
import dataclasses
import enum
import json
from typing import Any

import numpy as np

from . import _lib
from ._lib import Geometry, KernelConfig, RopeConfig


# --------------------------------------------------------------- errors --

class PortableError(Exception):
    """src/portable.rs:39-59."""


class InvalidGeometry(PortableError):
    pass


class ShapeMismatch(PortableError):
    pass


class NonFinite(PortableError):
    pass


class UnsupportedDevice(PortableError):
    pass


class BackendFailure(PortableError):
    pass


class DeviceTimeout(BackendFailure):
    """A bounded device-side wait gave up; the kernel recorded it and returned."""


class InvalidConfig(ValueError):
    """The anyhow error of AttentionKernelConfig::validate."""


_ERRORS = {
    _lib.ERR_INVALID_GEOMETRY: InvalidGeometry,
    _lib.ERR_SHAPE_MISMATCH: ShapeMismatch,
    _lib.ERR_NON_FINITE: NonFinite,
    _lib.ERR_UNSUPPORTED_DEVICE: UnsupportedDevice,
    _lib.ERR_BACKEND_FAILURE: BackendFailure,
    _lib.ERR_INVALID_CONFIG: InvalidConfig,
    _lib.ERR_DEVICE_TIMEOUT: DeviceTimeout,
}


def check(rc: int) -> None:
    if rc != _lib.OK:
        raise _ERRORS.get(rc, BackendFailure)(_lib.last_error())


# ------------------------------------------------------------- geometry --

@dataclasses.dataclass(frozen=True)
class AttentionGeometry:
    query_heads: int
    kv_heads: int
    head_dim: int

    @classmethod
    def new(cls, query_heads: int, kv_heads: int, head_dim: int) -> "AttentionGeometry":
        g = cls(query_heads, kv_heads, head_dim)
        if min(query_heads, kv_heads, head_dim) <= 0 or max(query_heads, kv_heads, head_dim) >= 2 ** 32:
            raise InvalidGeometry("heads and dimension must be positive, q_heads divisible by "
                                  "kv_heads, products finite")
        check(_lib.lib().mslim_cuda_geometry_validate(ctypes.byref(g.c())))
        return g

    def c(self) -> Geometry:
        return Geometry(self.query_heads, self.kv_heads, self.head_dim)

    def kv_head_for_query(self, query_head: int) -> int:
        if query_head >= self.query_heads:
            raise ShapeMismatch("query head out of range")
        return query_head // (self.query_heads // self.kv_heads)

    def query_elements(self) -> int:
        return self.query_heads * self.head_dim

    def kv_elements_per_token(self) -> int:
        return self.kv_heads * self.head_dim


# --------------------------------------------------------------- config --

class AttentionKernelMode(str, enum.Enum):
    """src/attention_kernel.rs:8-14 (serde snake_case)."""
    REFERENCE = "reference"
    STRICT_TILED = "strict_tiled"
    ONLINE_EXPERIMENTAL = "online_experimental"
    SPLIT_KV_EXPERIMENTAL = "split_kv_experimental"

    @property
    def code(self) -> int:
        return ["reference", "strict_tiled", "online_experimental", "split_kv_experimental"].index(self.value)


_CONFIG_FIELDS = ("mode", "block_queries", "block_keys", "work_group", "splits")


@dataclasses.dataclass(frozen=True)
class AttentionKernelConfig:
    """src/attention_kernel.rs:18-139; validation runs in the C library."""
    mode: AttentionKernelMode = AttentionKernelMode.REFERENCE
    block_queries: int = 1
    block_keys: int = 64
    work_group: int = 64
    splits: int = 1

    @classmethod
    def from_json(cls, value: str | dict | None) -> "AttentionKernelConfig":
        """serde(default, deny_unknown_fields)."""
        if value is None:
            return cls()
        d = json.loads(value) if isinstance(value, str) else dict(value)
        unknown = set(d) - set(_CONFIG_FIELDS)
        if unknown:
            raise InvalidConfig(f"unknown field(s) {sorted(unknown)}")
        kw: dict[str, Any] = {}
        for k, v in d.items():
            if k == "mode":
                try:
                    kw[k] = AttentionKernelMode(v)
                except ValueError as e:
                    raise InvalidConfig(f"unknown variant {v!r}") from e
            else:
                if not isinstance(v, int) or isinstance(v, bool) or v < 0:
                    raise InvalidConfig(f"{k} must be a non-negative integer")
                kw[k] = v
        return cls(**kw)

    def to_json(self) -> dict:
        return {"mode": self.mode.value, "block_queries": self.block_queries,
                "block_keys": self.block_keys, "work_group": self.work_group, "splits": self.splits}

    def c(self) -> KernelConfig:
        def u32(x):
            return x if 0 <= x < 2 ** 32 else 2 ** 32 - 1
        return KernelConfig(self.mode.code, u32(self.block_queries), u32(self.block_keys),
                            u32(self.work_group), u32(self.splits))

    def experimental(self) -> bool:
        return self.mode in (AttentionKernelMode.ONLINE_EXPERIMENTAL,
                             AttentionKernelMode.SPLIT_KV_EXPERIMENTAL)

    def validate(self) -> None:
        check(_lib.lib().mslim_cuda_config_validate(ctypes.byref(self.c()), -1))

    def validate_activation(self, allow_experimental: bool) -> None:
        check(_lib.lib().mslim_cuda_config_validate(ctypes.byref(self.c()), int(bool(allow_experimental))))

    def check_snapshot(self, recorded: dict | None) -> None:
        """src/attention_kernel.rs:80-91: legacy snapshots mean reference mode."""
        rec = AttentionKernelConfig.from_json(recorded)
        rec.validate()
        if rec != self:
            raise InvalidConfig("snapshot attention numeric configuration mismatch")

    def id(self) -> str:
        buf = ctypes.create_string_buffer(128)
        check(_lib.lib().mslim_cuda_config_id(ctypes.byref(self.c()), buf, 128))
        return buf.value.decode()

    def local_bytes(self, head_dim: int) -> int:
        out = ctypes.c_size_t()
        check(_lib.lib().mslim_cuda_config_local_bytes(ctypes.byref(self.c()), head_dim, ctypes.byref(out)))
        return out.value

    def decode_scratch_bytes(self, heads: int, head_dim: int) -> int:
        out = ctypes.c_size_t()
        h = heads if heads < 2 ** 32 else 2 ** 32 - 1
        check(_lib.lib().mslim_cuda_config_decode_scratch_bytes(ctypes.byref(self.c()), h, head_dim,
                                                                ctypes.byref(out)))
        return out.value


@dataclasses.dataclass(frozen=True)
class RopeKernelConfig:
    """src/gpu_llm/kernels.rs:16-47."""
    theta: float = 10000.0
    llama3_scaling: int = 0
    factor: float = 1.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 2.0
    original_max_position: float = 1.0

    def c(self) -> RopeConfig:
        return RopeConfig(self.theta, self.llama3_scaling, self.factor, self.low_freq_factor,
                          self.high_freq_factor, self.original_max_position)


# ---------------------------------------------------------------- plumbing --

def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _nbytes(t) -> int:
    return int(t.numel() * t.element_size())


def _stream(stream=None) -> int:
    if stream is not None:
        return int(stream) if isinstance(stream, int) else int(stream.cuda_stream)
    import torch
    return int(torch.cuda.current_stream().cuda_stream)


def device_status(device: int = 0, reset: bool = True) -> int:
    """Synchronises `device` and returns (and clears) its timeout status word."""
    st = ctypes.c_int(0)
    rc = _lib.lib().mslim_cuda_device_status(device, int(reset), ctypes.byref(st))
    if rc not in (_lib.OK, _lib.ERR_DEVICE_TIMEOUT, _lib.ERR_SHAPE_MISMATCH) or \
            (rc != _lib.OK and st.value == 0):
        check(rc)
    return st.value


DECODE_SPLIT_MERGE = 0
DECODE_PERSISTENT = 1


def set_decode_schedule(schedule: int) -> None:
    """Process-wide decode schedule: DECODE_SPLIT_MERGE (default) or
    DECODE_PERSISTENT (same bits)."""
    check(_lib.lib().mslim_cuda_set_decode_schedule(int(schedule)))


def get_decode_schedule() -> int:
    return int(_lib.lib().mslim_cuda_get_decode_schedule())


def kernel_launches() -> int:
    """Kernels the library has launched in this process (captures count once)."""
    return int(_lib.lib().mslim_cuda_kernel_launches())


def decode_workspace_bytes(geometry: AttentionGeometry, n_seq: int, max_tokens: int,
                           split_tokens: int = 0) -> int:
    out = ctypes.c_size_t()
    check(_lib.lib().mslim_cuda_decode_workspace_bytes(ctypes.byref(geometry.c()), n_seq, max_tokens,
                                                       split_tokens, ctypes.byref(out)))
    return out.value


def decode_split_tokens(geometry: AttentionGeometry, n_seq: int, max_tokens: int) -> int:
    """The split size the library picks when split_tokens is 0."""
    out = ctypes.c_uint32()
    check(_lib.lib().mslim_cuda_decode_split_tokens(ctypes.byref(geometry.c()), n_seq, max_tokens,
                                                    ctypes.byref(out)))
    return out.value


def decode_split_tokens_for_lengths(geometry: AttentionGeometry, lengths) -> int:
    """The split size for a batch whose token counts are known on the host
    (fewest waves of split CTAs times the split length)."""
    arr = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
    out = ctypes.c_uint32()
    check(_lib.lib().mslim_cuda_decode_split_tokens_for_lengths(ctypes.byref(geometry.c()), arr.size,
                                                                arr.ctypes.data, ctypes.byref(out)))
    return out.value


def decode_dense(geometry: AttentionGeometry, q, k_cache, v_cache, seq_tokens, n_seq: int,
                 max_tokens: int, workspace, out, split_tokens: int = 0, stream=None) -> None:
    """GpuEngine::attention for a batch of token-major caches."""
    check(_lib.lib().mslim_cuda_decode_dense(
        ctypes.byref(geometry.c()), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(seq_tokens), n_seq,
        max_tokens, split_tokens, _ptr(workspace), _nbytes(workspace), _ptr(out), _stream(stream)))


def decode_selected_workspace_bytes(geometry: AttentionGeometry, n_seq: int, max_selected: int,
                                    split_tokens: int = 0) -> int:
    out = ctypes.c_size_t()
    check(_lib.lib().mslim_cuda_decode_selected_workspace_bytes(ctypes.byref(geometry.c()), n_seq, max_selected,
                                                                split_tokens, ctypes.byref(out)))
    return out.value


def decode_selected(geometry: AttentionGeometry, q, k_cache, v_cache, max_tokens: int, seq_tokens, selected,
                    selected_counts, max_selected: int, n_seq: int, workspace, out, split_tokens: int = 0,
                    stream=None) -> None:
    """Certified sparse decode (epsilon > 0): attention restricted to the
    selected positions, GpuEngine::micro_sparse_scores / micro_hot_attention
    (src/gpu_llm/gpu_resources.rs:656-771)."""
    check(_lib.lib().mslim_cuda_decode_selected(
        ctypes.byref(geometry.c()), _ptr(q), _ptr(k_cache), _ptr(v_cache), max_tokens, _ptr(seq_tokens),
        _ptr(selected), _ptr(selected_counts), max_selected, n_seq, split_tokens, _ptr(workspace),
        _nbytes(workspace), _ptr(out), _stream(stream)))


def decode_selected_paged(geometry: AttentionGeometry, q, k_pool, v_pool, n_pages: int, page_tokens: int,
                          page_table, max_pages_per_seq: int, seq_tokens, selected, selected_counts,
                          max_selected: int, n_seq: int, workspace, out, split_tokens: int = 0, stream=None) -> None:
    """Certified sparse decode with the selected rows gathered straight out
    of ColdStore-exact pages."""
    check(_lib.lib().mslim_cuda_decode_selected_paged(
        ctypes.byref(geometry.c()), _ptr(q), _ptr(k_pool), _ptr(v_pool), n_pages, page_tokens, _ptr(page_table),
        max_pages_per_seq, _ptr(seq_tokens), _ptr(selected), _ptr(selected_counts), max_selected, n_seq,
        split_tokens, _ptr(workspace), _nbytes(workspace), _ptr(out), _stream(stream)))


def decode_paged(geometry: AttentionGeometry, q, k_pool, v_pool, n_pages: int, page_tokens: int,
                 page_table, max_pages_per_seq: int, seq_tokens, n_seq: int, workspace, out,
                 split_tokens: int = 0, stream=None) -> None:
    """Decode over ColdStore-exact pages through a device page table."""
    check(_lib.lib().mslim_cuda_decode_paged(
        ctypes.byref(geometry.c()), _ptr(q), _ptr(k_pool), _ptr(v_pool), n_pages, page_tokens,
        _ptr(page_table), max_pages_per_seq, _ptr(seq_tokens), n_seq, split_tokens, _ptr(workspace),
        _nbytes(workspace), _ptr(out), _stream(stream)))


STATIC_SCRATCH_BYTES = 16 << 20


def decode_paged_static_scratch(geometry: AttentionGeometry, q, k_pool, v_pool, n_pages: int,
                                page_tokens: int, page_table, max_pages_per_seq: int, seq_tokens,
                                n_seq: int, out, split_tokens: int = 0, stream=None) -> None:
    """Paged decode without a workspace: the split partials live in the
    library's 16 MiB static device array (shared by all calls on a device)."""
    check(_lib.lib().mslim_cuda_decode_paged_static_scratch(
        ctypes.byref(geometry.c()), _ptr(q), _ptr(k_pool), _ptr(v_pool), n_pages, page_tokens,
        _ptr(page_table), max_pages_per_seq, _ptr(seq_tokens), n_seq, split_tokens, _ptr(out),
        _stream(stream)))


def prefill_causal(geometry: AttentionGeometry, q, k, v, out, queries: int, prior: int,
                   stream=None) -> None:
    """BatchKernels::attention (src/gpu_llm/prefill.rs:363-435)."""
    check(_lib.lib().mslim_cuda_prefill_causal(ctypes.byref(geometry.c()), _ptr(q), _ptr(k), _ptr(v),
                                               _ptr(out), queries, prior, _stream(stream)))


def rope_append_decode_dense(geometry: AttentionGeometry, q_in, q_out, k_in, v_in, positions, n_seq: int,
                             cfg: RopeKernelConfig, k_cache, v_cache, max_tokens: int, stream=None) -> None:
    """Decode-step RoPE + K/V write into dense token-major caches
    [n_seq][max_tokens][KVH][D] at row positions[s] (run_layer, mod.rs:2099-2116)."""
    check(_lib.lib().mslim_cuda_rope_append_decode_dense(
        ctypes.byref(geometry.c()), _ptr(q_in), _ptr(q_out), _ptr(k_in), _ptr(v_in), _ptr(positions), n_seq,
        ctypes.byref(cfg.c()), _ptr(k_cache), _ptr(v_cache), max_tokens, _stream(stream)))


def residual_add(a, b, out, n: int, stream=None) -> None:
    """GpuEngine::add (src/gpu_llm/gpu_resources.rs:539-559): out = bf16(a + b)."""
    check(_lib.lib().mslim_cuda_residual_add(_ptr(a), _ptr(b), _ptr(out), n, _stream(stream)))


def swiglu(gate, up, out, n: int, stream=None) -> None:
    """GpuEngine::swiglu (src/gpu_llm/gpu_resources.rs:561-581)."""
    check(_lib.lib().mslim_cuda_swiglu(_ptr(gate), _ptr(up), _ptr(out), n, _stream(stream)))


def page_token_hashes(pool, n_pool_pages: int, kv_heads: int, page_tokens: int, head_dim: int, page_ids,
                      n_pages: int, tokens: int, hashes, stream=None) -> None:
    """Per-token FNV-1a of ColdStore pages from the device pool (cold_store.rs:725-742)."""
    check(_lib.lib().mslim_cuda_page_token_hashes(_ptr(pool), n_pool_pages, kv_heads, page_tokens, head_dim,
                                                  _ptr(page_ids), n_pages, tokens, _ptr(hashes), _stream(stream)))


def kv_canonical_dense(cache, kv_heads: int, head_dim: int, tokens: int, out, stream=None) -> None:
    """One session's token-major K (or V) rows -> out [kv_heads][tokens][head_dim]
    (the logical KV digest order, src/gpu_llm/mod.rs:1981-2023)."""
    check(_lib.lib().mslim_cuda_kv_canonical_dense(_ptr(cache), kv_heads, head_dim, tokens, _ptr(out),
                                                   _stream(stream)))


def kv_canonical_paged(pool, n_pages: int, kv_heads: int, page_tokens: int, head_dim: int, page_row,
                       max_pages: int, tokens: int, out, stream=None) -> None:
    """One session's ColdStore-exact pages -> out [kv_heads][tokens][head_dim]
    (src/gpu_region_store.rs:338-371, the read_keys/read_values gather)."""
    check(_lib.lib().mslim_cuda_kv_canonical_paged(_ptr(pool), n_pages, kv_heads, page_tokens, head_dim,
                                                   _ptr(page_row), max_pages, tokens, _ptr(out), _stream(stream)))


def gemv(x, w, y, m: int, n: int, k: int, ldy: int = 0, stream=None) -> None:
    """y[m][n] = bf16(x[m][k] . w[n][k]) for 1..16 rows (the decode
    projections) on the tensor cores; ldy: y's row stride (default n)."""
    check(_lib.lib().mslim_cuda_gemv(_ptr(x), _ptr(w), _ptr(y), m, n, k, ldy or n, _stream(stream)))


def gemv_swiglu(x, w_gu, out, m: int, width: int, k: int, ldo: int = 0, stream=None) -> None:
    """The gate|up projection and SwiGLU in one launch; w_gu in the layout of
    interleave_gate_up (gpu_llm.cl llm_prefill_fused_swiglu_reuse8)."""
    check(_lib.lib().mslim_cuda_gemv_swiglu(_ptr(x), _ptr(w_gu), _ptr(out), m, width, k, ldo or width,
                                            _stream(stream)))


def interleave_gate_up(gate, up):
    """[width][k] gate and up weight rows (torch) -> the [2 * width][k] layout
    of mslim_cuda_gemv_swiglu: blocks of 64 gate rows, each followed by the up
    rows of the same 64 features."""
    import torch
    width, k = gate.shape
    if width % 64 or up.shape != gate.shape:
        raise ShapeMismatch("gate and up must be equal [width][k] with width a multiple of 64")
    blocks = torch.stack([gate.reshape(width // 64, 64, k), up.reshape(width // 64, 64, k)], dim=1)
    return blocks.reshape(2 * width, k).contiguous()


def swiglu_rows(gate_up, out, rows: int, width: int, stream=None) -> None:
    """SwiGLU over rows of a fused [gate | up] projection output."""
    check(_lib.lib().mslim_cuda_swiglu_rows(_ptr(gate_up), _ptr(out), rows, width, _stream(stream)))


def residual_rmsnorm(x, delta, w, y, tokens: int, hidden: int, eps: float, stream=None) -> None:
    """x = bf16(x + delta) in place, then y = RMSNorm(x, w) (one pass)."""
    check(_lib.lib().mslim_cuda_residual_rmsnorm(_ptr(x), _ptr(delta), _ptr(w), _ptr(y), tokens, hidden, eps,
                                                 _stream(stream)))


def rope_append_decode_dense_qkv(geometry: AttentionGeometry, qkv, q_out, positions, n_seq: int,
                                 cfg: RopeKernelConfig, k_cache, v_cache, max_tokens: int, stream=None) -> None:
    """rope_append_decode_dense reading q|k|v from one fused projection output."""
    check(_lib.lib().mslim_cuda_rope_append_decode_dense_qkv(
        ctypes.byref(geometry.c()), _ptr(qkv), _ptr(q_out), _ptr(positions), n_seq, ctypes.byref(cfg.c()),
        _ptr(k_cache), _ptr(v_cache), max_tokens, _stream(stream)))


def rope_append_decode_paged_qkv(geometry: AttentionGeometry, qkv, q_out, positions, n_seq: int,
                                 cfg: RopeKernelConfig, k_pool, v_pool, n_pages: int, page_tokens: int,
                                 page_table, max_pages: int, stream=None) -> None:
    """rope_append_decode_paged reading q|k|v from one fused projection output."""
    check(_lib.lib().mslim_cuda_rope_append_decode_paged_qkv(
        ctypes.byref(geometry.c()), _ptr(qkv), _ptr(q_out), _ptr(positions), n_seq, ctypes.byref(cfg.c()),
        _ptr(k_pool), _ptr(v_pool), n_pages, page_tokens, _ptr(page_table), max_pages, _stream(stream)))


def gemv_qkv_rope_append_dense(geometry: AttentionGeometry, x, w_qkv, k: int, positions, n_seq: int,
                               cfg: RopeKernelConfig, q_out, k_cache, v_cache, max_tokens: int,
                               stream=None) -> None:
    """The decode q|k|v projection with rope_append_decode_dense_qkv in its
    epilogue (head_dim 128)."""
    check(_lib.lib().mslim_cuda_gemv_qkv_rope_append_dense(
        ctypes.byref(geometry.c()), _ptr(x), _ptr(w_qkv), k, _ptr(positions), n_seq, ctypes.byref(cfg.c()),
        _ptr(q_out), _ptr(k_cache), _ptr(v_cache), max_tokens, _stream(stream)))


def gemv_qkv_rope_append_paged(geometry: AttentionGeometry, x, w_qkv, k: int, positions, n_seq: int,
                               cfg: RopeKernelConfig, q_out, k_pool, v_pool, n_pages: int, page_tokens: int,
                               page_table, max_pages: int, stream=None) -> None:
    """The decode q|k|v projection with rope_append_decode_paged_qkv in its
    epilogue (head_dim 128)."""
    check(_lib.lib().mslim_cuda_gemv_qkv_rope_append_paged(
        ctypes.byref(geometry.c()), _ptr(x), _ptr(w_qkv), k, _ptr(positions), n_seq, ctypes.byref(cfg.c()),
        _ptr(q_out), _ptr(k_pool), _ptr(v_pool), n_pages, page_tokens, _ptr(page_table), max_pages,
        _stream(stream)))


def argmax(logits, rows: int, vocab: int, token_ids, ties_to_last: bool = True, stream=None) -> None:
    """GpuEngine::argmax (src/gpu_llm/gpu_resources.rs:1065) / the CPU greedy
    step (src/native_cpu_adapter.rs:582-587): int32 token id per row."""
    check(_lib.lib().mslim_cuda_argmax(_ptr(logits), rows, vocab, int(bool(ties_to_last)), _ptr(token_ids),
                                       _stream(stream)))


def rmsnorm(x, w, y, tokens: int, hidden: int, eps: float, stream=None) -> None:
    check(_lib.lib().mslim_cuda_rmsnorm(_ptr(x), _ptr(w), _ptr(y), tokens, hidden, eps, _stream(stream)))


def rope(inp, out, tokens: int, heads: int, head_dim: int, start_position: int,
         cfg: RopeKernelConfig, stream=None) -> None:
    check(_lib.lib().mslim_cuda_rope(_ptr(inp), _ptr(out), tokens, heads, head_dim, start_position,
                                     ctypes.byref(cfg.c()), _stream(stream)))


def rope_append_paged(geometry: AttentionGeometry, q_in, q_out, k_in, v_in, tokens: int,
                      start_position: int, cfg: RopeKernelConfig, k_pool, v_pool, n_pages: int,
                      page_tokens: int, page_table, max_pages: int, stream=None) -> None:
    check(_lib.lib().mslim_cuda_rope_append_paged(
        ctypes.byref(geometry.c()), _ptr(q_in), _ptr(q_out), _ptr(k_in), _ptr(v_in), tokens,
        start_position, ctypes.byref(cfg.c()), _ptr(k_pool), _ptr(v_pool), n_pages, page_tokens,
        _ptr(page_table), max_pages, _stream(stream)))


def rope_append_decode_paged(geometry: AttentionGeometry, q_in, q_out, k_in, v_in, positions,
                             n_seq: int, cfg: RopeKernelConfig, k_pool, v_pool, n_pages: int,
                             page_tokens: int, page_table, max_pages: int, stream=None) -> None:
    """One new token per session appended at positions[s] (decode step)."""
    check(_lib.lib().mslim_cuda_rope_append_decode_paged(
        ctypes.byref(geometry.c()), _ptr(q_in), _ptr(q_out), _ptr(k_in), _ptr(v_in), _ptr(positions),
        n_seq, ctypes.byref(cfg.c()), _ptr(k_pool), _ptr(v_pool), n_pages, page_tokens, _ptr(page_table),
        max_pages, _stream(stream)))


# ---------------------------------------------------------- TiledAttention --

class TiledAttention:
    """src/gpu_llm/tiled_attention.rs:22-293."""

    def __init__(self, handle: int, config: AttentionKernelConfig, geometry: AttentionGeometry):
        self._h = ctypes.c_void_p(handle)
        self.config = config
        self.geometry = geometry

    @classmethod
    def build(cls, config: AttentionKernelConfig, geometry: AttentionGeometry,
              device: int = 0) -> "TiledAttention":
        h = ctypes.c_void_p()
        check(_lib.lib().mslim_cuda_plan_build(ctypes.byref(config.c()), ctypes.byref(geometry.c()),
                                               device, ctypes.byref(h)))
        return cls(h.value, config, geometry)

    def run(self, q, k, v, output, queries: int, prior: int, geometry: AttentionGeometry | None = None,
            stream=None) -> None:
        g = geometry or self.geometry
        if g != self.geometry:
            raise ShapeMismatch("kernel specialization does not match geometry")
        if queries < 0 or prior < 0 or queries + prior > 0x7fffffff:
            # checked_add and the indexing bound (tiled_attention.rs:182-188; the kernels index in i32)
            raise ShapeMismatch("attention history exceeds the indexing bound")
        check(_lib.lib().mslim_cuda_plan_run(self._h, _ptr(q), _nbytes(q), _ptr(k), _nbytes(k), _ptr(v),
                                             _nbytes(v), _ptr(output), _nbytes(output), queries, prior,
                                             _stream(stream)))

    def diagnostics(self) -> dict:
        buf = ctypes.create_string_buffer(4096)
        check(_lib.lib().mslim_cuda_plan_diagnostics(self._h, buf, 4096))
        return json.loads(buf.value.decode())

    def close(self) -> None:
        if self._h:
            _lib.lib().mslim_cuda_plan_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# -------------------------------------------------------------- GpuEngine --

class GpuEngine:
    """The attention/prologue slice of src/gpu_llm/gpu_resources.rs::GpuEngine.

    The decode workspace is reserved when the engine is built, for histories
    of up to `max_tokens` tokens of `geometry` (the reference sizes its
    Workspace buffers from the model's context capacity when it creates the
    engine, src/gpu_llm/kernels.rs:272-293), so attention() never allocates;
    a longer history is a ShapeMismatch.  set_attention_kernel installs a
    TiledAttention plan, which owns its own scratch."""

    def __init__(self, device: int = 0, geometry: AttentionGeometry | None = None, max_tokens: int = 0):
        import torch
        self.device = device
        self._torch = torch
        self._seq = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")
        self.tiled_attention: TiledAttention | None = None
        self.geometry = geometry
        self.max_tokens = max_tokens
        self._workspace = None
        if geometry is not None and max_tokens > 0:
            # sized for the shortest split the library's policy takes (256
            # tokens), so the policy's split for any history up to max_tokens fits
            self._workspace = torch.zeros(max(decode_workspace_bytes(geometry, 1, max_tokens, 256), 16),
                                          dtype=torch.uint8, device=f"cuda:{device}")

    def set_attention_kernel(self, config: AttentionKernelConfig, geometry: AttentionGeometry,
                             allow_experimental: bool = False) -> None:
        """GpuLlm::set_attention_kernel / install_attention_kernel (src/gpu_llm/mod.rs:539-592)."""
        config.validate_activation(allow_experimental)
        self.tiled_attention = None if config.mode == AttentionKernelMode.REFERENCE else \
            TiledAttention.build(config, geometry, self.device)

    def norm(self, inp, weight, output, hidden: int, eps: float, tokens: int = 1, stream=None) -> None:
        rmsnorm(inp, weight, output, tokens, hidden, eps, stream)

    def rope(self, inp, output, heads: int, head_dim: int, position: int, cfg: RopeKernelConfig,
             tokens: int = 1, stream=None) -> None:
        rope(inp, output, tokens, heads, head_dim, position, cfg, stream)

    def attention(self, query, kv, output, tokens: int, geometry: AttentionGeometry, stream=None) -> None:
        """Decode over a token-major cache of `tokens` rows (gpu_resources.rs:583)."""
        if self.tiled_attention is not None:
            if tokens <= 0:
                raise ShapeMismatch("empty tiled decode")
            self.tiled_attention.run(query, kv[0], kv[1], output, 1, tokens - 1, geometry, stream)
            return
        if tokens <= 0:
            raise ShapeMismatch("atención nativa sin KV")
        cap = _nbytes(kv[0]) // (geometry.kv_elements_per_token() * 2)
        if tokens > cap or _nbytes(kv[1]) < tokens * geometry.kv_elements_per_token() * 2:
            raise ShapeMismatch("KV cache smaller than the token count")
        if self._workspace is None or tokens > self.max_tokens or \
                _nbytes(self._workspace) < decode_workspace_bytes(geometry, 1, tokens):
            raise ShapeMismatch("history beyond the decode workspace reserved when the engine was built")
        self._seq.fill_(tokens)
        decode_dense(geometry, query, kv[0], kv[1], self._seq, 1, tokens, self._workspace, output, 0, stream)

    exact_hot_fused_attention = attention

    def prefill_attention(self, queries_buf, keys, values, output, tokens: int, prior: int,
                          geometry: AttentionGeometry, stream=None) -> None:
        """BatchKernels::attention (src/gpu_llm/prefill.rs:363-435)."""
        if self.tiled_attention is not None:
            self.tiled_attention.run(queries_buf, keys, values, output, tokens, prior, geometry, stream)
            return
        prefill_causal(geometry, queries_buf, keys, values, output, tokens, prior, stream)


# ---------------------------------------------------- isolated backend --

_DTYPES = {"bf16": 1, "f16": 2, "f32": 3}
_DTYPE_BYTES = {"bf16": 2, "f16": 2, "f32": 4}


class ExactKvFrames:
    """src/portable.rs:461-559: [tokens, kv_heads, head_dim] frames, raw bits."""

    def __init__(self, geometry: AttentionGeometry):
        self.geometry = geometry
        self.frames: list[tuple[str, np.ndarray, str, np.ndarray]] = []
        self.tokens = 0

    def append(self, key: np.ndarray, value: np.ndarray, key_dtype: str = "bf16",
               value_dtype: str = "bf16") -> None:
        g = self.geometry
        if key.ndim != 3 or key.shape[1:] != (g.kv_heads, g.head_dim) or key.shape != value.shape:
            raise ShapeMismatch("KV frame needs [tokens, kv_heads, head_dim]")
        self.frames.append((key_dtype, np.ascontiguousarray(key), value_dtype, np.ascontiguousarray(value)))
        self.tokens += key.shape[0]

    def is_empty(self) -> bool:
        return not self.frames

    def decode(self, backend: "GpuBackend", query: np.ndarray) -> np.ndarray:
        return backend.decode(self, query)


class GpuBackend:
    """src/gpu_backend.rs: AttentionBackend on the B200 decode kernel."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(_lib.lib().mslim_cuda_backend_create(device, ctypes.byref(h)))
        self._h = h

    def name(self) -> str:
        return "b200-split-kv-decode"

    def decode(self, cache: ExactKvFrames, query: np.ndarray) -> np.ndarray:
        g = cache.geometry
        q = np.ascontiguousarray(query, np.float32).reshape(-1)
        if q.size != g.query_elements():
            raise ShapeMismatch("GPU Q shape")
        out = np.zeros(g.query_elements(), np.float32)
        if cache.is_empty():
            if not np.all(np.isfinite(q)):
                raise NonFinite("non-finite computation: GPU Q")
            return out
        kd, vd = cache.frames[0][0], cache.frames[0][2]
        if any(f[0] != kd or f[2] != vd for f in cache.frames) or kd != vd:
            raise BackendFailure("GPU backend requires uniform K and V formats across frames")
        k = np.concatenate([f[1].reshape(-1).view(np.uint8) for f in cache.frames])
        v = np.concatenate([f[3].reshape(-1).view(np.uint8) for f in cache.frames])
        check(_lib.lib().mslim_cuda_backend_decode(self._h, ctypes.byref(g.c()), q.ctypes.data,
                                                   k.ctypes.data, v.ctypes.data, _DTYPES[kd],
                                                   cache.tokens, out.ctypes.data))
        return out

    def last_timings(self) -> dict | None:
        buf = ctypes.create_string_buffer(1024)
        if _lib.lib().mslim_cuda_backend_last_timings(self._h, buf, 1024) != _lib.OK:
            return None
        return json.loads(buf.value.decode())

    def close(self) -> None:
        if self._h:
            _lib.lib().mslim_cuda_backend_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
