"""B200 (sm_100a) attention hot path of M-SLIM behind its attention API.

The compute lives in libmslim_cuda.so (vk-shei_b200/csrc, C ABI in
include/mslim_cuda.h); this package is the host-side mirror of the
reference's interfaces plus seeded workload generators.
"""
from . import _lib
from .attention import (AttentionGeometry, AttentionKernelConfig, AttentionKernelMode, BackendFailure,
                        DeviceTimeout, ExactKvFrames, GpuBackend, GpuEngine, InvalidConfig,
                        InvalidGeometry, NonFinite, PortableError, RopeKernelConfig, ShapeMismatch,
                        TiledAttention, UnsupportedDevice, check, decode_dense, decode_paged, decode_paged_static_scratch,
                        decode_workspace_bytes, decode_split_tokens, decode_split_tokens_for_lengths, device_status, kernel_launches, set_decode_schedule, get_decode_schedule, DECODE_SPLIT_MERGE, DECODE_PERSISTENT, prefill_causal, rmsnorm, rope,
                        rope_append_decode_dense, rope_append_decode_paged, rope_append_paged, residual_add, swiglu,
                        argmax, swiglu_rows, residual_rmsnorm, gemv, gemv_swiglu, interleave_gate_up, page_token_hashes, kv_canonical_dense, kv_canonical_paged,
                        decode_selected, decode_selected_paged, decode_selected_workspace_bytes,
                        rope_append_decode_dense_qkv,
                        rope_append_decode_paged_qkv, gemv_qkv_rope_append_dense,
                        gemv_qkv_rope_append_paged)

LIB_PATH = _lib.LIB_PATH


def load():
    """Loads the native library (raises if it was not built)."""
    return _lib.lib()
