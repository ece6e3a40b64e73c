"""ctypes binding of libmslim_cuda.so (include/mslim_cuda.h).

There is no fallback: if the native library is missing or does not load, every
entry point raises.  The library is built in-tree by vk-shei_b200/build.py.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmslim_cuda.so")

OK = 0
ERR_INVALID_GEOMETRY = 1
ERR_SHAPE_MISMATCH = 2
ERR_NON_FINITE = 3
ERR_UNSUPPORTED_DEVICE = 4
ERR_BACKEND_FAILURE = 5
ERR_INVALID_CONFIG = 6
ERR_DEVICE_TIMEOUT = 7


class Geometry(ctypes.Structure):
    _fields_ = [("query_heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32)]


class KernelConfig(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int32), ("block_queries", ctypes.c_uint32),
                ("block_keys", ctypes.c_uint32), ("work_group", ctypes.c_uint32),
                ("splits", ctypes.c_uint32)]


class TpComm(ctypes.Structure):
    _fields_ = [("world", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("max_rows", ctypes.c_uint32),
                ("hidden", ctypes.c_uint32), ("data", ctypes.c_void_p * 8), ("flags", ctypes.c_void_p * 8),
                ("epoch", ctypes.c_void_p)]


class RopeConfig(ctypes.Structure):
    _fields_ = [("theta", ctypes.c_float), ("llama3_scaling", ctypes.c_uint32),
                ("factor", ctypes.c_float), ("low_freq_factor", ctypes.c_float),
                ("high_freq_factor", ctypes.c_float), ("original_max_position", ctypes.c_float)]


_lock = threading.Lock()
_lib = None

_vp = ctypes.c_void_p
_u32 = ctypes.c_uint32
_sz = ctypes.c_size_t
_int = ctypes.c_int
_G = ctypes.POINTER(Geometry)
_C = ctypes.POINTER(KernelConfig)
_R = ctypes.POINTER(RopeConfig)

# name -> (restype, argtypes); the ABI test checks this list against the header.
SIGNATURES = {
    "mslim_cuda_last_error": (ctypes.c_char_p, []),
    "mslim_cuda_version": (ctypes.c_char_p, []),
    "mslim_cuda_implementation_digest": (ctypes.c_char_p, []),
    "mslim_cuda_device_status": (_int, [_int, _int, ctypes.POINTER(_int)]),
    "mslim_cuda_kernel_launches": (ctypes.c_uint64, []),
    "mslim_cuda_set_decode_schedule": (_int, [_int]),
    "mslim_cuda_get_decode_schedule": (_int, []),
    "mslim_cuda_geometry_validate": (_int, [_G]),
    "mslim_cuda_config_default": (KernelConfig, []),
    "mslim_cuda_config_validate": (_int, [_C, _int]),
    "mslim_cuda_config_id": (_int, [_C, ctypes.c_char_p, _sz]),
    "mslim_cuda_config_local_bytes": (_int, [_C, _u32, ctypes.POINTER(_sz)]),
    "mslim_cuda_config_decode_scratch_bytes": (_int, [_C, _u32, _u32, ctypes.POINTER(_sz)]),
    "mslim_cuda_plan_build": (_int, [_C, _G, _int, ctypes.POINTER(_vp)]),
    "mslim_cuda_plan_destroy": (None, [_vp]),
    "mslim_cuda_plan_run": (_int, [_vp, _vp, _sz, _vp, _sz, _vp, _sz, _vp, _sz, _u32, _u32, _vp]),
    "mslim_cuda_plan_diagnostics": (_int, [_vp, ctypes.c_char_p, _sz]),
    "mslim_cuda_decode_workspace_bytes": (_int, [_G, _u32, _u32, _u32, ctypes.POINTER(_sz)]),
    "mslim_cuda_decode_split_tokens": (_int, [_G, _u32, _u32, ctypes.POINTER(_u32)]),
    "mslim_cuda_decode_split_tokens_for_lengths": (_int, [_G, _u32, _vp, ctypes.POINTER(_u32)]),
    "mslim_cuda_exp2_eval": (_int, [_vp, _vp, _vp, _vp, _u32, _vp]),
    "mslim_cuda_decode_dense": (_int, [_G, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp, _sz, _vp, _vp]),
    "mslim_cuda_decode_paged": (_int, [_G, _vp, _vp, _vp, _u32, _u32, _vp, _u32, _vp, _u32, _u32, _vp,
                                       _sz, _vp, _vp]),
    "mslim_cuda_decode_paged_static_scratch": (_int, [_G, _vp, _vp, _vp, _u32, _u32, _vp, _u32, _vp, _u32,
                                                      _u32, _vp, _vp]),
    "mslim_cuda_prefill_causal": (_int, [_G, _vp, _vp, _vp, _vp, _u32, _u32, _vp]),
    "mslim_cuda_residual_add": (_int, [_vp, _vp, _vp, ctypes.c_uint64, _vp]),
    "mslim_cuda_swiglu": (_int, [_vp, _vp, _vp, ctypes.c_uint64, _vp]),
    "mslim_cuda_gemv": (_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp]),
    "mslim_cuda_gemv_swiglu": (_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp]),
    "mslim_cuda_page_token_hashes": (_int, [_vp, _u32, _u32, _u32, _u32, _vp, _u32, _u32, _vp, _vp]),
    "mslim_cuda_kv_canonical_dense": (_int, [_vp, _u32, _u32, _u32, _vp, _vp]),
    "mslim_cuda_decode_selected_workspace_bytes": (_int, [_vp, _u32, _u32, _u32, _vp]),
    "mslim_cuda_decode_selected": (_int, [_vp, _vp, _vp, _vp, _u32, _vp, _vp, _vp, _u32, _u32, _u32, _vp,
                                          ctypes.c_size_t, _vp, _vp]),
    "mslim_cuda_decode_selected_paged": (_int, [_vp, _vp, _vp, _vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp, _u32,
                                                _u32, _u32, _vp, ctypes.c_size_t, _vp, _vp]),
    "mslim_cuda_kv_canonical_paged": (_int, [_vp, _u32, _u32, _u32, _u32, _vp, _u32, _u32, _vp, _vp]),
    "mslim_cuda_swiglu_rows": (_int, [_vp, _vp, _u32, _u32, _vp]),
    "mslim_cuda_argmax": (_int, [_vp, _u32, _u32, _int, _vp, _vp]),
    "mslim_cuda_residual_rmsnorm": (_int, [_vp, _vp, _vp, _vp, _u32, _u32, ctypes.c_float, _vp]),
    "mslim_cuda_rope_append_decode_dense_qkv": (_int, [_G, _vp, _vp, _vp, _u32, _R, _vp, _vp, _u32, _vp]),
    "mslim_cuda_gemv_qkv_rope_append_dense": (_int, [_G, _vp, _vp, _u32, _vp, _u32, _R, _vp, _vp, _vp, _u32,
                                                     _vp]),
    "mslim_cuda_gemv_qkv_rope_append_paged": (_int, [_G, _vp, _vp, _u32, _vp, _u32, _R, _vp, _vp, _vp, _u32,
                                                     _u32, _vp, _u32, _vp]),
    "mslim_cuda_rope_append_decode_paged_qkv": (_int, [_G, _vp, _vp, _vp, _u32, _R, _vp, _vp, _u32, _u32, _vp,
                                                       _u32, _vp]),
    "mslim_cuda_rmsnorm": (_int, [_vp, _vp, _vp, _u32, _u32, ctypes.c_float, _vp]),
    "mslim_cuda_rope": (_int, [_vp, _vp, _u32, _u32, _u32, _u32, _R, _vp]),
    "mslim_cuda_rope_append_paged": (_int, [_G, _vp, _vp, _vp, _vp, _u32, _u32, _R, _vp, _vp, _u32, _u32,
                                            _vp, _u32, _vp]),
    "mslim_cuda_rope_append_decode_paged": (_int, [_G, _vp, _vp, _vp, _vp, _vp, _u32, _R, _vp, _vp, _u32,
                                                   _u32, _vp, _u32, _vp]),
    "mslim_cuda_rope_append_decode_dense": (_int, [_G, _vp, _vp, _vp, _vp, _vp, _u32, _R, _vp, _vp, _u32,
                                                   _vp]),
    "mslim_cuda_tp_alloc": (_int, [_sz, ctypes.POINTER(_vp)]),
    "mslim_cuda_tp_free": (_int, [_vp]),
    "mslim_cuda_ipc_handle": (_int, [_vp, _vp]),
    "mslim_cuda_ipc_open": (_int, [_vp, ctypes.POINTER(_vp)]),
    "mslim_cuda_ipc_close": (_int, [_vp]),
    "mslim_cuda_tp_allreduce_rmsnorm": (_int, [ctypes.POINTER(TpComm), _u32, _vp, _vp, _vp, _u32, ctypes.c_float,
                                               _vp]),
    "mslim_cuda_backend_create": (_int, [_int, ctypes.POINTER(_vp)]),
    "mslim_cuda_backend_destroy": (None, [_vp]),
    "mslim_cuda_backend_decode": (_int, [_vp, _G, _vp, _vp, _vp, _int, _u32, _vp]),
    "mslim_cuda_backend_last_timings": (_int, [_vp, ctypes.c_char_p, _sz]),
}


def lib() -> ctypes.CDLL:
    """Loads the native library once; raises if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python vk-shei_b200/build.py` "
                "(there is no CPU fallback for the attention path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
        return L


def last_error() -> str:
    return lib().mslim_cuda_last_error().decode(errors="replace")
