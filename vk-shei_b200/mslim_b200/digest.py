"""Validation digest of the logical K/V state, `logical_kv_sha256`.

The reference adapters expose one SHA-256 over the whole K/V state in a
canonical byte order, so that two storage routes (dense device caches and
ColdStore-exact pages) can be compared by content: "mslim-dense-kv-state-v1",
the token count as u64 little-endian, then for every layer its K and then its
V, each as bf16 rows ordered [kv_heads][tokens][head_dim]
(GpuLlm::logical_kv_sha256, src/gpu_llm/mod.rs:1981-2023;
GpuRegionStore::logical_kv_sha256, src/gpu_region_store.rs:338-371;
docs/VALIDATION.md:103-113).

The device writes each tensor in that order (mslim_cuda_kv_canonical_dense /
_paged, one gather kernel per tensor); the bytes are read back and hashed on
the host, as the reference does after its own read-back.
"""
from __future__ import annotations

import hashlib
import struct

KV_DIGEST_TAG = b"mslim-dense-kv-state-v1"


class LogicalKvHasher:
    """Streams the canonical serialisation into SHA-256.  Call add(k, v) once
    per layer in layer order with the layer's canonical K and V bytes."""

    def __init__(self, tokens: int):
        self.h = hashlib.sha256()
        self.h.update(KV_DIGEST_TAG)
        self.h.update(struct.pack("<Q", int(tokens)))

    def add(self, k_bytes: bytes, v_bytes: bytes) -> None:
        self.h.update(k_bytes)
        self.h.update(v_bytes)

    def hexdigest(self) -> str:
        return self.h.hexdigest()


def device_tensor_bytes(torch, t) -> bytes:
    """Host copy of a device bf16 tensor's raw bytes (little-endian u16)."""
    return t.contiguous().view(torch.int16).cpu().numpy().tobytes()
