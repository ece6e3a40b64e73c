"""The logical K/V validation digest (GpuLlm::logical_kv_sha256,
src/gpu_llm/mod.rs:1981-2023; GpuRegionStore::logical_kv_sha256,
src/gpu_region_store.rs:338-371) on the CPU: the oracle's row-by-row
restatement, its vectorised form, and the package's host-side hasher fed the
canonical [kv_heads][tokens][head_dim] bytes the device gather writes."""
import hashlib
import struct

import numpy as np
import pytest


def _layers(rng, n_layers, tokens, kvh, d):
    return [(rng.integers(0, 65536, size=(tokens, kvh, d), dtype=np.uint16),
             rng.integers(0, 65536, size=(tokens, kvh, d), dtype=np.uint16)) for _ in range(n_layers)]


def test_header_only_state_is_the_tag_and_a_zero_count(oracle):
    want = hashlib.sha256(b"mslim-dense-kv-state-v1" + struct.pack("<Q", 0)).hexdigest()
    assert oracle.logical_kv_sha256(0, [], 8, 128) == want
    # layers with no committed tokens add nothing
    assert oracle.logical_kv_sha256(0, [(np.zeros((0, 8, 128), np.uint16),) * 2] * 3, 8, 128) == want


@pytest.mark.parametrize("n_layers,tokens,kvh,d", [(1, 1, 1, 8), (2, 5, 3, 16), (3, 17, 8, 128), (1, 64, 2, 40)])
def test_row_loop_and_transposed_form_agree(oracle, n_layers, tokens, kvh, d):
    rng = np.random.default_rng(n_layers * 100 + tokens)
    layers = _layers(rng, n_layers, tokens, kvh, d)
    assert oracle.logical_kv_sha256(tokens, layers, kvh, d) == oracle.logical_kv_sha256_fast(tokens, layers, kvh, d)


def test_the_byte_order_is_head_major_and_k_before_v(oracle):
    rng = np.random.default_rng(7)
    tokens, kvh, d = 6, 2, 8
    layers = _layers(rng, 2, tokens, kvh, d)
    base = oracle.logical_kv_sha256(tokens, layers, kvh, d)
    # token-major bytes hashed as they lie give another digest
    h = hashlib.sha256(b"mslim-dense-kv-state-v1" + struct.pack("<Q", tokens))
    for k, v in layers:
        h.update(k.tobytes())
        h.update(v.tobytes())
    assert h.hexdigest() != base
    # K and V swapped, or layers swapped, change it
    assert oracle.logical_kv_sha256(tokens, [(v, k) for k, v in layers], kvh, d) != base
    assert oracle.logical_kv_sha256(tokens, layers[::-1], kvh, d) != base
    # rows past `tokens` are not part of the state
    longer = [(np.concatenate([k, k[:2]]), np.concatenate([v, v[:2]])) for k, v in layers]
    assert oracle.logical_kv_sha256(tokens, longer, kvh, d) == base
    # one flipped bit anywhere changes it
    k0 = layers[0][0].copy()
    k0[3, 1, 5] ^= 1
    assert oracle.logical_kv_sha256(tokens, [(k0, layers[0][1])] + layers[1:], kvh, d) != base


def test_package_hasher_matches_the_oracle(oracle):
    from mslim_b200.digest import LogicalKvHasher
    rng = np.random.default_rng(11)
    tokens, kvh, d = 33, 8, 128
    layers = _layers(rng, 4, tokens, kvh, d)
    hasher = LogicalKvHasher(tokens)
    for k, v in layers:
        # what mslim_cuda_kv_canonical_* writes: [kv_heads][tokens][head_dim]
        hasher.add(np.ascontiguousarray(k.transpose(1, 0, 2)).tobytes(),
                   np.ascontiguousarray(v.transpose(1, 0, 2)).tobytes())
    assert hasher.hexdigest() == oracle.logical_kv_sha256(tokens, layers, kvh, d)
