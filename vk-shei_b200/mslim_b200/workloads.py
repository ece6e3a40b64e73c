"""Seeded synthetic inputs for the benchmark configurations.

The reference quotes no public dataset for this path; every input is i.i.d.
N(0, 1) (weights N(0, 0.02)) rounded to bf16, drawn from numpy PCG64 with the
configuration's seed (GPU-sized tensors come from torch's CUDA generator with
the same seed).  Configurations (BASELINE.json "configs"):

  C1 decode     seed 0: q [32][128], K/V [1024][8][128], RoPE theta 1e4 on K at
                positions 0..1023 and on q at 1023 (the newest token attends
                over its own K, as run_layer appends before attending).
  C2 prefill    seed 1: Q [2048][32][128], K/V [2048][8][128], RoPE theta 5e5
                at positions 0..2047, causal.
  C4 batched    seed 3: 64 sessions with lengths uniform in [4096, 32768],
                K/V in 256-token ColdStore pages under a random physical
                page permutation, one query per session.
"""
from __future__ import annotations

import dataclasses

import numpy as np

QH, KVH, D = 32, 8, 128


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (NaN kept NaN, quiet bit set)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + np.uint32(0x7FFF) + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), r)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def normal_bf16(rng: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    x = rng.standard_normal(shape, dtype=np.float32)
    if scale != 1.0:
        x = x * np.float32(scale)
    return bf16_bits(x)


@dataclasses.dataclass
class DecodeCase:
    q_raw: np.ndarray   # bf16 [QH][D] before RoPE
    k_raw: np.ndarray   # bf16 [T][KVH][D] before RoPE
    v: np.ndarray       # bf16 [T][KVH][D]
    theta: float
    position: int       # position of the query (= T - 1)


def c1_decode(seed: int = 0, tokens: int = 1024, qh: int = QH, kvh: int = KVH,
              d: int = D) -> DecodeCase:
    rng = np.random.default_rng(seed)
    q = normal_bf16(rng, (qh, d))
    k = normal_bf16(rng, (tokens, kvh, d))
    v = normal_bf16(rng, (tokens, kvh, d))
    return DecodeCase(q, k, v, 10000.0, tokens - 1)


@dataclasses.dataclass
class PrefillCase:
    q_raw: np.ndarray   # bf16 [S][QH][D]
    k_raw: np.ndarray   # bf16 [S][KVH][D]
    v: np.ndarray
    theta: float


def c2_prefill(seed: int = 1, seq: int = 2048, qh: int = QH, kvh: int = KVH, d: int = D) -> PrefillCase:
    rng = np.random.default_rng(seed)
    q = normal_bf16(rng, (seq, qh, d))
    k = normal_bf16(rng, (seq, kvh, d))
    v = normal_bf16(rng, (seq, kvh, d))
    return PrefillCase(q, k, v, 500000.0)


@dataclasses.dataclass
class BatchedDecodeLayout:
    lengths: np.ndarray      # int32 [n_seq]
    page_table: np.ndarray   # int32 [n_seq][max_pages] physical page ids
    n_pages: int
    page_tokens: int
    max_pages: int


def c4_layout(seed: int = 3, n_seq: int = 64, lo: int = 4096, hi: int = 32768,
              page_tokens: int = 256) -> BatchedDecodeLayout:
    """Session lengths and the random physical page permutation of C4."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi, size=n_seq, endpoint=True).astype(np.int32)
    pages = (lengths + page_tokens - 1) // page_tokens
    n_pages = int(pages.sum())
    perm = rng.permutation(n_pages).astype(np.int32)
    max_pages = (hi + page_tokens - 1) // page_tokens
    table = np.zeros((n_seq, max_pages), np.int32)
    cursor = 0
    for s in range(n_seq):
        table[s, :pages[s]] = perm[cursor:cursor + pages[s]]
        cursor += pages[s]
    return BatchedDecodeLayout(lengths, table, n_pages, page_tokens, max_pages)


def c4_algorithmic_bytes(layout: BatchedDecodeLayout, qh: int = QH, kvh: int = KVH, d: int = D) -> int:
    """K+V bytes of every session + Q and O rows + the page-table entries read."""
    kv = int(layout.lengths.astype(np.int64).sum()) * kvh * d * 2 * 2
    qo = len(layout.lengths) * qh * d * 2 * 2
    pt = int(((layout.lengths + layout.page_tokens - 1) // layout.page_tokens).sum()) * 4
    return kv + qo + pt
