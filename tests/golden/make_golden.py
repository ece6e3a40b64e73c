"""Generates the golden fixtures in this directory from the CPU restatement
(oracle/), which is pinned to the reference's known-answer tests
(tests/test_oracle_kat.py).  The reference itself (Rust + OpenCL) cannot be
built or imported in this image, so its outputs are restated, not captured.

    python tests/golden/make_golden.py

Fixtures (numpy .npz, bf16 as uint16 bits):
  decode_small.npz   GQA decode, QH 8 / KVH 2 / D 128, 200 tokens, RoPE theta 1e4
                     (K at positions 0..199, q at 199), seed 11
  prefill_small.npz  causal prefill, QH 4 / KVH 1 / D 128, 96 queries after a
                     prior of 32 tokens, RoPE theta 5e5, seed 12
  prologue_small.npz RMSNorm (5 x 256, eps 1e-5) and RoPE (3 x 4 x 64, position 17)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "vk-shei_b200"))


def main():
    from oracle import oracle
    from mslim_b200 import workloads as wl

    rng = np.random.default_rng(11)
    qh, kvh, d, t = 8, 2, 128, 200
    q_raw = wl.normal_bf16(rng, (1, qh, d))
    k_raw = wl.normal_bf16(rng, (t, kvh, d))
    v = wl.normal_bf16(rng, (t, kvh, d))
    k = oracle.rope_rows_bf16(k_raw, 0, 10000.0)
    q = oracle.rope_rows_bf16(q_raw, t - 1, 10000.0)[0]
    out = oracle.dense_attention_bf16(qh, kvh, d, oracle.bf16_to_f32(q), k, v, threads=1)
    np.savez_compressed(os.path.join(HERE, "decode_small.npz"), q_raw=q_raw, k_raw=k_raw, v=v, q=q, k=k,
                        out=oracle.bf16_from_f32(out).reshape(qh, d), geometry=np.array([qh, kvh, d, t]))

    rng = np.random.default_rng(12)
    qh, kvh, d, prior, nq = 4, 1, 128, 32, 96
    hist = prior + nq
    q_raw = wl.normal_bf16(rng, (nq, qh, d))
    k_raw = wl.normal_bf16(rng, (hist, kvh, d))
    v = wl.normal_bf16(rng, (hist, kvh, d))
    q = oracle.rope_rows_bf16(q_raw, prior, 500000.0)
    k = oracle.rope_rows_bf16(k_raw, 0, 500000.0)
    out = oracle.causal_prefill_bf16(qh, kvh, d, q, k, v, nq, prior, threads=1)
    np.savez_compressed(os.path.join(HERE, "prefill_small.npz"), q=q, k=k, v=v, out=out,
                        geometry=np.array([qh, kvh, d, nq, prior]))

    rng = np.random.default_rng(13)
    x = wl.normal_bf16(rng, (5, 256))
    w = wl.normal_bf16(rng, (256,), 0.02)
    y = oracle.rms_norm_rows_bf16(x, w, 1e-5)
    r_in = wl.normal_bf16(rng, (3, 4, 64))
    r_out = oracle.rope_rows_bf16(r_in, 17, 10000.0)
    np.savez_compressed(os.path.join(HERE, "prologue_small.npz"), x=x, w=w, y=y, rope_in=r_in, rope_out=r_out)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
