"""Golden fixtures (tests/golden/, written by make_golden.py from the pinned
CPU restatement): the oracle must keep reproducing them bit for bit (CPU), and
the CUDA path must match them within the attention tolerance (GPU)."""
import os

import numpy as np
import pytest

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def test_oracle_reproduces_decode_fixture(oracle):
    f = load("decode_small.npz")
    qh, kvh, d, t = (int(x) for x in f["geometry"])
    assert np.array_equal(oracle.rope_rows_bf16(f["k_raw"], 0, 10000.0), f["k"])
    assert np.array_equal(oracle.rope_rows_bf16(f["q_raw"], t - 1, 10000.0)[0], f["q"])
    out = oracle.dense_attention_bf16(qh, kvh, d, oracle.bf16_to_f32(f["q"]), f["k"], f["v"], threads=2)
    assert np.array_equal(oracle.bf16_from_f32(out).reshape(qh, d), f["out"])


def test_oracle_reproduces_prefill_fixture(oracle):
    f = load("prefill_small.npz")
    qh, kvh, d, nq, prior = (int(x) for x in f["geometry"])
    out = oracle.causal_prefill_bf16(qh, kvh, d, f["q"], f["k"], f["v"], nq, prior, threads=2)
    assert np.array_equal(out, f["out"])


def test_oracle_reproduces_prologue_fixture(oracle):
    f = load("prologue_small.npz")
    assert np.array_equal(oracle.rms_norm_rows_bf16(f["x"], f["w"], 1e-5), f["y"])
    assert np.array_equal(oracle.rope_rows_bf16(f["rope_in"], 17, 10000.0), f["rope_out"])


@pytest.mark.gpu
def test_cuda_decode_matches_golden():
    import torch

    import mslim_b200 as m
    from gpu_util import bf16_f32, dev, empty_u16, host_u16
    f = load("decode_small.npz")
    qh, kvh, d, t = (int(x) for x in f["geometry"])
    g = m.AttentionGeometry.new(qh, kvh, d)
    ws = torch.zeros(m.decode_workspace_bytes(g, 1, t), dtype=torch.uint8, device="cuda:0")
    out = empty_u16((1, qh, d))
    m.decode_dense(g, dev(f["q"][None]), dev(f["k"][None]), dev(f["v"][None]), dev(np.array([t], np.int32)),
                   1, t, ws, out)
    torch.cuda.synchronize()
    got = bf16_f32(host_u16(out)[0])
    assert np.max(np.abs(got - bf16_f32(f["out"]))) <= 2e-2


@pytest.mark.gpu
def test_cuda_plan_prefill_matches_golden():
    import torch

    import mslim_b200 as m
    from gpu_util import bf16_f32, dev, empty_u16, host_u16
    f = load("prefill_small.npz")
    qh, kvh, d, nq, prior = (int(x) for x in f["geometry"])
    g = m.AttentionGeometry.new(qh, kvh, d)
    plan = m.TiledAttention.build(m.AttentionKernelConfig(mode=m.AttentionKernelMode.STRICT_TILED), g)
    out = empty_u16((nq, qh, d))
    plan.run(dev(f["q"]), dev(f["k"]), dev(f["v"]), out, nq, prior)
    torch.cuda.synchronize()
    assert np.max(np.abs(bf16_f32(host_u16(out)) - bf16_f32(f["out"]))) <= 2e-2
    plan.close()
