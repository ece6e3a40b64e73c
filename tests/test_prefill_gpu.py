"""GPU parity of the tcgen05/TMEM causal prefill kernel against the CPU path
(the reference prefills by running forward_token per prompt row,
src/native_cpu_adapter.rs:717-784, so row i attends over keys 0..=prior+i with
dense_attention_bf16)."""
import numpy as np
import pytest

from gpu_util import bf16_f32, dev, empty_u16, host_u16, max_abs, torch_mod

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def m():
    import mslim_b200
    mslim_b200.load()
    return mslim_b200


def run_prefill(m, g, q, k, v, queries, prior):
    torch = torch_mod()
    out = empty_u16((queries, g.query_heads, g.head_dim))
    kd, vd = dev(k), dev(v)
    m.prefill_causal(g, dev(q), kd, vd, out, queries, prior)
    torch.cuda.synchronize()
    assert m.device_status(0) == 0
    assert np.array_equal(host_u16(kd), k) and np.array_equal(host_u16(vd), v), "K/V modified"
    return host_u16(out)


CASES = [(1, 0), (5, 0), (128, 0), (129, 0), (200, 37), (256, 256), (64, 1000), (300, 129)]


@pytest.mark.parametrize("geom", [(32, 8, 128), (8, 2, 128), (4, 1, 128), (4, 4, 128), (32, 8, 64), (8, 4, 64),
                                  (16, 8, 64),
                                  # zero-padded head dims (the reference validates 80,
                                  # tiled_attention.rs:414-421) and head_dim 64 with an
                                  # odd group (the single-head kernel at 128)
                                  (4, 2, 80), (12, 4, 80), (4, 4, 64), (6, 2, 64), (8, 8, 96), (4, 2, 120),
                                  # head_dim 256 (64-key tiles; tiled_attention.rs:414-421) and
                                  # 192, zero-padded to it
                                  (4, 1, 256), (8, 2, 256), (6, 2, 256), (4, 2, 192)])
def test_prefill_matches_cpu_path(m, oracle, geom):
    from mslim_b200 import workloads as wl
    qh, kvh, d = geom
    g = m.AttentionGeometry.new(qh, kvh, d)
    rng = np.random.default_rng(qh * 7 + kvh)
    for queries, prior in CASES:
        hist = prior + queries
        q = wl.normal_bf16(rng, (queries, qh, d))
        k = wl.normal_bf16(rng, (hist, kvh, d))
        v = wl.normal_bf16(rng, (hist, kvh, d))
        got = run_prefill(m, g, q, k, v, queries, prior)
        ref = oracle.causal_prefill_bf16(qh, kvh, d, q, k, v, queries, prior)
        err = max_abs(bf16_f32(got), bf16_f32(ref))
        assert err <= TOL, (geom, queries, prior, err)
        again = run_prefill(m, g, q, k, v, queries, prior)
        assert again.tobytes() == got.tobytes(), "repeat run differs"


def test_c2_full_size_matches_cpu_path(m, oracle):
    """C2: S = 2048, 32/8 heads, D = 128, RoPE theta 5e5 on positions 0..2047."""
    from mslim_b200 import workloads as wl
    case = wl.c2_prefill()
    q = oracle.rope_rows_bf16(case.q_raw, 0, case.theta)
    k = oracle.rope_rows_bf16(case.k_raw, 0, case.theta)
    g = m.AttentionGeometry.new(32, 8, 128)
    got = run_prefill(m, g, q, k, case.v, 2048, 0)
    ref = oracle.causal_prefill_bf16(32, 8, 128, q, k, case.v, 2048, 0)
    err = max_abs(bf16_f32(got), bf16_f32(ref))
    assert err <= TOL, err
    # P enters the PV product as bf16 (relative 2^-9), so many outputs land one
    # bf16 ulp from the CPU's f32-weighted sum; none further than the tolerance.
    same = np.mean(got == ref)
    assert same > 0.5, same


@pytest.mark.parametrize("chunk,d", [(64, 128), (128, 128), (192, 128), (256, 128), (192, 64), (128, 80),
                                     (192, 256)])
def test_chunked_prefill_equals_one_shot(m, chunk, d):
    """Prefill in batches of 64/128/192/256 tokens (each chunk at prior =
    tokens so far, over the keys written so far; src/gpu_llm/mod.rs:5435)
    gives the same bits as one call over all 640 tokens: every row runs the
    same key tiles in the same order wherever its query tile starts."""
    from mslim_b200 import workloads as wl
    qh, kvh, S = 32, 8, 640
    g = m.AttentionGeometry.new(qh, kvh, d)
    rng = np.random.default_rng(5435)
    q = wl.normal_bf16(rng, (S, qh, d))
    k = wl.normal_bf16(rng, (S, kvh, d))
    v = wl.normal_bf16(rng, (S, kvh, d))
    whole = run_prefill(m, g, q, k, v, S, 0)
    parts = []
    for start in range(0, S, chunk):
        n = min(chunk, S - start)
        parts.append(run_prefill(m, g, q[start:start + n], k[:start + n], v[:start + n], n, start))
    assert np.concatenate(parts).tobytes() == whole.tobytes()


def test_prefill_rejects_unsupported(m):
    torch = torch_mod()
    b = torch.zeros(64, dtype=torch.int16, device="cuda:0")
    # head dims outside 64..256 or not a multiple of 8 have no prefill kernel
    with pytest.raises(m.InvalidGeometry):
        m.prefill_causal(m.AttentionGeometry.new(4, 4, 32), b, b, b, b.clone(), 1, 0)
    with pytest.raises(m.InvalidGeometry):
        m.prefill_causal(m.AttentionGeometry.new(4, 2, 84), b, b, b, b.clone(), 1, 0)
    with pytest.raises(m.ShapeMismatch):
        m.prefill_causal(m.AttentionGeometry.new(4, 1, 128), b, b, b, b, 1, 0)


def test_fma_pipe_exp2_meets_its_stated_error_bound():
    """The prefill softmax evaluates one exponential pair in eight with a
    polynomial on the FMA pipe (exp2_fma: round-to-integer split, the Remez
    minimax cubic for 2^f on [-1/2, 1/2], exponent-field add).  Over (-126, 0],
    the argument range of a softmax that subtracts the row maximum, its
    relative error against CUDA's exp2f (and against float64) stays within the
    stated 7.5e-5; at -126 and below it returns about 2^-126."""
    import ctypes
    import torch
    from mslim_b200 import _lib
    _lib.lib()
    grid = -126.0 + np.arange(126 * 4096 + 1, dtype=np.float64) / 4096.0      # every 2^-12 step
    rng = np.random.default_rng(9)
    x = np.concatenate([grid[1:], rng.uniform(-126.0, 0.0, 1 << 20), [-1e-30, -0.5, 0.5 - 1.0, -125.5]])
    x = x.astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    outs = [torch.empty_like(xd) for _ in range(3)]
    rc = _lib.lib().mslim_cuda_exp2_eval(xd.data_ptr(), outs[0].data_ptr(), outs[1].data_ptr(),
                                         outs[2].data_ptr(), x.size, None)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    poly, mufu, ref = (o.cpu().numpy().astype(np.float64) for o in outs)
    rel = np.abs(poly / ref - 1.0)
    assert rel.max() <= 7.5e-5, (rel.max(), x[np.argmax(rel)])
    exact = np.exp2(x.astype(np.float64))
    assert np.abs(poly / exact - 1.0).max() <= 7.5e-5 + 2e-7
    assert np.abs(mufu / exact - 1.0).max() <= 1e-6          # the MUFU path, for scale
    low = np.array([-126.0, -130.0, -1000.0], np.float32)
    xl = torch.from_numpy(low).cuda()
    outl = [torch.empty_like(xl) for _ in range(3)]
    assert _lib.lib().mslim_cuda_exp2_eval(xl.data_ptr(), outl[0].data_ptr(), outl[1].data_ptr(),
                                           outl[2].data_ptr(), low.size, None) == 0
    torch.cuda.synchronize()
    got = outl[0].cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got / 2.0 ** -126 - 1.0) <= 2e-4), got
