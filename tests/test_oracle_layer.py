"""The decoder-layer pieces of the CPU restatement (native_cpu_adapter.rs:
129-148, 186-191, 486-591) against direct numpy restatements, on the CPU."""
import numpy as np
import pytest

from mslim_b200 import workloads


def _bf16(rng, shape, scale=1.0):
    return workloads.bf16_bits(rng.standard_normal(shape).astype(np.float32) * np.float32(scale))


def _f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_matvec_is_a_sequential_f32_fold_rounded_to_bf16(oracle):
    rng = np.random.default_rng(0)
    w = _bf16(rng, (7, 53), 0.5)
    x = _f32(_bf16(rng, 53))
    got = oracle.matvec_bf16(w, x, threads=2)
    wf = _f32(w).reshape(7, 53)
    want = np.empty(7, np.float32)
    for r in range(7):
        acc = np.float32(-0.0)
        for c in range(53):
            acc = np.float32(acc + np.float32(wf[r, c] * x[c]))
        want[r] = _f32(workloads.bf16_bits(np.array([acc], np.float32)))[0]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_add_residual_rounds_once(oracle):
    rng = np.random.default_rng(1)
    a, b = _f32(_bf16(rng, 1000)), _f32(_bf16(rng, 1000, 3.0))
    got = oracle.add_residual(a, b)
    assert np.array_equal(got, _f32(workloads.bf16_bits(a + b)))


def test_swiglu_formula(oracle):
    rng = np.random.default_rng(2)
    g, u = _f32(_bf16(rng, 5000, 3.0)), _f32(_bf16(rng, 5000))
    got = oracle.swiglu(g, u)
    silu = _f32(workloads.bf16_bits(g / (np.float32(1) + np.exp(-g))))
    want = _f32(workloads.bf16_bits(silu * u))
    # numpy's float32 exp and glibc expf may differ in the last bit
    assert (got == want).mean() > 0.999
    assert np.abs(got - want).max() <= np.abs(want).max() * 2 ** -7


@pytest.mark.parametrize("values,expected", [
    ([1.0, 3.0, 3.0, 2.0], 2),                # last of equal maxima
    ([-0.0, 0.0, -0.0], 1),                   # +0 above -0 (total order)
    ([float("nan"), 1.0], 0),                 # +NaN above everything
    ([-np.inf, -np.inf], 1),
    ([5.0], 0),
])
def test_argmax_last_total_order(oracle, values, expected):
    assert oracle.argmax_last(np.array(values, np.float32)) == expected


def _tiny_layer(rng, zero_out=False):
    hidden, inter, qh, kvh, d = 32, 48, 4, 2, 8
    w = {
        "input_norm": _bf16(rng, hidden, 0.3), "wq": _bf16(rng, (qh * d, hidden), 0.2),
        "wk": _bf16(rng, (kvh * d, hidden), 0.2), "wv": _bf16(rng, (kvh * d, hidden), 0.2),
        "wo": _bf16(rng, (hidden, qh * d), 0.2), "post_norm": _bf16(rng, hidden, 0.3),
        "wg": _bf16(rng, (inter, hidden), 0.2), "wu": _bf16(rng, (inter, hidden), 0.2),
        "wd": _bf16(rng, (hidden, inter), 0.2),
    }
    if zero_out:
        w["wo"][:] = 0
        w["wd"][:] = 0
    return w, (hidden, inter, qh, kvh, d)


def test_layer_with_zero_output_projections_keeps_the_state(oracle):
    rng = np.random.default_rng(3)
    w, (hidden, inter, qh, kvh, d) = _tiny_layer(rng, zero_out=True)
    lo = oracle.LayerOracle(w, hidden, inter, qh, kvh, d, 1e-5, 10000.0, 4, threads=1)
    x = _f32(_bf16(rng, hidden))
    st, *_ = lo.forward(x)
    assert np.array_equal(st, x)  # bf16(x + 0) == x


def test_layer_is_the_composition_of_its_pieces(oracle):
    """forward_token's layer body (native_cpu_adapter.rs:503-577) restated
    with the separately pinned pieces, three tokens deep."""
    rng = np.random.default_rng(4)
    w, (hidden, inter, qh, kvh, d) = _tiny_layer(rng)
    eps, theta = 1e-5, 10000.0
    lo = oracle.LayerOracle(w, hidden, inter, qh, kvh, d, eps, theta, 3, threads=1)
    kc = np.zeros((3, kvh, d), np.uint16)
    vc = np.zeros_like(kc)
    for pos in range(3):
        x = _f32(_bf16(rng, hidden))
        st, q_got, k_got, att_got = lo.forward(x)
        n = oracle.rms_norm(x, _f32(w["input_norm"]), eps)
        q = oracle.matvec_bf16(w["wq"], n, 1)
        k = oracle.matvec_bf16(w["wk"], n, 1)
        v = oracle.matvec_bf16(w["wv"], n, 1)
        q = oracle.apply_rope(q, qh, d, pos, theta)
        k = oracle.apply_rope(k, kvh, d, pos, theta)
        kc[pos] = oracle.bf16_from_f32(k).reshape(kvh, d)
        vc[pos] = oracle.bf16_from_f32(v).reshape(kvh, d)
        att = oracle.dense_attention_bf16(qh, kvh, d, q, kc[:pos + 1], vc[:pos + 1], 1)
        s1 = oracle.add_residual(x, oracle.matvec_bf16(w["wo"], att, 1))
        n2 = oracle.rms_norm(s1, _f32(w["post_norm"]), eps)
        gated = oracle.swiglu(oracle.matvec_bf16(w["wg"], n2, 1), oracle.matvec_bf16(w["wu"], n2, 1))
        want = oracle.add_residual(s1, oracle.matvec_bf16(w["wd"], gated, 1))
        assert np.array_equal(q_got, q) and np.array_equal(k_got, k) and np.array_equal(att_got, att)
        assert np.array_equal(st, want)


def test_lm_head_argmax_is_norm_matvec_argmax(oracle):
    rng = np.random.default_rng(6)
    hidden, vocab = 32, 300
    state = _f32(_bf16(rng, hidden))
    fnorm = _bf16(rng, hidden, 0.5)
    lm = _bf16(rng, (vocab, hidden), 0.3)
    tok, logits = oracle.lm_head_argmax(state, fnorm, lm, 1e-5, threads=1)
    want = oracle.matvec_bf16(lm, oracle.rms_norm(state, _f32(fnorm), 1e-5), 1)
    assert np.array_equal(logits, want)
    assert tok == oracle.argmax_last(want)
