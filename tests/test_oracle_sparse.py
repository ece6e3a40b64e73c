"""CPU checks of the certified sparse decode restatement (epsilon > 0,
assets/gpu_llm.cl:847-964): attention restricted to the selected positions
is the hot-dense attention over those rows; selecting every position is the
dense attention; an omitted row cannot influence the result; the selection
must be strictly increasing."""
import numpy as np
import pytest


def _case(rng, t, kvh, d, qh):
    from mslim_b200 import workloads as wl
    q = rng.standard_normal(qh * d).astype(np.float32)
    k = wl.bf16_bits(rng.standard_normal(t * kvh * d).astype(np.float32)).reshape(t, kvh, d)
    v = wl.bf16_bits(rng.standard_normal(t * kvh * d).astype(np.float32)).reshape(t, kvh, d)
    return oracle_q(q), k, v


def oracle_q(q):
    # queries in the decode path hold bf16-representable values
    from mslim_b200 import workloads as wl
    return (wl.bf16_bits(q).astype(np.uint32) << 16).view(np.float32)


def test_every_position_equals_dense(oracle):
    rng = np.random.default_rng(1)
    q, k, v = _case(rng, 70, 2, 16, 8)
    full = oracle.dense_attention_bf16(8, 2, 16, q, k, v)
    assert np.array_equal(oracle.selected_attention_bf16(8, 2, 16, q, k, v, np.arange(70)), full)


def test_omitted_rows_do_not_matter(oracle):
    rng = np.random.default_rng(2)
    q, k, v = _case(rng, 50, 2, 16, 4)
    sel = np.array([0, 3, 4, 17, 49])
    a = oracle.selected_attention_bf16(4, 2, 16, q, k, v, sel)
    k2, v2 = k.copy(), v.copy()
    omitted = np.setdiff1d(np.arange(50), sel)
    k2[omitted] = 0x7F80            # +inf everywhere else
    v2[omitted] = 0x7FC0            # NaN everywhere else
    assert np.array_equal(oracle.selected_attention_bf16(4, 2, 16, q, k2, v2, sel), a)
    assert np.array_equal(a, oracle.dense_attention_bf16(4, 2, 16, q, np.ascontiguousarray(k[sel]),
                                                         np.ascontiguousarray(v[sel])))


def test_empty_and_unsorted_selections(oracle):
    rng = np.random.default_rng(3)
    q, k, v = _case(rng, 10, 1, 8, 2)
    assert not oracle.selected_attention_bf16(2, 1, 8, q, k, v, []).any()
    with pytest.raises(ValueError):
        oracle.selected_attention_bf16(2, 1, 8, q, k, v, [1, 1, 2])
    with pytest.raises(ValueError):
        oracle.selected_attention_bf16(2, 1, 8, q, k, v, [4, 2])
