"""C3: one Llama-3-8B-shaped decoder layer on the
device, 512-token prefill then 8 forced decode steps, against the CPU
restatement of forward_token (oracle/mslim_oracle.c, native_cpu_adapter.rs:
486-577), plus the elementwise layer kernels (residual add, SwiGLU, argmax).

Gates (the north star for C3): dense KV == ColdStore-exact KV bitwise on the
device path; attention outputs within max-abs 2e-2 of the CPU path."""
import numpy as np
import pytest

from gpu_util import bf16_f32, bf16_ulps, dev, host_u16


def u16(t):
    """bf16 (or int16) device tensor -> numpy bf16 bits."""
    import torch
    return host_u16(t.contiguous().view(torch.int16))


pytestmark = pytest.mark.gpu

SEED = 2
PREFILL, DECODE = 512, 8
VOCAB = 128256
TOL = 2e-2


@pytest.fixture(scope="module")
def c3(oracle):
    import torch
    from mslim_b200 import layer
    spec = layer.LayerSpec()
    weights = layer.random_layer_weights(spec, SEED)
    ids = np.random.default_rng(SEED).integers(0, VOCAB, size=PREFILL + DECODE)
    emb = layer.embedding_rows(ids, spec.hidden, SEED)
    x_dev = dev(emb).view(torch.bfloat16)
    cap = PREFILL + DECODE
    runs = {}
    for mode in ("dense", "coldstore"):
        L = layer.DeviceLayer(spec, weights, cap, kv_mode=mode, page_tokens=256, page_seed=SEED)
        out, q_r, k_r, v, attn = L.prefill(x_dev[:PREFILL])
        steps = [L.decode(x_dev[PREFILL + i:PREFILL + i + 1]) for i in range(DECODE)]
        torch.cuda.synchronize()
        runs[mode] = {
            "prefill": [u16(t) for t in (out, q_r, k_r, v, attn)],
            "decode": [[u16(t) for t in s] for s in steps],
        }
        if mode == "dense":
            runs[mode]["k_cache"] = u16(L.k_cache)
            runs[mode]["v_cache"] = u16(L.v_cache)
        runs[mode]["kv_sha256"] = L.logical_kv_sha256()
        del L
    # the CPU path, token by token (forward_token over one layer)
    lo = oracle.LayerOracle(weights, spec.hidden, spec.intermediate, spec.query_heads, spec.kv_heads,
                            spec.head_dim, spec.eps, spec.theta, cap)
    xf = oracle.bf16_to_f32(emb).reshape(emb.shape)
    cpu = [lo.forward(xf[t]) for t in range(cap)]
    return {"spec": spec, "runs": runs, "cpu": cpu}


def test_c3_dense_and_coldstore_are_bit_exact(c3):
    d, c = c3["runs"]["dense"], c3["runs"]["coldstore"]
    for a, b in zip(d["prefill"], c["prefill"]):
        assert np.array_equal(a, b)
    for sd, sc in zip(d["decode"], c["decode"]):
        for a, b in zip(sd, sc):
            assert np.array_equal(a, b), "decode step differs between dense and ColdStore KV"


def test_c3_logical_kv_digest_dense_equals_coldstore(c3, oracle):
    """The adapters' validation digest (src/gpu_llm/mod.rs:1981-2023,
    src/gpu_region_store.rs:338-371) over the 520 committed tokens: the dense
    caches and the ColdStore-exact pages hold the same bf16 K/V, and the
    device-ordered bytes hash like the CPU restatement of the serialisation."""
    d, c = c3["runs"]["dense"], c3["runs"]["coldstore"]
    spec = c3["spec"]
    T = PREFILL + DECODE
    assert d["kv_sha256"] == c["kv_sha256"]
    want = oracle.logical_kv_sha256_fast(T, [(d["k_cache"], d["v_cache"])], spec.kv_heads, spec.head_dim)
    assert d["kv_sha256"] == want


def test_c3_attention_matches_cpu_on_the_device_inputs(c3, oracle):
    """The device attention against the CPU hot-dense attention fed the very
    same post-RoPE q and K/V (isolates the attention kernels)."""
    spec = c3["spec"]
    d = c3["runs"]["dense"]
    _, q_r, k_r, v, attn = d["prefill"]
    qh, kvh, hd = spec.query_heads, spec.kv_heads, spec.head_dim
    ref = oracle.causal_prefill_bf16(qh, kvh, hd, q_r.reshape(PREFILL, qh, hd), k_r.reshape(PREFILL, kvh, hd),
                                     v.reshape(PREFILL, kvh, hd), PREFILL, 0)
    err = np.abs(bf16_f32(attn).reshape(ref.shape) - bf16_f32(ref)).max()
    print(f"C3 prefill attention vs CPU on device inputs: max-abs {err:.3g}")
    assert err <= TOL, f"prefill attention max-abs {err}"
    for i, (_, q_step, a_step) in enumerate(d["decode"]):
        T = PREFILL + i + 1
        ref = oracle.dense_attention_bf16(qh, kvh, hd, bf16_f32(q_step).reshape(-1),
                                          d["k_cache"][:T], d["v_cache"][:T])
        err = np.abs(bf16_f32(a_step).reshape(-1) - ref).max()
        print(f"C3 decode step {i} attention vs CPU on device inputs: max-abs {err:.3g}")
        assert err <= TOL, f"decode step {i} attention max-abs {err}"


def test_c3_layer_matches_cpu_path(c3):
    """End to end: every token's attention output of the device layer against
    the CPU decoder's own (its own projections, RoPE and caches)."""
    d = c3["runs"]["dense"]
    cpu = c3["cpu"]
    attn_dev = np.concatenate([bf16_f32(d["prefill"][4]).reshape(PREFILL, -1)] +
                              [bf16_f32(s[2]).reshape(1, -1) for s in d["decode"]])
    attn_cpu = np.stack([c[3] for c in cpu])
    err = np.abs(attn_dev - attn_cpu).max()
    print(f"C3 attention outputs vs the CPU path (all 520 tokens): max-abs {err:.3g}")
    assert err <= TOL, f"attention outputs max-abs {err} against the CPU path"
    state_dev = np.concatenate([bf16_f32(d["prefill"][0]).reshape(PREFILL, -1)] +
                               [bf16_f32(s[0]).reshape(1, -1) for s in d["decode"]])
    state_cpu = np.stack([c[0] for c in cpu])
    # layer outputs: GEMM vs sequential sums differ in rounding only
    rel = np.abs(state_dev - state_cpu).max() / np.abs(state_cpu).max()
    print(f"C3 layer outputs vs the CPU path: max-abs {np.abs(state_dev - state_cpu).max():.3g}, "
          f"relative to the largest output {rel:.3g}")
    assert rel < 2e-2, f"layer output relative max-abs {rel}"


# ------------------------------------------------------ elementwise ops --

def _rand_bf16(rng, n, scale=1.0):
    from mslim_b200 import workloads
    return workloads.bf16_bits(rng.standard_normal(n).astype(np.float32) * np.float32(scale))


@pytest.mark.parametrize("n", [1, 7, 8, 4096, 14336 * 3 + 5])
def test_residual_add_bitwise(n, oracle):
    import torch
    import mslim_b200 as m
    rng = np.random.default_rng(n)
    a, b = _rand_bf16(rng, n), _rand_bf16(rng, n)
    ta, tb = dev(a), dev(b)
    out = torch.empty_like(ta)
    m.residual_add(ta, tb, out, n)
    ref = oracle.bf16_from_f32(oracle.add_residual(oracle.bf16_to_f32(a), oracle.bf16_to_f32(b)))
    assert np.array_equal(u16(out), ref)


@pytest.mark.parametrize("n", [1, 9, 14336, 14336 * 8 + 3])
def test_swiglu_matches_cpu(n, oracle):
    import torch
    import mslim_b200 as m
    rng = np.random.default_rng(n + 1)
    g, u = _rand_bf16(rng, n, 3.0), _rand_bf16(rng, n)
    tg, tu = dev(g), dev(u)
    out = torch.empty_like(tg)
    m.swiglu(tg, tu, out, n)
    ref = oracle.bf16_from_f32(oracle.swiglu(oracle.bf16_to_f32(g), oracle.bf16_to_f32(u)))
    got = u16(out)
    # expf differs from glibc's in the last f32 bit at most; after the two bf16
    # roundings almost every output is identical and none is more than 1 ulp off
    ulps = bf16_ulps(got, ref)
    assert ulps.max() <= 1
    assert (ulps == 0).mean() > 0.999


def _argmax_case(oracle, logits_u16, ties_to_last):
    import torch
    import mslim_b200 as m
    rows, vocab = logits_u16.shape
    t = dev(np.ascontiguousarray(logits_u16))
    ids = torch.full((rows,), -7, dtype=torch.int32, device="cuda:0")
    m.argmax(t, rows, vocab, ids, ties_to_last=ties_to_last)
    return ids.cpu().numpy()


def test_argmax_last_matches_cpu_max_by(oracle):
    rng = np.random.default_rng(5)
    rows = _rand_bf16(rng, 8 * VOCAB, 1.3).reshape(8, VOCAB)
    got = _argmax_case(oracle, rows, True)
    want = [oracle.argmax_last(oracle.bf16_to_f32(r)) for r in rows]
    assert list(got) == want


def test_argmax_tie_rules(oracle):
    one, zero, nzero = 0x3F80, 0x0000, 0x8000
    nan = 0x7FC0
    cases = np.array([
        [0xBF80, one, 0x4000, one, 0x4000, 0xC000],    # 2.0 at 2 and 4
        [one] * 6,                                      # all equal
        [nzero, zero, nzero, zero, nzero, nzero],       # -0 vs +0
        [one, nan, 0x4000, one, 0x3F00, nan],           # NaN present
    ], np.uint16)
    last = _argmax_case(oracle, cases, True)
    first = _argmax_case(oracle, cases, False)
    # CPU path: f32::total_cmp, last of equal maxima (NaN is the largest)
    assert list(last) == [oracle.argmax_last(oracle.bf16_to_f32(r)) for r in cases] == [4, 5, 3, 5]
    # OpenCL llm_argmax: float order, first of equal maxima, NaN never chosen
    assert list(first) == [2, 0, 0, 2]


# ----------------------------------------------------- fused decode steps --

def test_residual_rmsnorm_is_add_then_norm_bitwise():
    import torch
    import mslim_b200 as m
    rng = np.random.default_rng(11)
    for tokens, hidden in [(8, 4096), (3, 136), (1, 4000), (5, 12)]:
        x, d = _rand_bf16(rng, tokens * hidden), _rand_bf16(rng, tokens * hidden, 0.5)
        w = _rand_bf16(rng, hidden)
        tx1, tx2, td, tw = dev(x), dev(x), dev(d), dev(w)
        y1, y2 = torch.empty_like(tx1), torch.empty_like(tx1)
        m.residual_add(tx1, td, tx1, tokens * hidden)
        m.rmsnorm(tx1, tw, y1, tokens, hidden, 1e-5)
        m.residual_rmsnorm(tx2, td, tw, y2, tokens, hidden, 1e-5)
        assert np.array_equal(u16(tx1), u16(tx2)) and np.array_equal(u16(y1), u16(y2))


def test_swiglu_rows_matches_split_buffers_bitwise():
    import torch
    import mslim_b200 as m
    rng = np.random.default_rng(12)
    rows, width = 8, 14336
    gu = _rand_bf16(rng, rows * 2 * width, 3.0).reshape(rows, 2 * width)
    out = torch.empty((rows, width), dtype=torch.int16, device="cuda:0")
    m.swiglu_rows(dev(gu), out, rows, width)
    ref = torch.empty_like(out)
    g, u = dev(np.ascontiguousarray(gu[:, :width])), dev(np.ascontiguousarray(gu[:, width:]))
    m.swiglu(g, u, ref, rows * width)
    assert np.array_equal(u16(out), u16(ref))


@pytest.mark.parametrize("paged", [False, True])
def test_fused_qkv_append_matches_separate_inputs(paged):
    import torch
    import mslim_b200 as m
    from mslim_b200 import attention as att
    rng = np.random.default_rng(13)
    QH, KVH, D, B, T = 32, 8, 128, 4, 600
    g = att.AttentionGeometry.new(QH, KVH, D)
    cfg = att.RopeKernelConfig(theta=500000.0)
    qkv = _rand_bf16(rng, B * (QH + 2 * KVH) * D).reshape(B, -1)
    q = np.ascontiguousarray(qkv[:, :QH * D])
    k = np.ascontiguousarray(qkv[:, QH * D:(QH + KVH) * D])
    v = np.ascontiguousarray(qkv[:, (QH + KVH) * D:])
    pos = dev(np.array([0, 17, 255, 599], np.int32))
    outs = []
    for fused in (False, True):
        q_out = torch.empty((B, QH * D), dtype=torch.int16, device="cuda:0")
        if paged:
            pt, mp = 256, 3
            table = dev(np.random.default_rng(1).permutation(B * mp).astype(np.int32).reshape(B, mp))
            kc = torch.zeros((B * mp, KVH, pt, D), dtype=torch.int16, device="cuda:0")
            vc = torch.zeros_like(kc)
            if fused:
                m.rope_append_decode_paged_qkv(g, dev(qkv), q_out, pos, B, cfg, kc, vc, B * mp, pt, table, mp)
            else:
                m.rope_append_decode_paged(g, dev(q), q_out, dev(k), dev(v), pos, B, cfg, kc, vc, B * mp, pt,
                                           table, mp)
        else:
            kc = torch.zeros((B, T, KVH, D), dtype=torch.int16, device="cuda:0")
            vc = torch.zeros_like(kc)
            if fused:
                m.rope_append_decode_dense_qkv(g, dev(qkv), q_out, pos, B, cfg, kc, vc, T)
            else:
                m.rope_append_decode_dense(g, dev(q), q_out, dev(k), dev(v), pos, B, cfg, kc, vc, T)
        outs.append([u16(q_out), u16(kc), u16(vc)])
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    assert m.device_status(0) == 0


def _qkv_rope_two_ways(m, g, cfg, x, w, pos, k, paged, T=600, pt=256):
    """(q_out, K store, V store) of the fused q|k|v projection + RoPE + append
    and of the plain projection followed by the q|k|v append, each from
    zeroed stores and a poisoned q_out; the fused one twice."""
    import torch
    B = x.shape[0]
    QH, KVH = g.query_heads, g.kv_heads
    mp = -(-T // pt)
    table = dev(np.random.default_rng(1).permutation(B * mp).astype(np.int32).reshape(B, mp))
    runs = []
    for form in ("two-step", "fused", "fused"):
        q_out = torch.full((B, QH * 128), 0x7FC1, dtype=torch.int16, device="cuda:0")
        shape = (B * mp, KVH, pt, 128) if paged else (B, T, KVH, 128)
        kc = torch.zeros(shape, dtype=torch.int16, device="cuda:0")
        vc = torch.zeros_like(kc)
        if form == "fused":
            if paged:
                m.gemv_qkv_rope_append_paged(g, x, w, k, pos, B, cfg, q_out, kc, vc, B * mp, pt, table, mp)
            else:
                m.gemv_qkv_rope_append_dense(g, x, w, k, pos, B, cfg, q_out, kc, vc, T)
        else:
            qkv = torch.empty((B, (QH + 2 * KVH) * 128), dtype=torch.int16, device="cuda:0")
            m.gemv(x, w, qkv, B, (QH + 2 * KVH) * 128, k)
            if paged:
                m.rope_append_decode_paged_qkv(g, qkv, q_out, pos, B, cfg, kc, vc, B * mp, pt, table, mp)
            else:
                m.rope_append_decode_dense_qkv(g, qkv, q_out, pos, B, cfg, kc, vc, T)
        status = m.device_status(0)
        runs.append(([u16(q_out), u16(kc), u16(vc)], status))
    return runs


@pytest.mark.parametrize("paged", [False, True])
@pytest.mark.parametrize("qh,kvh,b,k", [(32, 8, 8, 4096), (16, 4, 8, 4096), (4, 1, 8, 4096), (32, 8, 3, 512),
                                        (8, 2, 16, 72)])
def test_gemv_qkv_rope_append_equals_projection_then_append(paged, qh, kvh, b, k):
    """The decode q|k|v projection with RoPE + K/V append in its epilogue
    writes the bits of the projection followed by the q|k|v append kernel:
    q_out, the K and the V store (dense caches or ColdStore pages), on two
    calls in a row; at C5's TP 1, 2 and 8 head counts and small shapes."""
    import mslim_b200 as m
    from mslim_b200 import attention as att
    rng = np.random.default_rng(qh * 17 + b + k)
    g = att.AttentionGeometry.new(qh, kvh, 128)
    cfg = att.RopeKernelConfig(theta=500000.0)
    x = dev(_rand_bf16(rng, b * k).reshape(b, k))
    w = dev(_rand_bf16(rng, (qh + 2 * kvh) * 128 * k, 0.02).reshape(-1, k))
    pos = dev(rng.integers(0, 600, size=b).astype(np.int32))
    runs = _qkv_rope_two_ways(m, g, cfg, x, w, pos, k, paged)
    (want, s0), (got, s1), (again, s2) = runs
    assert s0 == s1 == s2 == 0
    for a, c, d in zip(want, got, again):
        assert np.array_equal(a, c) and np.array_equal(c, d)


@pytest.mark.parametrize("paged", [False, True])
def test_gemv_qkv_rope_append_skips_rows_outside_the_store(paged):
    """A position outside the store (and, paged, a page id outside the pool)
    writes nothing for that row, in the fused form as in the two-step one,
    and the status word reports it; the other rows are written."""
    import mslim_b200 as m
    from mslim_b200 import attention as att
    rng = np.random.default_rng(29)
    qh, kvh, b, k = 8, 2, 4, 256
    g = att.AttentionGeometry.new(qh, kvh, 128)
    cfg = att.RopeKernelConfig(theta=10000.0)
    x = dev(_rand_bf16(rng, b * k).reshape(b, k))
    w = dev(_rand_bf16(rng, (qh + 2 * kvh) * 128 * k, 0.02).reshape(-1, k))
    pos = dev(np.array([5, -1, 800, 599], np.int32))      # rows 1 and 2: outside the 600 / 768-token stores
    runs = _qkv_rope_two_ways(m, g, cfg, x, w, pos, k, paged)
    (want, s0), (got, s1), _ = runs
    assert s0 != 0 and s1 != 0
    for a, c in zip(want, got):
        assert np.array_equal(a, c)
    q_out = got[0]
    assert (q_out[1] == 0x7FC1).all() and (q_out[2] == 0x7FC1).all() and not (q_out[0] == 0x7FC1).all()


def test_gemv_qkv_rope_append_rejects_other_head_dims_and_batches():
    import torch
    import mslim_b200 as m
    from mslim_b200 import attention as att
    cfg = att.RopeKernelConfig(theta=10000.0)
    x = torch.zeros((17, 64), dtype=torch.int16, device="cuda:0")
    w = torch.zeros((6 * 128, 64), dtype=torch.int16, device="cuda:0")
    q_out = torch.zeros((17, 4 * 128), dtype=torch.int16, device="cuda:0")
    kc = torch.zeros((17, 16, 1, 128), dtype=torch.int16, device="cuda:0")
    pos = torch.zeros(17, dtype=torch.int32, device="cuda:0")
    with pytest.raises(m.InvalidGeometry):
        m.gemv_qkv_rope_append_dense(att.AttentionGeometry.new(4, 1, 64), x, w, 64, pos, 4, cfg, q_out, kc, kc, 16)
    with pytest.raises(m.ShapeMismatch):
        m.gemv_qkv_rope_append_dense(att.AttentionGeometry.new(4, 1, 128), x, w, 64, pos, 17, cfg, q_out, kc, kc, 16)
    assert m.device_status(0) == 0


@pytest.mark.parametrize("paged", [False, True])
@pytest.mark.parametrize("qh,kvh,d", [(32, 8, 128), (4, 1, 128), (8, 2, 80), (2, 2, 256)])
def test_rope_append_vector_and_scalar_forms_agree(paged, qh, kvh, d):
    """The launcher takes the 16-byte form when head_dim % 16 == 0 and every
    row is 16-byte aligned; an input view one element into its buffer forces
    the element-wise form.  Both must write the same bits."""
    import torch
    import mslim_b200 as m
    from mslim_b200 import attention as att
    rng = np.random.default_rng(qh * 31 + d)
    B, T = 5, 300
    g = att.AttentionGeometry.new(qh, kvh, d)
    cfg = att.RopeKernelConfig(theta=500000.0)
    width = (qh + 2 * kvh) * d
    qkv = _rand_bf16(rng, B * width).reshape(B, width)
    pos = dev(np.array([0, 1, 77, 255, 299], np.int32))
    outs = []
    for misaligned in (False, True):
        buf = torch.zeros(B * width + 8, dtype=torch.int16, device="cuda:0")
        off = 1 if misaligned else 0
        buf[off:off + B * width].copy_(dev(qkv).view(-1))
        src = buf[off:off + B * width].view(B, width)
        q_out = torch.empty((B, qh * d), dtype=torch.int16, device="cuda:0")
        if paged:
            pt, mp = 64, 5
            table = dev(np.random.default_rng(3).permutation(B * mp).astype(np.int32).reshape(B, mp))
            kc = torch.zeros((B * mp, kvh, pt, d), dtype=torch.int16, device="cuda:0")
            vc = torch.zeros_like(kc)
            m.rope_append_decode_paged_qkv(g, src, q_out, pos, B, cfg, kc, vc, B * mp, pt, table, mp)
        else:
            kc = torch.zeros((B, T, kvh, d), dtype=torch.int16, device="cuda:0")
            vc = torch.zeros_like(kc)
            m.rope_append_decode_dense_qkv(g, src, q_out, pos, B, cfg, kc, vc, T)
        outs.append([u16(q_out), u16(kc), u16(vc)])
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    assert m.device_status(0) == 0


@pytest.mark.parametrize("m,n,k", [(8, 6144, 4096), (8, 4096, 512), (8, 28672, 4096), (8, 4096, 14336),
                                   (8, 16032, 4096), (8, 768, 4096), (3, 1024, 1792), (16, 520, 256),
                                   (1, 8, 128), (5, 200, 72)])
def test_gemv_matches_fp32_reference(m, n, k):
    """The tcgen05 projection against a float64 product of the same bf16
    values: one bf16 rounding of an fp32 sum, and the same bits on a second
    call (fixed split order)."""
    import torch
    import mslim_b200 as mm
    rng = np.random.default_rng(m * 7 + n + k)
    x = _rand_bf16(rng, m * k).reshape(m, k)
    w = _rand_bf16(rng, n * k, 0.02).reshape(n, k)
    y = torch.full((m, n), 0x7FC1, dtype=torch.int16, device="cuda:0")
    xd, wd = dev(x), dev(w)
    mm.gemv(xd, wd, y, m, n, k)
    ref = bf16_f32(x).astype(np.float64) @ bf16_f32(w).astype(np.float64).T
    got = bf16_f32(u16(y))
    tol = np.abs(ref) * 2.0 ** -7 + 1e-6 * np.sqrt(k)
    assert (np.abs(got - ref) <= tol).all(), np.abs(got - ref).max()
    y2 = torch.empty_like(y)
    mm.gemv(xd, wd, y2, m, n, k)
    assert torch.equal(y, y2)
    assert mm.device_status(0) == 0


@pytest.mark.parametrize("m,width,k", [(8, 14336, 4096), (8, 7168, 4096), (8, 1792, 4096), (3, 3584, 4096),
                                       (1, 64, 128), (16, 192, 72)])
def test_gemv_swiglu_equals_projection_then_swiglu(m, width, k):
    """The fused gate|up projection + SwiGLU (gpu_llm.cl
    llm_prefill_fused_swiglu_reuse8) returns the bits of the two-step path:
    the projection over the interleaved weights, then SwiGLU over each
    [gate 64 | up 64] block -- and those equal the projection over the
    concatenated [gate | up] weights followed by SwiGLU over the halves; a
    second call gives the same bits."""
    import torch
    import mslim_b200 as mm
    rng = np.random.default_rng(m * 11 + width + k)
    x = _rand_bf16(rng, m * k).reshape(m, k)
    wg = _rand_bf16(rng, width * k, 0.02).reshape(width, k)
    wu = _rand_bf16(rng, width * k, 0.02).reshape(width, k)
    wgu = mm.interleave_gate_up(dev(wg), dev(wu))
    xd = dev(x)
    out = torch.full((m, width), 0x7FC1, dtype=torch.int16, device="cuda:0")
    mm.gemv_swiglu(xd, wgu, out, m, width, k)
    y = torch.empty((m, 2 * width), dtype=torch.int16, device="cuda:0")
    mm.gemv(xd, wgu, y, m, 2 * width, k)
    two_step = torch.empty((m, width), dtype=torch.int16, device="cuda:0")
    mm.swiglu_rows(y, two_step, m * width // 64, 64)
    assert torch.equal(out, two_step)
    cat = dev(np.concatenate([wg, wu]))
    y_cat = torch.empty((m, 2 * width), dtype=torch.int16, device="cuda:0")
    mm.gemv(xd, cat, y_cat, m, 2 * width, k)
    halves = torch.empty((m, width), dtype=torch.int16, device="cuda:0")
    mm.swiglu_rows(y_cat, halves, m, width)
    assert torch.equal(out, halves)
    again = torch.empty_like(out)
    mm.gemv_swiglu(xd, wgu, again, m, width, k)
    assert torch.equal(out, again)
    assert mm.device_status(0) == 0


def test_gemv_swiglu_writes_strided_rows_and_rejects_bad_arguments():
    import torch
    import mslim_b200 as mm
    rng = np.random.default_rng(9)
    m, width, k, ldo = 4, 128, 256, 200
    x = dev(_rand_bf16(rng, m * k).reshape(m, k))
    wgu = dev(_rand_bf16(rng, 2 * width * k, 0.02).reshape(2 * width, k))
    wide = torch.full((m, ldo), 0x1234, dtype=torch.int16, device="cuda:0")
    mm.gemv_swiglu(x, wgu, wide, m, width, k, ldo=ldo)
    dense = torch.empty((m, width), dtype=torch.int16, device="cuda:0")
    mm.gemv_swiglu(x, wgu, dense, m, width, k)
    got = u16(wide)
    assert np.array_equal(got[:, :width], u16(dense)) and (got[:, width:] == 0x1234).all()
    for bad in (dict(m=17), dict(width=96), dict(k=100), dict(ldo=width - 1)):
        args = dict(m=m, width=width, k=k, ldo=0)
        args.update(bad)
        with pytest.raises(mm.ShapeMismatch):
            mm.gemv_swiglu(x, wgu, dense, args["m"], args["width"], args["k"], ldo=args["ldo"])
    assert mm.device_status(0) == 0


def test_gemv_writes_strided_rows_and_rejects_bad_arguments():
    """ldy > n writes into a wider row (e.g. one slice of a fused output) and
    leaves the rest untouched; bad shapes are refused before any launch."""
    import torch
    import mslim_b200 as mm
    rng = np.random.default_rng(5)
    m, n, k, ldy = 4, 256, 4096, 384
    x = _rand_bf16(rng, m * k).reshape(m, k)
    w = _rand_bf16(rng, n * k, 0.02).reshape(n, k)
    y = torch.full((m, ldy), 0x1234, dtype=torch.int16, device="cuda:0")
    mm.gemv(dev(x), dev(w), y, m, n, k, ldy=ldy)
    dense = torch.empty((m, n), dtype=torch.int16, device="cuda:0")
    mm.gemv(dev(x), dev(w), dense, m, n, k)
    got = u16(y)
    assert np.array_equal(got[:, :n], u16(dense)) and (got[:, n:] == 0x1234).all()
    with pytest.raises(mm.ShapeMismatch):
        mm.gemv(dev(x), dev(w), dense, 17, n, k)
    with pytest.raises(mm.ShapeMismatch):
        mm.gemv(dev(x), dev(w), dense, m, n, 100)
    with pytest.raises(mm.ShapeMismatch):
        mm.gemv(dev(x), dev(w), dense, m, n, k, ldy=n - 1)