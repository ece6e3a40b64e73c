"""GPU parity of the RMSNorm / RoPE prologue and of RoPE fused with the
ColdStore page append, against the CPU restatement
(src/native_cpu_adapter.rs:194-221, src/gpu_region_store.rs:470-483)."""
import numpy as np
import pytest

from gpu_util import bf16_f32, bf16_ulps, dev, empty_u16, host_u16, max_abs, torch_mod

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def m():
    import mslim_b200
    mslim_b200.load()
    return mslim_b200


@pytest.fixture(scope="module")
def wl():
    from mslim_b200 import workloads
    return workloads


ulps = bf16_ulps


@pytest.mark.parametrize("tokens,hidden", [(1, 4096), (520, 4096), (3, 80), (7, 4100)])
def test_rmsnorm_matches_cpu(m, wl, oracle, tokens, hidden):
    rng = np.random.default_rng(tokens + hidden)
    x = wl.normal_bf16(rng, (tokens, hidden))
    w = wl.normal_bf16(rng, (hidden,), 0.02)
    ref = oracle.rms_norm_rows_bf16(x, w, 1e-5)
    y = empty_u16((tokens, hidden))
    m.rmsnorm(dev(x), dev(w), y, tokens, hidden, 1e-5)
    torch_mod().cuda.synchronize()
    got = host_u16(y)
    d = ulps(got, ref)
    # Only the sum-of-squares order differs (tree here and in the reference's
    # OpenCL kernel, sequential on the CPU).  That can move the f32 scale by an
    # ulp, which can flip each of the two cascaded bf16 roundings: <= 2 ulps.
    assert d.max() <= 2 and np.mean(d == 0) > 0.99, (d.max(), np.mean(d == 0))


def test_rope_c1_matches_cpu(m, wl, oracle):
    case = wl.c1_decode()
    ref = oracle.rope_rows_bf16(case.k_raw, 0, case.theta)
    out = empty_u16(case.k_raw.shape)
    m.rope(dev(case.k_raw), out, 1024, 8, 128, 0, m.RopeKernelConfig(theta=case.theta))
    torch_mod().cuda.synchronize()
    got = host_u16(out)
    d = ulps(got, ref)
    # Same angle bits (host-side theta^(2i/D) table, IEEE division on the
    # device); cos/sin are correctly rounded in double, glibc's sinf/cosf can
    # differ in the last bit, and a flipped bf16 rounding of cos or sin moves
    # the output by a few bf16 ulps at most.
    assert np.mean(d == 0) > 0.999, np.mean(d == 0)
    assert max_abs(bf16_f32(got), bf16_f32(ref)) <= 2e-2


def test_rope_at_zero_is_identity(m, wl):
    rng = np.random.default_rng(5)
    x = wl.normal_bf16(rng, (1, 4, 64))
    out = empty_u16(x.shape)
    m.rope(dev(x), out, 1, 4, 64, 0, m.RopeKernelConfig(theta=10000.0))
    torch_mod().cuda.synchronize()
    assert np.array_equal(host_u16(out), x)


def test_rope_llama3_scaling_matches_gpu_formula(m, wl, oracle):
    rng = np.random.default_rng(9)
    x = wl.normal_bf16(rng, (64, 8, 128))
    cfg = m.RopeKernelConfig(theta=500000.0, llama3_scaling=1, factor=8.0, low_freq_factor=1.0,
                             high_freq_factor=4.0, original_max_position=8192.0)
    ref = oracle.gpu_rope_rows_bf16(x, 9000, 500000.0, True, 8.0, 1.0, 4.0, 8192.0)
    out = empty_u16(x.shape)
    m.rope(dev(x), out, 64, 8, 128, 9000, cfg)
    torch_mod().cuda.synchronize()
    d = ulps(host_u16(out), ref)
    assert np.mean(d == 0) > 0.99 and max_abs(bf16_f32(host_u16(out)), bf16_f32(ref)) <= 2e-2


@pytest.mark.parametrize("page_tokens", [64, 256])
def test_rope_append_paged_then_decode_c1(m, wl, oracle, page_tokens):
    """The full C1 prologue on the device: RoPE(q, k) fused with the append of
    k and v into ColdStore pages, then paged decode, vs the CPU path
    (apply_rope + append + dense_attention_bf16)."""
    torch = torch_mod()
    case = wl.c1_decode()
    T = 1024
    g = m.AttentionGeometry.new(32, 8, 128)
    rng = np.random.default_rng(1)
    n_pages = T // page_tokens + 3
    perm = rng.permutation(n_pages).astype(np.int32)
    table = perm[:T // page_tokens].copy()
    k_pool = torch.zeros((n_pages, 8, page_tokens, 128), dtype=torch.int16, device="cuda:0")
    v_pool = torch.zeros_like(k_pool)
    # every token position carries its own q row here; only the last one is the
    # decode query, the rest exercise the fused q path too
    q_rows = np.repeat(case.q_raw[None], T, axis=0)
    q_out = empty_u16((T, 32, 128))
    cfg = m.RopeKernelConfig(theta=case.theta)
    m.rope_append_paged(g, dev(q_rows), q_out, dev(case.k_raw), dev(case.v), T, 0, cfg, k_pool, v_pool,
                        n_pages, page_tokens, dev(table), len(table))
    torch.cuda.synchronize()
    k_ref = oracle.rope_rows_bf16(case.k_raw, 0, case.theta)
    kp = host_u16(k_pool)
    vp = host_u16(v_pool)
    for lp, phys in enumerate(table):
        sl = slice(lp * page_tokens, (lp + 1) * page_tokens)
        assert np.array_equal(vp[phys], oracle.page_from_token_major(case.v[sl], 8, 128))
        d = ulps(kp[phys], oracle.page_from_token_major(k_ref[sl], 8, 128))
        assert np.mean(d == 0) > 0.999
    q_ref = oracle.rope_rows_bf16(case.q_raw[None], T - 1, case.theta)[0]
    qd = host_u16(q_out)[T - 1]
    assert np.mean(ulps(qd, q_ref) == 0) > 0.99
    ws = torch.zeros(m.decode_workspace_bytes(g, 1, T), dtype=torch.uint8, device="cuda:0")
    out = empty_u16((1, 32, 128))
    m.decode_paged(g, q_out[T - 1:T], k_pool, v_pool, n_pages, page_tokens,
                   dev(table[None].copy()), len(table), dev(np.array([T], np.int32)), 1, ws, out)
    torch.cuda.synchronize()
    ref = oracle.dense_attention_bf16(32, 8, 128, oracle.bf16_to_f32(q_ref), k_ref, case.v)
    assert max_abs(bf16_f32(host_u16(out)).reshape(-1), ref) <= 2e-2
