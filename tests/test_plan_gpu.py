"""The TiledAttention plan (mslim_cuda_plan_build / _run) under the reference's
physical protocol (src/gpu_llm/tiled_attention.rs:296-506): histories
1..4097, queries 1 and min(n, 5) with prior = n - queries, the reference's six
strict geometries / tilings and its online and split-KV configurations, its
modular bf16 input pattern; every output within the north-star tolerance of
the CPU path (each query row over keys 0..=prior+row), experimental modes
within the reference's 0.0078125 of strict, repeat runs bit-identical, K/V
unmodified, bad buffers and geometry rejected."""
import numpy as np
import pytest

from gpu_util import bf16_f32, dev, empty_u16, host_u16, max_abs, torch_mod

pytestmark = pytest.mark.gpu
TOL = 2e-2
EXPERIMENTAL_TOL = 0.0078125   # tiled_attention.rs:366-379
HISTORIES = [1, 2, 31, 33, 63, 65, 129, 375, 2049, 4097]


@pytest.fixture(scope="module")
def m():
    import mslim_b200
    mslim_b200.load()
    return mslim_b200


def modular_input(count: int, salt: int) -> np.ndarray:
    """The reference's deterministic pattern (tiled_attention.rs:305-312):
    value i = ((37 i + 13 salt) mod 257 - 128) / 128, rounded to bf16 (exact:
    every value is a multiple of 1/128 in [-1, 1))."""
    i = np.arange(count, dtype=np.int64)
    vals = (((i * 37 + salt * 13) % 257) - 128).astype(np.float32) / np.float32(128.0)
    return (vals.view(np.uint32) >> 16).astype(np.uint16)


def exercise(m, oracle, cfg, g, histories, strict_outputs=None):
    torch = torch_mod()
    plan = m.TiledAttention.build(cfg, g)
    qh, kvh, d = g.query_heads, g.kv_heads, g.head_dim
    outs = {}
    try:
        for n in histories:
            for queries in sorted({1, min(n, 5)}):
                prior = n - queries
                q = modular_input(queries * qh * d, 3).reshape(queries, qh, d)
                k = modular_input(n * kvh * d, 7).reshape(n, kvh, d)
                v = modular_input(n * kvh * d, 11).reshape(n, kvh, d)
                kd, vd = dev(k), dev(v)
                out = empty_u16((queries, qh, d))
                plan.run(dev(q), kd, vd, out, queries, prior)
                torch.cuda.synchronize()
                got = host_u16(out)
                ref = oracle.causal_prefill_bf16(qh, kvh, d, q, k, v, queries, prior)
                err = max_abs(bf16_f32(got), bf16_f32(ref))
                assert err <= TOL, (cfg, g.head_dim, n, queries, err)
                if strict_outputs is not None:
                    e2 = max_abs(bf16_f32(got), bf16_f32(strict_outputs[(n, queries)]))
                    assert e2 <= EXPERIMENTAL_TOL, (cfg, n, queries, e2)
                again = empty_u16((queries, qh, d))
                plan.run(dev(q), kd, vd, again, queries, prior)
                torch.cuda.synchronize()
                assert np.array_equal(host_u16(again), got), "repeatability failed"
                assert np.array_equal(host_u16(kd), k), "K was modified"
                assert np.array_equal(host_u16(vd), v), "V was modified"
                outs[(n, queries)] = got
        assert m.device_status(0) == 0
        diag = plan.diagnostics()
        assert diag and isinstance(diag, dict)
    finally:
        plan.close()
    return outs


# (head_dim, query heads, kv heads, block_queries, block_keys, work_group):
# tiled_attention.rs:410-417
STRICT_CASES = [(64, 4, 4, 1, 32, 32), (128, 8, 2, 1, 64, 64), (128, 4, 1, 2, 64, 64),
                (128, 4, 1, 4, 32, 128), (80, 4, 2, 2, 32, 32), (256, 4, 1, 1, 64, 128)]


@pytest.mark.parametrize("dim,qh,kh,bm,bn,wg", STRICT_CASES)
def test_strict_tiled_histories_and_causal_tails(m, oracle, dim, qh, kh, bm, bn, wg):
    cfg = m.AttentionKernelConfig(mode=m.AttentionKernelMode.STRICT_TILED, block_queries=bm, block_keys=bn,
                                  work_group=wg, splits=1)
    exercise(m, oracle, cfg, m.AttentionGeometry.new(qh, kh, dim), HISTORIES)


def test_online_and_split_within_the_experimental_tolerance_of_strict(m, oracle):
    # tiled_attention.rs:438-456: online (block_queries 2) and split-KV (8 splits)
    # on 8/2/128 over histories 1..4097
    g = m.AttentionGeometry.new(8, 2, 128)
    hist = [1, 2, 7, 33, 65, 129, 375, 2049, 4097]
    strict = exercise(m, oracle, m.AttentionKernelConfig(mode=m.AttentionKernelMode.STRICT_TILED), g, hist)
    for mode, splits, bm in [(m.AttentionKernelMode.ONLINE_EXPERIMENTAL, 1, 2),
                             (m.AttentionKernelMode.SPLIT_KV_EXPERIMENTAL, 8, 1)]:
        cfg = m.AttentionKernelConfig(mode=mode, block_queries=bm, splits=splits)
        exercise(m, oracle, cfg, g, hist, strict_outputs=strict)


def test_plan_rejects_bad_geometry_and_buffers(m):
    # tiled_attention.rs:479-506
    torch = torch_mod()
    g = m.AttentionGeometry.new(4, 1, 128)
    plan = m.TiledAttention.build(m.AttentionKernelConfig(mode=m.AttentionKernelMode.STRICT_TILED), g)
    try:
        b = torch.zeros(1, dtype=torch.int16, device="cuda:0")      # a 2-byte buffer
        with pytest.raises(m.ShapeMismatch):
            plan.run(b, b, b, b.clone(), 1, 0)
        with pytest.raises(m.ShapeMismatch):
            plan.run(b, b, b, b.clone(), 0, 0)
        with pytest.raises(m.ShapeMismatch):
            plan.run(b, b, b, b.clone(), 1, 2 ** 63)
        with pytest.raises(m.ShapeMismatch):
            plan.run(b, b, b, b.clone(), 1, 0, m.AttentionGeometry.new(4, 1, 64))
        assert m.device_status(0) == 0
    finally:
        plan.close()


@pytest.mark.parametrize("qh,kh,dim", [(8, 2, 128), (8, 2, 64), (4, 4, 64), (4, 2, 80), (4, 1, 256), (8, 2, 32)])
def test_long_runs_take_the_prefill_kernel_where_it_exists(m, oracle, qh, kh, dim):
    """Runs of >= 64 queries go to the tcgen05 prefill kernel when it takes the
    shape (head_dim 64..256, a multiple of 8) and to the split-KV kernel
    otherwise; both within tolerance of the CPU path."""
    cfg = m.AttentionKernelConfig(mode=m.AttentionKernelMode.STRICT_TILED)
    g = m.AttentionGeometry.new(qh, kh, dim)
    plan = m.TiledAttention.build(cfg, g)
    try:
        queries, prior = 200, 57
        n = prior + queries
        q = modular_input(queries * qh * dim, 3).reshape(queries, qh, dim)
        k = modular_input(n * kh * dim, 7).reshape(n, kh, dim)
        v = modular_input(n * kh * dim, 11).reshape(n, kh, dim)
        out = empty_u16((queries, qh, dim))
        plan.run(dev(q), dev(k), dev(v), out, queries, prior)
        torch_mod().cuda.synchronize()
        ref = oracle.causal_prefill_bf16(qh, kh, dim, q, k, v, queries, prior)
        assert max_abs(bf16_f32(host_u16(out)), bf16_f32(ref)) <= TOL
        took_prefill = plan.diagnostics()["prefill_dispatches_since_configuration"] == 1
        assert took_prefill == (64 <= dim <= 256 and dim % 8 == 0)
        assert m.device_status(0) == 0
    finally:
        plan.close()
