"""The isolated AttentionBackend on the B200 decode kernel vs the f64 CPU
reference backend, following the reference's physical test protocol
(src/gpu_backend.rs:379-469: tolerance 1e-4)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def m():
    import mslim_b200
    mslim_b200.load()
    return mslim_b200


@pytest.fixture(scope="module")
def backend(m):
    b = m.GpuBackend(0)
    yield b
    b.close()


def frames(m, wl, geometry, key, value, dtype):
    cache = m.ExactKvFrames(geometry)
    enc = {"bf16": wl.bf16_bits, "f16": lambda a: a.astype(np.float16).view(np.uint16),
           "f32": lambda a: a.astype(np.float32)}[dtype]
    t = key.shape[0]
    cache.append(enc(key).reshape(t, geometry.kv_heads, geometry.head_dim),
                 enc(value).reshape(t, geometry.kv_heads, geometry.head_dim), dtype, dtype)
    return cache, enc(key), enc(value)


def test_bf16_roundtrip_against_f64(m, backend, oracle):
    # gpu_backend.rs:384-412 gpu_roundtrip with bf16 frames
    from mslim_b200 import workloads as wl
    g = m.AttentionGeometry.new(4, 2, 4)
    k = np.array([(i % 11 - 5) * 0.0625 for i in range(32)], np.float32)
    v = np.array([(i % 13 - 6) * 0.0625 for i in range(32)], np.float32)
    cache, kb, vb = frames(m, wl, g, k.reshape(4, 2, 4), v.reshape(4, 2, 4), "bf16")
    q = np.full(16, 0.15, np.float32)
    cpu = oracle.cpu_reference_decode_f64(4, 2, 4, q, kb, vb, "bf16", "bf16")
    gpu = cache.decode(backend, q)
    assert np.max(np.abs(cpu - gpu)) < 1e-4, (cpu, gpu)
    t = backend.last_timings()
    assert t["kernel_ms"] > 0 and t["input_kv_bytes"] == 2 * 32 * 2


@pytest.mark.parametrize("qh,kvh", [(4, 4), (4, 1)])
def test_geometry_roundtrips_f32_frames(m, backend, oracle, qh, kvh):
    # gpu_backend.rs:414-441: f32 frames whose values are exact in bf16 are
    # carried losslessly; the query is an arbitrary f32 (hi + lo bf16 pair).
    from mslim_b200 import workloads as wl
    g = m.AttentionGeometry.new(qh, kvh, 8)
    count = 5 * kvh * 8
    key = np.array([((i % 19) - 9) * 0.0625 for i in range(count)], np.float32)
    value = np.array([((i % 17) - 8) * 0.0625 for i in range(count)], np.float32)
    cache, kb, vb = frames(m, wl, g, key.reshape(5, kvh, 8), value.reshape(5, kvh, 8), "f32")
    query = np.array([((i % 7) - 3) * 0.125 for i in range(qh * 8)], np.float32)
    cpu = oracle.cpu_reference_decode_f64(qh, kvh, 8, query, kb, vb, "f32", "f32")
    gpu = cache.decode(backend, query)
    assert np.max(np.abs(cpu - gpu)) < 1e-4


def test_values_off_the_bf16_grid_are_carried_not_quantized(m, backend, oracle):
    """0.1 is not a bf16 value: the frame goes up as a bf16 hi + lo pair and
    the result still meets the reference's 1e-4 against f64."""
    from mslim_b200 import workloads as wl
    g = m.AttentionGeometry.new(4, 2, 4)
    k = np.full((4, 2, 4), 0.1, np.float32)
    v = np.arange(32, dtype=np.float32).reshape(4, 2, 4) * np.float32(0.0371)
    cache, kb, vb = frames(m, wl, g, k, v, "f32")
    q = np.linspace(-1.3, 0.7, 16).astype(np.float32)
    cpu = oracle.cpu_reference_decode_f64(4, 2, 4, q, kb, vb, "f32", "f32")
    gpu = cache.decode(backend, q)
    assert np.max(np.abs(cpu - gpu)) < 1e-4, (cpu, gpu)
    assert backend.last_timings()["input_kv_bytes"] == 2 * 32 * 4


@pytest.mark.parametrize("dtype", ["f16", "f32"])
@pytest.mark.parametrize("qh,kvh,d,t", [(32, 8, 128, 700), (8, 2, 64, 129), (4, 4, 40, 33)])
def test_general_f16_f32_frames_against_f64(m, backend, oracle, dtype, qh, kvh, d, t):
    from mslim_b200 import workloads as wl
    rng = np.random.default_rng(d + t)
    g = m.AttentionGeometry.new(qh, kvh, d)
    k = rng.standard_normal((t, kvh, d)).astype(np.float32)
    v = rng.standard_normal((t, kvh, d)).astype(np.float32)
    cache, kb, vb = frames(m, wl, g, k, v, dtype)
    q = (rng.standard_normal(qh * d) * 0.5).astype(np.float32)
    cpu = oracle.cpu_reference_decode_f64(qh, kvh, d, q, kb, vb, dtype, dtype)
    gpu = cache.decode(backend, q)
    err = np.max(np.abs(cpu - gpu))
    print(f"{dtype} frames qh={qh} kvh={kvh} d={d} t={t}: max-abs vs f64 {err:.3g}")
    assert err < 1e-4, err


def test_split_frames_need_head_dim_at_most_128(m, backend):
    from mslim_b200 import workloads as wl
    g = m.AttentionGeometry.new(2, 1, 256)
    k = np.full((3, 1, 256), 0.1, np.float32)
    cache, _, _ = frames(m, wl, g, k, k, "f16")
    with pytest.raises(m.UnsupportedDevice):
        cache.decode(backend, np.zeros(512, np.float32))


def test_non_finite_frame_values_are_refused(m, backend):
    from mslim_b200 import workloads as wl
    g = m.AttentionGeometry.new(4, 2, 8)
    k = np.ones((2, 2, 8), np.float32)
    v = k.copy()
    v[1, 1, 3] = np.inf
    cache, _, _ = frames(m, wl, g, k, v, "f32")
    with pytest.raises(m.NonFinite):
        cache.decode(backend, np.ones(32, np.float32))


def test_long_history_and_large_head_dim(m, backend, oracle):
    from mslim_b200 import workloads as wl
    rng = np.random.default_rng(2)
    for (qh, kvh, d, t) in [(32, 8, 128, 3000), (8, 2, 256, 700), (4, 4, 40, 129)]:
        g = m.AttentionGeometry.new(qh, kvh, d)
        k = rng.standard_normal((t, kvh, d)).astype(np.float32)
        v = rng.standard_normal((t, kvh, d)).astype(np.float32)
        cache, kb, vb = frames(m, wl, g, k, v, "bf16")
        q = rng.standard_normal(qh * d).astype(np.float32)
        cpu = oracle.cpu_reference_decode_f64(qh, kvh, d, q, kb, vb)
        gpu = cache.decode(backend, q)
        # bench acceptance tolerance of the reference (mslim-attention-bench.rs:185)
        assert np.max(np.abs(cpu - gpu)) < 5e-4, (qh, kvh, d, t, np.max(np.abs(cpu - gpu)))


def test_empty_and_nonfinite(m, backend):
    g = m.AttentionGeometry.new(4, 2, 8)
    cache = m.ExactKvFrames(g)
    assert np.all(cache.decode(backend, np.ones(32, np.float32)) == 0)
    cache.append(np.zeros((1, 2, 8), np.uint16), np.zeros((1, 2, 8), np.uint16))
    q = np.ones(32, np.float32)
    q[3] = np.nan
    with pytest.raises(m.NonFinite):
        cache.decode(backend, q)
    with pytest.raises(m.ShapeMismatch):
        cache.decode(backend, np.ones(31, np.float32))
