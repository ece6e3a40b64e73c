"""Pins the CPU restatement (oracle/) against every known-answer test and
fixture the reference holds for the attention hot path.  CPU only."""
import numpy as np
import pytest


def test_bf16_decode_all_65536_encodings(oracle):
    # tests/fixed_width_decode.rs:11-21: every bf16 encoding decodes like
    # half::bf16::to_f32 (exact widening; NaN keeps its payload + quiet bit).
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = oracle.bf16_to_f32(bits).view(np.uint32)
    b32 = bits.astype(np.uint32)
    nan = (b32 & 0x7FFF) > 0x7F80
    want = np.where(nan, (b32 | 0x0040) << 16, b32 << 16).astype(np.uint32)
    assert np.array_equal(got, want)
    assert oracle.bf16_to_f32(np.array([0x3F80], np.uint16))[0] == 1.0
    assert np.isnan(oracle.bf16_to_f32(np.array([0x7FC1], np.uint16))[0])


def test_portable_exact_bits_all_formats(oracle):
    # src/portable.rs:661-681: 1.0 and NaN payloads for bf16/f16, f16
    # subnormal 1 -> 2^-24.
    L = oracle.lib()
    assert L.mo_bf16_to_f32(0x3F80) == 1.0
    assert L.mo_f16_to_f32(0x3C00) == 1.0
    assert np.isnan(L.mo_f16_to_f32(0x7E01))
    assert L.mo_f16_to_f32(0x0001) == 2.0 ** -24
    assert L.mo_f16_to_f32(0x8000) == 0.0 and np.signbit(L.mo_f16_to_f32(0x8000))
    for h in (0x0001, 0x03FF, 0x0400, 0x3555, 0x7BFF, 0xFBFF, 0x8001, 0x7C00, 0xFC00):
        want = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        assert L.mo_f16_to_f32(h) == want


@pytest.mark.parametrize("x_bits,want", [
    (0x3F800000, 0x3F80),  # 1.0
    (0x3F808000, 0x3F80),  # tie -> even (down)
    (0x3F818000, 0x3F82),  # tie -> even (up)
    (0x3F808001, 0x3F81),  # above half -> up
    (0x3F807FFF, 0x3F80),  # below half -> down
    (0x7F7FFFFF, 0x7F80),  # max finite rounds to +inf
    (0x7F800000, 0x7F80),  # +inf
    (0xFF800000, 0xFF80),  # -inf
    (0x7F800001, 0x7FC0),  # signalling NaN stays NaN (quiet bit forced)
    (0xFFFFFFFF, 0xFFFF),  # all-ones NaN does not wrap to zero
    (0x80000000, 0x8000),  # -0.0
    (0x00000001, 0x0000),  # tiny subnormal rounds to +0
])
def test_bf16_from_f32_rounding(oracle, x_bits, want):
    # half 2.7.1 bf16::from_f32 == write_bf16 (assets/gpu_llm.cl:10-21).
    x = np.array([x_bits], np.uint32).view(np.float32)
    assert int(oracle.bf16_from_f32(x)[0]) == want


def test_llama3_rope_inverse_frequency_kat(oracle):
    # src/gpu_llm/mod.rs:2849-2878: transformers 4.51.3
    # _compute_llama3_parameters for Llama-3.1-8B, relative tolerance 2e-6.
    table = [(0, 1.0), (20, 0.12868738), (40, 0.01656044), (60, 0.0013718937),
             (80, 0.000034281024), (100, 0.0000044115345), (120, 0.0000005677088),
             (126, 0.0000003068926)]
    for dim, expected in table:
        actual = oracle.rope_inverse_frequency(500000.0, dim, 128, llama3=True, factor=8.0, low=1.0,
                                               high=4.0, original_max_position=8192.0)
        assert abs(actual - expected) / max(expected, np.finfo(np.float32).tiny) <= 2e-6, (dim, actual)


def test_rope_at_zero_is_identity(oracle):
    # src/native_cpu_adapter.rs:997-1002
    out = oracle.apply_rope(np.array([1.0, 2.0, 3.0, 4.0], np.float32), 1, 4, 0, 10000.0)
    assert out.tolist() == [1.0, 2.0, 3.0, 4.0]


def test_rms_norm_is_finite_and_bf16_rounded(oracle):
    # src/native_cpu_adapter.rs:990-995
    out = oracle.rms_norm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 1e-5)
    assert np.all(np.isfinite(out))
    assert np.array_equal(oracle.bf16_to_f32(oracle.bf16_from_f32(out)), out)


def test_softmax_is_normalized(oracle):
    # src/native_cpu_adapter.rs:1004-1008
    v = oracle.softmax(np.array([1.0, 2.0, 3.0], np.float32))
    assert abs(float(v.sum(dtype=np.float32)) - 1.0) < 1e-6


@pytest.mark.parametrize("qheads,kvheads", [(2, 2), (4, 2), (8, 1)])
def test_mha_gqa_mqa_head_mapping(oracle, qheads, kvheads):
    # src/portable.rs:683-710: zero keys, distinct values per KV head; every
    # query head must return exactly its KV head's value row.
    keys = np.zeros(kvheads * 2, np.float32)
    values = np.array([x for h in range(kvheads) for x in (h + 1.0, -(h + 1.0))], np.float32)
    out = oracle.cpu_reference_decode_f64(qheads, kvheads, 2, np.zeros(qheads * 2, np.float32),
                                          keys, values, "f32", "f32")
    dense = oracle.dense_attention_bf16(qheads, kvheads, 2, np.zeros(qheads * 2, np.float32),
                                        oracle.bf16_from_f32(keys), oracle.bf16_from_f32(values))
    for head in range(qheads):
        kv = head // (qheads // kvheads)
        assert out[head * 2:head * 2 + 2].tolist() == [values[kv * 2], values[kv * 2 + 1]]
        assert dense[head * 2:head * 2 + 2].tolist() == [values[kv * 2], values[kv * 2 + 1]]


def test_streaming_softmax_stable_for_extreme_scores(oracle):
    # src/portable.rs:712-726
    out = oracle.cpu_reference_decode_f64(1, 1, 1, np.array([10000.0], np.float32),
                                          np.array([10000.0, -10000.0], np.float32),
                                          np.array([3.0, 9.0], np.float32), "f32", "f32")
    assert out.tolist() == [3.0]


def test_nonfinite_inputs_rejected(oracle):
    # src/portable.rs:806-825
    with pytest.raises(ArithmeticError):
        oracle.cpu_reference_decode_f64(1, 1, 2, np.array([np.nan, 1.0], np.float32),
                                        np.array([1.0, 2.0], np.float32), np.array([1.0, 2.0], np.float32),
                                        "f32", "f32")
    with pytest.raises(ValueError):
        oracle.cpu_reference_decode_f64(3, 2, 32, np.zeros(96, np.float32), np.zeros(64, np.float32),
                                        np.zeros(64, np.float32), "f32", "f32")


def test_fnv1a_published_vectors(oracle):
    # src/cold_store.rs:25-26,909-922 uses the published FNV-1a 64 parameters.
    assert oracle.fnv1a64(b"") == 0xCBF29CE484222325
    assert oracle.fnv1a64(b"a") == 0xAF63DC4C8601EC8C
    assert oracle.fnv1a64(b"foobar") == 0x85944171F73967E8


def test_pages_preserve_every_bf16_value_and_sparse_order(oracle):
    # src/gpu_region_store.rs:992-1042 with geometry (4, 2, 4): 37 tokens in
    # 8-token pages (5 pages); reading back token-major is byte identical,
    # sparse reads keep order.
    count, kvh, dim, page = 37, 2, 4, 8
    keys = oracle.bf16_from_f32(np.array([(i % 59 - 29) * 0.03125 for i in range(count * 8)], np.float32))
    values = oracle.bf16_from_f32(np.array([(i % 61 - 30) * 0.0625 for i in range(count * 8)], np.float32))
    pages_k, pages_v, hashes = [], [], []
    for start in range(0, count, page):
        n = min(page, count - start)
        pk = oracle.page_from_token_major(keys[start * 8:(start + n) * 8], kvh, dim)
        pv = oracle.page_from_token_major(values[start * 8:(start + n) * 8], kvh, dim)
        pages_k.append(pk)
        pages_v.append(pv)
        hashes.append(oracle.token_hashes(pv, kvh, n))
    assert len(pages_v) == 5

    def read(pages, positions):
        rows = []
        for t in positions:
            p = pages[t // page]
            rows.append(p[:, t % page, :].reshape(-1))
        return np.concatenate(rows)

    assert np.array_equal(read(pages_v, range(count)), values)
    assert np.array_equal(read(pages_k, range(count)), keys)
    sparse = [0, 2, 4, 7, 8, 11, 23, 24, 36]
    want = np.concatenate([values[i * 8:(i + 1) * 8] for i in sparse])
    assert np.array_equal(read(pages_v, sparse), want)
    # per-token hash == FNV-1a of that token's bytes across all heads
    for t in range(count):
        tok = pages_v[t // page][:, t % page, :].reshape(-1)
        assert hashes[t // page][t % page] == oracle.fnv1a64(tok.tobytes())


def test_dense_f32_oracle_agrees_with_f64_backend(oracle):
    # Two restatements of two reference paths (native_cpu_adapter.rs:253-307
    # and portable.rs:575-646) agree within the bench acceptance tolerance
    # (src/bin/mslim-attention-bench.rs:185, 5e-4) before the final bf16
    # rounding; after it, within one bf16 ulp of the output magnitude.
    rng = np.random.default_rng(7)
    qh, kvh, d, t = 8, 2, 64, 300
    q = oracle.bf16_to_f32(oracle.bf16_from_f32(rng.standard_normal(qh * d).astype(np.float32)))
    k = oracle.bf16_from_f32(rng.standard_normal(t * kvh * d).astype(np.float32))
    v = oracle.bf16_from_f32(rng.standard_normal(t * kvh * d).astype(np.float32))
    f64 = oracle.cpu_reference_decode_f64(qh, kvh, d, q, k, v)
    f32 = oracle.dense_attention_bf16(qh, kvh, d, q, k, v)
    assert np.max(np.abs(f64 - f32)) <= 2 ** -8 * max(1.0, float(np.max(np.abs(f64))))


def test_paged_equals_dense_bit_exact(oracle):
    # docs/VALIDATION.md:53-67: CPU hot-dense == CPU ColdStore-exact, bitwise.
    rng = np.random.default_rng(11)
    qh, kvh, d, t, pt = 8, 2, 32, 150, 16
    q = oracle.bf16_to_f32(oracle.bf16_from_f32(rng.standard_normal(qh * d).astype(np.float32)))
    k = oracle.bf16_from_f32(rng.standard_normal(t * kvh * d).astype(np.float32)).reshape(t, kvh, d)
    v = oracle.bf16_from_f32(rng.standard_normal(t * kvh * d).astype(np.float32)).reshape(t, kvh, d)
    npages = (t + pt - 1) // pt
    perm = rng.permutation(npages + 3)[:npages].astype(np.int32)
    pool_k = np.zeros((npages + 3, kvh, pt, d), np.uint16)
    pool_v = np.zeros_like(pool_k)
    for lp in range(npages):
        n = min(pt, t - lp * pt)
        pool_k[perm[lp], :, :n] = k[lp * pt:lp * pt + n].transpose(1, 0, 2)
        pool_v[perm[lp], :, :n] = v[lp * pt:lp * pt + n].transpose(1, 0, 2)
    dense = oracle.dense_attention_bf16(qh, kvh, d, q, k, v)
    paged = oracle.paged_attention_bf16(qh, kvh, d, q, pool_k, pool_v, perm, pt, t)
    assert dense.tobytes() == paged.tobytes()
