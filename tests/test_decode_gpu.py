"""GPU parity of the split-KV decode kernel against the CPU restatement of the
reference's hot-dense path (src/native_cpu_adapter.rs:253-307), plus the
bit-exact contracts: dense == ColdStore pages, run-to-run, K/V untouched."""
import numpy as np
import pytest

from gpu_util import bf16_f32, bf16_ulps, dev, empty_u16, f32_to_bf16_bits, host_u16, max_abs, torch_mod

pytestmark = pytest.mark.gpu

TOL = 2e-2  # north star: max-abs 2e-2 on attention outputs vs the CPU hot-dense path


@pytest.fixture(scope="module")
def m():
    import mslim_b200
    mslim_b200.load()
    return mslim_b200


@pytest.fixture(scope="module")
def wl():
    from mslim_b200 import workloads
    return workloads


def run_dense(m, g, q_bits, k_bits, v_bits, lengths=None, split_tokens=0):
    """q [n_seq][QH][D]; k/v [n_seq][max_tokens][KVH][D] (bf16 bits)."""
    torch = torch_mod()
    n_seq, max_tokens = k_bits.shape[0], k_bits.shape[1]
    if lengths is None:
        lengths = np.full(n_seq, max_tokens, np.int32)
    ws = torch.zeros(m.decode_workspace_bytes(g, n_seq, max_tokens, split_tokens), dtype=torch.uint8,
                     device="cuda:0")
    out = empty_u16((n_seq, g.query_heads, g.head_dim))
    m.decode_dense(g, dev(q_bits), dev(k_bits), dev(v_bits), dev(np.asarray(lengths, np.int32)), n_seq,
                   max_tokens, ws, out, split_tokens)
    torch.cuda.synchronize()
    assert m.device_status(0) == 0
    return host_u16(out)


def rand_bf16(wl, rng, shape):
    return wl.normal_bf16(rng, shape)


def test_c1_matches_cpu_hot_dense_oracle(m, wl, oracle):
    case = wl.c1_decode()
    k = oracle.rope_rows_bf16(case.k_raw, 0, case.theta)
    q = oracle.rope_rows_bf16(case.q_raw[None], case.position, case.theta)[0]
    ref = oracle.dense_attention_bf16(32, 8, 128, oracle.bf16_to_f32(q), k, case.v)
    g = m.AttentionGeometry.new(32, 8, 128)
    got = bf16_f32(run_dense(m, g, q[None], k[None], case.v[None]))[0].reshape(-1)
    err = max_abs(got, ref)
    assert err <= TOL, err
    # the only systematic difference is summation order: nearly every output
    # is the same bf16 value or its neighbour
    ulp = bf16_ulps(f32_to_bf16_bits(got), f32_to_bf16_bits(ref))
    assert np.mean(ulp == 0) > 0.99 and ulp.max() <= 2, (np.mean(ulp == 0), ulp.max())


GEOMETRIES = [(4, 4, 64), (8, 2, 128), (4, 1, 128), (4, 2, 80), (4, 1, 256), (32, 8, 128), (64, 2, 128)]
HISTORIES = [1, 2, 31, 33, 63, 65, 129, 375, 2049, 4097]


@pytest.mark.parametrize("geom", GEOMETRIES)
def test_histories_and_geometries_match_oracle(m, wl, oracle, geom):
    # The reference's tiled-attention protocol (src/gpu_llm/tiled_attention.rs:
    # 408-434): histories 1..4097 x geometries incl. D=80 and D=256.
    qh, kvh, d = geom
    g = m.AttentionGeometry.new(qh, kvh, d)
    rng = np.random.default_rng(100 + qh + kvh + d)
    for n in HISTORIES:
        q = rand_bf16(wl, rng, (qh, d))
        k = rand_bf16(wl, rng, (n, kvh, d))
        v = rand_bf16(wl, rng, (n, kvh, d))
        ref = oracle.dense_attention_bf16(qh, kvh, d, oracle.bf16_to_f32(q), k, v)
        got = bf16_f32(run_dense(m, g, q[None], k[None], v[None]))[0].reshape(-1)
        assert max_abs(got, ref) <= TOL, (geom, n, max_abs(got, ref))


def build_pool(wl, rng, lengths, kvh, d, page_tokens, spare_pages=5, garbage=True):
    """Random physical page permutation for a batch of sequences; unused slots
    and spare pages hold NaN bit patterns."""
    pages = [(int(L) + page_tokens - 1) // page_tokens for L in lengths]
    n_pages = sum(pages) + spare_pages
    perm = rng.permutation(n_pages).astype(np.int32)
    max_pages = max(max(pages), 1)
    table = np.zeros((len(lengths), max_pages), np.int32)
    fill = 0x7FC1 if garbage else 0
    k_pool = np.full((n_pages, kvh, page_tokens, d), fill, np.uint16)
    v_pool = np.full_like(k_pool, fill)
    max_tokens = max_pages * page_tokens
    k_dense = np.full((len(lengths), max_tokens, kvh, d), fill, np.uint16)
    v_dense = np.full_like(k_dense, fill)
    cursor = 0
    for s, L in enumerate(lengths):
        k = rand_bf16(wl, rng, (L, kvh, d))
        v = rand_bf16(wl, rng, (L, kvh, d))
        k_dense[s, :L], v_dense[s, :L] = k, v
        for lp in range(pages[s]):
            phys = perm[cursor]
            cursor += 1
            table[s, lp] = phys
            n = min(page_tokens, L - lp * page_tokens)
            k_pool[phys, :, :n] = k[lp * page_tokens:lp * page_tokens + n].transpose(1, 0, 2)
            v_pool[phys, :, :n] = v[lp * page_tokens:lp * page_tokens + n].transpose(1, 0, 2)
    return dict(k_pool=k_pool, v_pool=v_pool, table=table, k_dense=k_dense, v_dense=v_dense,
                n_pages=n_pages, max_pages=max_pages, max_tokens=max_tokens)


def run_paged(m, g, q, pool, lengths, page_tokens, split_tokens=0):
    torch = torch_mod()
    n_seq = len(lengths)
    ws = torch.zeros(m.decode_workspace_bytes(g, n_seq, pool["max_tokens"], split_tokens), dtype=torch.uint8,
                     device="cuda:0")
    out = empty_u16((n_seq, g.query_heads, g.head_dim))
    kp, vp = dev(pool["k_pool"]), dev(pool["v_pool"])
    m.decode_paged(g, dev(q), kp, vp, pool["n_pages"], page_tokens, dev(pool["table"]), pool["max_pages"],
                   dev(np.asarray(lengths, np.int32)), n_seq, ws, out, split_tokens)
    torch.cuda.synchronize()
    assert m.device_status(0) == 0
    assert np.array_equal(host_u16(kp), pool["k_pool"]), "K pool was modified"
    assert np.array_equal(host_u16(vp), pool["v_pool"]), "V pool was modified"
    return host_u16(out)


@pytest.mark.parametrize("page_tokens", [64, 256])
@pytest.mark.parametrize("split_tokens", [0, 64, 320])
def test_dense_and_coldstore_pages_bit_exact(m, wl, oracle, page_tokens, split_tokens):
    g = m.AttentionGeometry.new(32, 8, 128)
    rng = np.random.default_rng(7 + page_tokens + split_tokens)
    lengths = [1000, 1, 700, 0, 257, 64]
    pool = build_pool(wl, rng, lengths, 8, 128, page_tokens)
    q = rand_bf16(wl, rng, (len(lengths), 32, 128))
    paged = run_paged(m, g, q, pool, lengths, page_tokens, split_tokens)
    dense = run_dense(m, g, q, pool["k_dense"], pool["v_dense"], lengths, split_tokens)
    assert paged.tobytes() == dense.tobytes()
    again = run_paged(m, g, q, pool, lengths, page_tokens, split_tokens)
    assert again.tobytes() == paged.tobytes(), "repeat run differs"
    # garbage (NaN) rows past each sequence end do not leak into the result,
    # an empty sequence gives zeros, and every row is within tolerance
    assert not np.any(paged[3])
    for s, L in enumerate(lengths):
        if L == 0:
            continue
        ref = oracle.dense_attention_bf16(32, 8, 128, oracle.bf16_to_f32(q[s].reshape(-1)),
                                          pool["k_dense"][s, :L], pool["v_dense"][s, :L])
        assert max_abs(bf16_f32(paged[s]).reshape(-1), ref) <= TOL


def test_dense_and_coldstore_bit_exact_for_many_context_lengths(m, wl, oracle):
    """The reference's exact-hot parity sweep (src/gpu_llm/mod.rs:4311-4415,
    T in 1..2048): every context length around the 64-token tile and
    256-token page edges, one session each, dense caches against
    ColdStore-exact pages in one batched call, bitwise; each within the
    tolerance of the CPU path."""
    g = m.AttentionGeometry.new(32, 8, 128)
    rng = np.random.default_rng(4311)
    edges = [1, 2, 3, 7, 31, 32, 33, 63, 64, 65, 127, 128, 129, 191, 255, 256, 257, 383, 511, 512, 513,
             767, 1023, 1024, 1025, 1279, 1535, 1791, 2047, 2048]
    for page_tokens in (64, 256):
        pool = build_pool(wl, rng, edges, 8, 128, page_tokens)
        q = rand_bf16(wl, rng, (len(edges), 32, 128))
        paged = run_paged(m, g, q, pool, edges, page_tokens)
        dense = run_dense(m, g, q, pool["k_dense"], pool["v_dense"], edges)
        assert paged.tobytes() == dense.tobytes(), page_tokens
        for s in (0, 8, 15, 29):
            L = edges[s]
            ref = oracle.dense_attention_bf16(32, 8, 128, oracle.bf16_to_f32(q[s].reshape(-1)),
                                              pool["k_dense"][s, :L], pool["v_dense"][s, :L])
            assert max_abs(bf16_f32(paged[s]).reshape(-1), ref) <= TOL


def test_split_size_changes_only_rounding(m, wl, oracle):
    g = m.AttentionGeometry.new(32, 8, 128)
    rng = np.random.default_rng(3)
    q = rand_bf16(wl, rng, (1, 32, 128))
    k = rand_bf16(wl, rng, (1, 5000, 8, 128))
    v = rand_bf16(wl, rng, (1, 5000, 8, 128))
    ref = oracle.dense_attention_bf16(32, 8, 128, oracle.bf16_to_f32(q.reshape(-1)), k[0], v[0])
    for st in (64, 128, 1024, 4096, 8192):
        got = bf16_f32(run_dense(m, g, q, k, v, split_tokens=st)).reshape(-1)
        assert max_abs(got, ref) <= TOL, st
        again = bf16_f32(run_dense(m, g, q, k, v, split_tokens=st)).reshape(-1)
        assert got.tobytes() == again.tobytes()


def test_extreme_scores_are_stable(m, wl):
    # src/portable.rs:712-726 at kernel scale: one key dominates by a huge
    # margin; the output is exactly that key's value row.
    g = m.AttentionGeometry.new(4, 1, 64)
    q = np.zeros((1, 4, 64), np.uint16)
    q[..., 0] = wl.bf16_bits(np.array([100.0], np.float32))[0]
    k = np.zeros((1, 2, 1, 64), np.uint16)
    k[0, 0, 0, 0] = wl.bf16_bits(np.array([100.0], np.float32))[0]
    k[0, 1, 0, 0] = wl.bf16_bits(np.array([-100.0], np.float32))[0]
    v = np.zeros_like(k)
    v[0, 0, 0, :] = wl.bf16_bits(np.full(64, 3.0, np.float32))
    v[0, 1, 0, :] = wl.bf16_bits(np.full(64, 9.0, np.float32))
    out = bf16_f32(run_dense(m, g, q, k, v))
    assert np.all(out == 3.0)


def test_rejects_bad_arguments(m):
    torch = torch_mod()
    g = m.AttentionGeometry.new(32, 8, 128)
    b = torch.zeros(8, dtype=torch.int16, device="cuda:0")
    seq = torch.ones(1, dtype=torch.int32, device="cuda:0")
    ws = torch.empty(16, dtype=torch.uint8, device="cuda:0")
    with pytest.raises(m.ShapeMismatch):  # workspace too small
        m.decode_dense(g, b, b, b, seq, 1, 4096, ws, b.clone())
    with pytest.raises(m.ShapeMismatch):  # output aliases input
        m.decode_dense(g, b, b, b, seq, 1, 1, torch.empty(1 << 20, dtype=torch.uint8, device="cuda:0"), b)
    with pytest.raises(m.InvalidGeometry):
        m.decode_dense(m.AttentionGeometry.new(4, 1, 12), b, b, b, seq, 1, 1, ws, b.clone())
    with pytest.raises(m.ShapeMismatch):  # page size not a multiple of 64
        m.decode_paged(g, b, b, b, 1, 48, seq, 1, seq, 1, ws, b.clone())


def test_paged_decode_reports_page_ids_outside_the_pool(m, wl):
    """A page-table entry outside [0, n_pages) is never loaded: the decode
    records it in the device status word (mslim_cuda_device_status returns
    MSLIM_ERR_SHAPE_MISMATCH), and sessions whose rows are intact keep their
    exact outputs.  The reference rejects bad buffers before dispatch
    (src/gpu_llm/tiled_attention.rs:172-207); here the table lives on the
    device, so the check runs where the entry is read."""
    import ctypes
    from mslim_b200 import _lib
    torch = torch_mod()
    rng = np.random.default_rng(41)
    qh, kvh, d, pt = 32, 8, 128, 64
    lengths = [300, 200, 130, 64]
    pool = build_pool(wl, rng, lengths, kvh, d, pt)
    g = m.AttentionGeometry.new(qh, kvh, d)
    q = rand_bf16(wl, rng, (len(lengths), qh, d))
    want = run_paged(m, g, q, pool, lengths, pt)
    bad = dict(pool)
    bad["table"] = pool["table"].copy()
    bad["table"][0, 2] = pool["n_pages"]      # one past the pool
    bad["table"][2, 1] = -1                   # negative
    n_seq = len(lengths)
    ws = torch.zeros(m.decode_workspace_bytes(g, n_seq, pool["max_tokens"]), dtype=torch.uint8, device="cuda:0")
    out = empty_u16((n_seq, qh, d))
    m.decode_paged(g, dev(q), dev(pool["k_pool"]), dev(pool["v_pool"]), pool["n_pages"], pt, dev(bad["table"]),
                   pool["max_pages"], dev(np.asarray(lengths, np.int32)), n_seq, ws, out)
    st = ctypes.c_int(0)
    rc = _lib.lib().mslim_cuda_device_status(0, 1, ctypes.byref(st))
    assert rc == _lib.ERR_SHAPE_MISMATCH and st.value == 2, (rc, st.value)
    assert "outside the page pool" in _lib.last_error()
    got = host_u16(out)
    for s in (1, 3):                          # untouched table rows: same bits
        assert np.array_equal(got[s], want[s]), s
    # the status word was cleared; a good table decodes cleanly again
    assert np.array_equal(run_paged(m, g, q, pool, lengths, pt), want)


@pytest.mark.parametrize("tokens", [256, 100, 1])
def test_page_token_hashes_match_the_coldstore_record(m, oracle, tokens):
    """ColdStore page sealing from device pages (cold_store.rs:725-742): the
    per-token FNV-1a of pool pages equal the record hashes of their compact
    head-major payloads, full or partly filled."""
    import torch
    rng = np.random.default_rng(tokens)
    n_pool, kvh, pt, d = 12, 8, 256, 128
    pool = rng.integers(0, 1 << 16, size=(n_pool, kvh, pt, d), dtype=np.uint16)
    ids = np.array([7, 0, 11, 3], np.int32)
    hashes = torch.zeros((len(ids), tokens), dtype=torch.int64, device="cuda:0")
    m.page_token_hashes(dev(pool), n_pool, kvh, pt, d, dev(ids), len(ids), tokens, hashes)
    got = hashes.cpu().numpy().view(np.uint64)
    for i, p in enumerate(ids):
        payload = np.ascontiguousarray(pool[p][:, :tokens, :])
        assert np.array_equal(got[i], oracle.token_hashes(payload, kvh, tokens))
    assert m.device_status(0) == 0


def test_kv_canonical_paged_reads_pages_in_order_and_rejects_bad_ids():
    """mslim_cuda_kv_canonical_paged: the session's pages, listed by its page
    table row, come out head-major [kv_heads][tokens][head_dim]; a page id
    outside the pool writes nothing for its rows and sets the status word."""
    import torch
    import mslim_b200 as m
    from gpu_util import dev, host_u16
    rng = np.random.default_rng(17)
    kvh, pt, d, n_pages, tokens = 3, 16, 24, 6, 70
    pool = rng.integers(0, 65536, size=(n_pages, kvh, pt, d), dtype=np.uint16)
    row = np.array([4, 0, 5, 2, 1], np.int32)          # 5 logical pages for 70 tokens
    out = torch.zeros((kvh, tokens, d), dtype=torch.int16, device="cuda:0")
    m.kv_canonical_paged(dev(pool), n_pages, kvh, pt, d, dev(row), len(row), tokens, out)
    assert m.device_status(0) == 0
    want = np.stack([np.concatenate([pool[row[t // pt], h, t % pt][None] for t in range(tokens)])
                     for h in range(kvh)])
    assert np.array_equal(host_u16(out), want)
    bad = row.copy()
    bad[2] = n_pages                                     # outside the pool
    out.zero_()
    m.kv_canonical_paged(dev(pool), n_pages, kvh, pt, d, dev(bad), len(bad), tokens, out)
    assert m.device_status(0) == 2                       # MSLIM_ERR_SHAPE_MISMATCH
    got = host_u16(out)
    assert not got[:, 2 * pt:3 * pt].any() and np.array_equal(got[:, :2 * pt], want[:, :2 * pt])


def _selected_case(m, wl, rng, lengths, counts, max_selected, qh=32, kvh=8, d=128, split_tokens=0, sel=None):
    torch = torch_mod()
    g = m.AttentionGeometry.new(qh, kvh, d)
    n_seq, cap = len(lengths), max(lengths)
    k = np.full((n_seq, cap, kvh, d), 0x7FC1, np.uint16)      # NaN past each end
    v = np.full_like(k, 0x7FC1)
    for s_, L in enumerate(lengths):
        k[s_, :L] = rand_bf16(wl, rng, (L, kvh, d))
        v[s_, :L] = rand_bf16(wl, rng, (L, kvh, d))
    if sel is None:
        sel = np.zeros((n_seq, max_selected), np.int32)
        for s_, (L, c) in enumerate(zip(lengths, counts)):
            sel[s_, :c] = np.sort(rng.choice(L, size=c, replace=False))
    q = rand_bf16(wl, rng, (n_seq, qh, d))
    ws = torch.zeros(m.decode_selected_workspace_bytes(g, n_seq, max_selected, split_tokens), dtype=torch.uint8,
                     device="cuda:0")
    out = empty_u16((n_seq, qh, d))
    kd, vd = dev(k), dev(v)
    m.decode_selected(g, dev(q), kd, vd, cap, dev(np.asarray(lengths, np.int32)), dev(sel),
                      dev(np.asarray(counts, np.int32)), max_selected, n_seq, ws, out, split_tokens)
    torch.cuda.synchronize()
    assert np.array_equal(host_u16(kd), k) and np.array_equal(host_u16(vd), v), "K/V modified"
    return g, q, k, v, sel, host_u16(out)


def test_selected_decode_matches_cpu_over_the_certified_rows(m, wl, oracle):
    """epsilon > 0 path (gpu_resources.rs:656-771): attention over the
    selected positions only, against the CPU attention over those rows."""
    rng = np.random.default_rng(847)
    lengths, counts = [300, 2049, 65, 1000, 8], [1, 17, 64, 999, 8]
    g, q, k, v, sel, out = _selected_case(m, wl, rng, lengths, counts, 1024)
    assert m.device_status(0) == 0
    for s, c in enumerate(counts):
        ref = oracle.selected_attention_bf16(32, 8, 128, oracle.bf16_to_f32(q[s].reshape(-1)), k[s], v[s],
                                             sel[s, :c])
        assert max_abs(bf16_f32(out[s]).reshape(-1), ref) <= TOL, (s, c)


def test_selecting_every_position_gives_the_dense_decode_bits(m, wl):
    torch = torch_mod()
    rng = np.random.default_rng(964)
    lengths = [1, 77, 512, 700]
    sel = np.zeros((4, 768), np.int32)
    for s, L in enumerate(lengths):
        sel[s, :L] = np.arange(L)
    g, q, k, v, _, out = _selected_case(m, wl, rng, lengths, lengths, 768, split_tokens=128, sel=sel)
    assert m.device_status(0) == 0
    dense = run_dense(m, g, q, k, v, lengths, 128)
    assert dense.tobytes() == out.tobytes()


def test_selected_decode_empty_and_invalid_selections(m, wl):
    rng = np.random.default_rng(965)
    # count 0 -> zeros, no error
    _, _, _, _, _, out = _selected_case(m, wl, rng, [40, 50], [0, 3], 8)
    assert m.device_status(0) == 0 and not out[0].any() and out[1].any()
    # not strictly increasing
    sel = np.array([[3, 9, 9, 20], [0, 1, 2, 3]], np.int32)
    _selected_case(m, wl, rng, [40, 50], [4, 4], 4, sel=sel)
    assert m.device_status(0) == 2
    # a position at or past the committed length
    sel = np.array([[3, 9, 40, 0], [0, 1, 2, 3]], np.int32)
    _selected_case(m, wl, rng, [40, 50], [3, 4], 4, sel=sel)
    assert m.device_status(0) == 2
    # more selected than the capacity
    sel = np.zeros((2, 4), np.int32)
    _selected_case(m, wl, rng, [40, 50], [5, 1], 4, sel=sel)
    assert m.device_status(0) == 2


@pytest.mark.parametrize("page_tokens", [64, 256])
def test_selected_decode_over_coldstore_pages(m, wl, oracle, page_tokens):
    """epsilon > 0 over ColdStore-exact pages: the selected rows come straight
    out of the page pool (random physical order, NaN in unused slots) and give
    the bits of the dense-cache selection over the same K/V; selecting every
    position gives the paged decode's bits; a page id outside the pool is
    reported."""
    torch = torch_mod()
    rng = np.random.default_rng(1063 + page_tokens)
    qh, kvh, d = 32, 8, 128
    g = m.AttentionGeometry.new(qh, kvh, d)
    lengths, counts = [300, 1025, 64, 700], [5, 333, 64, 700]
    pool = build_pool(wl, rng, lengths, kvh, d, page_tokens)
    n_seq, cap = len(lengths), 768
    sel = np.zeros((n_seq, cap), np.int32)
    for s_, (L, c) in enumerate(zip(lengths, counts)):
        sel[s_, :c] = np.sort(rng.choice(L, size=c, replace=False))
    sel[3, :700] = np.arange(700)                            # every position of session 3
    q = rand_bf16(wl, rng, (n_seq, qh, d))
    st = 128
    ws = torch.zeros(m.decode_selected_workspace_bytes(g, n_seq, cap, st), dtype=torch.uint8, device="cuda:0")
    seq = dev(np.asarray(lengths, np.int32))
    cnt = dev(np.asarray(counts, np.int32))
    kp, vp = dev(pool["k_pool"]), dev(pool["v_pool"])

    def paged_sel(table):
        out = empty_u16((n_seq, qh, d))
        m.decode_selected_paged(g, dev(q), kp, vp, pool["n_pages"], page_tokens, dev(table), pool["max_pages"],
                                seq, dev(sel), cnt, cap, n_seq, ws, out, st)
        torch.cuda.synchronize()
        return host_u16(out)

    got = paged_sel(pool["table"])
    assert m.device_status(0) == 0
    dense_out = empty_u16((n_seq, qh, d))
    m.decode_selected(g, dev(q), dev(pool["k_dense"]), dev(pool["v_dense"]), pool["max_tokens"], seq, dev(sel), cnt,
                      cap, n_seq, ws, dense_out, st)
    torch.cuda.synchronize()
    assert got.tobytes() == host_u16(dense_out).tobytes()
    full = run_paged(m, g, q, pool, lengths, page_tokens, st)
    assert got[3].tobytes() == full[3].tobytes()
    for s_, c in enumerate(counts):
        ref = oracle.selected_attention_bf16(qh, kvh, d, oracle.bf16_to_f32(q[s_].reshape(-1)),
                                             pool["k_dense"][s_], pool["v_dense"][s_], sel[s_, :c])
        assert max_abs(bf16_f32(got[s_]).reshape(-1), ref) <= TOL, s_
    assert np.array_equal(host_u16(kp), pool["k_pool"]) and np.array_equal(host_u16(vp), pool["v_pool"])
    bad = pool["table"].copy()
    bad[1, 0] = pool["n_pages"] + 3
    paged_sel(bad)
    assert m.device_status(0) == 2


def test_gpu_engine_reserves_its_workspace_when_built(m, wl, oracle):
    """GpuEngine::attention (src/gpu_llm/gpu_resources.rs:583-643) through the
    Python mirror: the decode workspace is reserved when the engine is built
    (like the reference's Workspace), attention() allocates nothing, its
    output equals the dense entry point's, and a history beyond the reserved
    capacity is a ShapeMismatch."""
    torch = torch_mod()
    rng = np.random.default_rng(43)
    qh, kvh, d, cap = 32, 8, 128, 1024
    g = m.AttentionGeometry.new(qh, kvh, d)
    eng = m.GpuEngine(0, g, cap)
    ws_ptr = eng._workspace.data_ptr()
    k = rand_bf16(wl, rng, (cap, kvh, d))
    v = rand_bf16(wl, rng, (cap, kvh, d))
    q = rand_bf16(wl, rng, (qh, d))
    kd, vd, qd = dev(k), dev(v), dev(q)
    for T in (1, 300, cap):
        out = empty_u16((qh, d))
        eng.attention(qd, (kd, vd), out, T, g)
        torch.cuda.synchronize()
        assert eng._workspace.data_ptr() == ws_ptr
        want = run_dense(m, g, q[None], k[None, :T], v[None, :T])[0]
        ref = oracle.dense_attention_bf16(qh, kvh, d, bf16_f32(q).reshape(-1), k[:T], v[:T])
        got = host_u16(out)
        assert max_abs(bf16_f32(got).reshape(-1), ref) <= TOL
        assert got.tobytes() == want.tobytes()        # same call, same split policy
    with pytest.raises(m.ShapeMismatch):
        eng.attention(qd, (kd, vd), empty_u16((qh, d)), cap + 1, g)


@pytest.mark.parametrize("split_tokens", [1024, 256, 64])
def test_persistent_kernel_and_split_merge_pair_give_the_same_bits(m, wl, oracle, split_tokens):
    """The persistent decode schedule (one launch: splits taken from a work
    counter, units longest split first, each item merged in-kernel by the CTA
    whose split completes it -- from a bulk copy of its partials, at once or
    after that CTA's last split, or from plain loads when the partials do not
    fit shared memory) returns the bits of the default schedule, one CTA per
    split and a separate merge.  Under the persistent schedule a query buffer
    that is 4-byte but not 16-byte aligned falls back to the two-kernel form
    (the persistent kernel brings query rows in by bulk copies); the launch
    counter shows which form ran.  Split sizes 1024, 256 and 64 give items of
    up to 4, 16 and 64 splits (every merge form)."""
    torch = torch_mod()
    g = m.AttentionGeometry.new(32, 8, 128)
    rng = np.random.default_rng(1000 + split_tokens)
    pt = 256
    lengths = [4096, 1, 3000, 0, 777, 2500, 64, 4000]
    pool = build_pool(wl, rng, lengths, 8, 128, pt)
    q = rand_bf16(wl, rng, (len(lengths), 32, 128))
    n_seq = len(lengths)
    ws = torch.zeros(m.decode_workspace_bytes(g, n_seq, pool["max_tokens"], split_tokens), dtype=torch.uint8,
                     device="cuda:0")
    kp, vp, table = dev(pool["k_pool"]), dev(pool["v_pool"]), dev(pool["table"])
    seq = dev(np.asarray(lengths, np.int32))
    q_al = dev(q)
    buf = torch.zeros(q.size + 8, dtype=torch.int16, device="cuda:0")
    q_mis = buf[2:2 + q.size].view(q.shape)            # 4 bytes past a 16-byte boundary
    q_mis.copy_(q_al)
    assert q_al.data_ptr() % 16 == 0 and q_mis.data_ptr() % 16 == 4
    outs, launches = [], []
    runs = [(m.DECODE_PERSISTENT, q_al), (m.DECODE_PERSISTENT, q_mis), (m.DECODE_PERSISTENT, q_al),
            (m.DECODE_SPLIT_MERGE, q_al)]
    try:
        for schedule, qd in runs:
            m.set_decode_schedule(schedule)
            out = empty_u16((n_seq, 32, 128))
            out.fill_(0x7FC1)
            before = m.kernel_launches()
            m.decode_paged(g, qd, kp, vp, pool["n_pages"], pt, table, pool["max_pages"], seq, n_seq, ws, out,
                           split_tokens)
            launches.append(m.kernel_launches() - before)
            torch.cuda.synchronize()
            assert m.device_status(0) == 0
            outs.append(host_u16(out))
    finally:
        m.set_decode_schedule(m.DECODE_SPLIT_MERGE)
    assert launches == [1, 2, 1, 2], launches
    assert outs[0].tobytes() == outs[1].tobytes()        # persistent == split + merge (unaligned query)
    assert outs[0].tobytes() == outs[2].tobytes()        # and again (counters left at zero)
    assert outs[0].tobytes() == outs[3].tobytes()        # the default schedule
    for s, L in enumerate(lengths):
        if L == 0:
            assert not np.any(outs[0][s]), s
            continue
        ref = oracle.paged_attention_bf16(32, 8, 128, bf16_f32(q[s].reshape(-1)), pool["k_pool"], pool["v_pool"],
                                          pool["table"][s], pt, L, 1)
        assert max_abs(bf16_f32(outs[0][s].reshape(-1)), ref) <= TOL, s
