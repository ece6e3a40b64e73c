"""The allocation-free paged decode entry point.

mslim_cuda_decode_paged_static_scratch serves callers that cannot allocate
device memory (a serving loop that must not pay cudaMalloc/cudaFree's
implicit device synchronisation, an FFI host that only holds the K/V,
page-table and output pointers and has no device allocator).  Its split
partials live in the library's static 16 MiB device array instead of a
caller workspace.  These tests call it through the C ABI twice in a row and
compare with mslim_cuda_decode_paged, which takes a workspace.  This file is
collected last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from gpu_util import bf16_f32, dev, empty_u16, host_u16, max_abs, torch_mod

pytestmark = pytest.mark.gpu

TOL = 2e-2  # the attention tolerance of the other decode tests


@pytest.fixture(scope="module")
def m():
    import mslim_b200
    mslim_b200.load()
    return mslim_b200


def make_case(m, rng, lengths, page_tokens=256):
    from mslim_b200 import workloads as wl
    kvh, d, qh = 8, 128, 32
    pages = [(L + page_tokens - 1) // page_tokens for L in lengths]
    n_pages = sum(pages) + 2
    perm = rng.permutation(n_pages).astype(np.int32)
    max_pages = max(pages)
    table = np.zeros((len(lengths), max_pages), np.int32)
    cur = 0
    for s, npg in enumerate(pages):
        table[s, :npg] = perm[cur:cur + npg]
        cur += npg
    k_pool = wl.normal_bf16(rng, (n_pages, kvh, page_tokens, d))
    v_pool = wl.normal_bf16(rng, (n_pages, kvh, page_tokens, d))
    q = wl.normal_bf16(rng, (len(lengths), qh, d))
    return dict(q=dev(q), k=dev(k_pool), v=dev(v_pool), table=dev(table), n_pages=n_pages,
                max_pages=max_pages, seq=dev(np.asarray(lengths, np.int32)), n_seq=len(lengths),
                page_tokens=page_tokens)


def call_static(m, g, c, out, split_tokens):
    """Through the C ABI directly (no Python-side workspace anywhere)."""
    from mslim_b200 import _lib
    stream = torch_mod().cuda.current_stream().cuda_stream
    return _lib.lib().mslim_cuda_decode_paged_static_scratch(
        ctypes.byref(g.c()), c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(), c["n_pages"],
        c["page_tokens"], c["table"].data_ptr(), c["max_pages"], c["seq"].data_ptr(), c["n_seq"],
        split_tokens, out.data_ptr(), stream)


def call_workspace(m, g, c, split_tokens):
    torch = torch_mod()
    ws = torch.zeros(m.decode_workspace_bytes(g, c["n_seq"], c["max_pages"] * c["page_tokens"], split_tokens),
                     dtype=torch.uint8, device="cuda:0")
    out = empty_u16((c["n_seq"], g.query_heads, g.head_dim))
    m.decode_paged(g, c["q"], c["k"], c["v"], c["n_pages"], c["page_tokens"], c["table"], c["max_pages"],
                   c["seq"], c["n_seq"], ws, out, split_tokens)
    torch.cuda.synchronize()
    return host_u16(out)


@pytest.mark.parametrize("split_tokens", [0, 1024])
def test_static_scratch_matches_workspace_entry_point_twice(m, split_tokens):
    torch = torch_mod()
    g = m.AttentionGeometry.new(32, 8, 128)
    rng = np.random.default_rng(21)
    case_a = make_case(m, rng, [9000, 1, 4097, 300, 12000, 64])
    case_b = make_case(m, rng, [5000, 7000, 33])
    for case in (case_a, case_b, case_a):   # two calls in a row, contents of the
        want = call_workspace(m, g, case, split_tokens)  # shared array from the
        for _ in range(2):                                # previous call left behind
            out = empty_u16((case["n_seq"], 32, 128))
            out.fill_(0x7FC1)
            rc = call_static(m, g, case, out, split_tokens)
            assert rc == 0, m._lib.last_error()
            torch.cuda.synchronize()
            got = host_u16(out)
            assert max_abs(bf16_f32(got), bf16_f32(want)) <= TOL
            if split_tokens:
                # same split size -> same arithmetic -> same bits
                assert got.tobytes() == want.tobytes()
    assert m.device_status(0) == 0


def test_static_scratch_rejects_oversized_requests(m):
    g = m.AttentionGeometry.new(32, 8, 128)
    rng = np.random.default_rng(22)
    case = make_case(m, rng, [32768] * 4)
    out = empty_u16((4, 32, 128))
    # 4 sessions x 32 heads x 512 splits of 64 tokens x 132 floats > 16 MiB
    rc = call_static(m, g, case, out, 64)
    assert rc == m._lib.ERR_SHAPE_MISMATCH
    assert "static scratch" in m._lib.last_error()


def test_static_scratch_takes_larger_splits_when_the_policy_split_overflows(m):
    """96 sessions of 32768 tokens: at the library's own split size (3072
    tokens) the partials need more than the 16 MiB array, so split_tokens == 0
    doubles the split until they fit.  The result equals the workspace entry point at that
    doubled split, bit for bit, on two calls in a row."""
    torch = torch_mod()
    g = m.AttentionGeometry.new(32, 8, 128)
    n_seq, L, pt = 96, 32768, 256
    limit = 16 << 20
    policy = m.decode_split_tokens(g, n_seq, L)
    assert m.decode_workspace_bytes(g, n_seq, L, policy) > limit     # the case overflows
    st = policy
    while m.decode_workspace_bytes(g, n_seq, L, st) > limit and st < L:
        st *= 2
    assert st > policy and m.decode_workspace_bytes(g, n_seq, L, st) <= limit
    pages = L // pt
    n_pages = n_seq * pages
    gen = torch.Generator(device="cuda:0")
    gen.manual_seed(23)
    k = torch.randn((n_pages, 8, pt, 128), generator=gen, device="cuda:0", dtype=torch.bfloat16)
    v = torch.randn((n_pages, 8, pt, 128), generator=gen, device="cuda:0", dtype=torch.bfloat16)
    q = torch.randn((n_seq, 32, 128), generator=gen, device="cuda:0", dtype=torch.bfloat16)
    table = torch.randperm(n_pages, generator=gen, device="cuda:0").to(torch.int32).view(n_seq, pages)
    seq = torch.full((n_seq,), L, dtype=torch.int32, device="cuda:0")
    case = dict(q=q, k=k, v=v, table=table, n_pages=n_pages, max_pages=pages, seq=seq, n_seq=n_seq,
                page_tokens=pt)
    want = call_workspace(m, g, case, st)
    for _ in range(2):
        out = empty_u16((n_seq, 32, 128))
        out.fill_(0x7FC1)
        rc = call_static(m, g, case, out, 0)
        assert rc == 0, m._lib.last_error()
        torch.cuda.synchronize()
        assert host_u16(out).tobytes() == want.tobytes()
    assert m.device_status(0) == 0
