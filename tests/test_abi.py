"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, and its host-side contract checks match the reference's rules
(src/attention_kernel.rs:141-206, src/portable.rs:806-825)."""
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mslim_cuda.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mslim_cuda_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def m():
    import mslim_b200
    mslim_b200.load()
    return mslim_b200


def test_library_exports_every_declared_symbol(m):
    from mslim_b200 import _lib
    L = _lib.lib()
    declared = header_functions()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(L, name), f"{name} declared in the header but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert sorted(_lib.SIGNATURES) == declared


def test_static_archive_and_shared_library_built():
    base = os.path.join(ROOT, "vk-shei_b200", "mslim_b200")
    assert os.path.exists(os.path.join(base, "libmslim_cuda.so"))
    assert os.path.exists(os.path.join(base, "libmslim_cuda.a"))


def test_implementation_digest_names_the_sources_the_library_was_built_from(m):
    """mslim_cuda_implementation_digest, the library's share of the
    calibration profile identity (src/calibration_profile.rs:90-125): the
    digest the build recipe computes over the current sources."""
    import sys
    from mslim_b200 import _lib
    sys.path.insert(0, os.path.join(ROOT, "vk-shei_b200"))
    import build
    got = _lib.lib().mslim_cuda_implementation_digest().decode()
    assert re.fullmatch(r"[0-9a-f]{64}", got)
    assert got == build.source_digest(), "the loaded library was built from other sources"


def test_default_is_reference_and_experimental_opt_in_is_mandatory(m):
    # src/attention_kernel.rs:145-158
    assert m.AttentionKernelConfig.from_json("{}") == m.AttentionKernelConfig()
    c = m.AttentionKernelConfig(mode=m.AttentionKernelMode.ONLINE_EXPERIMENTAL)
    with pytest.raises(m.InvalidConfig):
        c.validate_activation(False)
    c.validate_activation(True)


@pytest.mark.parametrize("kw", [
    dict(work_group=0),
    dict(block_keys=33),
    dict(splits=2),
    dict(mode="strict_tiled", splits=2),
    dict(mode="split_kv_experimental", splits=65),
    dict(mode="split_kv_experimental", splits=1),
    dict(mode="split_kv_experimental", splits=8, block_queries=2),
    dict(block_queries=3),
    dict(block_queries=2),  # reference mode cannot carry tuning values
])
def test_reject_ignored_or_unbounded_configuration(m, kw):
    # src/attention_kernel.rs:159-187
    if "mode" in kw:
        kw = dict(kw, mode=m.AttentionKernelMode(kw["mode"]))
    with pytest.raises(m.InvalidConfig):
        m.AttentionKernelConfig(**kw).validate()


def test_unknown_fields_rejected(m):
    with pytest.raises(m.InvalidConfig):
        m.AttentionKernelConfig.from_json('{"epsilon":0.1}')
    with pytest.raises(m.InvalidConfig):
        m.AttentionKernelConfig.from_json('{"mode":"fast"}')


def test_scratch_is_bounded_and_strict_has_no_global_scores(m):
    # src/attention_kernel.rs:188-205
    strict = m.AttentionKernelConfig(mode=m.AttentionKernelMode.STRICT_TILED)
    assert strict.decode_scratch_bytes(32, 128) == 0
    assert strict.local_bytes(128) < 64 * 1024
    split = m.AttentionKernelConfig(mode=m.AttentionKernelMode.SPLIT_KV_EXPERIMENTAL, splits=8)
    assert split.decode_scratch_bytes(32, 128) == 32 * 8 * 130 * 4
    with pytest.raises(m.InvalidConfig):
        split.decode_scratch_bytes(2 ** 40, 128)
    with pytest.raises(m.InvalidConfig):
        strict.local_bytes(257)


def test_ids_follow_the_reference_format(m):
    # src/attention_kernel.rs:101-110: Debug name of the mode, lower-cased.
    assert m.AttentionKernelConfig().id() == "reference"
    c = m.AttentionKernelConfig(mode=m.AttentionKernelMode.SPLIT_KV_EXPERIMENTAL, splits=8)
    assert c.id() == "splitkvexperimental-q1-k64-wg64-s8"
    c = m.AttentionKernelConfig(mode=m.AttentionKernelMode.ONLINE_EXPERIMENTAL, block_queries=2)
    assert c.id() == "onlineexperimental-q2-k64-wg64-s1"


def test_snapshot_contract(m):
    # src/attention_kernel.rs:80-91
    m.AttentionKernelConfig().check_snapshot(None)
    strict = m.AttentionKernelConfig(mode=m.AttentionKernelMode.STRICT_TILED)
    with pytest.raises(m.InvalidConfig):
        strict.check_snapshot(None)
    strict.check_snapshot({"mode": "strict_tiled"})


def test_geometry_rules(m):
    # src/portable.rs:421-443, :808
    with pytest.raises(m.InvalidGeometry):
        m.AttentionGeometry.new(3, 2, 32)
    with pytest.raises(m.InvalidGeometry):
        m.AttentionGeometry.new(0, 1, 8)
    g = m.AttentionGeometry.new(32, 8, 128)
    assert [g.kv_head_for_query(h) for h in (0, 3, 4, 31)] == [0, 0, 1, 7]
    with pytest.raises(m.ShapeMismatch):
        g.kv_head_for_query(32)


def test_decode_workspace_bytes(m):
    g = m.AttentionGeometry.new(32, 8, 128)
    # a head of work counters (two words, then one arrival counter per item,
    # 16384 items) and the split partials {acc[128], m, l, 2 pad} in f32
    assert m.decode_workspace_bytes(g, 64, 32768, 2048) == 256 + 4 * 16384 + 64 * 32 * 16 * 132 * 4
    with pytest.raises(m.ShapeMismatch):
        m.decode_workspace_bytes(g, 1, 100, 100)


def _fluid_step_time(lengths, per_seq, slots, st, cap=2.5, fixed=300.0, exit_cost=8.0):
    """The split kernel's step time as the library models it: CTAs start in
    grid order as resident places free up; n running CTAs each stream at
    min(cap, slots / n) times their full-load rate."""
    import heapq
    lens = [int(x) for x in lengths if x > 0]
    max_splits = max([1] + [-(-L // st) for L in lens])
    running, level, t = [], 0.0, 0.0

    def finish():
        nonlocal level, t
        rate = min(cap, slots / len(running))
        top = heapq.heappop(running)
        t += (top - level) / rate
        level = top

    for L in [max(int(x), 0) for x in lengths]:
        n = -(-L // st) if L else 0
        slen = -(-(-(-L // n)) // 64) * 64 if n else 0
        for _ in range(per_seq):
            for k in range(max_splits):
                work = (min(slen, L - k * slen) + fixed) if k < n else exit_cost
                if len(running) == slots:
                    finish()
                heapq.heappush(running, level + work)
    while running:
        finish()
    return t


SPLIT_CANDIDATES = (3072, 2688, 2048, 1536, 1024, 768, 512, 256)


def _choose_split(lengths, per_seq, slots, cap, max_waves=16):
    """The library's choice among the split candidates: the shortest modelled
    step (per-CTA speed-up cap `cap`), the longer split within 0.5 %; a
    candidate needing more than max_waves waves of CTAs is skipped (except the
    longest); the result is at most the longest sequence rounded up to 64
    tokens, at least 256."""
    longest = max([0] + [int(x) for x in lengths])
    if len(lengths) * per_seq * max(1, -(-longest // SPLIT_CANDIDATES[0])) > max_waves * slots:
        return min(SPLIT_CANDIDATES[0], max(256, -(-longest // 64) * 64))   # only the longest is modelled
    best, best_st = 0.0, SPLIT_CANDIDATES[0]
    for st in SPLIT_CANDIDATES:
        grid = len(lengths) * per_seq * max(1, -(-longest // st))
        if st != SPLIT_CANDIDATES[0] and grid > max_waves * slots:
            continue
        t = _fluid_step_time(lengths, per_seq, slots, st, cap=cap)
        if best == 0.0 or t < best * 0.995:
            best, best_st = t, st
    return min(best_st, max(256, -(-longest // 64) * 64))


def _slots(head_dim):
    kd = 64 if head_dim <= 64 else 128 if head_dim <= 128 else 256
    return 148 * (3 if kd == 64 else 2 if kd == 128 else 1)


def test_split_tokens_for_host_lengths(m):
    """mslim_cuda_decode_split_tokens_for_lengths runs the model of the split
    kernel's CTAs on the GPU over the candidate split sizes and keeps the
    fastest: it equals this restatement of the model for the C4 draw and its
    shards of 2, 4 and 8 GPUs, where it picks the sizes measured best on B200
    (3072 tokens on 1 GPU and on the shards of 4, 2688 on those of 2 and 8),
    and is deterministic."""
    import numpy as np
    import bench
    from mslim_b200 import workloads
    g = m.AttentionGeometry.new(32, 8, 128)
    L = workloads.c4_layout(seed=3).lengths[:64]
    for world in (1, 2, 4, 8):
        for rank in sorted({0, world - 1}):
            lengths = L[bench.lpt_shard(L, world, rank)].astype(np.int32)
            st = m.decode_split_tokens_for_lengths(g, lengths)
            assert st in SPLIT_CANDIDATES
            assert st == m.decode_split_tokens_for_lengths(g, lengths)
            assert st == _choose_split(lengths, 8, 296, cap=2.5), (world, rank, st)
            if rank == 0:
                assert st == {1: 3072, 2: 2688, 4: 3072, 8: 2688}[world]
    assert m.decode_split_tokens_for_lengths(g, np.zeros(3, np.int32)) == 256
    assert m.decode_split_tokens_for_lengths(g, np.array([100, 7], np.int32)) == 256


def test_split_tokens_for_device_lengths(m):
    """split_tokens == 0 (lengths on the device, only the longest known):
    the same model with every sequence at max_tokens and a per-CTA speed-up
    cap of 1 (equal lengths: every CTA of a wave starts and ends together).
    The picks for C5's decode at TP 1, 2 and 8 (8 sessions of ~8.3 K tokens)
    are the splits measured fastest for those shapes on B200 (one full wave of
    CTAs each); short histories keep 256-token splits so their few items
    still spread over the GPU."""
    import numpy as np
    cases = [((32, 8, 128), 8, 8260), ((16, 4, 128), 8, 8260), ((4, 1, 128), 8, 8260),
             ((32, 8, 128), 1, 1025), ((32, 8, 128), 1, 520), ((32, 8, 128), 64, 32768),
             ((32, 8, 128), 4, 4096), ((32, 8, 64), 4, 4096), ((32, 8, 256), 2, 16384),
             ((64, 2, 128), 3, 5000), ((32, 8, 128), 1, 40)]
    for (qh, kvh, d), n_seq, max_tokens in cases:
        g = m.AttentionGeometry.new(qh, kvh, d)
        group = qh // kvh
        chunks = 1 if group <= 16 else group // 16
        want = _choose_split(np.full(n_seq, max_tokens, np.int32), kvh * chunks, _slots(d), cap=1.0)
        got = m.decode_split_tokens(g, n_seq, max_tokens)
        assert got == want, ((qh, kvh, d), n_seq, max_tokens, got, want)
        assert got == m.decode_split_tokens(g, n_seq, max_tokens)     # remembered, same answer
        assert 256 <= got <= 3072 and got % 64 == 0
    g = m.AttentionGeometry.new(32, 8, 128)
    assert m.decode_split_tokens(g, 8, 8260) == 2688          # C5, TP 1 (256 CTAs)
    assert m.decode_split_tokens(m.AttentionGeometry.new(16, 4, 128), 8, 8260) == 1024   # TP 2 (288 CTAs)
    assert m.decode_split_tokens(m.AttentionGeometry.new(4, 1, 128), 8, 8260) == 256     # TP 8 (264 CTAs)
    assert m.decode_split_tokens(g, 1, 1025) == 256           # C1
    # many waves at the longest split: the answer is the longest split, without
    # simulating millions of CTAs (a decode call pays for the policy)
    import time
    t0 = time.perf_counter()
    assert m.decode_split_tokens(g, 4096, 131072) == 3072
    lens = np.full(4096, 131072, np.int32)
    assert m.decode_split_tokens_for_lengths(g, lens) == 3072 == _choose_split(lens, 8, 296, cap=2.5)
    assert time.perf_counter() - t0 < 0.5
    # a workspace sized at split 256 holds the policy's partials for every
    # shorter history (the policy's split count is not monotone in the length)
    cap = 9000
    big = m.decode_workspace_bytes(g, 1, cap, 256)
    assert all(m.decode_workspace_bytes(g, 1, t) <= big for t in range(1, cap + 1, 97))


def test_kernel_launch_counter_reads_without_a_gpu(m):
    """mslim_cuda_kernel_launches is a host counter: it reads without a
    device and only grows."""
    a = m.kernel_launches()
    b = m.kernel_launches()
    assert 0 <= a <= b


def test_decode_schedule_setting(m):
    """mslim_cuda_set_decode_schedule: split + merge by default, persistent on
    request, anything else rejected (host state only, no device needed)."""
    assert m.get_decode_schedule() == m.DECODE_SPLIT_MERGE
    try:
        m.set_decode_schedule(m.DECODE_PERSISTENT)
        assert m.get_decode_schedule() == m.DECODE_PERSISTENT
        with pytest.raises(m.ShapeMismatch):
            m.set_decode_schedule(7)
        assert m.get_decode_schedule() == m.DECODE_PERSISTENT
    finally:
        m.set_decode_schedule(m.DECODE_SPLIT_MERGE)
    assert m.get_decode_schedule() == m.DECODE_SPLIT_MERGE
