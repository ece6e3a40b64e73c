"""The tensor-parallel decode reduction (mslim_cuda_tp_allreduce_rmsnorm):
with one rank it must equal the residual add + RMSNorm bitwise; with two ranks
(one per GPU, skipped below two GPUs) every rank must get the same bits, equal
to the fp32 rank-order sum rounded once."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROWS, HIDDEN, EPS = 8, 4096, 1e-5


def _bf16(rng, n, scale=1.0):
    from mslim_b200 import workloads
    return workloads.bf16_bits(rng.standard_normal(n).astype(np.float32) * np.float32(scale))


def _u16(t):
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_one_rank_equals_residual_rmsnorm():
    import torch
    import mslim_b200 as m
    from gpu_util import dev
    from mslim_b200.tp import TpComm
    rng = np.random.default_rng(21)
    comm = TpComm(1, 0, ROWS, HIDDEN)
    try:
        w = dev(_bf16(rng, HIDDEN))
        x0 = _bf16(rng, ROWS * HIDDEN).reshape(ROWS, HIDDEN)
        for call in range(5):      # both slots, the counters advancing
            part = _bf16(rng, ROWS * HIDDEN, 0.5).reshape(ROWS, HIDDEN)
            slot = comm.next_slot()
            comm.slot(slot, ROWS).view(torch.int16).copy_(dev(part))
            xa, xb = dev(x0), dev(x0)
            ya, yb = torch.empty_like(xa), torch.empty_like(xa)
            comm.allreduce_rmsnorm(slot, xa, w, ya, ROWS, EPS)
            m.residual_rmsnorm(xb, dev(part), w, yb, ROWS, HIDDEN, EPS)
            torch.cuda.synchronize()
            assert np.array_equal(_u16(xa), _u16(xb)) and np.array_equal(_u16(ya), _u16(yb)), call
        assert m.device_status(0) == 0
    finally:
        torch.cuda.synchronize()
        comm.close()


def _two_rank_worker(rank, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "vk-shei_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    import mslim_b200 as m
    from mslim_b200 import workloads
    from mslim_b200.tp import TpComm
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    comm = TpComm(2, rank, ROWS, HIDDEN)
    rng = np.random.default_rng(100)            # same draws on both ranks
    w = workloads.bf16_bits(rng.standard_normal(HIDDEN).astype(np.float32))
    x = workloads.bf16_bits(rng.standard_normal(ROWS * HIDDEN).astype(np.float32))
    parts = [workloads.bf16_bits(rng.standard_normal(ROWS * HIDDEN).astype(np.float32) * 0.5)
             for _ in range(2)]

    def t(a):
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)

    outs = []
    xt = t(x).view(ROWS, HIDDEN)
    for call in range(4):
        slot = comm.next_slot()
        comm.slot(slot, ROWS).copy_(t(parts[rank]).view(ROWS, HIDDEN))
        y = torch.empty_like(xt)
        comm.allreduce_rmsnorm(slot, xt, t(w), y, ROWS, EPS)
        torch.cuda.synchronize()
        outs.append((_u16(xt), _u16(y)))
    status = m.device_status(rank)
    dist.barrier()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, outs, status, x, w, parts))


def test_two_ranks_agree_and_sum_in_rank_order(oracle):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs (one rank per GPU)")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, rest) for r, *rest in [q.get(timeout=180) for _ in range(2)])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    (outs0, st0, x, w, parts), (outs1, st1, *_) = res[0], res[1]
    assert st0 == 0 and st1 == 0
    for (x0, y0), (x1, y1) in zip(outs0, outs1):
        assert np.array_equal(x0, x1) and np.array_equal(y0, y1)
    # call 0 against the restatement: bf16(x + bf16(p0 + p1)), then RMSNorm
    f = lambda b: (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    delta = oracle.bf16_from_f32(f(parts[0]) + f(parts[1]))
    xn = oracle.bf16_from_f32(f(x) + f(delta))
    assert np.array_equal(outs0[0][0].reshape(-1), xn)


def test_a_peer_that_never_arrives_times_out_and_the_context_survives():
    """Failure detection without a fault: a two-rank communicator whose second
    rank is never run (its slots alias this rank's, its ready counter is never
    written).  The kernel's bounded wait gives up (~2 s), records a timeout in
    the status word, leaves x and y untouched, and the context stays usable."""
    import ctypes

    import torch
    import mslim_b200 as m
    from gpu_util import dev
    from mslim_b200 import _lib
    from mslim_b200.tp import TpComm
    rng = np.random.default_rng(31)
    comm = TpComm(1, 0, ROWS, HIDDEN)
    try:
        c = _lib.TpComm()
        ctypes.memmove(ctypes.byref(c), ctypes.byref(comm.c), ctypes.sizeof(c))
        c.world = 2
        c.data[1], c.flags[1] = comm.c.data[0], comm.c.flags[0]
        x = dev(_bf16(rng, ROWS * HIDDEN).reshape(ROWS, HIDDEN))
        x_before = _u16(x)
        y = torch.zeros_like(x)
        w = dev(_bf16(rng, HIDDEN))
        assert m.device_status(0) == 0
        m.check(_lib.lib().mslim_cuda_tp_allreduce_rmsnorm(ctypes.byref(c), 0, x.data_ptr(), w.data_ptr(),
                                                           y.data_ptr(), ROWS, EPS,
                                                           torch.cuda.current_stream().cuda_stream))
        assert m.device_status(0) == _lib.ERR_DEVICE_TIMEOUT
        assert np.array_equal(_u16(x), x_before) and not _u16(y).any()
        # the context is intact: other kernels still run and the status is clear
        a = dev(_bf16(rng, 1024))
        out = torch.empty_like(a)
        m.residual_add(a, a, out, 1024)
        torch.cuda.synchronize()
        assert m.device_status(0) == 0
    finally:
        torch.cuda.synchronize()
        comm.close()


def _set_call_numbers(comm, value: int):
    """Writes every row's call counter of a communicator (uint32, set here as
    its int32 bit pattern) so a test can start next to the wrap."""
    import torch
    from mslim_b200.tp import _DeviceArray
    ep = torch.as_tensor(_DeviceArray(comm.c.epoch, (comm.max_rows,), "<i4"), device="cuda")
    ep.fill_(value)
    torch.cuda.synchronize()


def test_one_rank_across_the_call_number_wrap():
    """Call numbers are uint32 per row and wrap after 2^32 calls; the
    reduction compares them as serial numbers and skips 0, so calls on either
    side of the wrap still equal the residual add + RMSNorm bitwise."""
    import torch
    import mslim_b200 as m
    from gpu_util import dev
    from mslim_b200.tp import TpComm
    rng = np.random.default_rng(22)
    comm = TpComm(1, 0, ROWS, HIDDEN)
    try:
        _set_call_numbers(comm, -3)          # 0xFFFFFFFD: the next calls are ..FE, ..FF, 1, 2
        w = dev(_bf16(rng, HIDDEN))
        x0 = _bf16(rng, ROWS * HIDDEN).reshape(ROWS, HIDDEN)
        for call in range(4):
            part = _bf16(rng, ROWS * HIDDEN, 0.5).reshape(ROWS, HIDDEN)
            slot = comm.next_slot()
            comm.slot(slot, ROWS).view(torch.int16).copy_(dev(part))
            xa, xb = dev(x0), dev(x0)
            ya, yb = torch.empty_like(xa), torch.empty_like(xa)
            comm.allreduce_rmsnorm(slot, xa, w, ya, ROWS, EPS)
            m.residual_rmsnorm(xb, dev(part), w, yb, ROWS, HIDDEN, EPS)
            torch.cuda.synchronize()
            assert np.array_equal(_u16(xa), _u16(xb)) and np.array_equal(_u16(ya), _u16(yb)), call
        assert m.device_status(0) == 0
    finally:
        torch.cuda.synchronize()
        comm.close()


def test_a_missing_peer_still_times_out_at_the_call_number_wrap():
    """At the wrap the next call number would be 0, the value of a flag no peer
    has written; it is skipped, so a peer that never arrives is still waited
    for (and the bounded wait gives up) instead of being taken as arrived."""
    import ctypes

    import torch
    import mslim_b200 as m
    from gpu_util import dev
    from mslim_b200 import _lib
    from mslim_b200.tp import TpComm
    rng = np.random.default_rng(32)
    comm = TpComm(1, 0, ROWS, HIDDEN)
    try:
        _set_call_numbers(comm, -1)          # 0xFFFFFFFF: the next call number wraps
        c = _lib.TpComm()
        ctypes.memmove(ctypes.byref(c), ctypes.byref(comm.c), ctypes.sizeof(c))
        c.world = 2
        c.data[1], c.flags[1] = comm.c.data[0], comm.c.flags[0]
        x = dev(_bf16(rng, ROWS * HIDDEN).reshape(ROWS, HIDDEN))
        x_before = _u16(x)
        y = torch.zeros_like(x)
        w = dev(_bf16(rng, HIDDEN))
        assert m.device_status(0) == 0
        m.check(_lib.lib().mslim_cuda_tp_allreduce_rmsnorm(ctypes.byref(c), 0, x.data_ptr(), w.data_ptr(),
                                                           y.data_ptr(), ROWS, EPS,
                                                           torch.cuda.current_stream().cuda_stream))
        assert m.device_status(0) == _lib.ERR_DEVICE_TIMEOUT
        assert np.array_equal(_u16(x), x_before) and not _u16(y).any()
    finally:
        torch.cuda.synchronize()
        comm.close()
