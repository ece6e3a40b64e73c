"""Host logic of the multi-GPU decode path, run as world-size-2 gloo ranks on
the CPU: longest-processing-time session sharding (each session owned by
exactly one rank, loads balanced) and the max-over-ranks step time the bench
reports."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "vk-shei_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    import bench
    from mslim_b200 import workloads
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    layout = workloads.c4_layout(seed=3)
    mine = bench.lpt_shard(layout.lengths, world, rank)
    shards = [None] * world
    dist.all_gather_object(shards, mine)
    load = torch.tensor([float(layout.lengths[mine].sum())])
    dist.all_reduce(load, op=dist.ReduceOp.MAX)
    t = torch.tensor([10.0 + rank])       # a per-rank step time
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        q.put((shards, float(load.item()), float(t.item()), layout.lengths.tolist()))
    dist.barrier()
    dist.destroy_process_group()


def test_lpt_shards_cover_every_session_once_and_balance():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    shards, max_load, max_t, lengths = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(lengths)))
    assert not set(shards[0]) & set(shards[1])
    total = sum(lengths)
    # LPT keeps the heaviest rank within one session of the mean load
    assert max_load <= total / world + max(lengths)
    assert max_load >= total / world
    assert max_t == 11.0


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_lpt_shard_is_a_partition(world):
    import bench
    from mslim_b200 import workloads
    lengths = workloads.c4_layout(seed=3).lengths
    parts = [bench.lpt_shard(lengths, world, r) for r in range(world)]
    assert sorted(i for p in parts for i in p) == list(range(len(lengths)))
    loads = [int(np.asarray(lengths)[p].sum()) for p in parts]
    assert max(loads) - min(loads) <= max(lengths)


def _argmax_worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "vk-shei_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    from mslim_b200.model import pick_shard_argmax, shard_argmax_key
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(9)
    vocab, rows = 1000, 6
    logits = rng.standard_normal((rows, vocab)).astype(np.float32)
    logits[1, 100] = logits[1, 900] = 50.0        # tie across shards: the later index wins
    logits[2, 10] = logits[2, 11] = 60.0          # tie inside a shard
    logits[3, :] = -0.0
    logits[3, 700] = 0.0                          # +0 above -0
    bits = torch.from_numpy(logits).to(torch.bfloat16).view(torch.int16).clone()
    bits[4, 3] = 0x7FC0                           # a positive NaN is the largest
    per = (vocab + world - 1) // world
    lo, hi = rank * per, min(vocab, (rank + 1) * per)
    shard = bits[:, lo:hi]
    # local argmax under total_cmp, last index among equals (what mslim_argmax does)
    s32 = shard.to(torch.int32)
    key = torch.where(s32 < 0, s32 ^ 0x7FFF, s32)
    order = key * (hi - lo) + torch.arange(hi - lo)
    local = order.argmax(dim=1).to(torch.int32)
    mine = shard_argmax_key(torch, shard.gather(1, local.long().view(-1, 1)).view(-1), local, lo)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    best = pick_shard_argmax(torch, torch.stack(every))
    if rank == 0:
        q.put((best.tolist(), bits.numpy()))
    dist.barrier()
    dist.destroy_process_group()


def test_vocab_sharded_argmax_keeps_the_cpu_tie_rule(oracle):
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_argmax_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    best, bits = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    f32 = (bits.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    want = [oracle.argmax_last(r) for r in f32]
    assert best == want
    assert best[1] == 900 and best[2] == 11 and best[3] == 700 and best[4] == 3
