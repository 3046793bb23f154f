"""Host-side logic of the multi-GPU bench on CPU ranks (gloo, world size 2):
sequence sharding covers the global batch exactly once, every rank draws the
same prompts, and timings reduce to the slowest rank."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def test_shard_partitions_global_batch():
    for world in (1, 2, 4, 8, 3):
        seen = []
        for r in range(world):
            s, n = bench.shard(256, world, r)
            seen.extend(range(s, s + n))
        assert seen == list(range(256))
    assert bench.shard(256, 8, 7) == (224, 32)


def test_lpt_partition_of_the_long_context_prompts():
    """Long-context run: LPT over prompt + new tokens covers every sequence
    once, and no rank exceeds another by more than the heaviest sequence."""
    lens = [len(p) + bench.LONG_NEW for p in bench.long_prompts()]
    assert len(lens) == bench.LONG_SEQS
    for world in (1, 2, 4, 8):
        parts, loads = bench.lpt_partition(lens, world)
        assert sorted(i for part in parts for i in part) == list(range(len(lens)))
        assert [sum(lens[i] for i in part) for part in parts] == loads
        assert max(loads) - min(loads) <= max(lens)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        start, count = bench.shard(256, world, rank)
        prompts = bench.prompts_for(start, count, 16, 256)
        # every rank must agree on the global prompt set
        full = torch.zeros(256, 16, dtype=torch.long)
        full[start:start + count] = prompts
        dist.all_reduce(full)
        ms = bench.max_over_ranks(10.0 + rank, world)
        bench.barrier(world)
        q.put((rank, start, count, int(full.sum()), ms))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharding_and_max_timing():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    ref_sum = int(bench.prompts_for(0, 256, 16, 256).sum())
    assert [r[1:3] for r in res] == [(0, 128), (128, 128)]
    assert all(r[3] == ref_sum for r in res)
    assert all(r[4] == 11.0 for r in res)
