"""Multi-rank host logic of bench.py on CPU: prompt sharding across ranks, the call sites' shares,
and the gather of the outputs to rank 0, run as two gloo ranks (world size 2, 127.0.0.1)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def test_shards_cover_every_prompt_once_and_balance_lengths():
    lengths = bench.workload_lengths(1024, 5)
    for world in (1, 2, 4, 8):
        shards = [bench.shard_prompts(lengths, world, r) for r in range(world)]
        flat = sorted(p for s in shards for p in s)
        assert flat == list(range(1024))
        assert len({len(s) for s in shards}) == 1  # the same number of prompts (CFG pairs) per rank
        sums = [sum(lengths[2 * p] + lengths[2 * p + 1] for p in s) for s in shards]
        assert max(sums) - min(sums) <= 0.01 * max(sums)  # K/V work within 1 %


def test_call_site_shards():
    """bench.py's call sites at N GPUs: every problem on exactly one rank when sharded; batches
    smaller than N, and the B = 2 self-attention pair, run whole on every rank (replicas)."""
    for n in (2, 8, 64, 128, 256):
        for world in (1, 2, 4, 8):
            parts = [bench.site_shard(n, r, world) for r in range(world)]
            if n >= world:
                assert sorted(i for idx, rep in parts for i in idx) == list(range(n))
                assert not any(rep for _, rep in parts)
                assert max(len(p[0]) for p in parts) - min(len(p[0]) for p in parts) <= 1
            else:
                assert all(rep and p == list(range(n)) for p, rep in parts)
    assert bench.site_shard(2, 1, 4, shardable=False) == ([0, 1], True)
    assert bench.site_shard(2, 0, 1, shardable=False) == ([0, 1], False)


def test_cpulist_parsing():
    """bench.py pins each rank to its GPU's local CPUs, read from sysfs lists like these."""
    assert bench.parse_cpulist("0-3,8,10-11") == {0, 1, 2, 3, 8, 10, 11}
    assert bench.parse_cpulist("0-47,96-143\n".strip()) == set(range(48)) | set(range(96, 144))
    assert bench.parse_cpulist("") == set()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths = bench.workload_lengths(64, 5)
        mine = bench.shard_prompts(lengths, world, rank)
        seqs = [s for p in mine for s in (2 * p, 2 * p + 1)]
        # each rank's "output" rows tagged with their sequence ids, padded to the largest shard
        # like bench.py's send buffers, gathered to rank 0
        shard_max = max(len(bench.shard_prompts(lengths, world, r)) for r in range(world)) * 2
        send = torch.full((shard_max,), -1.0)
        send[: len(seqs)] = torch.tensor(seqs, dtype=torch.float32)
        recv = [torch.empty(shard_max) for _ in range(world)] if rank == 0 else None
        dist.gather(send, recv, dst=0)
        t = torch.tensor([float(10 + rank)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the bench's max-over-ranks timing
        if rank == 0:
            got = sorted(int(x) for r in recv for x in r.tolist() if x >= 0)
            out.put((got, float(t.item())))
    finally:
        dist.destroy_process_group()


def test_gather_to_rank0_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got, tmax = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert got == list(range(128))  # every sequence of the 64 prompts arrives exactly once
    assert tmax == 11.0
    assert all(p.exitcode == 0 for p in procs)
