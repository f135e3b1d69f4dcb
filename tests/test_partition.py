"""Length-balanced sharding of decode sequences across GPUs (host logic, CPU).

Includes a two-rank gloo run: every rank derives its shard of the global batch
independently (as bench.py's ranks do) and the union of the shards, gathered
over the process group, is the whole batch exactly once."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from paged_decode import partition as P
from paged_decode import workloads as W


def test_lpt_covers_every_sequence_once():
    lens = W.long_tail_lengths(0)
    for n in (1, 2, 4, 8):
        shards = P.lpt_assign(lens, n)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(lens)))


def test_lpt_is_balanced_within_its_bound():
    for seed in range(4):
        lens = W.qwen3b_decode(seed, batch=512).seq_lens
        for n in (2, 4, 8):
            loads = P.shard_loads(lens, P.lpt_assign(lens, n))
            bound = P.makespan_bound(lens, n)
            # LPT is within 4/3 of optimal; uniform lengths land much closer
            assert max(loads) <= bound * 4 / 3 + max(lens)
            assert max(loads) / bound < 1.01


def test_lpt_heavy_tail_respects_longest_sequence():
    lens = W.long_tail_lengths(0)
    loads = P.shard_loads(lens, P.lpt_assign(lens, 8))
    assert max(loads) >= max(lens)
    assert max(loads) <= P.makespan_bound(lens, 8) + max(lens)


def test_lpt_rejects_zero_ranks():
    with pytest.raises(ValueError):
        P.lpt_assign([1, 2], 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench

    spec = bench.rank_spec(rank, world, seed=0, layer=0)
    lens = torch.tensor(spec.seq_lens, dtype=torch.int64)
    n = torch.tensor([lens.numel()], dtype=torch.int64)
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, n)
    mx = int(max(s.item() for s in sizes))
    padded = torch.full((mx,), -1, dtype=torch.int64)
    padded[: lens.numel()] = lens
    gathered = [torch.zeros(mx, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(gathered, padded)
    if rank == 0:
        out.put([g[g >= 0].tolist() for g in gathered])
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_shard_the_global_batch():
    import bench

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    shards = q.get()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    glob = sorted(bench.global_lengths(world, 0))
    assert sorted(shards[0] + shards[1]) == glob
    loads = [sum(s) for s in shards]
    assert max(loads) / (sum(loads) / world) < 1.01
