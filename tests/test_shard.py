"""Head-sharding host logic on CPU: the shard plan, and a world_size-2 gloo run of the
one-process-per-GPU layout (each rank takes its shard of heads, computes it, the outputs are
gathered for verification only). The per-rank compute here is the CPU oracle, planted by the
test in place of the GPU kernel; the code under test is the partitioning and reassembly."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fa.shard import Shard, plan_shards


@pytest.mark.parametrize("total,world", [(64, 1), (64, 2), (64, 8), (10, 4), (3, 8), (0, 2), (256, 3)])
def test_plan_shards_balanced_contiguous(total, world):
    shards = plan_shards(total, world)
    assert len(shards) == world
    assert shards[0].start == 0 and shards[-1].stop == total
    for a, b in zip(shards, shards[1:]):
        assert a.stop == b.start
    sizes = [s.heads for s in shards]
    assert max(sizes) - min(sizes) <= 1
    assert sum(sizes) == total


def test_plan_shards_rejects_bad_world():
    with pytest.raises(ValueError):
        plan_shards(4, 0)


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fa.synthetic import make_qkv
        from oracle import attention as oracle

        q, k, v = make_qkv(2, 3, 40, 64, seed=5)
        n, d = q.shape[2:]
        shard = plan_shards(6, world)[rank]
        flat = lambda t: t.reshape(6, n, d)[shard.start : shard.stop]  # noqa: E731
        part = torch.from_numpy(oracle.attention(flat(q).numpy(), flat(k).numpy(), flat(v).numpy(), causal=True))
        # timing reduction used by bench.py: max over ranks
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        if rank == 0:
            full = torch.cat(parts, dim=0).reshape(q.shape)
            ref = torch.from_numpy(oracle.attention(q.numpy(), k.numpy(), v.numpy(), causal=True))
            result_q.put((float(t), bool(torch.equal(full, ref))))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_shard_and_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    tmax, same = q.get(timeout=10)
    assert tmax == 2.0
    assert same
