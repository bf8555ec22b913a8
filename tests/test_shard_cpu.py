"""CPU (gloo) tests of the batch x head data-parallel split: every (batch, head) slice is
owned by exactly one rank, shards are views, results reassemble to the single-process
answer, and the job time is the maximum over ranks.  fp32 SDPA on the CPU stands in for
the GPU kernels (the split itself moves no data)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastflashattention_b200 import shard


@pytest.mark.parametrize("bh,world", [(64, 8), (5, 2), (5, 3), (3, 4), (1, 1)])
def test_bh_range_partitions(bh, world):
    ranges = [shard.bh_range(bh, r, world) for r in range(world)]
    owned = [i for s, e in ranges for i in range(s, e)]
    assert owned == list(range(bh))
    assert all(e - s <= -(-bh // world) for s, e in ranges)


def test_shard_is_a_view_and_roundtrips():
    x = torch.randn(2, 3, 16, 8)
    shards = [shard.shard_heads(x, r, 2) for r in range(2)]
    assert shards[0].data_ptr() == x.data_ptr()
    assert [s.shape[1] for s in shards] == [3, 3]
    assert torch.equal(shard.unshard_heads(shards, 2, 3), x)


def test_max_over_ranks_without_group():
    assert shard.max_over_ranks(1.5) == 1.5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        B, H, S, D = 2, 5, 32, 16
        q, k, v = (torch.randn(B, H, S, D, generator=g) for _ in range(3))
        qs, ks, vs = (shard.shard_heads(t, rank, world) for t in (q, k, v))
        out = torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, is_causal=True)
        gathered = [None] * world
        dist.all_gather_object(gathered, out)
        whole = shard.unshard_heads(gathered, B, H)
        ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
        results[rank] = (float((whole - ref).abs().max()), shard.max_over_ranks(10.0 + rank))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_reassemble_and_time_is_max(world):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(world):
        err, tmax = results[r]
        assert err < 1e-6
        assert tmax == 10.0 + world - 1
