"""CPU (gloo) tests of the context-parallel ring: schedule, zig-zag layout, LSE merge and
the fixed-order dK/dV accumulation, against full fp32 attention, at world sizes 2 and 3."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastflashattention_b200 import ring

B, H, S, D = 1, 2, 96, 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_reference(q, k, v, do, scale):
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr, is_causal=True, scale=scale)
    o.backward(do)
    return o.detach(), qr.grad, kr.grad, vr.grad


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.ring_blocks import CpuBlockOps
        g = torch.Generator().manual_seed(0)
        q, k, v, do = (torch.randn(B, H, S, D, generator=g) for _ in range(4))
        scale = D ** -0.5
        shards = [ring.shard_sequence(t, rank, world) for t in (q, k, v, do)]
        outs = []
        for _ in range(2):  # twice: the backward must be bitwise reproducible
            qs, ks, vs = (t.clone().requires_grad_(True) for t in shards[:3])
            o = ring.ring_attention(qs, ks, vs, scale=scale, ops=CpuBlockOps())
            o.backward(shards[3])
            outs.append((o.detach(), qs.grad, ks.grad, vs.grad))
        ref = _full_reference(q, k, v, do, scale)
        errs = []
        for got, want in zip(outs[0], ref):
            want_s = ring.shard_sequence(want, rank, world)
            errs.append(float((got - want_s).norm() / want_s.norm()))
        same = all(torch.equal(a, b) for a, b in zip(outs[0], outs[1]))
        results[rank] = (errs, same)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ring_matches_full_attention_on_gloo(world):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    for r in range(world):
        errs, same = results[r]
        assert max(errs) < 1e-5, (r, errs)
        assert same, r


def test_zigzag_layout_roundtrip_and_balance():
    x = torch.arange(2 * 4 * 8).reshape(1, 1, 64, 1).float()
    shards = [ring.shard_sequence(x, r, 4) for r in range(4)]
    assert torch.equal(ring.unshard_sequence(shards), x)
    # causal work per rank (number of visible (q, k) chunk pairs) is the same on every rank
    work = []
    for r in range(4):
        mine = ring.chunk_ids(r, 4)
        work.append(sum(1 for x_ in mine for y in range(8) if ring.block_kind(x_, y) is not None))
    assert len(set(work)) == 1


def test_shard_rejects_indivisible_length():
    with pytest.raises(ValueError):
        ring.shard_sequence(torch.zeros(1, 1, 10, 4), 0, 3)
