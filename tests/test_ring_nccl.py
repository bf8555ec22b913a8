"""GPU (>= 2 devices): the context-parallel ring over NCCL point-to-point, one process per
GPU, against full attention computed on rank 0.  Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastflashattention_b200 import ring

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        B, H, S, D = 1, 4, 512 * world, 128
        g = torch.Generator(device="cuda").manual_seed(0)
        q, k, v, do = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(4))
        qs, ks, vs, dos = (ring.shard_sequence(t, rank, world) for t in (q, k, v, do))
        for t in (qs, ks, vs):
            t.requires_grad_(True)
        o = ring.ring_attention(qs, ks, vs)
        o.backward(dos)
        qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
        ref = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr, is_causal=True)
        ref.backward(do.float())
        errs = []
        for a, b in zip((o, qs.grad, ks.grad, vs.grad), (ref, qr.grad, kr.grad, vr.grad)):
            bs = ring.shard_sequence(b.detach(), rank, world)
            errs.append(float((a.float() - bs).norm() / bs.norm()))
        results[rank] = errs
    finally:
        dist.destroy_process_group()


def test_ring_over_nccl():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least two GPUs")
    world = min(world, 8)
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(world):
        assert max(results[r]) < 5e-3, (r, results[r])
