"""GPU: the context-parallel ring running the sm_100a kernels.

P ranks are emulated as P threads of one process on one GPU with an in-memory ring
exchange (no inter-GPU traffic and no kernels waiting on each other: every kernel is an
ordinary independent launch).  The product code path — ``ring_attention`` with the
default ``CudaBlockOps`` (C ABI) — is what runs; only the transport is replaced.
"""
import threading

import pytest
import torch
import torch.nn.functional as F

from fastflashattention_b200 import ring

pytestmark = pytest.mark.gpu

TOL = 5e-3


class ThreadExchange:
    """In-memory ring exchange among `world` threads (post deposits, wait collects)."""

    def __init__(self, world):
        self.world = world
        self.barrier = threading.Barrier(world)
        self.slots = {}
        self.lock = threading.Lock()
        self.round = [0] * world

    def for_rank(self, rank):
        ex = self

        class _View:
            def post(self, tensors):
                k = ex.round[rank]
                ex.round[rank] += 1
                torch.cuda.synchronize()
                with ex.lock:
                    ex.slots[(k, rank)] = tensors

                def wait():
                    ex.barrier.wait(timeout=60)
                    got = ex.slots[(k, (rank - 1) % ex.world)]
                    ex.barrier.wait(timeout=60)
                    return got

                return wait

        return _View()


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def _run_ring(q, k, v, do, world, D):
    """Every rank's (o, dq, dk, dv), reassembled to full-sequence tensors."""
    ex = ThreadExchange(world)
    out = [None] * world
    errors = []

    def run(rank):
        try:
            torch.cuda.set_device(0)
            qs, ks, vs, dos = (ring.shard_sequence(t, rank, world) for t in (q, k, v, do))
            # the ring's forward and backward are called directly: autograd would run every
            # thread's backward on its one worker thread per device, one after the other
            state = ring.RingState(rank, world, ex.for_rank(rank))
            ops = ring.CudaBlockOps()
            o, lse = ring.ring_forward(qs, ks, vs, state, D ** -0.5, ops)
            dq, dk, dv = ring.ring_backward(qs, ks, vs, o, lse, dos, state, D ** -0.5, ops)
            torch.cuda.synchronize()
            out[rank] = (o, dq, dk, dv)
        except Exception as e:  # surface thread failures in the test
            errors.append(e)
            ex.barrier.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    return [ring.unshard_sequence([out[r][i] for r in range(world)]) for i in range(4)]


@pytest.mark.parametrize("world,S,D", [(2, 1024, 128), (4, 2048, 128), (3, 768, 64)])
def test_ring_threads_match_full_attention(world, S, D):
    torch.manual_seed(0)
    B, H = 1, 4
    q, k, v, do = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16) for _ in range(4))
    got = _run_ring(q, k, v, do, world, D)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = F.scaled_dot_product_attention(qr, kr, vr, is_causal=True)
    ref.backward(do.float())
    for name, a, b in zip(("o", "dq", "dk", "dv"), got, (ref, qr.grad, kr.grad, vr.grad)):
        assert _rel(a, b) < TOL, (name, _rel(a, b))


def test_ring_configs4_sampled_rows():
    """BASELINE configs[4] (B1 H32 S131072 D128 causal) over 8 ring ranks (threads on one
    GPU), checked against exact float64 attention on sampled rows and key columns of four
    heads, and bitwise against a second run (the ring backward is deterministic)."""
    from test_parity_large import _exact_slice, _rel as rel64, _samples
    world, B, H, S, D = 8, 1, 32, 131072, 128
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, do = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(4))
    got = _run_ring(q, k, v, do, world, D)
    again = _run_ring(q, k, v, do, world, D)
    for a, b in zip(got, again):
        assert torch.equal(a, b)
    o, dq, dk, dv = got
    want = {n: [] for n in ("o", "dq", "dk", "dv")}
    have = {n: [] for n in want}
    for h in (0, 9, 22, 31):
        R, C = _samples(S, gen, 32), _samples(S, gen, 32)
        ex = _exact_slice(q[0, h], k[0, h], v[0, h], do[0, h], D ** -0.5, True, R, C)
        for n, g_, w in zip(("o", "dq", "dk", "dv"), (o[0, h, R], dq[0, h, R], dk[0, h, C], dv[0, h, C]),
                            (ex[0], ex[2], ex[3], ex[4])):
            have[n].append(g_.double())
            want[n].append(w)
    for n in want:
        err = rel64(torch.cat(have[n]), torch.cat(want[n]))
        assert err < TOL, (n, err)
