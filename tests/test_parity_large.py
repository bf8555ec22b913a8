"""GPU: forward and backward parity at the benchmarked and configured sizes.

The O(S^2) fp32 oracle does not fit these sizes, so every (batch, head) slice is checked
against exact float64 attention on sampled rows and sampled key columns, which needs no
S x S tensor in memory at once:

* O, the LSE and dQ on sampled query rows R: each needs only its own row of P and dP;
* dK and dV on sampled key columns C: they need P[:, C] for every query row, hence the
  exact LSE of every row (chunked float64 Q K^T) and delta_i = dO_i . O_i with the exact O.

Shapes: the bench workload (B4 H16 S8192 D128 causal) and S=16384 of BASELINE configs[1];
configs[2] (B8 H16 D64 non-causal, S in {1024, 4096, 16384}) and its q*8 stress variant.
Gate: rel-L2 over the sampled entries 5e-3 (BASELINE's 0.5 %); the q*8 gradients use the
reference tests' 1e-2, as everywhere else in this suite.  The 5-run bitwise determinism
of the headline shape at S=8192 and 16384 is checked here too.
"""
import math

import pytest
import torch

from fastflashattention_b200 import _lib, fast_attention
from fastflashattention_b200._kernel import fastflash_attn

pytestmark = pytest.mark.gpu

TOL = 5e-3
TOL_PEAKY_GRAD = 1e-2
LOG2E = 1.4426950408889634
CHUNK = 2048  # query rows per float64 block


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def _mask(rows, cols, causal):
    """Additive float64 mask for rows x cols (0 or -inf)."""
    if not causal:
        return None
    return torch.where(cols[None, :] > rows[:, None], float("-inf"), 0.0).double()


def _exact_slice(q, k, v, do, scale, causal, R, C):
    """Exact float64 quantities of one [S, D] slice: (O[R], lse2[R], dQ[R], dK[C], dV[C])."""
    S = q.shape[0]
    dev = q.device
    qd, kd, vd, dod = (t.double() for t in (q, k, v, do))
    cols = torch.arange(S, device=dev)
    lse = torch.empty(S, dtype=torch.float64, device=dev)
    o = torch.empty(S, q.shape[1], dtype=torch.float64, device=dev)
    for r0 in range(0, S, CHUNK):
        rows = cols[r0:r0 + CHUNK]
        s = (qd[rows] @ kd.T) * scale
        m = _mask(rows, cols, causal)
        if m is not None:
            s = s + m
        lse[rows] = torch.logsumexp(s, dim=1)
        o[rows] = torch.softmax(s, dim=1) @ vd
    delta = (dod * o).sum(dim=1)
    # query side: rows R
    s = (qd[R] @ kd.T) * scale
    m = _mask(R, cols, causal)
    if m is not None:
        s = s + m
    p = torch.exp(s - lse[R, None])
    dp = dod[R] @ vd.T
    dq = (p * (dp - delta[R, None])) @ kd * scale
    # key side: columns C, all rows
    s = (qd @ kd[C].T) * scale
    m = _mask(cols, C, causal)
    if m is not None:
        s = s + m
    p = torch.exp(s - lse[:, None])
    dv = p.T @ dod
    dp = dod @ vd[C].T
    dk = (p * (dp - delta[:, None])).T @ qd * scale
    return o[R], lse[R] * LOG2E, dq, dk, dv


def _samples(S, gen, n=48):
    """Sorted sample of row indices: the first and last 8 and n random ones."""
    mid = torch.randint(8, S - 8, (n,), device="cuda", generator=gen)
    return torch.unique(torch.cat([torch.arange(0, 8, device="cuda"), mid, torch.arange(S - 8, S, device="cuda")]))


def _run_and_check(B, H, S, D, causal, qmul, seed, grad_tol):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v, do = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(4))
    if qmul != 1.0:
        q = (q.float() * qmul).to(torch.bfloat16)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    out = fast_attention(qg, kg, vg, is_causal=causal)
    dq, dk, dv = torch.autograd.grad(out, (qg, kg, vg), do)
    _, lse = fastflash_attn(q, k, v, causal, return_lse=True)
    scale = 1.0 / math.sqrt(D)
    got = {n: [] for n in ("o", "lse", "dq", "dk", "dv")}
    want = {n: [] for n in got}
    for b in range(B):
        for h in range(H):
            R, C = _samples(S, gen), _samples(S, gen)
            ex = _exact_slice(q[b, h], k[b, h], v[b, h], do[b, h], scale, causal, R, C)
            for n, g, w in zip(("o", "lse", "dq", "dk", "dv"),
                               (out[b, h, R], lse[b, h, R], dq[b, h, R], dk[b, h, C], dv[b, h, C]), ex):
                got[n].append(g.detach().double())
                want[n].append(w)
    for n in ("o", "dq", "dk", "dv"):
        err = _rel(torch.cat(got[n]), torch.cat(want[n]))
        assert err < (TOL if n == "o" else grad_tol), (n, err)
        # no single slice may hide behind the average (a mis-mapped CTA would hit one)
        worst = max(_rel(g, w) for g, w in zip(got[n], want[n]))
        assert worst < 2 * (TOL if n == "o" else grad_tol), (n, "worst slice", worst)
    assert float((torch.cat(got["lse"]) - torch.cat(want["lse"])).abs().max()) < 3e-3
    assert _lib.device_status() == (0, 0, 0, 0)


@pytest.mark.parametrize("B,H,S", [(4, 16, 8192), (1, 16, 16384)], ids=["bench-B4H16S8192", "B1H16S16384"])
def test_headline_causal_d128_fwd_bwd(B, H, S):
    _run_and_check(B, H, S, 128, True, 1.0, 0, TOL)


@pytest.mark.parametrize("S", [1024, 4096, 16384])
def test_configs2_noncausal_d64(S):
    _run_and_check(8, 16, S, 64, False, 1.0, 1, TOL)


@pytest.mark.parametrize("S", [1024, 16384])
def test_configs2_peaky_q8(S):
    _run_and_check(8, 16, S, 64, False, 8.0, 2, TOL_PEAKY_GRAD)


def _grads(q, k, v, g):
    qs, ks, vs = (t.detach().requires_grad_(True) for t in (q, k, v))
    out = fast_attention(qs, ks, vs, is_causal=True)
    return (out.detach(), *torch.autograd.grad(out, (qs, ks, vs), g))


@pytest.mark.parametrize("S", [8192, 16384])
def test_headline_bitwise_five_runs(S):
    gen = torch.Generator(device="cuda").manual_seed(3)
    q, k, v, g = (torch.randn(4, 16, S, 128, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(4))
    first = _grads(q, k, v, g)
    for _ in range(4):
        for a, b in zip(first, _grads(q, k, v, g)):
            assert torch.equal(a, b)
