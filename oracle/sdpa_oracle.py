"""fp32 SDPA oracle (test infrastructure only; see ``oracle/__init__.py``).

Restates the reference's parity oracle (``tests/test_parity.py:32-35``): inputs are
upcast to fp32 and passed to ``F.scaled_dot_product_attention`` with the math backend
forced; gradients come from autograd.  Runs on the CPU.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel


def sdpa_fwd_bwd(q, k, v, do, causal: bool, scale: float | None = None, need_grad: bool = True):
    """q,k,v,do: [B,H,S,D] tensors (any float dtype, any device).  Returns fp32
    (O, LSE_natural[B,H,S], dq, dk, dv) — the grads are None when need_grad is False."""
    qf, kf, vf = (t.detach().float().requires_grad_(need_grad) for t in (q, k, v))
    with sdpa_kernel(SDPBackend.MATH):
        o = F.scaled_dot_product_attention(qf, kf, vf, is_causal=causal, scale=scale)
    D = q.shape[-1]
    sm = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    with torch.no_grad():
        s = (qf @ kf.transpose(-1, -2)) * sm
        if causal:
            S = q.shape[-2]
            s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device=s.device), 1), float("-inf"))
        lse = torch.logsumexp(s, dim=-1)
    if not need_grad:
        return o.detach(), lse, None, None, None
    o.backward(do.float())
    return o.detach(), lse, qf.grad, kf.grad, vf.grad


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    """‖a−b‖/‖b‖ in fp32 (reference tests/test_parity.py:26-29)."""
    a = a.float()
    b = b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))
