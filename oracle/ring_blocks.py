"""fp32 CPU block operations for testing the context-parallel ring (test infrastructure).

Implements the ``BlockOps`` interface of ``fastflashattention_b200.ring`` in plain torch
fp32 with the same base-2 LSE convention as the kernels (reference
``fastflash_attention/_kernel.py:274-279``): block forward merged into an fp32 running
result by its LSE, delta = rowsum(O*dO), and the block backward from the global LSE/delta
added into fp32 accumulators
(``_kernel.py:379-448, 487-564``).  Used only by tests to check the ring's schedule,
masking, merge and accumulation order on CPU ranks.
"""
from __future__ import annotations

import torch

LOG2E = 1.4426950408889634


def _scores(q, k, causal, scale):
    s = (q.float() @ k.float().transpose(-1, -2)) * (scale * LOG2E)
    if causal:
        C = q.shape[-2]
        s = s.masked_fill(torch.triu(torch.ones(C, C, dtype=torch.bool), 1), float("-inf"))
    return s


class CpuBlockOps:
    def _fwd(self, q, k, v, causal, scale):
        s = _scores(q, k, causal, scale)
        m = s.amax(dim=-1, keepdim=True)
        l = torch.exp2(s - m).sum(dim=-1, keepdim=True)
        lse = (m + torch.log2(l))
        p = torch.exp2(s - lse)
        return p @ v.float(), lse[..., 0]

    def fwd_merge(self, q, k, v, causal, scale, acc, acc_lse, first):
        o, lse = self._fwd(q, k, v, causal, scale)
        if first:
            acc.copy_(o)
            acc_lse.copy_(lse)
            return
        m = torch.maximum(acc_lse, lse)
        wa, wb = torch.exp2(acc_lse - m), torch.exp2(lse - m)
        acc.copy_((wa[..., None] * acc + wb[..., None] * o) / (wa + wb)[..., None])
        acc_lse.copy_(m + torch.log2(wa + wb))

    def delta(self, o, do):
        return (o.float() * do.float()).sum(dim=-1)

    def bwd_acc(self, q, k, v, do, lse, delta, causal, scale, dq_acc, dk_acc, dv_acc):
        s = _scores(q, k, causal, scale)
        p = torch.exp2(s - lse[..., None])
        dv_acc += p.transpose(-1, -2) @ do.float()
        dp = do.float() @ v.float().transpose(-1, -2)
        ds = p * (dp - delta[..., None])
        dq_acc += ds @ k.float() * scale
        dk_acc += ds.transpose(-1, -2) @ q.float() * scale
