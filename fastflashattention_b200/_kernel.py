"""Host launchers and the autograd Function over the sm_100a C ABI.

Mirrors the reference module ``fastflash_attention/_kernel.py``:
  * ``fastflash_attn(q, k, v, causal, return_lse=False, scale=None)``   (:282-318)
  * ``FastFlashAttn`` autograd Function                                   (:773-906)
  * ``fastflash_attn_train(q, k, v, causal, scale=None)``                 (:909-911)
  * ``LOG2E``                                                             (:40)
with the Triton kernels replaced by calls into ``libffa_sm100.so`` (``include/ffa.h``).
Outputs are allocated by the torch caching allocator on the inputs' device and every
launch goes on the current torch CUDA stream.  Inputs are made contiguous first, as
the reference does (:294, :791).  Head dims below 64 are zero-padded to 64 for the
kernels (padding q/k with zeros leaves q.k unchanged and padded v columns are dropped),
while the softmax scale keeps using the true head dim.
"""
from __future__ import annotations

import contextlib

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable

from . import _lib

LOG2E = 1.4426950408889634  # 1/ln(2): exp(x) = exp2(x*log2e)

_KERNEL_DIMS = (64, 128)


def _default_scale(head_dim: int) -> float:
    return 1.0 / (head_dim ** 0.5)


def _kdim(d: int) -> int:
    return 64 if d <= 64 else 128


def _prep(t: torch.Tensor, kd: int) -> torch.Tensor:
    """[B,H,S,D] -> contiguous [B*H,S,kd] (zero-padded along D when D < kd)."""
    B, H, S, D = t.shape
    t = t.contiguous()
    if D != kd:
        t = F.pad(t, (0, kd - D))
    return t.reshape(B * H, S, kd)


def _stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _on_device(dev: torch.device):
    """Context that makes `dev` current for the launch (a no-op when it already is)."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(dev)


def fastflash_attn(q, k, v, causal: bool, return_lse: bool = False, scale=None):
    """Exact bf16 attention forward. [B,H,S,D] bf16 -> [B,H,S,D] bf16 (+ base-2 LSE [B,H,S]).

    ``scale`` overrides the default ``1/sqrt(D)``.  With ``return_lse`` also returns the
    per-row base-2 log-sum-exp ``m + log2(l)`` in fp32, as the reference does (:274-279).
    """
    B, H, S, D = q.shape
    assert D <= 128 and (D & (D - 1)) == 0, "HEAD_DIM must be a power of two <= 128"
    assert q.is_cuda and k.is_cuda and v.is_cuda
    lib = _lib.load()
    kd = _kdim(D)
    qf, kf, vf = (_prep(t, kd) for t in (q, k, v))
    o = torch.empty_like(qf)
    lse = torch.empty(B * H, S, device=q.device, dtype=torch.float32) if return_lse else None
    sm = _default_scale(D) if scale is None else float(scale)
    with _on_device(q.device):
        rc = lib.ffa_fwd(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), o.data_ptr(),
                         lse.data_ptr() if lse is not None else None,
                         B * H, S, kd, qf.stride(0), qf.stride(1), sm, int(bool(causal)),
                         _stream_ptr(q.device))
    _lib.check(rc, "ffa_fwd")
    o = o.reshape(B, H, S, kd)
    if kd != D:
        o = o[..., :D].contiguous()
    if return_lse:
        return o, lse.reshape(B, H, S)
    return o


def _bwd(q, k, v, o, do, lse, causal: bool, scale):
    """dq, dk, dv for the saved forward state; all [B,H,S,D]."""
    B, H, S, D = q.shape
    lib = _lib.load()
    kd = _kdim(D)
    qf, kf, vf, of, dof = (_prep(t, kd) for t in (q, k, v, o, do))
    lf = lse.reshape(B * H, S).contiguous()
    dq = torch.empty_like(qf)
    dk = torch.empty_like(kf)
    dv = torch.empty_like(vf)
    delta = torch.empty(B * H, S, device=q.device, dtype=torch.float32)
    sm = _default_scale(D) if scale is None else float(scale)
    with _on_device(q.device):
        rc = lib.ffa_bwd(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), of.data_ptr(), dof.data_ptr(),
                         lf.data_ptr(), delta.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                         B * H, S, kd, qf.stride(0), qf.stride(1), sm, int(bool(causal)),
                         _stream_ptr(q.device))
    _lib.check(rc, "ffa_bwd")
    out = []
    for g in (dq, dk, dv):
        g = g.reshape(B, H, S, kd)
        if kd != D:
            g = g[..., :D].contiguous()
        out.append(g)
    return tuple(out)


class FastFlashAttn(torch.autograd.Function):
    """Differentiable attention: sm_100a forward + deterministic two-kernel backward."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale=None):
        o, lse = fastflash_attn(q, k, v, causal, return_lse=True, scale=scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal = causal
        ctx.scale = scale
        return o

    @staticmethod
    @once_differentiable
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = _bwd(q, k, v, o, do, lse, ctx.causal, ctx.scale)
        return dq, dk, dv, None, None


def fastflash_attn_train(q, k, v, causal: bool, scale=None):
    """Differentiable entry point. [B,H,S,D] bf16 -> [B,H,S,D] bf16, grads on q,k,v."""
    return FastFlashAttn.apply(q, k, v, causal, scale)
