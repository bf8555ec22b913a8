"""Host launchers and the autograd Function over the sm_100a C ABI.

Mirrors the reference module ``fastflash_attention/_kernel.py``:
  * ``fastflash_attn(q, k, v, causal, return_lse=False, scale=None)``   (:282-318)
  * ``FastFlashAttn`` autograd Function                                   (:773-906)
  * ``fastflash_attn_train(q, k, v, causal, scale=None)``                 (:909-911)
  * ``LOG2E``                                                             (:40)
with the Triton kernels replaced by calls into ``libffa_sm100.so`` (``include/ffa.h``).
``attention_train`` is the same differentiable attention as ``FastFlashAttn`` with its
autograd node in C++; ``fast_attention`` uses it.
The host work (contiguous inputs as the reference makes them, :294, :791; zero-padding of
head dims below 64, which leaves q.k unchanged and drops the padded v columns while the
softmax scale keeps the true head dim; output allocation by the torch caching allocator on
the inputs' device; the launch on the current stream) runs in C++ as the torch operators
``torch.ops.ffa_b200.*`` of ``libffa_torch.so`` (csrc/ffa_torch.cpp), over the C ABI.
"""
from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from . import _lib

LOG2E = 1.4426950408889634  # 1/ln(2): exp(x) = exp2(x*log2e)


def _default_scale(head_dim: int) -> float:
    return 1.0 / (head_dim ** 0.5)


def fastflash_attn(q, k, v, causal: bool, return_lse: bool = False, scale=None):
    """Exact bf16 attention forward. [B,H,S,D] bf16 -> [B,H,S,D] bf16 (+ base-2 LSE [B,H,S]).

    ``scale`` overrides the default ``1/sqrt(D)``.  With ``return_lse`` also returns the
    per-row base-2 log-sum-exp ``m + log2(l)`` in fp32, as the reference does (:274-279).
    """
    B, H, S, D = q.shape
    assert D <= 128 and (D & (D - 1)) == 0, "HEAD_DIM must be a power of two <= 128"
    assert q.is_cuda and k.is_cuda and v.is_cuda
    sc = None if scale is None else float(scale)
    if return_lse:
        return _lib.ops().forward_lse(q, k, v, bool(causal), sc)
    return _lib.ops().forward(q, k, v, bool(causal), sc)


def _bwd(q, k, v, o, do, lse, causal: bool, scale):
    """dq, dk, dv for the saved forward state; all [B,H,S,D]."""
    return _lib.ops().backward(q, k, v, o, do, lse, bool(causal), None if scale is None else float(scale))


def attention_train(q, k, v, causal: bool, scale=None):
    """Differentiable attention through the C++ autograd node ``ffa_b200::attention``
    (forward with LSE, saved q, k, v, o, lse, deterministic backward): the same work as
    ``FastFlashAttn`` with no Python on the forward or backward path."""
    return _lib.ops().attention(q, k, v, bool(causal), None if scale is None else float(scale))


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
