"""fastflashattention_b200 — exact bf16 flash-attention for NVIDIA B200 (sm_100a).

Drop-in for the ``fastflash_attention`` package (AlcAI-Haven/FastFlashAttention):
the same four public names with the same arguments, the same strict input contract
and the same error messages (reference ``fastflash_attention/__init__.py:35-142``)::

    from fastflashattention_b200 import fast_attention
    out = fast_attention(q, k, v, is_causal=True)   # q,k,v: [B,H,S,D] bf16, CUDA

Inputs outside the contract raise :class:`UnsupportedConfig`; there is no hidden slow
path and no CPU fallback.  The kernels are hand-written CUDA for sm_100a (tcgen05 MMA
with TMEM accumulators, TMA-fed shared-memory rings) behind the C ABI in
``include/ffa.h``; the backward is deterministic (disjoint writes, no atomics).

Supported contract:
  * dtype ``bfloat16``, q/k/v CUDA tensors
  * shape ``[B, H, S, D]`` identical for q, k and v
  * ``head_dim`` a power of two ``<= 128``
  * ``attn_mask is None`` and ``dropout_p == 0`` (causal masking via ``is_causal``)
  * ``scale`` optional (defaults to ``1/sqrt(head_dim)``)
"""
from __future__ import annotations

import torch
from torch import nn

from ._kernel import attention_train, fastflash_attn, fastflash_attn_train, FastFlashAttn, LOG2E  # noqa: F401

__all__ = [
    "fast_attention",
    "FastFlashAttention",
    "is_eligible",
    "UnsupportedConfig",
    "__version__",
]

__version__ = "0.2.0"

# head dims the contract accepts (reference __init__.py:45)
_HEAD_DIMS = frozenset(1 << i for i in range(8))


class UnsupportedConfig(ValueError):
    """Raised by :func:`fast_attention` when an input falls outside the supported contract.

    The message names the violated constraint; :func:`is_eligible` performs the same
    check without raising.
    """


def _tensor_problem(name, t):
    if not isinstance(t, torch.Tensor):
        return f"{name} is not a torch.Tensor"
    if not t.is_cuda:
        return f"{name} is on device '{t.device}'; a CUDA tensor is required"
    if t.dtype is not torch.bfloat16:
        return f"{name} dtype is {t.dtype}; only bfloat16 is supported"
    if t.dim() != 4:
        return f"{name} has {t.dim()} dims; expected 4 ([B, H, S, D])"
    return None


def _reason(query, key, value, attn_mask, dropout_p, is_causal, scale, enable_gqa):
    """Why the input is unsupported (a message), or ``None`` if it is supported.

    Checks run in the reference order (``__init__.py:56-80``): mask, dropout, GQA flag,
    then per-tensor type / device / dtype / rank, then equal shapes, then head_dim.
    """
    if attn_mask is not None:
        return "attn_mask is not supported (strict policy); pass attn_mask=None and use is_causal"
    if dropout_p:
        return f"dropout_p={dropout_p} is not supported (strict policy); pass dropout_p=0"
    if enable_gqa:
        return "GQA/MQA (enable_gqa=True) is not supported (strict policy)"
    for name, t in (("query", query), ("key", key), ("value", value)):
        problem = _tensor_problem(name, t)
        if problem is not None:
            return problem
    shapes = (tuple(query.shape), tuple(key.shape), tuple(value.shape))
    if len(set(shapes)) != 1:
        return (f"shapes differ (query {shapes[0]}, key {shapes[1]}, value {shapes[2]}); GQA/MQA and "
                "differing key/value length are not supported (strict policy)")
    head_dim = shapes[0][-1]
    if head_dim not in _HEAD_DIMS:
        return f"head_dim={head_dim}; must be a power of two <= 128"
    return None


def is_eligible(query, key, value, attn_mask=None, dropout_p=0.0,
                is_causal=False, scale=None, enable_gqa=False) -> bool:
    """True iff :func:`fast_attention` accepts this input (never raises)."""
    return _reason(query, key, value, attn_mask, dropout_p, is_causal, scale, enable_gqa) is None


def fast_attention(query, key, value, attn_mask=None, dropout_p=0.0,
                   is_causal=False, scale=None, enable_gqa=False):
    """Exact bf16 attention, drop-in for ``F.scaled_dot_product_attention``.

    q, k, v are ``[B, H, S, D]`` bfloat16 CUDA tensors; returns ``[B, H, S, D]`` bfloat16.
    When autograd needs gradients of any input the call goes through the deterministic
    backward; otherwise it runs the forward alone without writing the LSE
    (reference dispatch, ``__init__.py:108-112``).
    """
    reason = _reason(query, key, value, attn_mask, dropout_p, is_causal, scale, enable_gqa)
    if reason is not None:
        raise UnsupportedConfig(reason)
    wants_grad = torch.is_grad_enabled() and any(t.requires_grad for t in (query, key, value))
    if wants_grad:
        return attention_train(query, key, value, is_causal, scale)
    return fastflash_attn(query, key, value, is_causal, scale=scale)


class FastFlashAttention(nn.Module):
    """``nn.Module`` around :func:`fast_attention`.

    ``is_causal`` and ``scale`` given to the constructor are defaults; the same
    arguments passed to ``forward`` take precedence when not ``None``.
    """

    def __init__(self, is_causal: bool = False, scale=None):
        super().__init__()
        self.is_causal = is_causal
        self.scale = scale

    def forward(self, query, key, value, attn_mask=None, dropout_p=0.0,
                is_causal=None, scale=None, enable_gqa=False):
        causal = self.is_causal if is_causal is None else is_causal
        sc = self.scale if scale is None else scale
        return fast_attention(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                              is_causal=causal, scale=sc, enable_gqa=enable_gqa)

    def extra_repr(self) -> str:
        return f"is_causal={self.is_causal}, scale={self.scale}"
