"""Strict-policy contract: is_eligible mirrors fast_attention's raise decision.

Port of the reference tests/test_eligibility.py:14-79 onto this package; the message
regexes are part of the drop-in contract.  CPU-only cases run without a GPU.
"""
import pytest
import torch

from fastflashattention_b200 import FastFlashAttention, UnsupportedConfig, fast_attention, is_eligible

gpu = pytest.mark.gpu


def _bf16(B, H, S, D, device="cuda"):
    return torch.randn(B, H, S, D, device=device, dtype=torch.bfloat16)


@gpu
def test_eligible_supported():
    q = _bf16(2, 4, 128, 64)
    assert is_eligible(q, q, q, is_causal=True)
    fast_attention(q, q, q, is_causal=True)


@gpu
@pytest.mark.parametrize("kwargs, needle", [
    ({"attn_mask": "MASK"}, "attn_mask"),
    ({"dropout_p": 0.1}, "dropout_p"),
    ({"enable_gqa": True}, "GQA"),
])
def test_unsupported_args_raise(kwargs, needle):
    q = _bf16(2, 4, 128, 64)
    if kwargs.get("attn_mask") == "MASK":
        kwargs["attn_mask"] = torch.zeros(128, 128, device="cuda", dtype=torch.bfloat16)
    assert not is_eligible(q, q, q, **kwargs)
    with pytest.raises(UnsupportedConfig, match=needle):
        fast_attention(q, q, q, **kwargs)


@gpu
def test_fp16_and_fp32_raise():
    for dt in (torch.float16, torch.float32):
        q = torch.randn(2, 4, 128, 64, device="cuda", dtype=dt)
        assert not is_eligible(q, q, q)
        with pytest.raises(UnsupportedConfig, match="bfloat16"):
            fast_attention(q, q, q)


@gpu
def test_gqa_shape_mismatch_raises():
    q = _bf16(2, 8, 128, 64)
    kv = _bf16(2, 2, 128, 64)
    assert not is_eligible(q, kv, kv)
    with pytest.raises(UnsupportedConfig, match="GQA|shapes differ"):
        fast_attention(q, kv, kv)


@gpu
def test_bad_head_dim_raises():
    q = _bf16(2, 4, 128, 96)
    assert not is_eligible(q, q, q)
    with pytest.raises(UnsupportedConfig, match="head_dim"):
        fast_attention(q, q, q)


def test_cpu_raises():
    q = torch.randn(2, 4, 16, 64, dtype=torch.bfloat16)
    assert not is_eligible(q, q, q)
    with pytest.raises(UnsupportedConfig, match="CUDA"):
        fast_attention(q, q, q)


@gpu
def test_module_forwards_defaults():
    q = _bf16(2, 4, 128, 64)
    attn = FastFlashAttention(is_causal=True)
    out = attn(q, q, q)
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    with pytest.raises(UnsupportedConfig, match="dropout_p"):
        attn(q, q, q, dropout_p=0.5)


# ---- CPU-only checks of the contract order (no kernel launch needed) -------------------

def test_cpu_contract_messages_in_reference_order():
    q = torch.randn(1, 1, 8, 64, dtype=torch.bfloat16)
    assert "attn_mask" in _reason_of(q, attn_mask=torch.zeros(8, 8))
    assert "dropout_p" in _reason_of(q, dropout_p=0.2)
    assert "GQA" in _reason_of(q, enable_gqa=True)
    assert "not a torch.Tensor" in _reason_of("x")
    assert "CUDA" in _reason_of(q)


def test_cpu_module_repr_and_defaults():
    m = FastFlashAttention(is_causal=True, scale=0.1)
    assert "is_causal=True" in repr(m) and "scale=0.1" in repr(m)


def test_cpu_head_dims_accepted():
    from fastflashattention_b200 import _HEAD_DIMS
    assert _HEAD_DIMS == frozenset((1, 2, 4, 8, 16, 32, 64, 128))


def _reason_of(q, **kw):
    from fastflashattention_b200 import _reason
    args = dict(attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, enable_gqa=False)
    args.update(kw)
    return _reason(q, q, q, **args)
