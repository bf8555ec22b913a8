"""The backward is deterministic: identical inputs -> bitwise-identical grads.

Port of the reference tests/test_determinism.py:22-39 (two runs) extended to the five
repeats BASELINE asks for, plus the headline shape.  Each output tile of the dK/dV and
dQ kernels is written by exactly one CTA with a fixed accumulation order, so repeats
must agree bit for bit; a race would show up here.
"""
import pytest
import torch

from fastflashattention_b200 import fast_attention

pytestmark = pytest.mark.gpu


def _grads(q, k, v, g, is_causal):
    for t in (q, k, v):
        t.grad = None
    out = fast_attention(q, k, v, is_causal=is_causal)
    out.backward(g)
    return out.detach().clone(), q.grad.clone(), k.grad.clone(), v.grad.clone()


@pytest.mark.parametrize("is_causal", [False, True])
@pytest.mark.parametrize("shape", [(2, 4, 512, 64), (1, 2, 1024, 128), (1, 3, 333, 128)])
def test_backward_bitwise_deterministic(shape, is_causal):
    torch.manual_seed(0)
    B, H, S, D = shape
    q, k, v = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, requires_grad=True) for _ in range(3))
    g = torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16)
    first = _grads(q, k, v, g, is_causal)
    for _ in range(4):
        again = _grads(q, k, v, g, is_causal)
        for a, b in zip(first, again):
            assert torch.equal(a, b)


def test_headline_shape_bitwise_five_runs():
    B, H, S, D = 4, 16, 2048, 128
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, g = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(4))
    for t in (q, k, v):
        t.requires_grad_(True)
    first = _grads(q, k, v, g, True)
    for _ in range(4):
        again = _grads(q, k, v, g, True)
        for a, b in zip(first, again):
            assert torch.equal(a, b)
