"""GPU: a training step allocates nothing of size O(S^2).

The reference measures peak memory in a fresh process per point (``bench/mem.py:37-118``)
and reports a flat training overhead (``README.md:162-169``).  Here the backward
recomputes P and dS tile by tile, so beyond its inputs a forward + backward may hold only
O, dQ, dK, dV ([B,H,S,D] bf16 each) plus the fp32 LSE and delta ([B,H,S] each), and a
little allocator slack.  At S=8192 a single [B,H,S,S] bf16 score tensor would be 8 GiB,
far above the bound.
"""
import gc

import pytest
import torch

from fastflashattention_b200 import fast_attention

pytestmark = pytest.mark.gpu

SLACK = 8 << 20  # allocator rounding and tiny host-side tensors


@pytest.mark.parametrize("S,D,causal", [(8192, 128, True), (4096, 64, False)])
def test_training_step_peak_memory_is_linear_in_S(S, D, causal):
    B, H = 4, 16
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, do = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(4))
    qg, kg, vg = (t.requires_grad_(True) for t in (q, k, v))

    def step():
        out = fast_attention(qg, kg, vg, is_causal=causal)
        return torch.autograd.grad(out, (qg, kg, vg), do)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    gc.collect()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    grads = step()
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    tensor = B * H * S * D * 2
    rows = B * H * S * 4
    bound = 4 * tensor + 2 * rows + SLACK  # O, dQ, dK, dV + LSE, delta
    assert peak <= bound, (peak, bound)
    del grads
