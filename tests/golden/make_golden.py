"""Generate the golden vectors in this folder (run on a CPU: ``python tests/golden/make_golden.py``).

Each case stores seeded bf16 inputs (q, k, v, dO as raw bf16 bits) and the outputs of
the reference's own parity oracle — ``F.scaled_dot_product_attention`` on fp32-upcast
inputs with autograd for the gradients (reference ``tests/test_parity.py:32-35, 62-85``,
restated in ``oracle/sdpa_oracle.py``) — together with the natural-log LSE.  Inputs are
drawn on the CPU from ``torch.Generator().manual_seed(seed)`` (q, k, v, dO in that order,
as ``bench/benchmark.py:44-48`` draws them), so the files do not depend on any GPU RNG.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.sdpa_oracle import sdpa_fwd_bwd  # noqa: E402

HERE = Path(__file__).resolve().parent

# name: (B, H, S, D, causal, scale, q_multiplier, seed)
CASES = {
    "tiny_causal_b1h2s256d64": (1, 2, 256, 64, True, None, 1.0, 0),
    "ragged_noncausal_b1h2s200d64": (1, 2, 200, 64, False, None, 1.0, 2),
    "ragged_causal_b1h1s200d64": (1, 1, 200, 64, True, None, 1.0, 5),
    "causal_b1h1s256d128": (1, 1, 256, 128, True, None, 1.0, 1),
    "custom_scale_b1h1s128d64": (1, 1, 128, 64, True, 0.05, 1.0, 3),
    "peaky_noncausal_b1h1s256d64": (1, 1, 256, 64, False, None, 8.0, 4),
    "small_d16_causal_b1h2s128d16": (1, 2, 128, 16, True, None, 1.0, 6),
}


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make(name, B, H, S, D, causal, scale, qmul, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda: torch.randn(B, H, S, D, generator=g, dtype=torch.float32).to(torch.bfloat16)  # noqa: E731
    q, k, v, do = mk(), mk(), mk(), mk()
    if qmul != 1.0:
        q = (q.float() * qmul).to(torch.bfloat16)
    o, lse, dq, dk, dv = sdpa_fwd_bwd(q, k, v, do, causal, scale)
    np.savez_compressed(
        HERE / f"{name}.npz",
        q=bits(q), k=bits(k), v=bits(v), do=bits(do),
        o=o.numpy(), lse=lse.numpy(), dq=dq.numpy(), dk=dk.numpy(), dv=dv.numpy(),
        meta=np.array([B, H, S, D, int(causal), seed], np.int64),
        scale=np.array([np.nan if scale is None else scale], np.float64),
        torch_version=np.array(torch.__version__),
    )


if __name__ == "__main__":
    for name, args in CASES.items():
        make(name, *args)
        print("wrote", name)
