"""pytest configuration: the `gpu` marker and shared helpers for the test suite.

`-m gpu` tests need a B200 (sm_100a) and call the kernels through the C ABI; every
other test runs on the CPU (oracle vs golden vectors, contract, library symbols,
multi-process host logic over gloo).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def golden_cases():
    return sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load_golden(name):
    """Returns dict with fp32 numpy arrays q,k,v,do ([B,H,S,D]) and fp32 reference outputs."""
    from oracle.flash_oracle import bf16_bits_to_f32
    z = np.load(GOLDEN / f"{name}.npz")
    B, H, S, D, causal, seed = (int(x) for x in z["meta"])
    sc = float(z["scale"][0])
    out = {k: bf16_bits_to_f32(z[k]).reshape(B, H, S, D) for k in ("q", "k", "v", "do")}
    for k in ("o", "lse", "dq", "dk", "dv"):
        out[k] = z[k]
    out.update(B=B, H=H, S=S, D=D, causal=bool(causal), scale=None if np.isnan(sc) else sc)
    return out
