"""GPU parity of the sm_100a kernels (through the C ABI) against the oracles.

* the reference's own parity tests (tests/test_parity.py:18-85 of the reference), same
  shapes, seeds and fp32-SDPA truth, with the tighter B200 gate of 5e-3 rel-L2 on O and
  on dQ/dK/dV;
* the committed golden vectors (tests/golden/, fp32 SDPA) and the numpy restatement of
  the reference algorithm (oracle/flash_oracle.py) on the same inputs;
* full-size shapes of the headline config checked by size-independent properties:
  exact fp64 attention recomputed for sampled rows of every head, and the base-2 LSE.
"""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import golden_cases, load_golden
from fastflashattention_b200 import fast_attention
from fastflashattention_b200._kernel import fastflash_attn
from oracle import flash_oracle as fo

pytestmark = pytest.mark.gpu

TOL = 5e-3            # rel-L2 for O and dQ/dK/dV (BASELINE tolerance: 0.5%)
TOL_PEAKY_GRAD = 1e-2  # q*8 stress case: the reference algorithm itself sits at 5.0e-3 on dQ

SHAPES = [
    (2, 4, 128, 64),
    (1, 8, 512, 128),
    (2, 2, 200, 64),   # ragged S
    (1, 3, 1024, 128),
]


def _rel_l2(a, b):
    a = a.float()
    b = b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


def _ref(q, k, v, is_causal, scale):
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=is_causal, scale=scale)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", torch.bfloat16)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("is_causal", [False, True])
def test_forward_parity(shape, is_causal):
    torch.manual_seed(0)
    B, H, S, D = shape
    q, k, v = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    out = fast_attention(q, k, v, is_causal=is_causal)
    ref = _ref(q, k, v, is_causal, None)
    assert _rel_l2(out, ref) < TOL


def test_forward_custom_scale():
    torch.manual_seed(1)
    B, H, S, D = 2, 4, 256, 64
    q, k, v = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    scale = 0.05
    out = fast_attention(q, k, v, is_causal=True, scale=scale)
    ref = _ref(q, k, v, True, scale)
    assert _rel_l2(out, ref) < TOL
    out_default = fast_attention(q, k, v, is_causal=True)
    assert _rel_l2(out, out_default) > 1e-2


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("is_causal", [False, True])
def test_backward_parity(shape, is_causal):
    torch.manual_seed(2)
    B, H, S, D = shape
    q, k, v = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
               for _ in range(3))
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    out = fast_attention(q, k, v, is_causal=is_causal)
    ref = _ref(qr, kr, vr, is_causal, None)
    torch.manual_seed(3)
    g = torch.randn_like(out)
    out.backward(g)
    ref.backward(g.float())
    for name, got, want in (("dq", q.grad, qr.grad), ("dk", k.grad, kr.grad), ("dv", v.grad, vr.grad)):
        assert _rel_l2(got, want) < TOL, f"{name} shape={shape} causal={is_causal}"


# ---------------------------------------------------------------------- golden vectors

@pytest.mark.parametrize("name", golden_cases())
def test_forward_golden(name):
    g = load_golden(name)
    q, k, v = (_cuda(g[x]) for x in ("q", "k", "v"))
    o, lse = fastflash_attn(q, k, v, g["causal"], return_lse=True, scale=g["scale"])
    assert _rel_l2(o.cpu(), torch.from_numpy(g["o"])) < TOL
    lse_nat = lse.cpu().numpy() / fo.LOG2E
    np.testing.assert_allclose(lse_nat, g["lse"], rtol=0, atol=2e-3)


@pytest.mark.parametrize("name", golden_cases())
def test_backward_golden(name):
    g = load_golden(name)
    q, k, v = (_cuda(g[x]).requires_grad_(True) for x in ("q", "k", "v"))
    do = _cuda(g["do"])
    out = fast_attention(q, k, v, is_causal=g["causal"], scale=g["scale"])
    out.backward(do)
    tol = TOL_PEAKY_GRAD if name.startswith("peaky") else TOL
    for got, ref in ((q.grad, "dq"), (k.grad, "dk"), (v.grad, "dv")):
        assert _rel_l2(got.cpu(), torch.from_numpy(g[ref])) < tol, ref


@pytest.mark.parametrize("name", ["tiny_causal_b1h2s256d64", "ragged_noncausal_b1h2s200d64",
                                  "causal_b1h1s256d128"])
def test_matches_flash_oracle(name):
    """Same inputs through the numpy restatement of the reference algorithm: the two
    bf16 pipelines agree far inside the tolerance to the fp32 truth."""
    g = load_golden(name)
    flat = lambda a: a.reshape(-1, a.shape[2], a.shape[3])  # noqa: E731
    q, k, v, do = (flat(g[x]) for x in ("q", "k", "v", "do"))
    o_ref, l_ref = fo.forward(q, k, v, g["causal"], g["scale"])
    qc, kc, vc = (_cuda(g[x]) for x in ("q", "k", "v"))
    o, lse = fastflash_attn(qc, kc, vc, g["causal"], return_lse=True, scale=g["scale"])
    assert fo.rel_l2(o.float().cpu().numpy().reshape(o_ref.shape), o_ref) < 3e-3
    np.testing.assert_allclose(lse.cpu().numpy().reshape(l_ref.shape), l_ref, atol=1e-3)


# ------------------------------------------------------------------ full-size properties

def _sampled_rows_exact(q, k, v, causal, scale, rows):
    """fp64 attention for the given query rows of every head. q,k,v [B,H,S,D]."""
    qs = q[:, :, rows].double()
    s = torch.einsum("bhid,bhjd->bhij", qs, k.double()) * scale
    if causal:
        S = k.shape[2]
        cols = torch.arange(S, device=q.device)
        s = s.masked_fill(cols[None, None, None, :] > rows[None, None, :, None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.einsum("bhij,bhjd->bhid", torch.softmax(s, dim=-1), v.double())
    return o, lse


@pytest.mark.parametrize("S,causal", [(4096, True), (8192, True), (2048, False)])
def test_forward_full_size_sampled_rows(S, causal):
    B, H, D = 4, 16, 128
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(3))
    o, lse = fastflash_attn(q, k, v, causal, return_lse=True)
    rows = torch.cat([torch.arange(0, 8, device="cuda"), torch.randint(0, S, (56,), device="cuda", generator=gen),
                      torch.arange(S - 8, S, device="cuda")])
    o_ref, lse_ref = _sampled_rows_exact(q, k, v, causal, 1.0 / math.sqrt(D), rows)
    assert _rel_l2(o[:, :, rows], o_ref) < TOL
    torch.testing.assert_close(lse[:, :, rows].double() / fo.LOG2E, lse_ref, rtol=0, atol=2e-3)


def test_forward_peaky_rows_lse_path():
    """q*8 makes rows peaky: exercises the online max and the lazy rescale."""
    B, H, S, D = 2, 4, 2048, 64
    gen = torch.Generator(device="cuda").manual_seed(7)
    q, k, v = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(3))
    q = (q.float() * 8).to(torch.bfloat16)
    for causal in (False, True):
        out = fast_attention(q, k, v, is_causal=causal)
        assert _rel_l2(out, _ref(q, k, v, causal, None)) < TOL



@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("is_causal", [False, True])
@pytest.mark.parametrize("boost", [(128, 192), (192, 256), (320, 384)], ids=["tile1-first-half",
                                                                            "tile1-second-half",
                                                                            "tile2-second-half"])
@pytest.mark.parametrize("scale", [None, -0.09])
def test_late_max_growth(D, is_causal, boost, scale):
    """Scores that jump by far more than 2^8 inside a later 128-key tile, in its first or
    second 64-key half (keys boosted x8).  This drives the forward's lazy rescale through
    both of its late paths: the row max taken before the first half is handed over, and
    the rescale of O after the first half's P.V has already run.  A negative scale turns
    the max into a min."""
    torch.manual_seed(5)
    B, H, S = 1, 2, 512
    q, k, v = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    k[:, :, boost[0]:boost[1]] *= 8
    q, k, v = (t.requires_grad_(True) for t in (q, k, v))
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    out = fast_attention(q, k, v, is_causal=is_causal, scale=scale)
    ref = _ref(qr, kr, vr, is_causal, scale)
    assert _rel_l2(out, ref) < TOL
    _, lse = fastflash_attn(q.detach(), k.detach(), v.detach(), is_causal, return_lse=True, scale=scale)
    sc = (1.0 / math.sqrt(D)) if scale is None else scale
    logits = (qr.detach().double() @ kr.detach().double().transpose(-1, -2)) * sc
    if is_causal:
        logits = logits.masked_fill(torch.ones(S, S, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    lse_true = torch.logsumexp(logits, dim=-1) / math.log(2.0)
    assert float((lse.double() - lse_true).abs().max()) < 2e-3
    torch.manual_seed(6)
    g = torch.randn_like(out)
    out.backward(g)
    ref.backward(g.float())
    for name, got, want in (("dq", q.grad, qr.grad), ("dk", k.grad, kr.grad), ("dv", v.grad, vr.grad)):
        assert _rel_l2(got, want) < TOL_PEAKY_GRAD, name

@pytest.mark.parametrize("D", [1, 2, 4, 8, 16, 32])
def test_small_head_dims_padded(D):
    torch.manual_seed(4)
    q, k, v = (torch.randn(2, 3, 160, D, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    for causal in (False, True):
        out = fast_attention(q, k, v, is_causal=causal)
        assert out.shape == q.shape
        assert _rel_l2(out, _ref(q, k, v, causal, None)) < TOL


def test_strided_inputs_are_copied():
    torch.manual_seed(5)
    base = torch.randn(2, 256, 4, 64, device="cuda", dtype=torch.bfloat16)
    q = base.transpose(1, 2)  # [B,H,S,D] view, non-contiguous
    out = fast_attention(q, q, q, is_causal=True)
    assert _rel_l2(out, _ref(q, q, q, True, None)) < TOL


def test_no_device_timeouts_recorded():
    from fastflashattention_b200 import _lib
    torch.manual_seed(6)
    q, k, v = (torch.randn(1, 2, 700, 128, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    fast_attention(q, k, v, is_causal=True)
    assert _lib.device_status() == (0, 0, 0, 0)
