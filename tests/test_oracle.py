"""CPU: pin the numpy restatement of the reference algorithm against the golden vectors.

The golden vectors are the reference's own test oracle (fp32 SDPA, see
tests/golden/make_golden.py); the gates are the reference's (forward 5e-3,
tests/test_parity.py:47; backward 1e-2, :85) and the tighter 5e-3 the B200 build is
held to for every output.
"""
import numpy as np
import pytest

from conftest import golden_cases, load_golden
from oracle import flash_oracle as fo

TOL = 5e-3  # rel-L2, O and dQ/dK/dV


def grad_tol(name):
    """Gradient gate: 5e-3, except the q*8 stress case, where the reference algorithm
    itself (bf16 dS) lands at ~5.0e-3 on dQ; there the reference's own 1e-2 gate applies."""
    return 1e-2 if name.startswith("peaky") else TOL


def _flat(a):
    B, H, S, D = a.shape
    return a.reshape(B * H, S, D)


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_golden(name):
    g = load_golden(name)
    q, k, v, do = (_flat(g[x]) for x in ("q", "k", "v", "do"))
    o, lse2 = fo.forward(q, k, v, g["causal"], g["scale"])
    assert fo.rel_l2(o, _flat(g["o"])) < TOL
    # base-2 LSE of the oracle vs natural-log LSE of the golden
    np.testing.assert_allclose(lse2 / fo.LOG2E, g["lse"].reshape(lse2.shape), rtol=0, atol=2e-4)
    dq, dk, dv = fo.backward(q, k, v, o, do, lse2, g["causal"], g["scale"])
    for mine, ref in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        assert fo.rel_l2(mine, _flat(g[ref])) < grad_tol(name), ref


def test_oracle_block_size_invariance():
    g = load_golden("tiny_causal_b1h2s256d64")
    q, k, v = (_flat(g[x]) for x in ("q", "k", "v"))
    o1, l1 = fo.forward(q, k, v, True, None, 128, 128)
    o2, l2 = fo.forward(q, k, v, True, None, 64, 64)
    assert fo.rel_l2(o1, o2) < 2e-3
    np.testing.assert_allclose(l1, l2, atol=1e-4)


def test_oracle_exact_f64_agrees():
    g = load_golden("ragged_noncausal_b1h2s200d64")
    q, k, v = (_flat(g[x]) for x in ("q", "k", "v"))
    o, lse = fo.exact_forward_f64(q, k, v, False)
    assert fo.rel_l2(o, _flat(g["o"])) < 1e-5
    np.testing.assert_allclose(lse, g["lse"].reshape(lse.shape), atol=1e-4)


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0], np.float32)
    r = fo.bf16_round(x)
    assert r[0] == 1.0
    assert r[1] == 1.0                     # tie -> even mantissa
    assert r[2] == np.float32(1.0 + 4 * 2 ** -8)
    assert r[3] == -2.5 and r[4] == 0.0
