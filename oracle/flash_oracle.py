"""CPU oracle (test infrastructure only): a numpy restatement of the reference algorithm.

Used only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg, as the checker.  The product path never imports this module.

It restates the arithmetic of the reference Triton kernels in
``fastflash_attention/_kernel.py`` step for step, in fp32 numpy with explicit bf16
rounding where the reference casts:

* forward  ``_fastflash_fwd`` (:194-279): blockwise online softmax in base 2 with
  ``qk_scale = scale * LOG2E`` (:304-305); per key block ``m_new = max(m, rowmax)``,
  ``alpha = exp2(m - m_new)``, ``p = exp2(qk - m_new)``, ``l = l*alpha + rowsum(p)``,
  ``acc = acc*alpha + bf16(p) @ v`` (:238-246); masked blocks use the ``m_safe`` guard
  (:257-266); ``O = acc / l_safe`` (:269-272); ``LSE = m_safe + log2(l_safe)`` (:274-279).
* backward preprocess (:323-338): ``delta = rowsum(O * dO)`` in fp32.
* dK/dV (:379-448): ``p = exp2(qk - lse)`` masked, ``dv += bf16(p)^T dO``,
  ``dp = dO V^T``, ``ds = p (dp - delta)``, ``dk += bf16(ds)^T Q``, ``dk *= scale``.
* dQ (:487-564, recompute path): ``dq += bf16(ds) K``, ``dq *= scale``.

Parity pin: ``tests/test_oracle.py`` checks this restatement against the fp32
``F.scaled_dot_product_attention`` golden vectors in ``tests/golden/`` (the reference's
own test oracle, ``tests/test_parity.py:32-35``) at the reference's gates
(5e-3 forward, 1e-2 backward, ``tests/test_parity.py:47, :85``).
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 -> bf16 (nearest, ties to even) and return as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def _mask(S: int, m0: int, m1: int, n0: int, n1: int, causal: bool) -> np.ndarray:
    rows = np.arange(m0, m1)[:, None]
    cols = np.arange(n0, n1)[None, :]
    valid = cols < S
    if causal:
        valid = valid & (rows >= cols)
    return valid


def forward(q, k, v, causal: bool, scale: float | None = None, block_m: int = 128, block_n: int = 128):
    """q, k, v: [BH, S, D] fp32 arrays holding bf16 values.  Returns (O bf16-rounded fp32, LSE2)."""
    BH, S, D = q.shape
    sm = (1.0 / np.sqrt(D)) if scale is None else float(scale)
    qk_scale = np.float32(sm * LOG2E)
    O = np.zeros((BH, S, D), np.float32)
    L = np.zeros((BH, S), np.float32)
    for z in range(BH):
        for m0 in range(0, S, block_m):
            m1 = min(m0 + block_m, S)
            qb = q[z, m0:m1]
            m_i = np.full(m1 - m0, -np.inf, np.float32)
            l_i = np.zeros(m1 - m0, np.float32)
            acc = np.zeros((m1 - m0, D), np.float32)
            n_end = min(m0 + block_m, S) if causal else S
            for n0 in range(0, n_end, block_n):
                n1 = min(n0 + block_n, S)
                qk = (qb @ k[z, n0:n1].T).astype(np.float32) * qk_scale
                qk = np.where(_mask(S, m0, m1, n0, n1, causal), qk, -np.inf).astype(np.float32)
                m_new = np.maximum(m_i, qk.max(axis=1))
                m_safe = np.where(m_new == -np.inf, 0.0, m_new).astype(np.float32)
                alpha = np.exp2(m_i - m_safe).astype(np.float32)
                p = np.exp2(qk - m_safe[:, None]).astype(np.float32)
                l_i = l_i * alpha + p.sum(axis=1, dtype=np.float32)
                acc = acc * alpha[:, None] + bf16_round(p) @ v[z, n0:n1]
                m_i = m_safe
            l_safe = np.where(l_i == 0.0, 1.0, l_i).astype(np.float32)
            O[z, m0:m1] = bf16_round(acc / l_safe[:, None])
            m_fin = np.where(m_i == -np.inf, 0.0, m_i)
            L[z, m0:m1] = m_fin + np.log2(l_safe)
    return O, L


def backward(q, k, v, o, do, lse, causal: bool, scale: float | None = None, block: int = 128):
    """Returns (dq, dk, dv) as bf16-rounded fp32 arrays, each [BH, S, D]."""
    BH, S, D = q.shape
    sm = np.float32((1.0 / np.sqrt(D)) if scale is None else float(scale))
    qk_scale = np.float32(float(sm) * LOG2E)
    delta = (o.astype(np.float32) * do.astype(np.float32)).sum(axis=2, dtype=np.float32)
    dq = np.zeros((BH, S, D), np.float32)
    dk = np.zeros((BH, S, D), np.float32)
    dv = np.zeros((BH, S, D), np.float32)
    for z in range(BH):
        qk = (q[z] @ k[z].T).astype(np.float32) * qk_scale
        p = np.exp2(qk - lse[z][:, None]).astype(np.float32)
        p = np.where(_mask(S, 0, S, 0, S, causal), p, 0.0).astype(np.float32)
        dp = (do[z] @ v[z].T).astype(np.float32)
        ds = (p * (dp - delta[z][:, None])).astype(np.float32)
        pb, dsb = bf16_round(p), bf16_round(ds)
        # blockwise accumulation order of the reference kernels is immaterial at fp32
        dv[z] = bf16_round(pb.T @ do[z])
        dk[z] = bf16_round((dsb.T @ q[z]) * sm)
        dq[z] = bf16_round((dsb @ k[z]) * sm)
    return dq, dk, dv


def exact_forward_f64(q, k, v, causal: bool, scale: float | None = None):
    """Plain softmax attention in float64 (no tiling, no bf16 rounding): O and natural-log LSE."""
    BH, S, D = q.shape
    sm = (1.0 / np.sqrt(D)) if scale is None else float(scale)
    s = np.einsum("zid,zjd->zij", q.astype(np.float64), k.astype(np.float64)) * sm
    if causal:
        s = np.where(np.tril(np.ones((S, S), bool))[None], s, -np.inf)
    m = s.max(axis=2, keepdims=True)
    e = np.exp(s - m)
    l = e.sum(axis=2, keepdims=True)
    o = np.einsum("zij,zjd->zid", e / l, v.astype(np.float64))
    return o, (m + np.log(l))[..., 0]


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12))
