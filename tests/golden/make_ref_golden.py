"""Generate the reference-implementation fixtures in ``tests/golden/ref/`` (needs a CUDA GPU).

    python tests/golden/make_ref_golden.py [--out DIR]

Runs the UNMODIFIED reference package (``fastflash_attention``, installed under
``baseline/_ref`` with ``pip install --target``) as a black box on the GPU: its public
``fast_attention`` forward and its ``torch.autograd`` backward (``FastFlashAttn``,
reference ``fastflash_attention/_kernel.py:773-906``), plus its base-2 LSE from
``fastflash_attn(..., return_lse=True)`` (``_kernel.py:282-318``).  Nothing of this
repository's kernels is on that path.

Inputs are drawn on the CPU from ``torch.Generator().manual_seed(seed)`` (q, k, v, then
dO), so any machine regenerates them bit for bit; each fixture stores the SHA-256 of the
input bytes so a test can prove it regenerated the same ones.  The seeds and shapes are
the reference tests' own (``tests/test_parity.py:18-23`` shapes; seed 2 / dO seed 3 of
``test_backward_parity``, ``:64-79``; seed 1 and scale 0.05 of
``test_forward_custom_scale``, ``:50-61``), plus BASELINE configs[0] (B1 H2 S256 D64
causal, seed 0), S=2048 at D=64 and D=128, and the q*8 peaky stress case.

Outputs are kept as the reference produced them: O, dQ, dK, dV as raw bf16 bits, the LSE
as fp32.  For S > 256 only a fixed sample of rows per (batch, head) slice is stored
(``rows``), which keeps the files small; rel-L2 over the sampled rows is the statistic
the tests compare.
"""
from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
REF = ROOT / "baseline" / "_ref"

# name: (B, H, S, D, causal, scale, q_multiplier, seed, dO seed)
CASES = {
    "cfg0_causal_b1h2s256d64": (1, 2, 256, 64, True, None, 1.0, 0, 100),
    "shape0_noncausal_b2h4s128d64": (2, 4, 128, 64, False, None, 1.0, 2, 3),
    "shape0_causal_b2h4s128d64": (2, 4, 128, 64, True, None, 1.0, 2, 3),
    "shape1_noncausal_b1h8s512d128": (1, 8, 512, 128, False, None, 1.0, 2, 3),
    "shape1_causal_b1h8s512d128": (1, 8, 512, 128, True, None, 1.0, 2, 3),
    "shape2_noncausal_b2h2s200d64": (2, 2, 200, 64, False, None, 1.0, 2, 3),
    "shape2_causal_b2h2s200d64": (2, 2, 200, 64, True, None, 1.0, 2, 3),
    "shape3_noncausal_b1h3s1024d128": (1, 3, 1024, 128, False, None, 1.0, 2, 3),
    "shape3_causal_b1h3s1024d128": (1, 3, 1024, 128, True, None, 1.0, 2, 3),
    "custom_scale_causal_b2h4s256d64": (2, 4, 256, 64, True, 0.05, 1.0, 1, 3),
    "s2048_causal_b1h2s2048d64": (1, 2, 2048, 64, True, None, 1.0, 11, 12),
    "s2048_causal_b1h2s2048d128": (1, 2, 2048, 128, True, None, 1.0, 13, 14),
    "peaky_noncausal_b1h2s1024d64": (1, 2, 1024, 64, False, None, 8.0, 4, 5),
}

ROWS_PER_SLICE = 32  # sampled rows per (batch, head) slice when S > 256


def make_inputs(B, H, S, D, qmul, seed, dseed):
    """Seeded CPU inputs: q, k, v from `seed`, dO from `dseed`; all bf16 [B,H,S,D]."""
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    if qmul != 1.0:
        q = (q.float() * qmul).to(torch.bfloat16)
    do = torch.randn(B, H, S, D, generator=torch.Generator().manual_seed(dseed)).to(torch.bfloat16)
    return q, k, v, do


def input_digest(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def sample_rows(S, seed):
    """Sorted row indices kept for one fixture: all rows when S <= 256, else a fixed
    sample that always includes the first and last rows (the causal diagonal's ends)."""
    if S <= 256:
        return np.arange(S, dtype=np.int64)
    rng = np.random.default_rng(1000 + seed)
    pick = rng.choice(np.arange(1, S - 1), ROWS_PER_SLICE - 2, replace=False)
    return np.sort(np.concatenate([[0, S - 1], pick])).astype(np.int64)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE / "ref"))
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    sys.path.insert(0, str(REF))
    import fastflash_attention as ref  # the unmodified reference, black box
    from fastflash_attention._kernel import fastflash_attn as ref_fwd_lse
    dev = torch.device("cuda", 0)
    for name, (B, H, S, D, causal, scale, qmul, seed, dseed) in CASES.items():
        q, k, v, do = make_inputs(B, H, S, D, qmul, seed, dseed)
        qd, kd, vd = (t.to(dev).requires_grad_(True) for t in (q, k, v))
        o = ref.fast_attention(qd, kd, vd, is_causal=causal, scale=scale)
        o.backward(do.to(dev))
        with torch.no_grad():
            o2, lse = ref_fwd_lse(q.to(dev), k.to(dev), v.to(dev), causal, return_lse=True, scale=scale)
        torch.cuda.synchronize()
        assert torch.equal(o2, o.detach()), "reference forward with and without LSE disagree"
        rows = sample_rows(S, seed)
        ridx = torch.from_numpy(rows).to(dev)
        pick = lambda t: t.detach().index_select(2, ridx)  # noqa: E731
        np.savez_compressed(
            out / f"{name}.npz",
            rows=rows,
            o=bits(pick(o)), dq=bits(pick(qd.grad)), dk=bits(pick(kd.grad)), dv=bits(pick(vd.grad)),
            lse=lse.index_select(2, ridx).cpu().numpy(),
            meta=np.array([B, H, S, D, int(causal), seed, dseed], np.int64),
            scale=np.array([np.nan if scale is None else scale], np.float64),
            qmul=np.array([qmul], np.float64),
            input_sha256=np.array(input_digest(q, k, v, do)),
            generator=np.array(f"reference fastflash_attention {getattr(ref, '__version__', '?')} "
                               f"on {torch.cuda.get_device_name(dev)}, torch {torch.__version__}"),
        )
        print("wrote", name, "rows", len(rows), flush=True)


if __name__ == "__main__":
    main()
