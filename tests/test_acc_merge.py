"""GPU: the fp32 accumulate and merge entry points the context-parallel ring uses.

* ``ffa_bwd_dkdv_acc`` / ``ffa_bwd_dq_acc`` add exactly the fp32 values the bf16 entry
  points round: into zeroed accumulators, their bf16 rounding equals ``ffa_bwd_dkdv`` /
  ``ffa_bwd_dq`` bit for bit, and a second call doubles them exactly.
* ``ffa_fwd_merge`` with ``first`` reproduces ``ffa_fwd`` (O bit for bit after rounding,
  the LSE to float precision), and merging two key halves equals attention over all keys.
"""
import math

import pytest
import torch

from fastflashattention_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(BH, S, D, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(BH, S, D, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(4)]


def _st():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("BH,S,D,causal", [(3, 700, 128, 1), (2, 512, 64, 0), (4, 256, 128, 0)])
def test_bwd_acc_matches_bf16_entry_points(BH, S, D, causal):
    lib = _lib.load()
    q, k, v, do = _inputs(BH, S, D, 1)
    sm = 1.0 / math.sqrt(D)
    st = (S * D, D)
    o = torch.empty_like(q)
    lse = torch.empty(BH, S, device="cuda", dtype=torch.float32)
    _lib.check(lib.ffa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), BH, S, D, *st, sm,
                           causal, _st()), "ffa_fwd")
    delta = torch.empty(BH, S, device="cuda", dtype=torch.float32)
    _lib.check(lib.ffa_bwd_preprocess(o.data_ptr(), do.data_ptr(), delta.data_ptr(), BH, S, D, *st, _st()), "pre")
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(), delta.data_ptr())
    _lib.check(lib.ffa_bwd_dkdv(*args, dk.data_ptr(), dv.data_ptr(), BH, S, D, *st, sm, causal, _st()), "dkdv")
    _lib.check(lib.ffa_bwd_dq(*args, dq.data_ptr(), BH, S, D, *st, sm, causal, _st()), "dq")
    aq, ak, av = (torch.zeros(BH, S, D, device="cuda", dtype=torch.float32) for _ in range(3))
    for call in range(2):
        _lib.check(lib.ffa_bwd_dkdv_acc(*args, ak.data_ptr(), av.data_ptr(), BH, S, D, *st, sm, causal, _st()),
                   "dkdv_acc")
        _lib.check(lib.ffa_bwd_dq_acc(*args, aq.data_ptr(), BH, S, D, *st, sm, causal, _st()), "dq_acc")
        torch.cuda.synchronize()
        if call == 0:
            first = [t.clone() for t in (aq, ak, av)]
            for name, a, b in (("dq", aq, dq), ("dk", ak, dk), ("dv", av, dv)):
                assert torch.equal(a.to(torch.bfloat16), b), name
    for a, f in zip((aq, ak, av), first):
        assert torch.equal(a, 2 * f)
    assert _lib.device_status() == (0, 0, 0, 0)


@pytest.mark.parametrize("BH,S,D,causal", [(3, 700, 128, 1), (2, 512, 64, 0)])
def test_fwd_merge_first_equals_forward(BH, S, D, causal):
    lib = _lib.load()
    q, k, v, _ = _inputs(BH, S, D, 2)
    sm = 1.0 / math.sqrt(D)
    st = (S * D, D)
    o = torch.empty_like(q)
    lse = torch.empty(BH, S, device="cuda", dtype=torch.float32)
    _lib.check(lib.ffa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), BH, S, D, *st, sm,
                           causal, _st()), "ffa_fwd")
    acc = torch.full((BH, S, D), float("nan"), device="cuda")
    acc_lse = torch.full((BH, S), float("nan"), device="cuda")
    _lib.check(lib.ffa_fwd_merge(q.data_ptr(), k.data_ptr(), v.data_ptr(), acc.data_ptr(), acc_lse.data_ptr(), BH, S,
                                 D, *st, sm, causal, 1, _st()), "ffa_fwd_merge")
    torch.cuda.synchronize()
    assert torch.equal(acc.to(torch.bfloat16), o)
    torch.testing.assert_close(acc_lse, lse, rtol=0, atol=2e-5)


@pytest.mark.parametrize("D", [64, 128])
def test_fwd_merge_of_two_key_halves_is_full_attention(D):
    """Queries of one chunk against two key chunks, merged in order, equal attention over
    the concatenated keys (the ring's non-causal blocks)."""
    lib = _lib.load()
    BH, C = 4, 512
    q, _, _, _ = _inputs(BH, C, D, 3)
    kf, vf = (torch.randn(BH, 2 * C, D, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    sm = 1.0 / math.sqrt(D)
    acc = torch.empty(BH, C, D, device="cuda")
    acc_lse = torch.empty(BH, C, device="cuda")
    for h in range(2):
        kh, vh = kf[:, h * C:(h + 1) * C].contiguous(), vf[:, h * C:(h + 1) * C].contiguous()
        _lib.check(lib.ffa_fwd_merge(q.data_ptr(), kh.data_ptr(), vh.data_ptr(), acc.data_ptr(), acc_lse.data_ptr(),
                                     BH, C, D, C * D, D, sm, 0, int(h == 0), _st()), "ffa_fwd_merge")
    torch.cuda.synchronize()
    s = (q.double() @ kf.double().transpose(1, 2)) * sm
    want = torch.softmax(s, dim=-1) @ vf.double()
    assert float((acc.double() - want).norm() / want.norm()) < 2e-3
    lse_true = torch.logsumexp(s, dim=-1) / math.log(2.0)
    assert float((acc_lse.double() - lse_true).abs().max()) < 1e-3
