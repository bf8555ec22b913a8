"""The allocation-free backward entry point `ffa_bwd_noalloc` (include/ffa.h).

Some callers cannot call cudaMalloc: their device memory belongs to another allocator
(frameworks that preallocate nearly the whole GPU, serving runtimes with a fixed pool),
or they run where allocating is forbidden.  `ffa_bwd_noalloc` keeps the backward's only
scratch (the fp32 delta = rowsum(O*dO) workspace) in a fixed array inside the library.
This test calls it through the C ABI twice in a row and checks both results against
the regular `ffa_bwd` (which takes a caller-allocated workspace).  It lives in its own
file, collected last, and passes both alone in a fresh process and after the others.
"""
import math

import pytest
import torch

from fastflashattention_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 5e-3  # rel-L2, the tolerance of the parity tests


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))


@pytest.mark.parametrize("BH,S,D,causal", [(8, 700, 128, 1), (3, 256, 64, 0)])
def test_noalloc_backward_matches_regular_backward_twice(BH, S, D, causal):
    lib = _lib.load()
    torch.manual_seed(11)
    dev = "cuda"
    q, k, v, do = (torch.randn(BH, S, D, device=dev, dtype=torch.bfloat16) for _ in range(4))
    o = torch.empty_like(q)
    lse = torch.empty(BH, S, device=dev, dtype=torch.float32)
    sm = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream().cuda_stream
    strides = (S * D, D)
    _lib.check(lib.ffa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), BH, S, D,
                           *strides, sm, causal, stream), "ffa_fwd")
    delta = torch.empty(BH, S, device=dev, dtype=torch.float32)
    ref = [torch.empty_like(q) for _ in range(3)]
    _lib.check(lib.ffa_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                           delta.data_ptr(), ref[0].data_ptr(), ref[1].data_ptr(), ref[2].data_ptr(), BH, S, D,
                           *strides, sm, causal, stream), "ffa_bwd")
    for _ in range(2):
        got = [torch.full_like(q, float("nan")) for _ in range(3)]
        _lib.check(lib.ffa_bwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                       lse.data_ptr(), got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(),
                                       BH, S, D, *strides, sm, causal, stream), "ffa_bwd_noalloc")
        torch.cuda.synchronize()
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            assert torch.isfinite(a).all(), name
            assert _rel(a, b) < TOL, name
    assert _lib.device_status() == (0, 0, 0, 0)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    S, D = 8192, 128
    BH = (4 << 20) // S + 1  # one slice more than the fixed scratch holds
    rc = lib.ffa_bwd_noalloc(16, 16, 16, 16, 16, 16, 16, 16, 16, BH, S, D, S * D, D, 0.1, 1, None)
    assert rc == _lib.FFA_ERR_INVALID
    assert "scratch" in _lib.last_error()
