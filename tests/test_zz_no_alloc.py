"""The allocation-free backward entry point `ffa_bwd_noalloc` (include/ffa.h).

Some callers cannot call cudaMalloc: their device memory belongs to another allocator
(frameworks that preallocate nearly the whole GPU, serving runtimes with a fixed pool),
or they run where allocating is forbidden.  `ffa_bwd_noalloc` keeps the backward's only
scratch (the fp32 delta = rowsum(O*dO) workspace) in a fixed array inside the library.
This test calls it through the C ABI twice in a row (with a different dO each time) and
checks that both results equal, bit for bit, those of the regular `ffa_bwd` (which takes a
caller-allocated workspace).  It lives in its own file, collected last, and passes both
alone in a fresh process and after the others.
"""
import math

import pytest
import torch

from fastflashattention_b200 import _lib

pytestmark = pytest.mark.gpu


def _bwd_pair(lib, q, k, v, o, do, lse, BH, S, D, causal, stream):
    """(ffa_bwd result with a caller-allocated workspace, ffa_bwd_noalloc result)."""
    sm = 1.0 / math.sqrt(D)
    strides = (S * D, D)
    delta = torch.empty(BH, S, device=q.device, dtype=torch.float32)
    ref = [torch.empty_like(q) for _ in range(3)]
    _lib.check(lib.ffa_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                           delta.data_ptr(), ref[0].data_ptr(), ref[1].data_ptr(), ref[2].data_ptr(), BH, S, D,
                           *strides, sm, causal, stream), "ffa_bwd")
    got = [torch.full_like(q, float("nan")) for _ in range(3)]
    _lib.check(lib.ffa_bwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                   lse.data_ptr(), got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(),
                                   BH, S, D, *strides, sm, causal, stream), "ffa_bwd_noalloc")
    torch.cuda.synchronize()
    return ref, got


@pytest.mark.parametrize("BH,S,D,causal", [(8, 700, 128, 1), (3, 256, 64, 0)])
def test_noalloc_backward_matches_regular_backward_twice(BH, S, D, causal):
    """Two calls in a row, the second with a different dO: the shared scratch keeps the
    first call's delta, so a second call that failed to rewrite it would show up here.
    Both entry points run the same deterministic kernels on the same delta, so their
    outputs must be bitwise equal."""
    lib = _lib.load()
    torch.manual_seed(11)
    dev = "cuda"
    q, k, v = (torch.randn(BH, S, D, device=dev, dtype=torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    lse = torch.empty(BH, S, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.ffa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), BH, S, D,
                           S * D, D, 1.0 / math.sqrt(D), causal, stream), "ffa_fwd")
    firsts = []
    for call in range(2):
        do = torch.randn(BH, S, D, device=dev, dtype=torch.bfloat16)
        ref, got = _bwd_pair(lib, q, k, v, o, do, lse, BH, S, D, causal, stream)
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            assert torch.isfinite(a).all(), (call, name)
            assert torch.equal(a, b), (call, name)
        firsts.append(got[0])
    assert not torch.equal(firsts[0], firsts[1])  # the second dO really changed the result
    assert _lib.device_status() == (0, 0, 0, 0)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    S, D = 8192, 128
    BH = (4 << 20) // S + 1  # one slice more than the fixed scratch holds
    rc = lib.ffa_bwd_noalloc(16, 16, 16, 16, 16, 16, 16, 16, 16, BH, S, D, S * D, D, 0.1, 1, None)
    assert rc == _lib.FFA_ERR_INVALID
    assert "scratch" in _lib.last_error()
