"""The backward's two-stream launch (dQ on a per-device side stream beside dK/dV).

* Host threads that run backward passes at the same time, each on its own stream, get
  bitwise the results of running them one after the other (the shared fork/join events
  are serialised inside the library).
* A backward captured into a CUDA graph replays to the eager result (the side stream is
  forked and joined with events, which capture records as parallel branches).
"""
import threading

import pytest
import torch

from fastflashattention_b200._kernel import _bwd, fastflash_attn

pytestmark = pytest.mark.gpu


def _inputs(seed, B=1, H=4, S=1024, D=128):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v, do = (torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16, generator=gen) for _ in range(4))
    o, lse = fastflash_attn(q, k, v, True, return_lse=True)
    return q, k, v, o, do, lse


def test_concurrent_threads_match_sequential():
    cases = [_inputs(seed) for seed in range(4)]
    want = [_bwd(*c, True, None) for c in cases]
    torch.cuda.synchronize()
    got = [None] * len(cases)
    errors = []

    def run(idx):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                for _ in range(3):
                    got[idx] = _bwd(*cases[idx], True, None)
            s.synchronize()
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    threads = [threading.Thread(target=run, args=(i,)) for i in range(len(cases))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    for w, g in zip(want, got):
        for a, b in zip(w, g):
            assert torch.equal(a, b)


def test_backward_in_cuda_graph_replays_eager_result():
    q, k, v, o, do, lse = _inputs(7, B=2, H=2, S=777)
    want = _bwd(q, k, v, o, do, lse, True, None)
    # warm up on a side stream before capture, as torch.cuda.graph expects
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _bwd(q, k, v, o, do, lse, True, None)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = _bwd(q, k, v, o, do, lse, True, None)
    for x in out:
        x.zero_()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(want, out):
        assert torch.equal(a, b)


def test_capture_beside_plain_backward_on_another_thread():
    """One thread captures a backward into a CUDA graph while another runs plain backward
    passes on its own stream.  Side streams are kept per caller stream, so the plain
    passes never land in the graph: both the plain results and the graph's replay equal
    the sequential results."""
    cap_in = _inputs(21, B=2, H=2, S=900)
    plain_in = _inputs(22)
    want_cap = _bwd(*cap_in, True, None)
    want_plain = _bwd(*plain_in, True, None)
    torch.cuda.synchronize()
    cs, ps = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(cs):  # first backward on this caller stream outside capture
        _bwd(*cap_in, True, None)
    cs.synchronize()
    started, errors, plain_out = threading.Event(), [], []

    def plain():
        try:
            started.wait(timeout=60)
            with torch.cuda.stream(ps):
                for _ in range(5):
                    plain_out.append(_bwd(*plain_in, True, None))
            ps.synchronize()
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    t = threading.Thread(target=plain)
    t.start()
    g = torch.cuda.CUDAGraph()
    # "thread_local" keeps the other thread's plain launches legal during this capture
    with torch.cuda.graph(g, stream=cs, capture_error_mode="thread_local"):
        started.set()
        out = _bwd(*cap_in, True, None)
        for _ in range(20):  # stay in capture while the other thread launches
            out = _bwd(*cap_in, True, None)
    t.join(timeout=120)
    assert not errors, errors
    for x in out:
        x.zero_()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(want_cap, out):
        assert torch.equal(a, b)
    assert plain_out
    for res in plain_out:
        for a, b in zip(want_plain, res):
            assert torch.equal(a, b)
