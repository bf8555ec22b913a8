"""CPU: the CTA -> (block rank, slice) order the forward and backward grids use
(`cta_work_at` / `work_group` in csrc/ffa_common.cuh), compiled for the host with nvcc.

Every (rank, slice) pair must be produced by exactly one CTA (each output tile is
written once), a group's rank-r blocks must all launch before any rank-(r+1) block
(longest job first, rank 0 being the heaviest), and a group of one slice must be the
plain block-major order the non-causal grids keep.
"""
import shutil
import subprocess
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parents[1] / "fastflashattention_b200" / "csrc"

PROGRAM = r"""
#include <cstdio>
#include <cstdlib>
#include "ffa_common.cuh"
int main(int argc, char** argv) {
  if (argv[1][0] == 'g') {  // g BH S D causal -> work_group
    std::printf("%d\n", ffa::work_group(std::atoi(argv[2]), std::atoi(argv[3]), std::atoi(argv[4]), std::atoi(argv[5]) != 0));
    return 0;
  }
  const int nblk = std::atoi(argv[1]), BH = std::atoi(argv[2]), group = std::atoi(argv[3]);
  for (int L = 0; L < nblk * BH; ++L) {
    const ffa::CtaWork w = ffa::cta_work_at(L, nblk, BH, group);
    std::printf("%d %d\n", w.rank, w.bh);
  }
  return 0;
}
"""


@pytest.fixture(scope="module")
def order_bin(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc not available")
    d = tmp_path_factory.mktemp("cta_order")
    src = d / "order.cu"
    src.write_text(PROGRAM)
    exe = d / "order"
    subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I", str(CSRC),
                    str(src), "-o", str(exe)], check=True, capture_output=True)
    return exe


def _order(exe, nblk, bh, group):
    out = subprocess.run([str(exe), str(nblk), str(bh), str(group)], check=True, capture_output=True, text=True)
    return [tuple(map(int, ln.split())) for ln in out.stdout.split("\n") if ln.strip()]


@pytest.mark.parametrize("nblk,bh,group", [(1, 1, 1), (3, 5, 2), (64, 64, 12), (32, 64, 64), (4, 64, 48),
                                           (16, 128, 1), (7, 13, 13), (5, 9, 4), (64, 3, 8)])
def test_every_tile_once_longest_first(order_bin, nblk, bh, group):
    order = _order(order_bin, nblk, bh, group)
    assert len(order) == nblk * bh
    assert sorted(order) == [(r, b) for r in range(nblk) for b in range(bh)]
    g = min(group, bh)
    for g0 in range(0, bh, g):
        members = [(L, r) for L, (r, b) in enumerate(order) if g0 <= b < g0 + g]
        Ls = [L for L, _ in members]
        assert Ls == list(range(Ls[0], Ls[0] + len(Ls))), "a group's CTAs are contiguous in launch order"
        ranks = [r for _, r in members]
        assert ranks == sorted(ranks), "rank r of every slice in a group launches before rank r+1"


def test_group_of_one_is_block_major(order_bin):
    nblk, bh = 6, 4
    assert _order(order_bin, nblk, bh, 1) == [(L % nblk, L // nblk) for L in range(nblk * bh)]


@pytest.mark.parametrize("bh,s,d,causal,want", [
    (64, 8192, 128, 1, 12),   # 4 MiB of streamed tiles per slice: 12 slices in 48 MiB
    (64, 1024, 128, 1, 64),   # everything fits: one group
    (8, 65536, 128, 1, 1),
    (64, 8192, 128, 0, 1),    # non-causal keeps block-major order
])
def test_work_group(order_bin, bh, s, d, causal, want):
    out = subprocess.run([str(order_bin), "g", str(bh), str(s), str(d), str(causal)], check=True,
                         capture_output=True, text=True)
    assert int(out.stdout) == want
