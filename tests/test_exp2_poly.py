"""The FMA-pipe exp2 of the softmax (`exp2_fma` / `exp2_fma2` in csrc/sm100.cuh).

CPU: a Remez exchange for the minimax relative error of a degree-3 polynomial p(f) ~ 2^f
on [-1/2, 1/2] re-derives the coefficients committed in sm100.cuh, and their float32
Horner evaluation stays within the stated 7.5e-5 relative error.

GPU: a small program built with nvcc evaluates exp2_fma and exp2_fma2 on the device over
x in [-125, 8] and compares them with CUDA's exp2f and with exact 2^x (max relative error
<= 1e-4); below -126 both clamp to about 2^-126 (a value far below anything a softmax
row sums to), and -inf gives that same clamped value, not 0.
"""
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

CSRC = Path(__file__).resolve().parents[1] / "fastflashattention_b200" / "csrc"


def committed_coefficients():
    src = (CSRC / "sm100.cuh").read_text()
    body = src[src.index("float exp2_fma(float x)"):]
    vals = dict(re.findall(r"(c[0-3]) = ([0-9.eE+-]+)f", body[:800]))
    return np.array([float(vals[f"c{i}"]) for i in range(4)])


def remez(deg, a=-0.5, b=0.5, iters=30):
    """Minimax relative-error polynomial for 2^x on [a, b] (Remez exchange)."""
    n = deg + 2
    x = 0.5 * (a + b) + 0.5 * (b - a) * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    g = np.linspace(a, b, 200001)
    for _ in range(iters):
        A = np.zeros((n, n))
        A[:, :deg + 1] = x[:, None] ** np.arange(deg + 1)
        A[:, deg + 1] = (-1.0) ** np.arange(n) * 2.0 ** x
        c = np.linalg.solve(A, 2.0 ** x)[:deg + 1]
        err = (np.polyval(c[::-1], g) - 2.0 ** g) / 2.0 ** g
        # the extremum of |err| inside every run of constant sign
        cuts = np.flatnonzero(np.diff(np.sign(err)) != 0) + 1
        ext = np.array([seg[np.argmax(np.abs(err[seg]))] for seg in np.split(np.arange(len(g)), cuts)])
        while len(ext) > n:
            ext = ext[1:] if abs(err[ext[0]]) < abs(err[ext[-1]]) else ext[:-1]
        if len(ext) == n:
            x = g[ext]
    return c, float(np.abs(err).max())


def test_coefficients_are_the_minimax_fit():
    c, err = remez(3)
    mine = committed_coefficients()
    np.testing.assert_allclose(mine, c.astype(np.float32), rtol=1e-6, atol=0)
    assert err < 7.5e-5
    f = np.linspace(-0.5, 0.5, 100001).astype(np.float32)
    p = np.zeros_like(f)
    for ck in mine.astype(np.float32)[::-1]:
        p = (p * f + ck).astype(np.float32)
    rel = np.abs(p.astype(np.float64) - 2.0 ** f.astype(np.float64)) / 2.0 ** f.astype(np.float64)
    assert rel.max() < 7.6e-5


PROGRAM = r"""
#include <cstdio>
#include <cmath>
#include "sm100.cuh"
__global__ void eval(const float* x, float* a, float* b, float* c, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * i + 1 < n) {
    float2 r = ffa::exp2_fma2(make_float2(x[2 * i], x[2 * i + 1]));
    b[2 * i] = r.x; b[2 * i + 1] = r.y;
  }
  for (int j = i; j < n; j += gridDim.x * blockDim.x) { a[j] = ffa::exp2_fma(x[j]); c[j] = exp2f(x[j]); }
}
int main() {
  const int n = 1 << 20;
  float *x, *a, *b, *c;
  if (cudaMallocManaged(&x, n * 4) || cudaMallocManaged(&a, n * 4) || cudaMallocManaged(&b, n * 4) ||
      cudaMallocManaged(&c, n * 4)) return 2;
  const int m = n - 64;
  for (int i = 0; i < m; ++i) x[i] = -125.0f + 133.0f * (float)i / (float)(m - 1);  // [-125, 8]
  for (int i = m; i < n - 1; ++i) x[i] = -126.0f - 2.0f * (float)(i - m);           // -126 ... -250
  x[n - 1] = -INFINITY;
  eval<<<(n / 2 + 255) / 256, 256>>>(x, a, b, c, n);
  if (cudaDeviceSynchronize() != cudaSuccess) return 3;
  double worst_f = 0, worst_f2 = 0, worst_cuda = 0, pair_mismatch = 0;
  for (int i = 0; i < m; ++i) {
    const double t = exp2((double)x[i]);
    worst_f = fmax(worst_f, fabs(a[i] - t) / t);
    worst_f2 = fmax(worst_f2, fabs(b[i] - t) / t);
    worst_cuda = fmax(worst_cuda, fabs((double)a[i] - c[i]) / c[i]);
    if (a[i] != b[i]) pair_mismatch += 1;
  }
  double tail_max = 0, tail_min = 1;
  for (int i = m; i < n; ++i) { tail_max = fmax(tail_max, a[i]); tail_max = fmax(tail_max, b[i]); tail_min = fmin(tail_min, fmin(a[i], b[i])); }
  printf("%.9g %.9g %.9g %.0f %.9g %.9g %.9g\n", worst_f, worst_f2, worst_cuda, pair_mismatch, tail_min, tail_max,
         (double)a[n - 1]);
  return 0;
}
"""


@pytest.mark.gpu
def test_exp2_fma_accuracy_on_device(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    src = tmp_path / "exp2.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "exp2"
    subprocess.run([nvcc, "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-I", str(CSRC),
                    str(src), "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, timeout=120).stdout.split()
    worst_f, worst_f2, worst_cuda, mismatch, tail_min, tail_max, at_neg_inf = map(float, out)
    assert worst_f <= 1e-4 and worst_f2 <= 1e-4, (worst_f, worst_f2)
    assert worst_cuda <= 1e-4, worst_cuda
    assert mismatch == 0  # the packed form rounds exactly like the scalar one
    # clamp: everything at or below -126 (and -inf) comes out at most about 2^-126, never 0 or negative
    assert 0 < tail_min and tail_max <= 2.0 ** -125
    assert 0 < at_neg_inf <= 2.0 ** -125
