"""Derivation of the exp2 polynomial used by exp2_fma() in sm100.cuh (not run at build time).

Remez exchange for the minimax *relative* error of p(f) ~ 2^f on [-1/2, 1/2] at degrees
3, 4 and 5; prints the float32 coefficients and the maximum relative error of the
float32 Horner evaluation.  The kernels use the degree-3 row.
"""
import numpy as np


def remez(deg, a=-0.5, b=0.5, iters=30):
    n = deg + 2
    x = 0.5*(a+b) + 0.5*(b-a)*np.cos(np.pi*np.arange(n)[::-1]/(n-1))
    for _ in range(iters):
        A = np.zeros((n, n)); rhs = 2.0**x
        for i in range(n):
            A[i,:deg+1] = x[i]**np.arange(deg+1)
            A[i,deg+1] = (-1)**i * 2.0**x[i]
        sol = np.linalg.solve(A, rhs)
        c = sol[:deg+1]
        g = np.linspace(a, b, 200001)
        err = (np.polyval(c[::-1], g) - 2.0**g)/2.0**g
        # new extrema
        idx = [0]
        s = np.sign(err)
        ext=[]
        # split into sign-runs and pick max |err| in each
        start=0
        for i in range(1,len(g)):
            if s[i]!=s[start]:
                seg=np.arange(start,i); ext.append(seg[np.argmax(np.abs(err[seg]))]); start=i
        seg=np.arange(start,len(g)); ext.append(seg[np.argmax(np.abs(err[seg]))])
        if len(ext) >= n:
            # keep the n largest consecutive alternating
            ext = np.array(ext)
            while len(ext) > n:
                if abs(err[ext[0]]) < abs(err[ext[-1]]): ext = ext[1:]
                else: ext = ext[:-1]
            x = g[ext]
    return c, np.abs(err).max()
for d in (3,4,5):
    c, e = remez(d)
    c32 = c.astype(np.float32)
    g = np.linspace(-0.5,0.5,1000001).astype(np.float32)
    p = np.zeros_like(g)
    for k in range(d, -1, -1): p = (p*g + c32[k]).astype(np.float32)
    rel = np.abs(p.astype(np.float64) - 2.0**g.astype(np.float64))/2.0**g
    print(d, [float(v) for v in c32], "maxrel(f64 fit)", e, "maxrel(f32 eval)", rel.max())
