"""Fits the polynomial behind ptx::exp2_poly3 (ptx_sm100.cuh).

2^x is evaluated as 2^n * p(f) with n = round(x), f = x - n in [-0.5, 0.5]
(Cody-Waite range reduction) and p the degree-3 polynomial minimising the
maximum RELATIVE error of p(f) against 2^f on [-0.5, 0.5], found here with a
Remez exchange.  Run: python fit_exp2_poly.py (prints degrees 3-5; the kernel
uses degree 3, max relative error 7.5e-5, below FP16's half-ulp 2.4e-4).
"""
import numpy as np
# Minimax (relative error) polynomial for 2^f on f in [-0.5, 0.5] via a Remez exchange.
def remez(deg, lo=-0.5, hi=0.5, iters=30):
    n = deg + 2
    x = 0.5*(lo+hi) + 0.5*(hi-lo)*np.cos(np.pi*np.arange(n)[::-1]/(n-1))
    f = lambda t: np.exp2(t)
    for _ in range(iters):
        # solve sum c_k x^k - f(x) = (-1)^i E f(x)   (relative error weight)
        A = np.zeros((n, n))
        for i in range(n):
            A[i, :deg+1] = x[i]**np.arange(deg+1)
            A[i, deg+1] = (-1)**i * f(x[i])
        sol = np.linalg.solve(A, f(x))
        c, E = sol[:deg+1], sol[deg+1]
        t = np.linspace(lo, hi, 200001)
        err = (np.polyval(c[::-1], t) - f(t)) / f(t)
        # new extrema: sign changes
        idx = [0]
        s = np.sign(err)
        for k in range(1, len(t)):
            if s[k] != s[idx[-1]]:
                idx.append(k)
            elif abs(err[k]) > abs(err[idx[-1]]):
                idx[-1] = k
        if len(idx) >= n:
            # pick n with largest alternating
            while len(idx) > n:
                if abs(err[idx[0]]) < abs(err[idx[-1]]): idx.pop(0)
                else: idx.pop()
            x = t[idx]
    return c, np.abs(err).max()
for d in (3, 4, 5):
    c, e = remez(d)
    c32 = c.astype(np.float32)
    t = np.linspace(-0.5, 0.5, 400001).astype(np.float32)
    # evaluate in float32 Horner
    p = np.full_like(t, c32[d])
    for k in range(d-1, -1, -1): p = (p * t + c32[k]).astype(np.float32)
    rel = np.abs(p.astype(np.float64) - np.exp2(t.astype(np.float64))) / np.exp2(t.astype(np.float64))
    print(d, "minimax rel err", e, "float32 eval max rel err", rel.max(), "coeffs", [float(v) for v in c32])
