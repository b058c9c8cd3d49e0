"""Fits the polynomial p(f) ~ 2^f on f in [-1/2, 1/2] used by the attention kernel's
FMA-pipe exponential (2^x = 2^round(x) * p(x - round(x))).

Method: minimise the maximum relative error |p(f) / 2^f - 1| with a Remez-style
exchange started from a least-squares fit on Chebyshev nodes. Prints the
coefficients (c0 + c1 f + c2 f^2 + ...) as float32 literals and the achieved bound.

    python kernelpilot_b200/csrc/fit_exp2_poly.py [degree]
"""
import sys

import numpy as np


def fit(degree: int, iters: int = 30):
    n = degree + 2
    # start: weighted least squares on dense Chebyshev nodes
    xs = np.cos(np.linspace(0, np.pi, 2000)) * 0.5
    w = 2.0 ** -xs
    V = np.vander(xs, degree + 1, increasing=True) * w[:, None]
    c = np.linalg.lstsq(V, np.ones_like(xs), rcond=None)[0]
    grid = np.linspace(-0.5, 0.5, 200001)
    ref = np.cos(np.linspace(0, np.pi, n))[::-1] * 0.5
    for _ in range(iters):
        # solve p(x_i)/2^x_i - 1 = (-1)^i E on the reference points
        A = np.zeros((n, n))
        for i, x in enumerate(ref):
            A[i, :degree + 1] = x ** np.arange(degree + 1) / 2.0 ** x
            A[i, degree + 1] = (-1) ** i
        sol = np.linalg.solve(A, np.ones(n))
        c = sol[:degree + 1]
        err = np.polyval(c[::-1], grid) / 2.0 ** grid - 1
        # new reference: extrema of the error between sign changes
        idx = [0]
        for k in range(1, len(grid) - 1):
            if (err[k] - err[k - 1]) * (err[k + 1] - err[k]) <= 0:
                idx.append(k)
        idx.append(len(grid) - 1)
        cand = grid[idx]
        vals = np.abs(err[idx])
        if len(cand) >= n:
            order = np.argsort(-vals)[:n]
            ref = np.sort(cand[order])
    c32 = np.array(c, dtype=np.float32)
    err32 = np.polyval(c32.astype(np.float64)[::-1], grid) / 2.0 ** grid - 1
    return c32, float(np.abs(err32).max())


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 3
    c, e = fit(deg)
    print("degree", deg, "max relative error", f"{e:.3e}")
    for i, v in enumerate(c):
        print(f"c{i} = {float(v)!r}f")
