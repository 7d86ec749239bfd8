"""Coefficients of the degree-3 polynomial p(f) ~ 2**f on [-1/2, 1/2] that
the forward kernel's FMA-pipe exponential uses (``exp2_poly`` in
``ring_fwd.cuh``): minimax in relative error, found by the Remez exchange
algorithm (equioscillation of the weighted error at 5 alternation points).
Prints the coefficients and the maximum relative error; the test
``tests/test_exp2_poly.py`` checks the header's constants against this."""

import numpy as np


def remez_exp2(deg: int = 3, lo: float = -0.5, hi: float = 0.5, iters: int = 30):
    n = deg + 2
    # start from Chebyshev extrema
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    grid = np.linspace(lo, hi, 200001)
    for _ in range(iters):
        # solve p(x_i) - 2**x_i = (-1)**i * E * 2**x_i   (relative error weight)
        a = np.zeros((n, n))
        for i, xi in enumerate(x):
            a[i, :deg + 1] = xi ** np.arange(deg + 1)
            a[i, deg + 1] = -((-1) ** i) * 2.0 ** xi
        sol = np.linalg.solve(a, 2.0 ** x)
        c = sol[:deg + 1]
        err = (np.polyval(c[::-1], grid) - 2.0 ** grid) / 2.0 ** grid
        # new alternation points: extrema of err between sign changes
        idx = [0]
        for k in range(1, len(grid) - 1):
            if (err[k] - err[k - 1]) * (err[k + 1] - err[k]) <= 0:
                idx.append(k)
        idx.append(len(grid) - 1)
        ext = np.array(idx)
        # keep n alternating extrema of largest magnitude
        pts = []
        for k in ext:
            if pts and np.sign(err[k]) == np.sign(err[pts[-1]]):
                if abs(err[k]) > abs(err[pts[-1]]):
                    pts[-1] = k
            else:
                pts.append(k)
        while len(pts) > n:
            if abs(err[pts[0]]) < abs(err[pts[-1]]):
                pts.pop(0)
            else:
                pts.pop()
        if len(pts) == n:
            x = grid[pts]
    return c, float(np.max(np.abs(err)))


if __name__ == "__main__":
    c, e = remez_exp2()
    for i, v in enumerate(c):
        print(f"c{i} = {np.float32(v)!r}  ({v:.10f})")
    print(f"max relative error {e:.3e}")
