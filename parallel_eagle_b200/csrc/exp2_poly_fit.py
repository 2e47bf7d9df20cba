"""Derive the coefficients of ``exp2_poly2`` (sm100.cuh): the degree-3 polynomial
p(f) minimising max |p(f) - 2^f| / 2^f over f in [-1/2, 1/2], by Remez exchange.

    python parallel_eagle_b200/csrc/exp2_poly_fit.py

prints the fp32 coefficients c0..c3 and the relative error they reach.
"""

import numpy as np


def fit(deg: int = 3, iters: int = 30):
    nodes = np.cos(np.linspace(0.0, np.pi, deg + 2))[::-1] * 0.5
    grid = np.linspace(-0.5, 0.5, 200001)
    for _ in range(iters):
        # p(f_i) - 2^f_i = (-1)^i E 2^f_i at the deg + 2 reference points
        A = np.zeros((deg + 2, deg + 2))
        for i, f in enumerate(nodes):
            A[i, : deg + 1] = f ** np.arange(deg + 1)
            A[i, deg + 1] = (-1) ** i * 2.0 ** f
        sol = np.linalg.solve(A, 2.0 ** nodes)
        coef = sol[: deg + 1]
        err = (np.polyval(coef[::-1], grid) - 2.0 ** grid) / 2.0 ** grid
        turn = [0] + [i for i in range(1, len(grid) - 1)
                      if (err[i] - err[i - 1]) * (err[i + 1] - err[i]) <= 0] + [len(grid) - 1]
        if len(turn) == deg + 2:
            nodes = grid[turn]
    c32 = coef.astype(np.float32)
    err32 = (np.polyval(c32[::-1].astype(np.float64), grid) - 2.0 ** grid) / 2.0 ** grid
    return c32, float(np.abs(err32).max())


if __name__ == "__main__":
    c, e = fit()
    print("c0..c3 =", ", ".join(f"{float(x):.8g}f" for x in c))
    print(f"max relative error {e:.3g}")
