"""Minimax (Remez exchange) fit of the quartic behind ``exp2_poly_x2`` (csrc/common.cuh).

The selection kernel evaluates 2^x = 2^n * q(f) with n = rint(x) and f in
[-0.5, 0.5]. The coefficients of q minimise the maximum *relative* error
max |q(f) / 2^f - 1| over that interval. This module reproduces them with the
classical Remez exchange algorithm for a weighted (relative-error) minimax
fit, in float64:

1. start from the Chebyshev extrema of the interval as the reference set of
   degree + 2 points;
2. solve the linear system q(x_i) - 2^x_i = (-1)^i E 2^x_i for the degree + 1
   coefficients and the levelled error E;
3. move every reference point to the local extremum of the weighted error
   q(x) / 2^x - 1 in its bracket (a dense grid, refined by golden-section
   search), and repeat until E and the extrema agree.

Run ``python tests/exp2_poly_fit.py`` to print the coefficients, highest degree
first (the Horner order of the header), rounded to float32.
"""

from __future__ import annotations

import numpy as np

LO, HI, DEGREE = -0.5, 0.5, 4


def _weighted_error(c: np.ndarray, x: np.ndarray) -> np.ndarray:
    """q(x) / 2^x - 1 for coefficients c (lowest degree first)."""
    return np.polynomial.polynomial.polyval(x, c) / np.exp2(x) - 1.0


def _local_extremum(c: np.ndarray, a: float, b: float, sign: float) -> float:
    """Golden-section search for the extremum of sign * error on [a, b]."""
    g = (np.sqrt(5.0) - 1.0) / 2.0
    x1, x2 = b - g * (b - a), a + g * (b - a)
    f = lambda t: -sign * _weighted_error(c, np.array([t]))[0]  # noqa: E731
    f1, f2 = f(x1), f(x2)
    for _ in range(200):
        if f1 < f2:
            b, x2, f2 = x2, x1, f1
            x1 = b - g * (b - a)
            f1 = f(x1)
        else:
            a, x1, f1 = x1, x2, f2
            x2 = a + g * (b - a)
            f2 = f(x2)
    return 0.5 * (a + b)


def remez_exp2(degree: int = DEGREE, lo: float = LO, hi: float = HI, iters: int = 30):
    """Return (coefficients lowest degree first, levelled relative error)."""
    n = degree + 2
    k = np.arange(n)
    ref = 0.5 * (lo + hi) - 0.5 * (hi - lo) * np.cos(np.pi * k / (n - 1))
    c = np.zeros(degree + 1)
    err = 0.0
    for _ in range(iters):
        a = np.zeros((n, n))
        for i, x in enumerate(ref):
            a[i, : degree + 1] = x ** np.arange(degree + 1)
            a[i, degree + 1] = -((-1.0) ** i) * np.exp2(x)
        sol = np.linalg.solve(a, np.exp2(ref))
        c, err = sol[: degree + 1], sol[degree + 1]
        grid = np.linspace(lo, hi, 20001)
        e = _weighted_error(c, grid)
        new = [lo]
        for i in range(1, n - 1):   # interior extrema, alternating in sign
            left, right = 0.5 * (ref[i - 1] + ref[i]), 0.5 * (ref[i] + ref[i + 1])
            sign = np.sign(e[np.argmin(np.abs(grid - ref[i]))]) or 1.0
            new.append(_local_extremum(c, left, right, sign))
        new.append(hi)
        ref = np.array(new)
    return c, abs(err)


def float32_coefficients() -> list[float]:
    """The fitted coefficients rounded to float32, highest degree first."""
    c, _ = remez_exp2()
    return [float(np.float32(v)) for v in c[::-1]]


if __name__ == "__main__":
    c, err = remez_exp2()
    print("levelled relative error", err)
    print(", ".join(f"{v:.8g}" for v in float32_coefficients()))
