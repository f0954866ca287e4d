"""Fit the polynomial behind the kernel's FMA-pipe exp2.

Method (Cody-Waite style range reduction with a minimax core):
  2^x = 2^n * 2^f,  n = round(x),  f = x - n in [-1/2, 1/2]
  2^f ~= p(f) = c0 + c1 f + c2 f^2 + c3 f^3
The coefficients minimise the maximum *relative* error of p(f) against 2^f
on [-1/2, 1/2], found with the Remez exchange algorithm below (equioscillation
on degree+2 points, linear solve, exchange of extrema, repeated until the
levelled error stops moving).  The kernel then inserts n into the exponent
field with an integer add.

Run:  python fa_b200/csrc/fit_exp2_poly.py   (prints C constants + error)
The constants are written into fa_kernel.cuh by hand; tests/test_exp2_poly.py
checks them against this fit and against the error bound.
"""

from __future__ import annotations

import numpy as np

DEGREE = 3
LO, HI = -0.5, 0.5


def _solve(points: np.ndarray) -> tuple[np.ndarray, float]:
    """p(x_i) - 2^x_i = (-1)^i E 2^x_i on the reference points (relative error E)."""
    m = len(points)
    A = np.zeros((m, DEGREE + 2))
    for j in range(DEGREE + 1):
        A[:, j] = points ** j
    t = 2.0 ** points
    A[:, DEGREE + 1] = -((-1.0) ** np.arange(m)) * t
    sol = np.linalg.solve(A, t)
    return sol[: DEGREE + 1], float(sol[DEGREE + 1])


def rel_error(coef: np.ndarray, x: np.ndarray) -> np.ndarray:
    return np.polyval(coef[::-1], x) / 2.0 ** x - 1.0


def remez(iterations: int = 50) -> tuple[np.ndarray, float]:
    n = DEGREE + 2
    k = np.arange(n)
    points = 0.5 * (LO + HI) + 0.5 * (HI - LO) * np.cos(np.pi * (n - 1 - k) / (n - 1))  # Chebyshev
    grid = np.linspace(LO, HI, 200001)
    coef, level = _solve(points)
    for _ in range(iterations):
        coef, level = _solve(points)
        err = rel_error(coef, grid)
        # Extrema: endpoints plus interior sign-change segment maxima.
        sign = np.sign(err)
        cuts = np.flatnonzero(np.diff(sign) != 0) + 1
        segs = np.split(np.arange(len(grid)), cuts)
        ext = [seg[np.argmax(np.abs(err[seg]))] for seg in segs if len(seg)]
        if len(ext) < n:
            break
        # Keep the n largest alternating extrema.
        while len(ext) > n:
            vals = np.abs(err[ext])
            drop = 0 if vals[0] < vals[-1] else len(ext) - 1
            ext.pop(drop)
        new_points = grid[ext]
        if np.allclose(new_points, points, atol=1e-12):
            break
        points = new_points
    return coef, float(np.max(np.abs(rel_error(coef, grid))))


def main():
    coef, err = remez()
    c32 = coef.astype(np.float32)
    err32 = float(np.max(np.abs(rel_error(c32.astype(np.float64), np.linspace(LO, HI, 200001)))))
    print(f"degree {DEGREE} minimax relative error on [{LO}, {HI}]: {err:.3e} (float32 coefficients {err32:.3e})")
    for i, c in enumerate(c32):
        print(f"constexpr float kExp2C{i} = {float(c)!r}f;  // {np.float32(c).view(np.uint32):#010x}")
    return coef


if __name__ == "__main__":
    main()
