#!/usr/bin/env python3
"""Coefficients of the FMA-pipe 2^x used by the attention softmax (sdpa.cu, EXP2_C*).

Method (both published and standard):
* Cody-Waite style range reduction for base 2: x = j + f with j = round-to-nearest(x)
  (the 1.5 * 2^23 "magic number" addition) and f = x - j in [-1/2, 1/2]; 2^x = 2^j * 2^f,
  the 2^j factor added to the exponent field.
* 2^f on [-1/2, 1/2] by a degree-N polynomial whose coefficients minimise the maximum
  RELATIVE error, found with the Remez exchange algorithm (E. Remez, 1934): solve for the
  coefficients and the levelled error on N + 2 reference points, move the points to the
  extrema of the new error function, repeat until the extrema are level.

Run:  python gen_exp2_poly.py [degree]   -> prints the coefficients (float32, hex and
decimal) and the float32-evaluated maximum relative error on a dense grid.
"""
from __future__ import annotations

import sys

import numpy as np


def remez_exp2(degree: int, iters: int = 60) -> np.ndarray:
    """Minimax-relative coefficients c[0..degree] of 2^f on [-1/2, 1/2] (float64)."""
    a, b = -0.5, 0.5
    n = degree + 2
    # Chebyshev extrema as the initial reference
    pts = 0.5 * (a + b) + 0.5 * (b - a) * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    grid = np.linspace(a, b, 200001)
    f_grid = np.exp2(grid)
    c = None
    for _ in range(iters):
        # c0 + c1 p + ... + cd p^d + (-1)^i E 2^p = 2^p   (relative error levelled at E)
        A = np.zeros((n, n))
        for i, p in enumerate(pts):
            A[i, :degree + 1] = p ** np.arange(degree + 1)
            A[i, degree + 1] = (-1) ** i * np.exp2(p)
        sol = np.linalg.solve(A, np.exp2(pts))
        c = sol[:degree + 1]
        err = (np.polyval(c[::-1], grid) - f_grid) / f_grid
        # new reference: the extrema of err between its sign changes
        idx = np.where(np.diff(np.sign(err)) != 0)[0]
        bounds = np.concatenate([[0], idx + 1, [len(grid)]])
        ext = [s + np.argmax(np.abs(err[s:e])) for s, e in zip(bounds[:-1], bounds[1:]) if e > s]
        if len(ext) < n:
            break
        # keep n alternating extrema with the largest magnitudes
        while len(ext) > n:
            k = int(np.argmin([abs(err[e]) for e in ext]))
            ext.pop(k)
        new = grid[np.array(ext)]
        if np.allclose(new, pts, atol=1e-12, rtol=0):
            break
        pts = new
    return c


def eval_f32(c32: np.ndarray, f: np.ndarray) -> np.ndarray:
    """Horner in float32 with fused multiply-adds (each step rounded once, as fmaf)."""
    r = np.full(f.shape, c32[-1], np.float32)
    for ck in c32[-2::-1]:
        r = (r.astype(np.float64) * f.astype(np.float64) + np.float64(ck)).astype(np.float32)
    return r


def main() -> int:
    degree = int(sys.argv[1]) if len(sys.argv) > 1 else 5
    c = remez_exp2(degree)
    c32 = c.astype(np.float32)
    f = np.linspace(-0.5, 0.5, 1 << 21).astype(np.float32)
    rel = np.abs(eval_f32(c32, f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)
    for k, v in enumerate(c32):
        print(f"EXP2_C{k} = {float(v).hex()}  ({float(v):.9g})")
    print(f"max relative error, float32 Horner on [-1/2, 1/2]: {rel.max():.3e} (2^{np.log2(rel.max()):.2f})")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
