"""Derive the minimax polynomial behind the FMA-pipe exp2 in kvbm_tc.cu.

The tensor-core kernels evaluate 2^x for part of their score elements on the
FMA pipe instead of the MUFU unit (Cody-Waite style range reduction with an
exact integer split, as in textbook exp implementations):

    j = rint(x)   (x + 1.5*2^23 rounds to the nearest integer),  f = x - j in [-1/2, 1/2]
    2^x = 2^j * p(f),   p(f) ~= 2^f

2^j is applied by adding j to the IEEE-754 exponent field of p(f).  The
n + 1 coefficients of p minimise the maximum RELATIVE error
max |p(f) / 2^f - 1| on [-1/2, 1/2]; they are found with the Remez exchange
algorithm (equioscillation of the weighted error at n + 2 points).  The
kernels clamp x at -126.75, so every result below 2^-126 comes out as a
positive denormal, never a wrapped exponent, and their flush-to-zero
accumulation adds it as an exact 0.

    python kv-block-mass_b200/csrc/gen_exp2_poly.py [--degree 4]

prints the float32 coefficients (lowest order first) and the maximum relative
error of their float32 Horner evaluation on a dense grid.
"""

from __future__ import annotations

import argparse

import numpy as np

LO, HI = -0.5, 0.5


def remez_exp2(n: int, iters: int = 60, grid: int = 400001):
    """c0..cn minimising max |sum_k c_k f^k / 2^f - 1| on [LO, HI]."""
    xs = np.linspace(LO, HI, grid)
    k = np.arange(n + 2)
    ref = (LO + HI) / 2 - (HI - LO) / 2 * np.cos(np.pi * k / (n + 1))  # Chebyshev extrema
    c = None
    for _ in range(iters):
        # sum_j c_j x_i^j - 2^{x_i} = (-1)^i E 2^{x_i}, i = 0..n+1
        A = np.zeros((n + 2, n + 2))
        for i, x in enumerate(ref):
            A[i, : n + 1] = x ** np.arange(n + 1)
            A[i, n + 1] = -((-1) ** i) * 2.0 ** x
        sol = np.linalg.solve(A, 2.0 ** ref)
        c = sol[: n + 1]
        err = (np.polyval(c[::-1], xs) - 2.0 ** xs) / 2.0 ** xs
        sign = np.sign(err)
        sign[sign == 0] = 1
        runs = np.flatnonzero(np.diff(sign)) + 1
        bounds = np.concatenate(([0], runs, [len(xs)]))
        ext = [lo + int(np.argmax(np.abs(err[lo:hi]))) for lo, hi in zip(bounds[:-1], bounds[1:])]
        while len(ext) > n + 2:
            ext = ext[1:] if abs(err[ext[0]]) < abs(err[ext[-1]]) else ext[:-1]
        if len(ext) < n + 2:
            break
        new_ref = xs[ext]
        if np.allclose(new_ref, ref, atol=1e-13):
            break
        ref = new_ref
    return c


def horner_f32(c32, f):
    p = np.full_like(f, c32[-1], dtype=np.float32)
    for cj in c32[-2::-1]:
        p = (p.astype(np.float64) * f.astype(np.float64) + np.float64(cj)).astype(np.float32)
    return p


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--degree", type=int, default=4)
    n = ap.parse_args().degree
    c = remez_exp2(n)
    c32 = c.astype(np.float32)
    f = np.linspace(LO, HI, 1_000_001, dtype=np.float32)
    rel = np.abs(horner_f32(c32, f).astype(np.float64) / 2.0 ** f.astype(np.float64) - 1.0)
    print(f"degree {n} on [{LO}, {HI}]: max relative error (float32 Horner) {rel.max():.3e}")
    for j, cj in enumerate(c32):
        print(f"  c{j} = {float(cj)!r:>24}f  // {np.float32(cj).view(np.uint32):#010x}")


if __name__ == "__main__":
    main()
