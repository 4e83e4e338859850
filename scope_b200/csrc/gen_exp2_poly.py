"""Generates the polynomial of the FMA-pipe exp2 in ``tc_ptx.cuh`` (``ex2_fma2``).

Method: Cody-Waite style range reduction for base 2, which is exact in
binary floating point (x = n + f, n = round(x), f in [-1/2, 1/2], since the
subtraction x - n is exact for |x| < 2^22), followed by a polynomial p(f) ~
2^f whose coefficients minimise the maximum RELATIVE error over [-1/2, 1/2]
(a minimax fit, computed here by the Remez exchange algorithm).  2^x is
then p(f) with n added to its exponent field.

The fit is carried out in float64; the printed coefficients are rounded to
float32, and the relative error of the whole float32 evaluation (Horner in
fma, as the kernel does it) is re-measured over a dense grid.

Run:  python scope_b200/csrc/gen_exp2_poly.py [degree]
"""
from __future__ import annotations

import sys

import numpy as np


def remez_rel(degree: int, a: float = -0.5, b: float = 0.5, iters: int = 60):
    """Minimax polynomial c[0] + c[1] f + ... for 2^f on [a, b], relative error."""
    n = degree + 2                                     # reference points: degree + 2
    k = np.arange(n)
    x = (a + b) / 2 + (b - a) / 2 * np.cos(np.pi * (n - 1 - k) / (n - 1))   # Chebyshev extrema
    grid = np.linspace(a, b, 200001)
    c = None
    for _ in range(iters):
        # solve sum c_j x_i^j - 2^x_i = (-1)^i E 2^x_i  (equioscillating relative error)
        f = np.exp2(x)
        A = np.zeros((n, n))
        for j in range(degree + 1):
            A[:, j] = x ** j
        A[:, degree + 1] = -((-1.0) ** k) * f
        sol = np.linalg.solve(A, f)
        c = sol[: degree + 1]
        err = (np.polyval(c[::-1], grid) - np.exp2(grid)) / np.exp2(grid)
        # new reference: the extrema of the error between its sign changes
        s = np.sign(err)
        idx = np.concatenate(([0], np.nonzero(np.diff(s))[0] + 1, [len(grid)]))
        if len(idx) - 1 != n:
            break
        x = np.array([grid[lo + np.argmax(np.abs(err[lo:hi]))] for lo, hi in zip(idx[:-1], idx[1:])])
    return c


def eval_f32(c32, xs):
    """The kernel's float32 evaluation: n = round(x), f = x - n, Horner in fma, exponent add."""
    xs = xs.astype(np.float32)
    magic = np.float32(12582912.0)                     # 1.5 * 2^23: x + magic rounds x to an integer
    t = (xs + magic).astype(np.float32)
    r = (t - magic).astype(np.float32)
    f = (xs - r).astype(np.float32)
    p = np.full_like(f, c32[-1])
    for cj in c32[-2::-1]:
        p = (p.astype(np.float64) * f + cj).astype(np.float32)   # fma: one rounding
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.view(np.float32)


def main():
    degree = int(sys.argv[1]) if len(sys.argv) > 1 else 3
    c = remez_rel(degree)
    c32 = c.astype(np.float32)
    xs = np.linspace(-125.0, 8.0, 4_000_001, dtype=np.float64).astype(np.float32)
    got = eval_f32(c32, xs).astype(np.float64)
    ref = np.exp2(xs.astype(np.float64))
    rel = np.abs(got - ref) / ref
    print(f"degree {degree}: max relative error of the float32 evaluation on [-125, 8]: {rel.max():.3e}")
    for j, v in enumerate(c32):
        print(f"  c{j} = {float(v)!r:>24}   # bits 0x{np.float32(v).view(np.uint32):08x}")


if __name__ == "__main__":
    main()
