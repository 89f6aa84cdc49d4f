"""Fits the polynomial that prefill.cu uses to evaluate 2^x on the FMA pipe.

Method (Cody-Waite range reduction plus a minimax polynomial, fitted here from first
principles):
  2^x = 2^n * 2^f   with n = rint(x) and f = x - n in [-1/2, 1/2];
  2^n is applied by adding n to the IEEE-754 exponent field;
  2^f ~= c0 + c1 f + c2 f^2 + c3 f^3, the polynomial of degree 3 that minimises the maximum
  RELATIVE error on [-1/2, 1/2], computed with the Remez exchange algorithm below.

The coefficients are rounded to fp32 and the final error is measured in fp32 Horner arithmetic
(the kernel evaluates the same expression with fma.rn.f32x2), so the printed bound is the one the
kernel achieves. P is then rounded to bf16 (relative step 2^-8), far coarser than this error.

    python flash-attention-lab_b200/csrc/fit_exp2_poly.py
"""

from __future__ import annotations

import numpy as np

DEGREE = 3
LO, HI = -0.5, 0.5


def remez(degree: int, iters: int = 50):
    n = degree + 2  # equioscillation points
    # Chebyshev extrema as the initial reference set.
    k = np.arange(n)
    xs = (LO + HI) / 2 + (HI - LO) / 2 * np.cos(np.pi * k / (n - 1))[::-1]
    dense = np.linspace(LO, HI, 200001)
    for _ in range(iters):
        # Solve p(x_i) - 2^x_i = (-1)^i E * 2^x_i for the coefficients and E (relative error).
        a = np.zeros((n, n))
        for j in range(degree + 1):
            a[:, j] = xs ** j
        a[:, -1] = -((-1.0) ** k) * np.exp2(xs)
        sol = np.linalg.solve(a, np.exp2(xs))
        coef = sol[:-1]
        err = np.polyval(coef[::-1], dense) / np.exp2(dense) - 1.0
        # New reference: the extremum of each sign-alternating segment.
        sign = np.sign(err)
        idx = np.flatnonzero(np.diff(sign) != 0)
        bounds = np.concatenate([[0], idx + 1, [len(dense)]])
        ext = [b0 + np.argmax(np.abs(err[b0:b1])) for b0, b1 in zip(bounds[:-1], bounds[1:])]
        if len(ext) != n:
            break
        xs = dense[ext]
    return coef


def fp32_horner_error(c32: np.ndarray) -> float:
    f = np.linspace(LO, HI, 400001).astype(np.float32)
    p = np.full_like(f, c32[-1])
    for c in c32[-2::-1]:
        p = (p * f + c).astype(np.float32)
    exact = np.exp2(f.astype(np.float64))
    return float(np.max(np.abs(p.astype(np.float64) / exact - 1.0)))


def main() -> None:
    coef = remez(DEGREE)
    c32 = coef.astype(np.float32)
    print(f"degree {DEGREE} minimax 2^f on [{LO}, {HI}]")
    for i, c in enumerate(c32):
        print(f"  c{i} = {float(c)!r}f  (hex {c.view(np.uint32):#010x})")
    print(f"max relative error, fp32 Horner: {fp32_horner_error(c32):.3e} "
          f"(bf16 half-ulp is {2.0 ** -9:.3e})")


if __name__ == "__main__":
    main()
