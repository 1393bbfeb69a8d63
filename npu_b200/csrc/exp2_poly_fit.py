"""Fit the polynomials the prefill softmax uses to evaluate 2^f, f in [-1/2, 1/2],
on the FMA pipe (exp2_fma2 in softmax.cuh): degree 3 and degree 2.

Method: relative-error minimax by iteratively reweighted least squares
(Lawson's algorithm) on a dense grid, weights 1 / 2^f. The results are printed as
C float literals with their max relative error in fp32 Horner form (cubic
7.5e-5, quadratic 1.7e-3; the bf16 P tile itself is rounded to 2^-9).

    python npu_b200/csrc/exp2_poly_fit.py
"""
import numpy as np


def fit(degree: int = 3, n: int = 20001, iters: int = 200):
    f = np.linspace(-0.5, 0.5, n)
    y = np.exp2(f)
    A = np.vander(f, degree + 1, increasing=True)
    w = np.ones(n)
    for _ in range(iters):
        sw = np.sqrt(w) / y
        c, *_ = np.linalg.lstsq(A * sw[:, None], y * sw, rcond=None)
        err = np.abs(A @ c - y) / y
        w = w * err
        w /= w.sum()
    return c, err.max()


if __name__ == "__main__":
    for degree in (2, 3):
        c, _ = fit(degree)
        c32 = c.astype(np.float32)
        f = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
        p = np.zeros_like(f)
        for cc in c32[::-1]:
            p = p * f + cc
        err = float(np.max(np.abs(p / np.exp2(f.astype(np.float64)) - 1)))
        print(f"degree {degree}: c0..c{degree} =", ", ".join(f"{x:.9e}f" for x in c32), f"max rel. error {err:.3e}")
