"""Fit the cubic used by the prefill softmax to evaluate 2^f, f in [-1/2, 1/2],
on the FMA pipe (exp2_fma in prefill.cu).

Method: relative-error minimax by iteratively reweighted least squares
(Lawson's algorithm) on a dense grid, weights 1 / 2^f. The result is printed as
C float literals; the cubic's max relative error (~8.8e-5) is far below the
bf16 rounding (2^-9) the P tile gets anyway.

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
    c, e = fit()
    c32 = c.astype(np.float32)
    f = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    p = ((c32[3] * f + c32[2]) * f + c32[1]) * f + c32[0]
    print("coefficients c0..c3:", ", ".join(f"{x:.9e}f" for x in c32))
    print("max relative error (fp32 Horner):", float(np.max(np.abs(p / np.exp2(f.astype(np.float64)) - 1))))
