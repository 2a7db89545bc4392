"""Fit the polynomial the attention kernel uses for part of its exp2 work.

2^x is split as 2^n * 2^f with n = round(x) and f = x - n in [-0.5, 0.5];
2^f is approximated by a cubic c0 + c1 f + c2 f^2 + c3 f^3 fitted here by
iteratively reweighted least squares on the relative error over a dense
grid (converging to the equioscillating, minimax fit — the Remez
criterion).  The kernel multiplies by 2^n by adding n to the exponent bits.

    python repercep_runtime_b200/csrc/gen_exp2_poly.py

prints the coefficients (pasted into attention.cu) and the worst relative
error; e4m3 keeps 3 mantissa bits (relative step 2^-3), the row sum tolerates
far less than the ~1e-4 this fit reaches.
"""

from __future__ import annotations

import numpy as np


def fit(degree: int = 3, iters: int = 60) -> tuple[np.ndarray, float]:
    f = np.linspace(-0.5, 0.5, 20001)
    target = np.exp2(f)
    V = np.vander(f, degree + 1, increasing=True)
    w = np.ones_like(f)
    coef = np.zeros(degree + 1)
    for _ in range(iters):
        A = V / target[:, None] * w[:, None]
        b = np.ones_like(f) * w
        coef, *_ = np.linalg.lstsq(A, b, rcond=None)
        err = np.abs(V @ coef / target - 1.0)
        w = w * (1.0 + err / err.max())
        w /= w.mean()
    err = np.abs(V @ coef / target - 1.0).max()
    return coef, float(err)


if __name__ == "__main__":
    c, e = fit()
    c32 = c.astype(np.float32)
    for i, v in enumerate(c32):
        print(f"c{i} = {float(v)!r}f  // {v.view(np.uint32):#010x}")
    print(f"max relative error {e:.3e}")
