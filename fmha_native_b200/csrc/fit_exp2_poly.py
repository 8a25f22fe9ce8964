"""Fits the polynomial used by exp2_poly2() in sm100_ptx.cuh.

2^x = 2^n * 2^f with n = round(x), f = x - n in [-0.5, 0.5]; 2^f is a
degree-3 polynomial minimising the maximum RELATIVE error on that interval
(Lawson iteratively reweighted least squares on Chebyshev points).  The
printed float32 coefficients are the ones compiled into the kernel; the
float32 Horner evaluation of them has max relative error ~7.5e-5, well below
the bf16 rounding (2^-8) that P undergoes before the P.V product.

Run: python fmha_native_b200/csrc/fit_exp2_poly.py
"""
import numpy as np


def fit(deg: int = 3, iters: int = 200):
    f = np.cos(np.linspace(0, np.pi, 4001)) * 0.5
    y = np.exp2(f)
    w = np.ones_like(f)
    V = np.vander(f, deg + 1, increasing=True)
    for _ in range(iters):
        A = V / y[:, None]
        sw = np.sqrt(w)
        c, *_ = np.linalg.lstsq(A * sw[:, None], sw, rcond=None)
        err = (V @ c - y) / y
        w = w * np.abs(err) + 1e-30
        w /= w.sum()
    c32 = c.astype(np.float32)
    ff = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    p = np.float32(c32[deg])
    for k in range(deg - 1, -1, -1):
        p = (p * ff + c32[k]).astype(np.float32)
    rel = np.abs(p.astype(np.float64) / np.exp2(ff.astype(np.float64)) - 1).max()
    return c32, rel


if __name__ == "__main__":
    c, rel = fit()
    print("coefficients c0..c3:", ", ".join(f"{x:.9e}f" for x in c))
    print(f"max relative error (fp32 Horner): {rel:.3e}")
