"""Fit the cubic that the attention kernel's FMA-pipe exp2 evaluates.

The kernel computes 2^x as 2^n * p(f) with n = round-to-nearest(x) and
f = x - n in [-0.5, 0.5] (Cody-Waite range reduction), so p must approximate
2^f on that interval.  The coefficients below minimise the maximum RELATIVE
error over a dense grid (a linear program: minimise E subject to
|p(f_i) / 2^f_i - 1| <= E), which is the minimax fit up to the grid spacing.
The result is then checked by evaluating Horner's rule in float32, as the
kernel does.  Run: python exp2_poly_fit.py  (prints the constants used in
pkv_attn.cu and the measured error; the bf16 P it feeds has a relative
rounding step of 2^-8, so an error well under 1e-3 is invisible after rounding).
"""
import numpy as np
from scipy.optimize import linprog

DEG = 3


def fit(deg=DEG, n=4001):
    f = np.linspace(-0.5, 0.5, n)
    w = np.exp2(-f)
    V = np.stack([f ** k * w for k in range(deg + 1)], axis=1)  # p(f)/2^f
    # variables: c_0..c_deg, E ; minimise E
    cost = np.zeros(deg + 2)
    cost[-1] = 1.0
    ones = np.ones((n, 1))
    A = np.vstack([np.hstack([V, -ones]), np.hstack([-V, -ones])])
    b = np.concatenate([np.ones(n), -np.ones(n)])
    res = linprog(cost, A_ub=A, b_ub=b, bounds=[(None, None)] * (deg + 2), method="highs")
    return res.x[:-1], res.x[-1]


def horner_f32(c, f):
    c = [np.float32(x) for x in c]
    p = np.full_like(f, c[-1], dtype=np.float32)
    for k in range(len(c) - 2, -1, -1):
        p = (p * f + c[k]).astype(np.float32)
    return p


if __name__ == "__main__":
    c, e = fit()
    f = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    rel = np.abs(horner_f32(c, f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1)
    for k, x in enumerate(c):
        print(f"c{k} = {np.float32(x).item()!r:>24}  ({np.float32(x).view(np.uint32):#010x})")
    print(f"LP max rel error {e:.3e}; float32 Horner max rel error {rel.max():.3e}")
