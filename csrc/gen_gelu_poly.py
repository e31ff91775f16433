"""Coefficients of the division-free normal CDF used by the GELU epilogues
(``norm_cdf_poly`` in csrc/common.cuh).

Phi(x) = sat(1/2 + x * R(t)),  t = min(2 x^2 / c^2 - 1, 1),  c = 4.5,

sat clamping to [0, 1]. R (degree 9 in t) minimises max |x R(t) - (Phi(x) - 1/2)|
over x in [0, c]: a discrete L-infinity fit on 400k points by Lawson's
algorithm (iteratively reweighted least squares whose weights grow with the
local error), under the equality constraint c R(1) = 1/2 + 2e-6, so that for
|x| >= c, where t is held at 1, |x R(1)| exceeds 1/2 and the saturation
returns exactly 0 or 1 (no select needed). The
printed error is measured on the fp32 evaluation the kernel performs, over
x in [-8, 8].
Run: python csrc/gen_gelu_poly.py
"""
import numpy as np
from scipy.special import erf

C, DEG = 4.5, 9


def fit(c=C, deg=DEG, iters=80):
    x = np.linspace(1e-9, c, 400001)
    t = 2 * x * x / (c * c) - 1
    target = 0.5 * erf(x / np.sqrt(2)) / x
    V = np.vander(t, deg + 1, increasing=True)
    # equality constraint c R(1) = 1/2 + 2e-6 (so fp32 saturates beyond c),
    # solved with the weighted least squares through its KKT system
    e = np.ones(deg + 1)
    w = x.copy()
    for _ in range(iters):
        A = V * w[:, None]
        kkt = np.block([[2 * A.T @ A, e[:, None]], [e[None, :], np.zeros((1, 1))]])
        rhs = np.concatenate([2 * A.T @ (target * w), [(0.5 + 2e-6) / c]])
        coef = np.linalg.solve(kkt, rhs)[:-1]
        err = x * (V @ coef - target)
        w = w * (np.abs(err) / np.abs(err).max() + 1e-4) ** 0.7
        w /= w.max()
    return coef.astype(np.float32)


def cdf_f32(a, xs, c=C):
    xs = np.asarray(xs, np.float32)
    t = np.minimum((xs * xs * np.float32(2 / (c * c)) - np.float32(1)).astype(np.float32), np.float32(1))
    r = np.full_like(t, a[-1])
    for k in a[-2::-1]:
        r = (r * t + k).astype(np.float32)
    return np.clip((np.float32(0.5) + xs * r).astype(np.float32), 0, 1)


if __name__ == "__main__":
    a = fit()
    xs = np.linspace(-8, 8, 4000001).astype(np.float32)
    ref = 0.5 + 0.5 * erf(xs.astype(np.float64) / np.sqrt(2))
    print(f"max |Phi_poly - Phi| = {np.abs(cdf_f32(a, xs) - ref).max():.3e}")
    big = np.array([C, 5.0, 50.0, 1e4], np.float32)
    print("tails exact:", (cdf_f32(a, big) == 1).all() and (cdf_f32(a, -big) == 0).all())
    print(f"2 / c^2 = {np.float32(2 / (C * C)):.9g}f")
    for i, k in enumerate(a):
        print(f"  a{i} = {k:.9g}f")
