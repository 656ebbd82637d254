"""Fit of the cubic used for the FMA-pipe exp2 in the attention kernel.

The kernel computes 2^x = 2^j * 2^f with j = round-to-nearest(x) and
f = x - j in [-0.5, 0.5]; 2^f is a cubic p(f) = 1 + c1 f + c2 f^2 + c3 f^3.
The constant term is pinned to 1 so that x = 0 -- the running row maximum
itself -- is exact. c1..c3 minimise the maximum RELATIVE error over
[-0.5, 0.5]; the minimax problem is solved as a linear program on a dense
grid (minimise t subject to |p(f_i)/2^f_i - 1| <= t). Running this file prints
the coefficients that csrc/attn_fwd_sm100.cuh hard-codes; the CPU tests re-run
the fit and check the constants and the error bound.
"""
from __future__ import annotations

import numpy as np

LO, HI = -0.5, 0.5
# The constants compiled into the kernel (FP32 values of the fit below).
KERNEL_COEFFS = (0.6932829022407532, 0.2422109693288803, 0.055009059607982635)


def rel_error(c, f):
    c1, c2, c3 = c
    p = ((c3 * f + c2) * f + c1) * f + 1.0
    return p / np.exp2(f) - 1.0


def fit(points: int = 4001):
    """Minimax relative-error cubic with p(0) = 1, via a linear program."""
    from scipy.optimize import linprog

    f = np.linspace(LO, HI, points)
    w = np.exp2(-f)  # relative error = w * (1 + c1 f + c2 f^2 + c3 f^3) - 1
    basis = np.stack([w * f, w * f * f, w * f ** 3], axis=1)
    const = w - 1.0
    # variables (c1, c2, c3, t): minimise t, |basis c + const| <= t
    a_ub = np.vstack([np.hstack([basis, -np.ones((points, 1))]), np.hstack([-basis, -np.ones((points, 1))])])
    b_ub = np.concatenate([-const, const])
    res = linprog(c=[0, 0, 0, 1], A_ub=a_ub, b_ub=b_ub, bounds=[(None, None)] * 3 + [(0, None)], method="highs")
    if not res.success:
        raise RuntimeError(res.message)
    coeffs = res.x[:3]
    return coeffs, float(np.abs(rel_error(coeffs, np.linspace(LO, HI, 400001))).max())


def max_rel_error_f32(c) -> float:
    """Max relative error of the FP32 evaluation (Horner, as the kernel does)."""
    f = np.linspace(LO, HI, 2000001, dtype=np.float32)
    c1, c2, c3 = (np.float32(v) for v in c)
    p = ((c3 * f + c2) * f + c1) * f + np.float32(1.0)
    return float(np.abs(p.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0).max())


if __name__ == "__main__":
    coeffs, e = fit()
    print("c1..c3 =", [float(np.float32(v)) for v in coeffs], "max rel err", e,
          "fp32 eval", max_rel_error_f32(coeffs), "kernel constants", max_rel_error_f32(KERNEL_COEFFS))
