"""Coefficients of the GELU used by the CUDA kernels (csrc/sm100.cuh).

GELU(x) = x * Phi(x) with the normal CDF written through the tail mass
h(x) = 1 - Phi(|x|) = 0.5 * exp(-x^2 / 2) * erfcx(z),  z = |x| / sqrt(2),

    Phi(x) = 1 - h (x >= 0),   Phi(x) = h (x < 0),
    GELU(x) = max(x, 0) - |x| * h.

erfcx (the scaled complementary error function exp(z^2) erfc(z)) is evaluated
in the rational form of Hastings' approximation to erfc (Abramowitz & Stegun,
Handbook of Mathematical Functions, formula 7.1.26):

    erfcx(z) ~ t * (C0 + C1 t + C2 t^2 + C3 t^3 + C4 t^4),   t = 1 / (1 + P z),

with P and C0..C4 refit here for the kernels' use: they minimise
(|x| + 1) * |delta h| on [0, 12], which bounds both the GELU error
|x| * |delta h| and the Phi error |delta h| (weighted least squares for the
C_k on a fine grid, P by a bounded scalar search).  The form holds for every z >= 0
(t -> 0 as z grows), so no clamp is needed.  The kernels compute t with one
rcp.approx and exp(-x^2 / 2) with one ex2.approx, and the polynomial by
Horner's rule on packed fp32 pairs.  Run this file to regenerate the
constants and print the fp32 error bounds; the values in sm100.cuh are the
committed ones.
"""

import numpy as np

NCOEF = 5
X_MAX = 12.0
GRID = 200_001


def _fit_coefficients(p, xs):
    from scipy.special import erfcx
    z = xs / np.sqrt(2.0)
    t = 1.0 / (1.0 + p * z)
    # d GELU = |x| * 0.5 exp(-x^2/2) * d erfcx and d Phi = 0.5 exp(-x^2/2) * d erfcx:
    # weighting by (|x| + 1) bounds both
    w = 0.5 * (xs + 1.0) * np.exp(-0.5 * xs ** 2)
    v = np.stack([t ** (k + 1) for k in range(NCOEF)], 1)
    c, *_ = np.linalg.lstsq(v * w[:, None], erfcx(z) * w, rcond=None)
    return c, np.abs((v @ c - erfcx(z)) * w).max()


def fit():
    """Returns (P, [C0..C4]) for the rational erfcx form."""
    from scipy.optimize import minimize_scalar
    xs = np.linspace(0.0, X_MAX, GRID)
    r = minimize_scalar(lambda p: _fit_coefficients(p, xs)[1], bounds=(0.1, 2.0), method="bounded")
    c, _ = _fit_coefficients(r.x, xs)
    return float(r.x), c


def tail_fp32(x, p, c):
    """h(x) = 1 - Phi(|x|) as the kernels compute it: fp32 rational form,
    reciprocal and exponential rounded to fp32."""
    x = np.asarray(x, dtype=np.float32)
    c32 = np.asarray(c, dtype=np.float32)
    kp = np.float32(p / np.sqrt(2.0))
    d = (np.abs(x) * kp + np.float32(1)).astype(np.float32)
    t = (np.float32(1) / d).astype(np.float32)
    q = np.full_like(t, c32[-1])
    for k in range(len(c32) - 2, -1, -1):
        q = (q * t + c32[k]).astype(np.float32)
    q = (q * t).astype(np.float32)
    e = (0.5 * np.exp(-0.5 * x.astype(np.float64) ** 2)).astype(np.float32)
    return (e * q).astype(np.float32)


def phi_fp32(x, p, c):
    """Phi(x) from the fp32 tail."""
    x = np.asarray(x, dtype=np.float32)
    h = tail_fp32(x, p, c).astype(np.float64)
    return np.where(x >= 0, 1 - h, h)


if __name__ == "__main__":
    from scipy.special import ndtr
    p, c = fit()
    xs = np.linspace(-12, 12, 2_000_001)
    err = np.abs(phi_fp32(xs, p, c) - ndtr(xs))
    print("max |Phi error| = %.2e" % err.max())
    print("max |GELU error| = %.2e" % (np.abs(xs) * err).max())
    print("  kP = %.9ef  (P / sqrt 2, P = %.9f)" % (np.float32(p / np.sqrt(2.0)), p))
    for k, v in enumerate(np.asarray(c, dtype=np.float32)):
        print("  C%d = %.9ef" % (k, v))
