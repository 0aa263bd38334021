"""Coefficients of the GELU used by the CUDA kernels (csrc/sm100.cuh).

GELU(x) = x * Phi(x) with the normal CDF written through its tail mass
h(a) = 1 - Phi(a) = Phi(-a) for a = |x|:

    Phi(x) = 1 - h (x >= 0),   Phi(x) = h (x < 0),
    GELU(x) = max(x, 0) - |x| * h.

The tail mass is evaluated as one power of two,

    h(a) = 0.5 exp(-a^2 / 2) erfcx(a / sqrt 2) = 2^(KE a^2 + Q(a)),
    KE = -1 / (2 ln 2),   Q(a) = log2(0.5 erfcx(a / sqrt 2)),

where erfcx(z) = exp(z^2) erfc(z) is the scaled complementary error function.
Q is smooth and slowly varying on [0, inf) (from -1 at 0 to about
-log2(a sqrt(2 pi)) in the tail), so a polynomial of low degree in
u = a * (2 / A) - 1 on [0, A] holds it well; for a > A the kernels clamp
a to A, which keeps the Gaussian factor exact and leaves an error below 2e-9
at A = 5.5.  The coefficients minimise the weighted maximum error
(|x| + 1) * |delta h| -- a bound on both the GELU error |x| * |delta h| and
the Phi error |delta h| -- by Lawson's algorithm (iteratively reweighted least
squares converging to the minimax solution; C. L. Lawson, "Contributions to
the theory of linear least maximum approximation", 1961).

The kernels evaluate Q by Horner's rule on packed fp32 pairs, the exponent
KE x^2 + Q with one more FMA and the power of two with one ex2.approx; the
derivative GELU'(x) = Phi(x) + x phi(x) takes the density from a second ex2,
phi(x) = 2^(KE x^2 + log2(1 / sqrt(2 pi))).  Run this file to regenerate the
constants and print the fp32 error bounds; the values in sm100.cuh are the
committed ones.
"""

import numpy as np

DEGREE = 7
A = 5.5
GRID = 200_001
ITERATIONS = 200
KE = -0.5 / np.log(2.0)
LOG2_PDF0 = np.log2(1.0 / np.sqrt(2.0 * np.pi))


def fit():
    """Returns the coefficients Q0..Q7 of Q(u), u = a * (2 / A) - 1, for a in [0, A]."""
    from scipy.special import erfcx, ndtr
    a = np.linspace(0.0, A, GRID)
    u = a * (2.0 / A) - 1.0
    q = np.log2(0.5 * erfcx(a / np.sqrt(2.0)))
    # d h = h ln 2 d Q, weighted by (|x| + 1)
    w = (a + 1.0) * ndtr(-a) * np.log(2.0)
    v = np.vander(u, DEGREE + 1, increasing=True)
    ww = np.ones_like(a)
    for _ in range(ITERATIONS):
        W = w * ww
        c, *_ = np.linalg.lstsq(v * W[:, None], q * W, rcond=None)
        e = np.abs((v @ c - q) * w)
        ww = ww * np.sqrt(e / e.max()) + 1e-14
        ww /= ww.max()
    return c


def _fma32(x, y, z):
    """fp32 fused multiply-add: the exact product and sum, rounded once."""
    return (np.asarray(x, np.float64) * np.asarray(y, np.float64) + np.asarray(z, np.float64)).astype(np.float32)


def tail_fp32(x, c):
    """h(x) = 1 - Phi(|x|) as the kernels compute it: fp32 FMAs in the same
    order, the power of two rounded to fp32."""
    x = np.asarray(x, dtype=np.float32)
    c32 = np.asarray(c, dtype=np.float32)
    a = np.minimum(np.abs(x), np.float32(A))
    u = _fma32(a, np.float32(2.0 / A), np.float32(-1.0))
    q = np.full_like(u, c32[-1])
    for k in range(len(c32) - 2, -1, -1):
        q = _fma32(q, u, c32[k])
    xx = (x.astype(np.float64) * x).astype(np.float32)
    s = _fma32(xx, np.float32(KE), q)
    return np.exp2(s.astype(np.float64)).astype(np.float32)


def phi_fp32(x, c):
    """Phi(x) from the fp32 tail."""
    x = np.asarray(x, dtype=np.float32)
    h = tail_fp32(x, c).astype(np.float64)
    return np.where(x >= 0, 1 - h, h)


def gelu_fp32(x, c):
    """GELU(x) = max(x, 0) - |x| h in the kernels' fp32 order."""
    x = np.asarray(x, dtype=np.float32)
    h = tail_fp32(x, c)
    return _fma32(-np.abs(x), h, np.maximum(x, np.float32(0)))


if __name__ == "__main__":
    from scipy.special import erf, ndtr
    c = fit()
    xs = np.linspace(-12, 12, 2_000_001).astype(np.float32)
    xd = xs.astype(np.float64)
    g_ref = 0.5 * xd * (1 + erf(xd / np.sqrt(2)))
    print("max |Phi error| = %.2e" % np.abs(phi_fp32(xs, c) - ndtr(xd)).max())
    excess = np.abs(gelu_fp32(xs, c) - g_ref) - 2.0 ** -23 * np.abs(g_ref)
    print("max |GELU error| - 2^-23 |GELU| = %.2e" % excess.max())
    print("  kA = %.9ef, kU = %.9ef, kE = %.9ef, kPdf2 = %.9ef"
          % (np.float32(A), np.float32(2.0 / A), np.float32(KE), np.float32(LOG2_PDF0)))
    for k, v in enumerate(np.asarray(c, dtype=np.float32)):
        print("  Q%d = %.9ef" % (k, v))
