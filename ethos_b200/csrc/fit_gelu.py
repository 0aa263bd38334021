"""Coefficients of the GELU used by the CUDA kernels (csrc/sm100.cuh).

GELU(x) = x * Phi(x) with the normal CDF written through the scaled
complementary error function erfcx(z) = exp(z^2) erfc(z):

    Phi(x) = 1 - 0.5 * exp(-z^2) * erfcx(z)   (x >= 0, z = x / sqrt(2))
    Phi(x) = 0.5 * exp(-z^2) * erfcx(z)       (x <  0, z = |x| / sqrt(2))

erfcx is smooth and bounded on [0, Z] (from 1 down to 0.137 at Z = 4.2), so
a least-squares polynomial in s = z / Z fits it closely; for z > Z the
factor exp(-z^2) < 2e-8 makes the clamped value irrelevant.  The kernels
evaluate the polynomial by Horner's rule in fp32 and exp(-z^2) with one
ex2.  Run this file to regenerate the constants and print the fp32 error
bounds; the values below are the committed ones.
"""

import numpy as np

Z = 4.2
DEGREE = 11


def fit(degree=DEGREE, z_max=Z, nodes=4000):
    from scipy.special import erfcx
    s = (1 - np.cos(np.linspace(0, np.pi, nodes))) / 2  # Chebyshev nodes on [0, 1]
    v = np.vander(s, degree + 1, increasing=True)
    c, *_ = np.linalg.lstsq(v, erfcx(s * z_max), rcond=None)
    return c


def phi_fp32(x, c, z_max=Z):
    """Phi(x) as the kernels compute it (fp32 Horner, exact exp)."""
    x = np.asarray(x, dtype=np.float32)
    c32 = np.asarray(c, dtype=np.float32)
    s = np.minimum(np.abs(x) * np.float32(1 / (np.sqrt(2) * z_max)), np.float32(1))
    p = np.full_like(s, c32[-1])
    for k in range(len(c32) - 2, -1, -1):
        p = (p * s + c32[k]).astype(np.float32)
    h = 0.5 * np.exp(-0.5 * x.astype(np.float64) ** 2) * p
    return np.where(x >= 0, 1 - h, h)


if __name__ == "__main__":
    from scipy.special import ndtr
    c = fit()
    xs = np.linspace(-12, 12, 2_000_001)
    err = np.abs(phi_fp32(xs, c) - ndtr(xs))
    print("max |Phi error| = %.2e" % err.max())
    print("max |GELU error| = %.2e" % (np.abs(xs) * err).max())
    for k, v in enumerate(np.asarray(c, dtype=np.float32)):
        print("  C%d = %.9ef" % (k, v))
