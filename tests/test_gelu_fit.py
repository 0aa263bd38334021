"""The kernels' GELU (csrc/sm100.cuh) against the erf definition.

The device code evaluates the tail mass h = 1 - Phi(|x|) as one power of two,
h = 2^(KE x^2 + Q(u)), with Q(a) = log2(0.5 erfcx(a / sqrt 2)) a degree-7
polynomial in u = min(|x|, A) * (2 / A) - 1 fitted by weighted minimax
(csrc/fit_gelu.py); this checks that the constants compiled into the kernels
are the fitted ones and that the fp32 evaluation order the kernels use stays
within the stated bounds of the exact normal CDF (scipy.special.ndtr) and of
erf-GELU."""

import importlib.util
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "ethos_b200", "csrc")


def _fit_module():
    spec = importlib.util.spec_from_file_location("fit_gelu", os.path.join(CSRC, "fit_gelu.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _header_constants():
    text = open(os.path.join(CSRC, "sm100.cuh")).read()
    found = dict(re.findall(r"\bQ(\d) = ([-+0-9.e]+)f", text))
    q = np.array([float(found[str(k)]) for k in range(len(found))], dtype=np.float32)
    named = {k: float(re.search(r"\b%s = ([-+0-9.e]+)f" % k, text).group(1)) for k in ("kA", "kU", "kE", "kPdf2")}
    return q, named


def test_header_constants_are_the_fit():
    pytest.importorskip("scipy")
    fit = _fit_module()
    q, named = _header_constants()
    assert len(q) == fit.DEGREE + 1
    # the least-squares iterations may differ in their last bits between
    # LAPACK builds; the committed fp32 values must agree to within an ulp
    np.testing.assert_allclose(q, np.asarray(fit.fit(), dtype=np.float32), rtol=3e-7, atol=1e-9)
    assert np.float32(named["kA"]) == np.float32(fit.A)
    assert np.float32(named["kU"]) == np.float32(2.0 / fit.A)
    assert np.float32(named["kE"]) == np.float32(fit.KE)
    assert np.float32(named["kPdf2"]) == np.float32(fit.LOG2_PDF0)


def test_gelu_error_bounds():
    scipy_special = pytest.importorskip("scipy.special")
    fit = _fit_module()
    q, _ = _header_constants()
    xs = np.linspace(-12, 12, 1_200_001).astype(np.float32)
    xd = xs.astype(np.float64)
    phi = fit.phi_fp32(xs, q)
    ref = scipy_special.ndtr(xd)
    assert np.abs(phi - ref).max() <= 2.5e-7
    gelu_ref = 0.5 * xd * (1 + scipy_special.erf(xd / np.sqrt(2)))
    # the form the kernels assemble, max(x, 0) - |x| h, rounded to fp32: the
    # fit's error plus the rounding of a result of that magnitude
    err = np.abs(fit.gelu_fp32(xs, q) - gelu_ref) - 2.0 ** -23 * np.abs(gelu_ref)
    assert err.max() <= 1e-7
    # derivative Phi + x phi, as the backward tables compute it
    pdf = np.exp(-0.5 * xd ** 2) / np.sqrt(2 * np.pi)
    assert np.abs((phi + xd * pdf) - (ref + xd * pdf)).max() <= 2.5e-7
    # the clamp: beyond |x| = A the tail keeps the exact Gaussian factor
    big = np.linspace(fit.A, 40.0, 100_001).astype(np.float32)
    hb = fit.tail_fp32(big, q).astype(np.float64)
    true = scipy_special.ndtr(-big.astype(np.float64))
    assert (np.abs(hb - true) * (big + 1.0)).max() <= 1e-8
