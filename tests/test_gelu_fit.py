"""The kernels' GELU (csrc/sm100.cuh) against the erf definition.

The device code evaluates Phi(x) = 1 - 0.5 exp(-x^2/2) erfcx(|x|/sqrt 2)
(mirrored for x < 0) with a degree-11 polynomial for erfcx; this checks that
the constants compiled into the kernels are the fitted ones and that the
fp32 evaluation order the kernels use stays within the stated bounds of the
exact normal CDF (scipy.special.ndtr) and of erf-GELU."""

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


def _header_coefficients():
    text = open(os.path.join(CSRC, "sm100.cuh")).read()
    found = dict(re.findall(r"\bC(\d+) = ([-+0-9.e]+)f", text))
    return np.array([float(found[str(k)]) for k in range(len(found))], dtype=np.float32)


def test_header_constants_are_the_fit():
    pytest.importorskip("scipy")
    fit = _fit_module()
    c = np.asarray(fit.fit(), dtype=np.float32)
    np.testing.assert_array_equal(_header_coefficients(), c)


def test_gelu_error_bounds():
    scipy_special = pytest.importorskip("scipy.special")
    fit = _fit_module()
    c = _header_coefficients()
    xs = np.linspace(-12, 12, 1_200_001)
    phi = fit.phi_fp32(xs, c)
    ref = scipy_special.ndtr(xs)
    assert np.abs(phi - ref).max() <= 2e-6
    gelu = xs * phi
    gelu_ref = 0.5 * xs * (1 + scipy_special.erf(xs / np.sqrt(2)))
    assert np.abs(gelu - gelu_ref).max() <= 1.5e-6
    # the form the kernels assemble: max(x, 0) - |x| h with h = 1 - Phi(|x|)
    h = np.where(xs >= 0, 1 - phi, phi)
    assert np.abs(np.maximum(xs, 0) - np.abs(xs) * h - gelu_ref).max() <= 1.5e-6
    # derivative Phi + x phi, as the backward tables compute it
    d = phi + xs * np.exp(-0.5 * xs ** 2) / np.sqrt(2 * np.pi)
    d_ref = ref + xs * np.exp(-0.5 * xs ** 2) / np.sqrt(2 * np.pi)
    assert np.abs(d - d_ref).max() <= 2e-6
