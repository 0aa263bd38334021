"""The kernels' GELU (csrc/sm100.cuh) against the erf definition.

The device code evaluates the tail mass h = 1 - Phi(|x|) =
0.5 exp(-x^2/2) erfcx(|x|/sqrt 2) with erfcx in a refit rational form of
Hastings' approximation (Abramowitz & Stegun 7.1.26), t = 1 / (1 + P z);
this checks that the constants compiled into the kernels are the fitted ones
and that the fp32 evaluation order the kernels use stays within the stated
bounds of the exact normal CDF (scipy.special.ndtr) and of erf-GELU."""

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
    found = dict(re.findall(r"\bC(\d+) = ([-+0-9.e]+)f", text))
    c = np.array([float(found[str(k)]) for k in range(len(found))], dtype=np.float32)
    kp = float(re.search(r"\bkP = ([-+0-9.e]+)f", text).group(1))
    return kp * np.sqrt(2.0), c


def test_header_constants_are_the_fit():
    pytest.importorskip("scipy")
    fit = _fit_module()
    p, c = fit.fit()
    hp, hc = _header_constants()
    np.testing.assert_array_equal(hc, np.asarray(c, dtype=np.float32))
    assert np.float32(hp / np.sqrt(2.0)) == np.float32(p / np.sqrt(2.0))


def test_gelu_error_bounds():
    scipy_special = pytest.importorskip("scipy.special")
    fit = _fit_module()
    p, c = _header_constants()
    xs = np.linspace(-12, 12, 1_200_001)
    phi = fit.phi_fp32(xs, p, c)
    ref = scipy_special.ndtr(xs)
    assert np.abs(phi - ref).max() <= 5e-7
    gelu = xs * phi
    gelu_ref = 0.5 * xs * (1 + scipy_special.erf(xs / np.sqrt(2)))
    assert np.abs(gelu - gelu_ref).max() <= 2.5e-7
    # the form the kernels assemble: max(x, 0) - |x| h with h = 1 - Phi(|x|)
    h = np.where(xs >= 0, 1 - phi, phi)
    assert np.abs(np.maximum(xs, 0) - np.abs(xs) * h - gelu_ref).max() <= 2.5e-7
    # derivative Phi + x phi, as the backward tables compute it
    d = phi + xs * np.exp(-0.5 * xs ** 2) / np.sqrt(2 * np.pi)
    d_ref = ref + xs * np.exp(-0.5 * xs ** 2) / np.sqrt(2 * np.pi)
    assert np.abs(d - d_ref).max() <= 5e-7
