"""The device GELU against the exact erf GELU, on the GPU.

The kernels evaluate GELU(x) = x Phi(x) and its derivative through the tail
mass h = 1 - Phi(|x|) = 2^(KE x^2 + Q(u)), Q a fitted degree-7 polynomial,
with the hardware's approximate exp2 (ethos_b200/csrc/sm100.cuh,
csrc/fit_gelu.py).  Here every
variant the kernels use runs through ethos_test_gelu on 2^21 points spread
over [-12, 12] plus a dense grid around 0, and is compared with a float64
reference (torch's erfc in double) and, for scale, with torch's own fp32 CUDA
F.gelu on the same points.

Bound asserted (absolute, per point): |GELU error| <= 2.5e-7 + 2^-23 |GELU(x)|
and |GELU' error| <= 5e-7 + 2^-23 |GELU'(x)| -- the fitted form's error plus
the fp32 rounding of a result of that magnitude."""

import ctypes
import math

import pytest
import torch

from ethos_b200 import _lib

pytestmark = pytest.mark.gpu


def _points():
    g = torch.Generator().manual_seed(0)
    grid = torch.linspace(-12.0, 12.0, 1 << 20, dtype=torch.float64)
    near0 = torch.linspace(-1.0, 1.0, 1 << 19, dtype=torch.float64)
    rnd = (torch.rand(1 << 19, generator=g, dtype=torch.float64) * 24.0 - 12.0)
    return torch.cat([grid, near0, rnd]).to(torch.float32)


def _reference(x):
    xd = x.double()
    phi_cdf = 0.5 * torch.erfc(-xd / math.sqrt(2.0))
    pdf = torch.exp(-0.5 * xd * xd) / math.sqrt(2.0 * math.pi)
    return xd * phi_cdf, phi_cdf + xd * pdf


def test_device_gelu_and_derivative_match_erf_gelu():
    L = _lib.lib()
    x = _points()
    n = x.numel()
    xg = x.cuda()
    out = torch.empty((5, n), dtype=torch.float32, device="cuda")
    st = L.ethos_test_gelu(ctypes.c_void_p(xg.data_ptr()), ctypes.c_void_p(out.data_ptr()), n,
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, st
    torch.cuda.synchronize()
    out = out.cpu().double()
    g_ref, d_ref = _reference(x)
    ulp = 2.0 ** -23
    report = {}
    for row, name in ((0, "gelu scalar"), (1, "gelu pair"), (2, "gelu (with grad)")):
        err = (out[row] - g_ref).abs()
        report[name] = err.max().item()
        assert (err <= 2.5e-7 + ulp * g_ref.abs()).all(), (name, err.max().item())
    for row, name in ((3, "grad (with gelu)"), (4, "grad scalar")):
        err = (out[row] - d_ref).abs()
        report[name] = err.max().item()
        assert (err <= 5e-7 + ulp * d_ref.abs()).all(), (name, err.max().item())
    # the paired forms share one evaluation, and the scalar form performs the
    # same fp32 operations one value at a time
    assert torch.equal(out[1], out[2])
    assert torch.equal(out[0], out[1])
    assert torch.equal(out[3], out[4])
    # torch's fp32 CUDA erf GELU on the same points, for scale
    torch_err = (torch.nn.functional.gelu(xg).cpu().double() - g_ref).abs().max().item()
    report["torch fp32 F.gelu"] = torch_err
    print(f"max |error| {report}")
    import json
    import os
    path = os.environ.get("ETHOS_TEST_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(dict(test="device_gelu_max_abs_error", **report)) + "\n")
