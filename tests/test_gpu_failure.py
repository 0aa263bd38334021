"""Failure detection without a GPU fault: a bounded wait that runs out.

Every mbarrier wait in the kernels gives up after the wait limit, records
ETHOS_ERR_TIMEOUT_BASE + site in the device error word, drains the CTA's
in-flight copies and MMAs, frees its tensor memory and exits.  Here the limit
is shortened to 1 ms and a GEMM is launched with one work unit's operand loads
withheld (ethos_test_gemm_withhold), so the MMA issuer's wait for them runs
out.  The call must report the timeout through the error word, the other
output tiles must still be right, and the same context must then run a normal
GEMM correctly.  Nothing traps, faults or hangs: the withheld loads are simply
never issued, and every wait involved ends by the time limit."""

import ctypes

import pytest
import torch

from ethos_b200 import _lib, ops
from helpers import rel_err

pytestmark = pytest.mark.gpu

M, N, K = 256, 256, 256  # 2 x 2 output tiles of 128 x 128: units 0..3, one CTA each


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def test_withheld_stage_times_out_and_context_survives():
    L = _lib.lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    ref = a.double() @ b.double().t()
    d = torch.full((M, N), float("nan"), device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.ethos_set_wait_limit_ns(1_000_000) == 0  # 1 ms
    try:
        st = L.ethos_test_gemm_withhold(_vp(a), _vp(b), _vp(d), M, N, K, 0, _vp(err), stream)
        assert st == 0, _lib.STATUS.get(st, st)
        torch.cuda.synchronize()  # the context is intact: no sticky error
    finally:
        assert L.ethos_set_wait_limit_ns(0) == 0  # back to the 2 s default
    code = int(err[0].item())
    assert _lib.ETHOS_ERR_TIMEOUT_BASE < code < _lib.ETHOS_ERR_TIMEOUT_BASE + 100, code
    # unit 0 is the top-left tile; the three others were computed normally
    assert rel_err(d[:128, 128:], ref[:128, 128:]) <= 1e-5
    assert rel_err(d[128:, :], ref[128:, :]) <= 1e-5

    # the same device keeps working: a normal GEMM through the public op
    dd = ops.gemm_bf16(a, b)
    torch.cuda.synchronize()
    ops.check_device_error("cuda")
    assert rel_err(dd, ref) <= 1e-5
    # and a withhold-free launch of the test entry point is complete as well
    d2 = torch.empty((M, N), device="cuda")
    err.zero_()
    assert L.ethos_test_gemm_withhold(_vp(a), _vp(b), _vp(d2), M, N, K, 1 << 20, _vp(err), stream) == 0
    torch.cuda.synchronize()
    assert int(err[0].item()) == 0
    assert rel_err(d2, ref) <= 1e-5
