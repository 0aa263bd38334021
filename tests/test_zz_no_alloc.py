"""The router entry point that allocates nothing, checked through the C ABI.

Some callers cannot allocate device memory per call -- a serving process that
runs under a memory plan reserved at start-up, or an embedding runtime that
owns no device allocator and only hands over its input and output buffers.
ethos_router_forward_noalloc serves them: its scratch is a static device array
inside the library.  This test drives it directly with ctypes and checks, on
two calls in a row (different inputs, so the shared scratch is reused), that
it reproduces ethos_router_forward exactly, and that an oversized request is
refused before any launch.  It sits in a file of its own that pytest collects
last and passes alone in a fresh process as well as after the other tests.
"""

import ctypes

import pytest
import torch

from ethos_b200 import EthosConfig, EthosExpertLayer, _lib, ops
from ethos_b200.init import seeded_input, seeded_state_dict

pytestmark = pytest.mark.gpu

CFG = dict(d_model=1024, num_experts=512 * 512, top_k=16, num_routing_heads=8, d_latent=128,
           d_intermediate_hypernet=512, d_query=512)


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_router_matches_router_forward_twice():
    layer = EthosExpertLayer(EthosConfig(**CFG))
    layer.load_state_dict(seeded_state_dict(layer, seed=4))
    layer = layer.to("cuda", torch.bfloat16).eval()
    pw = layer._packed(torch.device("cuda"))
    L = _lib.lib()
    err = ops.device_error_word("cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    H, k = CFG["num_routing_heads"], CFG["top_k"]
    for call, (T, seed) in enumerate([(200, 1), (258, 2)]):
        x = seeded_input(T, CFG["d_model"], seed=seed).to("cuda", torch.bfloat16)
        w_ref, ids_ref = ops.router_forward(x, pw, False, 1e-5, 0.1)
        ids = torch.full((T, H, k), -1, dtype=torch.int32, device="cuda")
        w = torch.full((T, H, k), -1.0, dtype=torch.float32, device="cuda")
        dims = ops.make_dims(T, pw.dims)
        st = L.ethos_router_forward_noalloc(ctypes.byref(dims), _vp(x), _vp(pw.w_cat), _vp(pw.bn), 1e-5,
                                            _vp(pw.key_cat), _vp(ids), _vp(w), _vp(err), stream)
        assert st == 0, (call, L.ethos_status_string(st))
        torch.cuda.synchronize()
        ops.check_device_error("cuda")
        assert torch.equal(ids, ids_ref), call
        assert (w - w_ref).abs().max().item() <= 1e-6, call


def test_noalloc_router_rejects_oversized_requests():
    layer = EthosExpertLayer(EthosConfig(**CFG))
    pw = layer.to("cuda", torch.bfloat16).eval()._packed(torch.device("cuda"))
    L = _lib.lib()
    T = 259
    x = torch.zeros((T, CFG["d_model"]), dtype=torch.bfloat16, device="cuda")
    ids = torch.empty((T, 8, 16), dtype=torch.int32, device="cuda")
    w = torch.empty((T, 8, 16), dtype=torch.float32, device="cuda")
    dims = ops.make_dims(T, pw.dims)
    st = L.ethos_router_forward_noalloc(ctypes.byref(dims), _vp(x), _vp(pw.w_cat), _vp(pw.bn), 1e-5,
                                        _vp(pw.key_cat), _vp(ids), _vp(w),
                                        _vp(ops.device_error_word("cuda")),
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 8  # ETHOS_ERR_SCRATCH_LIMIT
    assert b"static scratch" in L.ethos_status_string(st)
