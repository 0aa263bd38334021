"""CPU-side checks of the C ABI: the library loads, exports every entry point
that include/ethos_b200.h declares, and its host-only functions (dimension
checks, workspace sizing, status strings) behave.  No kernel is launched."""

import ctypes
import os
import re

import pytest

from ethos_b200 import _lib
from ethos_b200.build import LIB_PATH, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ethos_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|size_t|uint64_t|const char\s*\*)\s*(ethos_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def L():
    build()
    return _lib.lib()


def test_library_built_in_tree():
    build()
    assert os.path.exists(LIB_PATH)


def test_every_declared_symbol_is_exported(L):
    names = declared_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.EXPORTS), "ctypes table and header disagree"


def test_ctypes_argument_counts_match_header():
    """Every ctypes prototype has as many arguments as the header declares."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for m in re.finditer(r"^\s*(?:int|int64_t|size_t|uint64_t|const char\s*\*)\s*(ethos_\w+)\s*\(([^)]*)\)\s*;", text,
                         flags=re.M):
        name, args = m.group(1), m.group(2).strip()
        n = 0 if args in ("", "void") else len(args.split(","))
        assert len(_lib.EXPORTS[name][1]) == n, (name, n, len(_lib.EXPORTS[name][1]))


def test_abi_version_and_status_strings(L):
    assert L.ethos_abi_version() >= 1
    assert L.ethos_status_string(0) == b"ok"
    assert b"unsupported" in L.ethos_status_string(2)
    assert b"timed out" in L.ethos_status_string(1003)


def _dims(**kw):
    base = dict(tokens=16384, d_model=1024, num_experts=512 * 512, num_sub_keys=512, d_query=512,
                d_latent=128, d_hidden=512, num_heads=8, top_k=16)
    base.update(kw)
    return _lib.EthosDims(**base)


@pytest.mark.parametrize("kw,ok", [
    ({}, True),
    (dict(d_model=512, num_experts=4096, num_sub_keys=64), True),      # config 1
    (dict(tokens=1), True),
    (dict(d_latent=64), False),
    (dict(d_hidden=256), False),
    (dict(top_k=32), False),
    (dict(top_k=12), False),
    (dict(num_experts=512 * 511), False),
    (dict(num_sub_keys=1024, num_experts=1024 * 1024), False),
    (dict(d_query=96), False),
    (dict(d_model=1000), False),
    (dict(tokens=0), False),
])
def test_check_dims(L, kw, ok):
    d = _dims(**kw)
    st = L.ethos_check_dims(ctypes.byref(d))
    assert (st == 0) == ok, (kw, st)


def test_workspace_size(L):
    d = _dims()
    T, H, dq, dh, N = 16384, 8, 512, 512, 512 * 512
    ev = L.ethos_forward_workspace_size(ctypes.byref(d), 0, 1)
    tr = L.ethos_forward_workspace_size(ctypes.byref(d), 1, 1)
    tab = L.ethos_forward_workspace_size(ctypes.byref(d), 0, 2)
    auto = L.ethos_forward_workspace_size(ctypes.byref(d), 0, 0)
    assert ev >= H * 2 * T * dq * 2 + T * dh * (4 + 2)
    assert tr >= ev + T * H * dq * 4
    assert tab >= ev + N * dh * 2
    assert auto == tab  # 16384 * 128 selections >= 262144 experts: table path
    small = _dims(tokens=64)
    assert L.ethos_forward_workspace_size(ctypes.byref(small), 0, 0) == \
        L.ethos_forward_workspace_size(ctypes.byref(small), 0, 1)
    assert L.ethos_expert_workspace_size(ctypes.byref(d), 2) >= N * dh * 2
    assert L.ethos_expert_workspace_size(ctypes.byref(d), 1) < 4096
    bad = _dims(top_k=32)
    assert L.ethos_forward_workspace_size(ctypes.byref(bad), 0, 0) == 0


def test_fp32_workspace_and_shape_rule(L):
    """The fp32 path needs d_query / 2 to be a multiple of 128 (its score
    GEMMs' N tile); other shapes are rejected before any launch."""
    d = _dims()
    assert L.ethos_forward_workspace_size_f32(ctypes.byref(d), 0) > 2 * 8 * 16384 * 512 * 4
    assert L.ethos_backward_workspace_size_f32(ctypes.byref(d)) > 2 * 8 * 16384 * 512 * 4
    small_q = _dims(d_query=128)
    assert L.ethos_check_dims(ctypes.byref(small_q)) == 0          # fine for the bf16 path
    assert L.ethos_forward_workspace_size_f32(ctypes.byref(small_q), 0) == 0
    assert L.ethos_backward_workspace_size_f32(ctypes.byref(small_q)) == 0
    st = L.ethos_layer_forward_f32(ctypes.byref(small_q), *([None] * 3), 1e-5, 0.1, 0, *([None] * 15), None, 0,
                                   None, None)
    assert st == 2  # ETHOS_ERR_UNSUPPORTED_SHAPE


def test_null_arguments_rejected_without_gpu(L):
    d = _dims()
    st = L.ethos_layer_forward(ctypes.byref(d), None, None, None, 1e-5, 0.1, 0, None, None, None, None, 0, None, None,
                               None, None, None, None, None, None, None, None, None, None, 0, None, None, None)
    assert st == 1  # ETHOS_ERR_INVALID_ARG
    st = L.ethos_layer_backward(ctypes.byref(d), 0, 1e-5, None, 0, *([None] * 17), None, 0, *([None] * 6), None,
                                0, None, None, None)
    assert st == 1
    assert L.ethos_backward_workspace_size(ctypes.byref(d)) > 2 * 512 * 512 * 512 * 2


def test_split_backward_host_checks(L):
    """The expert-only and router-only backward calls reject missing
    arguments and unpaired tables before any launch, and size their
    workspaces below the whole layer's (each needs only its half)."""
    d = _dims()
    v = ctypes.c_void_p(256)
    assert L.ethos_expert_backward(ctypes.byref(d), *([None] * 14), 0, None, None) == 1
    # htab without gtab
    args = [v] * 7 + [v, None] + [v] * 4
    assert L.ethos_expert_backward(ctypes.byref(d), *args, v, 1 << 40, v, None) == 1
    assert L.ethos_router_backward(ctypes.byref(d), 0, 1e-5, *([None] * 10), 0, *([None] * 4), 0, None, None) == 1
    # training mode needs the forward's batch statistics
    args = [v] * 8 + [None] + [v]
    assert L.ethos_router_backward(ctypes.byref(d), 1, 1e-5, *args, 0, v, v, v, v, 1 << 40, v, None) == 1
    whole = L.ethos_backward_workspace_size(ctypes.byref(d))
    ex = L.ethos_expert_backward_workspace_size(ctypes.byref(d))
    ro = L.ethos_router_backward_workspace_size(ctypes.byref(d))
    assert 0 < ex < whole and 0 < ro < whole
    bad = _dims(d_query=100)
    assert L.ethos_expert_backward_workspace_size(ctypes.byref(bad)) == 0
    assert L.ethos_router_backward_workspace_size(ctypes.byref(bad)) == 0


def test_failure_test_hook_and_counter_host_checks(L):
    """Argument checks of the bounded-wait test entry point (no launch), and
    the launch counter is readable without a device."""
    v = ctypes.c_void_p(256)
    assert L.ethos_test_gemm_withhold(None, v, v, 256, 256, 256, 0, v, None) == 1
    assert L.ethos_test_gemm_withhold(v, v, v, 256, 256, 256, -1, v, None) == 1   # no unit to hold
    assert L.ethos_test_gemm_withhold(v, v, v, 256, 200, 256, 0, v, None) == 2    # N % 128
    assert L.ethos_test_gemm_withhold(v, v, v, 256, 256, 100, 0, v, None) == 2    # K % 8
    assert L.ethos_launch_count() == L.ethos_launch_count()


def test_no_cpu_fallback():
    """The ops refuse CPU tensors instead of computing on the host."""
    import torch
    from ethos_b200 import ops
    with pytest.raises(RuntimeError, match="no CPU path"):
        ops.gemm_bf16(torch.zeros(128, 64, dtype=torch.bfloat16), torch.zeros(256, 64, dtype=torch.bfloat16))


def test_python_path_rule_matches_library(L):
    """ops.resolve_expert_path (which decides whether the forward keeps the
    expert tables for the backward) agrees with the library's own choice, as
    seen in the workspace it asks for (the table path needs N x dh fp16)."""
    from ethos_b200 import ops
    base = dict(d_model=1024, num_experts=512 * 512, num_sub_keys=512, d_query=512, d_latent=128, d_hidden=512)
    for H, k in ((8, 16), (1, 4), (2, 8), (4, 4)):
        for T in (1, 64, 2047, 2048, 16384, 65536):
            for path in (ops.EXPERT_AUTO, ops.EXPERT_FUSED, ops.EXPERT_TABLE):
                d = _dims(tokens=T, num_heads=H, top_k=k)
                if L.ethos_check_dims(ctypes.byref(d)) != 0:
                    continue
                ws = L.ethos_forward_workspace_size(ctypes.byref(d), 0, path)
                ws_fused = L.ethos_forward_workspace_size(ctypes.byref(d), 0, ops.EXPERT_FUSED)
                lib_table = ws >= ws_fused + d.num_experts * d.d_hidden * 2
                py = ops.resolve_expert_path(T, dict(base, num_heads=H, top_k=k), path)
                assert (py == ops.EXPERT_TABLE) == lib_table, (H, k, T, path)
