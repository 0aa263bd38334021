"""ctypes binding of ``libethos_b200.so`` (the C ABI in ``include/ethos_b200.h``).

The library is built in tree by :mod:`ethos_b200.build`.  There is no fallback:
if the shared library cannot be loaded, every op raises ``EthosLibraryError``.
"""

import ctypes
import os
import threading

from .build import LIB_PATH

__all__ = ["EthosDims", "EthosError", "EthosLibraryError", "lib", "check", "EXPORTS", "STATUS"]

STATUS = {
    0: "ETHOS_OK", 1: "ETHOS_ERR_INVALID_ARG", 2: "ETHOS_ERR_UNSUPPORTED_SHAPE",
    3: "ETHOS_ERR_ALIGNMENT", 4: "ETHOS_ERR_WORKSPACE", 5: "ETHOS_ERR_CUDA",
    6: "ETHOS_ERR_TENSOR_MAP", 7: "ETHOS_ERR_NO_DEVICE", 8: "ETHOS_ERR_SCRATCH_LIMIT",
    16: "ETHOS_ERR_ID_OUT_OF_RANGE",
}
ETHOS_ERR_TIMEOUT_BASE = 1000


class EthosError(RuntimeError):
    """A C-ABI call returned a non-zero status (or the device error word was set)."""

    def __init__(self, status, what=""):
        self.status = int(status)
        name = STATUS.get(self.status)
        if name is None and self.status >= ETHOS_ERR_TIMEOUT_BASE:
            name = f"ETHOS_ERR_TIMEOUT(site {self.status - ETHOS_ERR_TIMEOUT_BASE})"
        super().__init__(f"{what}: {name or 'status %d' % self.status}")


class EthosLibraryError(RuntimeError):
    """The CUDA extension is missing or failed to load."""


class EthosDims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "tokens", "d_model", "num_experts", "num_sub_keys", "d_query", "d_latent",
        "d_hidden", "num_heads", "top_k")]


_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_I64 = ctypes.c_int64
_DIMS = ctypes.POINTER(EthosDims)

# name -> (restype, argtypes); must match include/ethos_b200.h
EXPORTS = {
    "ethos_abi_version": (_I, []),
    "ethos_launch_count": (ctypes.c_uint64, []),
    "ethos_status_string": (ctypes.c_char_p, [_I]),
    "ethos_read_device_error": (_I, [_P, ctypes.POINTER(_I), _I, _P]),
    "ethos_check_dims": (_I, [_DIMS]),
    "ethos_forward_workspace_size": (_SZ, [_DIMS, _I, _I]),
    "ethos_expert_workspace_size": (_SZ, [_DIMS, _I]),
    "ethos_layer_forward": (_I, [_DIMS, _P, _P, _P, _F, _F, _I, _P, _P, _P, _P, _I, _P, _P, _P,
                                 _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P, _P]),
    "ethos_backward_workspace_size": (_SZ, [_DIMS]),
    "ethos_layer_backward": (_I, [_DIMS, _I, _F, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                  _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P, _P]),
    "ethos_router_forward": (_I, [_DIMS, _P, _P, _P, _F, _F, _I, _P, _P, _P, _P, _P, _P, _SZ,
                                  _P, _P]),
    "ethos_expert_backward_workspace_size": (_SZ, [_DIMS]),
    # dims, latents, w1, ids, weights, xp, dot, dhacc, htab, gtab, dxp, d_weights, d_latents,
    # d_w1, workspace, workspace_bytes, dev_err, stream
    "ethos_expert_backward": (_I, [_DIMS] + [_P] * 14 + [_SZ, _P, _P]),
    "ethos_router_backward_workspace_size": (_SZ, [_DIMS]),
    # dims, bn_training, eps, x, w_cat, bn, keys, ids, weights, d_weights, save_qpre, save_bn,
    # dx, accumulate_dx, d_wq, d_bn, d_keys, workspace, workspace_bytes, dev_err, stream
    "ethos_router_backward": (_I, [_DIMS, _I, _F] + [_P] * 10 + [_I] + [_P] * 4 + [_SZ, _P, _P]),
    "ethos_expert_forward": (_I, [_DIMS, _I, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "ethos_expert_table_build": (_I, [_DIMS, _P, _P, _P, _P, _P, _P]),
    "ethos_router_forward_noalloc": (_I, [_DIMS, _P, _P, _P, _F, _P, _P, _P, _P, _P]),
    "ethos_product_key_topk": (_I, [_DIMS, _P, _P, _P, _P, _P, _P]),
    "ethos_gemm_bf16": (_I, [_P, _P, _P, _I64, _I64, _I64, _F, _I, _P, _P]),
    "ethos_gemm_bf16_ex": (_I, [_P, _I64, _I, _P, _I64, _I, _P, _I64, _I64, _I64, _I64, _F, _I, _P, _P]),
    "ethos_adamw_step": (_I, [_P, _I, _I64, _F, _F, _F, _F, _F, _I64, _P, _P, _P]),
    "ethos_grad_clip_workspace_size": (_SZ, []),
    "ethos_grad_clip_coef": (_I, [_P, _I, _F, _P, _SZ, _P, _P, _P]),
    "ethos_set_wait_limit_ns": (_I, [ctypes.c_uint64]),
    "ethos_test_gelu": (_I, [_P, _P, _I64, _P]),
    "ethos_forward_workspace_size_f32": (_SZ, [_DIMS, _I]),
    # dims, x, w_cat, bn, eps, momentum, bn_training, keys, latents, w1, wv, y, ids, weights,
    # save_xp, save_hacc, save_dot, save_qpre, save_bn, save_qhat, save_htab, save_gtab,
    # workspace, workspace_bytes, dev_err, stream
    "ethos_layer_forward_f32": (_I, [_DIMS, _P, _P, _P, _F, _F, _I] + [_P] * 15 + [_P, _SZ, _P, _P]),
    "ethos_backward_workspace_size_f32": (_SZ, [_DIMS]),
    # dims, bn_training, eps, dy, x, w_cat, bn, keys, latents, w1, wv, ids, weights, save_xp,
    # save_hacc, save_dot, save_qpre, save_bn, save_qhat, htab, gtab, dx, d_latents, d_w1, d_w2,
    # d_wq, d_bn, d_keys, workspace, workspace_bytes, dev_err, stage_events, stream
    "ethos_layer_backward_f32": (_I, [_DIMS, _I, _F] + [_P] * 26 + [_SZ, _P, _P, _P]),
    "ethos_test_gemm_withhold": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _P, _P]),
}

_lock = threading.Lock()
_lib = None


def lib(path=None):
    """Load (once) and return the ctypes handle; raises EthosLibraryError."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or os.environ.get("ETHOS_B200_LIB", LIB_PATH)
        if not os.path.exists(p):
            raise EthosLibraryError(
                f"{p} is missing: build it with `python -m ethos_b200.build` "
                "(the ETHOS layer has no CPU fallback)")
        try:
            handle = ctypes.CDLL(p)
        except OSError as e:
            raise EthosLibraryError(f"cannot load {p}: {e}") from e
        for name, (res, args) in EXPORTS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = handle
        return handle


def check(status, what):
    if status != 0:
        raise EthosError(status, what)
