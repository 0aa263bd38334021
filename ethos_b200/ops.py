"""Torch-tensor wrappers over the C ABI (device pointers in, device pointers out).

PyTorch only provides device memory and the current stream here; every
computation runs in ``libethos_b200.so``.  All tensors must already live on a
CUDA device: there is no CPU path.
"""

import ctypes

import torch

from ._lib import EthosDims, EthosError, check, lib

__all__ = [
    "make_dims", "gemm_bf16", "gemm_ex", "product_key_topk", "expert_forward", "router_forward", "layer_forward",
    "device_error_word", "check_device_error", "PackedWeights", "layer_backward", "layer_forward_f32",
    "router_forward_f32", "layer_backward_f32",
]

_ERR_WORDS = {}


def _vp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _events(evs):
    """ctypes array of raw cudaEvent_t handles (events are created on first
    record, so each is recorded once here if it has no handle yet)."""
    if evs is None:
        return None
    handles = []
    for e in evs:
        if e is None:
            handles.append(None)
            continue
        if e.cuda_event == 0:
            e.record()
        handles.append(e.cuda_event)
    return (ctypes.c_void_p * len(handles))(*handles)


def _require_cuda(t, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor: the ETHOS B200 layer has no CPU path")


def device_error_word(device):
    """The per-device int32 word where kernels record bounds/timeout errors."""
    device = torch.device(device)
    key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
    w = _ERR_WORDS.get(key)
    if w is None:
        w = torch.zeros(4, dtype=torch.int32, device=device)
        _ERR_WORDS[key] = w
    return w


def check_device_error(device, reset=True):
    """Synchronises the current stream and raises EthosError if a kernel set
    the device error word (expert id out of range, bounded wait timeout)."""
    w = device_error_word(device)
    code = ctypes.c_int(0)
    check(lib().ethos_read_device_error(_vp(w), ctypes.byref(code), 1 if reset else 0,
                                        _stream(w.device)), "ethos_read_device_error")
    if code.value != 0:
        raise EthosError(code.value, "device error word")


def make_dims(tokens, d):
    return EthosDims(tokens=int(tokens), d_model=d["d_model"], num_experts=d["num_experts"],
                     num_sub_keys=d["num_sub_keys"], d_query=d["d_query"], d_latent=d["d_latent"],
                     d_hidden=d["d_hidden"], num_heads=d["num_heads"], top_k=d["top_k"])


def gemm_bf16(a, b, scale=1.0, out_dtype=torch.float32):
    """``a [M, K] @ b[N, K]^T * scale`` on the tcgen05 GEMM (bf16 in, fp32 acc)."""
    _require_cuda(a, "a")
    _require_cuda(b, "b")
    a = a.contiguous()
    b = b.contiguous()
    M, K = a.shape
    N = b.shape[0]
    out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    err = device_error_word(a.device)
    check(lib().ethos_gemm_bf16(_vp(a), _vp(b), _vp(out), M, N, K, float(scale),
                                1 if out_dtype == torch.bfloat16 else 0, _vp(err), _stream(a.device)),
          "ethos_gemm_bf16")
    return out


def gemm_ex(a, b, a_mn=False, b_mn=False, out=None, mode="f32", scale=1.0):
    """General tcgen05 GEMM ``D[m, n] = scale * sum_k A(m, k) B(n, k)``.

    ``a`` is ``[M, K]`` (K-major) or ``[K, M]`` (``a_mn=True``, read in place);
    ``b`` is ``[N, K]`` or ``[K, N]`` (``b_mn=True``).  ``mode``: "f32" or
    "bf16" (store) or "acc" (fp32 ``out +=``, split-K atomics)."""
    _require_cuda(a, "a")
    _require_cuda(b, "b")
    if a.stride(-1) != 1 or b.stride(-1) != 1:
        raise ValueError("operands must have unit stride in their last dimension")
    K, M = (a.shape[0], a.shape[1]) if a_mn else (a.shape[1], a.shape[0])
    N = b.shape[1] if b_mn else b.shape[0]
    Kb = b.shape[0] if b_mn else b.shape[1]
    if Kb != K:
        raise ValueError(f"K mismatch {K} vs {Kb}")
    om = {"f32": 0, "bf16": 1, "acc": 2}[mode]
    if out is None:
        dt = torch.bfloat16 if mode == "bf16" else torch.float32
        out = (torch.zeros if mode == "acc" else torch.empty)((M, N), dtype=dt, device=a.device)
    err = device_error_word(a.device)
    check(lib().ethos_gemm_bf16_ex(_vp(a), a.stride(0), int(a_mn), _vp(b), b.stride(0), int(b_mn), _vp(out),
                                   out.stride(0), M, N, K, float(scale), om, _vp(err), _stream(a.device)),
          "ethos_gemm_bf16_ex")
    return out


def product_key_topk(q, keys, top_k):
    """Product-key selection from normalised queries.

    ``q`` bf16 ``[H, T, dq]``, ``keys`` bf16 ``[2, K, dq/2]``.  Returns
    ``(weights fp32 [T, H, k], ids int32 [T, H, k])`` (model.py:217-245)."""
    _require_cuda(q, "q")
    H, T, dq = q.shape
    K = keys.shape[1]
    dims = EthosDims(tokens=T, d_model=0, num_experts=K * K, num_sub_keys=K, d_query=dq,
                     d_latent=0, d_hidden=0, num_heads=H, top_k=int(top_k))
    ids = torch.empty((T, H, top_k), dtype=torch.int32, device=q.device)
    w = torch.empty((T, H, top_k), dtype=torch.float32, device=q.device)
    err = device_error_word(q.device)
    check(lib().ethos_product_key_topk(ctypes.byref(dims), _vp(q.contiguous()), _vp(keys.contiguous()),
                                       _vp(ids), _vp(w), _vp(err), _stream(q.device)),
          "ethos_product_key_topk")
    return w, ids


EXPERT_AUTO, EXPERT_FUSED, EXPERT_TABLE, EXPERT_TABLE_CACHED = 0, 1, 2, 3


def expert_forward(latents, w1, ids, weights, xp, dims, save_dot=False, path=EXPERT_AUTO):
    """Experts alone on given routing decisions: returns ``(hacc bf16 [T, dh],
    dot fp32 [T, H*k] or None)``.  ``ids`` int32 / ``weights`` fp32 ``[T, H, k]``.
    ``path``: EXPERT_FUSED (per token), EXPERT_TABLE (per-expert hidden
    table) or EXPERT_AUTO."""
    _require_cuda(ids, "ids")
    T = ids.shape[0]
    ed = make_dims(T, dims)
    L = lib()
    hacc = torch.empty((T, dims["d_hidden"]), dtype=torch.bfloat16, device=ids.device)
    dot = (torch.empty((T, dims["num_heads"] * dims["top_k"]), dtype=torch.float32, device=ids.device)
           if save_dot else None)
    ws_bytes = L.ethos_expert_workspace_size(ctypes.byref(ed), int(path))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=ids.device)
    err = device_error_word(ids.device)
    check(L.ethos_expert_forward(ctypes.byref(ed), int(path), _vp(latents), _vp(w1), _vp(ids.contiguous()),
                                 _vp(weights.contiguous()), _vp(xp.contiguous()), _vp(hacc), _vp(dot), _vp(ws),
                                 ws_bytes, _vp(err), _stream(ids.device)), "ethos_expert_forward")
    return hacc, dot


def expert_table_build(latents, w1, dims, with_grad=False):
    """The expert table ``H = fp16(gelu(latents @ w1^T))`` [N, dh] (and, with
    ``with_grad``, ``G = fp16(gelu'(latents @ w1^T))``) that
    ``EXPERT_TABLE_CACHED`` gathers from.  ``latents`` bf16 [N, dl], ``w1``
    bf16 [dh, dl].  Returns ``(htab, gtab or None)``."""
    _require_cuda(latents, "latents")
    N, dh = dims["num_experts"], dims["d_hidden"]
    htab = torch.empty((N, dh), dtype=torch.float16, device=latents.device)
    gtab = torch.empty_like(htab) if with_grad else None
    ed = make_dims(1, dims)
    err = device_error_word(latents.device)
    check(lib().ethos_expert_table_build(ctypes.byref(ed), _vp(latents.contiguous()), _vp(w1.contiguous()),
                                         _vp(htab), _vp(gtab), _vp(err), _stream(latents.device)),
          "ethos_expert_table_build")
    return htab, gtab


class PackedWeights:
    """Kernel-layout copies of the layer parameters (derived caches, never
    state): ``w_cat [H*dq + dh, d]`` (query projections stacked, then
    ``W_u^T``), ``key_cat``, ``latents [N, dl]``, ``w1 [dh, dl]``,
    ``wv [d, dh]`` and the fp32 ``bn [5, H*dq]`` (bias, gamma, beta, running
    mean, running var).  bf16 path (``fp32`` False): bf16 tensors, key_cat
    ``[2, K, dq]`` with each sub-key row written twice (split-bf16 scoring).
    fp32 path: fp32 tensors, key_cat ``[2, K, dq/2]`` (the two sub-key
    tables)."""

    __slots__ = ("w_cat", "key_cat", "latents", "w1", "wv", "bn", "dims", "fp32")

    def __init__(self, w_cat, key_cat, latents, w1, wv, bn, dims, fp32=False):
        self.w_cat, self.key_cat, self.latents = w_cat, key_cat, latents
        self.w1, self.wv, self.bn, self.dims = w1, wv, bn, dims
        self.fp32 = fp32


def router_forward(x2d, pw, bn_training, eps, momentum, save_qpre=None, save_bn=None):
    """``(weights fp32 [T,H,k], ids int32 [T,H,k])`` for bf16 ``x2d [T, d]``."""
    _require_cuda(x2d, "x")
    d = pw.dims
    T = x2d.shape[0]
    dims = make_dims(T, d)
    L = lib()
    ws_bytes = L.ethos_forward_workspace_size(ctypes.byref(dims), 1 if bn_training else 0, EXPERT_FUSED)
    if ws_bytes == 0:
        check(L.ethos_check_dims(ctypes.byref(dims)), "ethos_check_dims")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x2d.device)
    ids = torch.empty((T, d["num_heads"], d["top_k"]), dtype=torch.int32, device=x2d.device)
    w = torch.empty((T, d["num_heads"], d["top_k"]), dtype=torch.float32, device=x2d.device)
    err = device_error_word(x2d.device)
    check(L.ethos_router_forward(ctypes.byref(dims), _vp(x2d), _vp(pw.w_cat), _vp(pw.bn), float(eps),
                                 float(momentum), 1 if bn_training else 0, _vp(pw.key_cat), _vp(ids), _vp(w),
                                 _vp(save_qpre), _vp(save_bn), _vp(ws), ws_bytes, _vp(err),
                                 _stream(x2d.device)), "ethos_router_forward")
    return w, ids


STAGES = ("start", "projection", "batchnorm", "topk", "expert_table", "experts", "end")


def resolve_expert_path(tokens, dims, path=EXPERT_AUTO):
    """The expert path the library runs (its resolve rule, include/ethos_b200.h):
    the table once the step makes at least one selection per expert and
    H * k >= 16, otherwise the fused per-token kernel."""
    R = dims["num_heads"] * dims["top_k"]
    if path == EXPERT_TABLE_CACHED:
        return EXPERT_TABLE_CACHED
    if path == EXPERT_FUSED:
        return EXPERT_FUSED
    if path == EXPERT_TABLE:
        return EXPERT_TABLE if R >= 16 else EXPERT_FUSED
    return EXPERT_TABLE if (tokens * R >= dims["num_experts"] and R >= 16) else EXPERT_FUSED


def layer_forward(x2d, pw, bn_training, eps, momentum, save=False, path=EXPERT_AUTO, stage_events=None,
                  htab=None):
    """Router + experts.  Returns a dict with ``y`` (bf16 [T, d]), ``ids``,
    ``weights`` and, when ``save``, the tensors the backward pass needs.
    ``stage_events``: optional list of len(STAGES) ``torch.cuda.Event`` that
    the library records at each stage boundary (per-kernel timing).
    ``htab``: a prebuilt expert table (``expert_table_build``) for the
    current latents and W1; the experts then gather from it and skip the
    expansion (inference only: not with ``save``)."""
    _require_cuda(x2d, "x")
    if htab is not None:
        if save:
            raise ValueError("a cached expert table serves inference only (save=False)")
        path = EXPERT_TABLE_CACHED
    d = pw.dims
    T = x2d.shape[0]
    dev = x2d.device
    dims = make_dims(T, d)
    L = lib()
    ws_bytes = L.ethos_forward_workspace_size(ctypes.byref(dims), 1 if bn_training else 0, int(path))
    if ws_bytes == 0:
        check(L.ethos_check_dims(ctypes.byref(dims)), "ethos_check_dims")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    H, k, dh, HQ = d["num_heads"], d["top_k"], d["d_hidden"], d["num_heads"] * d["d_query"]
    out = dict(
        y=torch.empty((T, d["d_model"]), dtype=torch.bfloat16, device=dev),
        ids=torch.empty((T, H, k), dtype=torch.int32, device=dev),
        weights=torch.empty((T, H, k), dtype=torch.float32, device=dev),
    )
    if save:
        out["xp"] = torch.empty((T, dh), dtype=torch.float32, device=dev)
        out["hacc"] = torch.empty((T, dh), dtype=torch.bfloat16, device=dev)
        out["dot"] = torch.empty((T, H * k), dtype=torch.float32, device=dev)
        out["qpre"] = torch.empty((T, HQ), dtype=torch.float32, device=dev)
        out["qs"] = torch.empty((2, H, T, d["d_query"]), dtype=torch.bfloat16, device=dev)
        if bn_training:
            out["bn_stats"] = torch.empty((2, HQ), dtype=torch.float32, device=dev)
        if resolve_expert_path(T, d, path) == EXPERT_TABLE:
            # the expert table and its GELU derivative, kept for the backward
            out["htab"] = torch.empty((d["num_experts"], dh), dtype=torch.float16, device=dev)
            out["gtab"] = torch.empty((d["num_experts"], dh), dtype=torch.float16, device=dev)
    g = out.get
    if htab is not None:
        out["htab"] = htab
    err = device_error_word(dev)
    check(L.ethos_layer_forward(ctypes.byref(dims), _vp(x2d), _vp(pw.w_cat), _vp(pw.bn), float(eps),
                                float(momentum), 1 if bn_training else 0, _vp(pw.key_cat), _vp(pw.latents),
                                _vp(pw.w1), _vp(pw.wv), int(path), _vp(out["y"]), _vp(out["ids"]),
                                _vp(out["weights"]),
                                _vp(g("xp")), _vp(g("hacc")), _vp(g("dot")), _vp(g("qpre")),
                                _vp(g("bn_stats")), _vp(g("qs")), _vp(g("htab")), _vp(g("gtab")), _vp(ws), ws_bytes,
                                _vp(err), _events(stage_events), _stream(dev)),
          "ethos_layer_forward")
    if htab is not None:
        del out["htab"]
    return out


def _numel(shape):
    n = 1
    for s in shape:
        n *= s
    return n


BWD_STAGE_EXPERTS, BWD_STAGE_END = 0, 1  # ETHOS_BWD_STAGE_* (include/ethos_b200.h)


def layer_backward(dy, x16, pw, saved, bn_training, eps, stage_events=None, dx_dtype=torch.float32):
    """Gradients of the layer (see ethos_layer_backward).  ``dy`` [T, d] bf16
    or fp32; ``saved`` is the dict returned by ``layer_forward(save=True)``.
    Returns a dict of fp32 tensors (dx in ``dx_dtype``, fp32 or bf16): dx,
    d_latents, d_w1, d_w2, d_wq [H*dq, d],
    d_bn [3, H*dq] (bias, gamma, beta), d_keys [2, K, dq/2], and the flat fp32
    buffer holding all parameter gradients (``flat``, ``layout``).
    ``stage_events``: optional [experts_done, end] ``torch.cuda.Event`` (or
    None entries), recorded as ETHOS_BWD_STAGE_* describe."""
    if stage_events is not None and len(stage_events) != 2:
        raise ValueError("stage_events: one event (or None) per ETHOS_BWD_STAGE_*")
    _require_cuda(dy, "dy")
    d = pw.dims
    T = dy.shape[0]
    dev = dy.device
    dims = make_dims(T, d)
    L = lib()
    ws_bytes = L.ethos_backward_workspace_size(ctypes.byref(dims))
    if ws_bytes == 0:
        check(L.ethos_check_dims(ctypes.byref(dims)), "ethos_check_dims")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    HQ = d["num_heads"] * d["d_query"]
    # all parameter gradients live in one flat fp32 buffer (256-B aligned
    # slices), so that a caller can convert them with a single kernel
    shapes = [("d_latents", (d["num_experts"], d["d_latent"])), ("d_w1", (d["d_hidden"], d["d_latent"])),
              ("d_w2", (2 * d["d_model"], d["d_hidden"])), ("d_wq", (HQ, d["d_model"])), ("d_bn", (3, HQ)),
              ("d_keys", (2, d["num_sub_keys"], d["d_query"] // 2))]
    layout, off = [], 0
    for name, shp in shapes:
        n = 1
        for s_ in shp:
            n *= s_
        layout.append((name, off, shp))
        off += (n + 63) // 64 * 64
    flat = torch.empty(off, dtype=torch.float32, device=dev)
    g = {name: flat[o:o + _numel(shp)].view(shp) for name, o, shp in layout}
    if dx_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("dx_dtype: torch.float32 or torch.bfloat16")
    g["dx"] = torch.empty((T, d["d_model"]), dtype=dx_dtype, device=dev)
    g["flat"] = flat
    g["layout"] = layout
    dy = dy.contiguous()
    if dy.dtype not in (torch.bfloat16, torch.float32):
        dy = dy.float()
    err = device_error_word(dev)
    check(L.ethos_layer_backward(ctypes.byref(dims), 1 if bn_training else 0, float(eps), _vp(dy),
                                 1 if dy.dtype == torch.float32 else 0, _vp(x16), _vp(pw.w_cat), _vp(pw.bn),
                                 _vp(pw.key_cat), _vp(pw.latents), _vp(pw.w1), _vp(pw.wv), _vp(saved["ids"]),
                                 _vp(saved["weights"]), _vp(saved["xp"]), _vp(saved["hacc"]), _vp(saved["dot"]),
                                 _vp(saved["qpre"]), _vp(saved.get("bn_stats")), _vp(saved["qs"]),
                                 _vp(saved.get("htab")), _vp(saved.get("gtab")), _vp(g["dx"]),
                                 1 if dx_dtype == torch.bfloat16 else 0,
                                 _vp(g["d_latents"]), _vp(g["d_w1"]), _vp(g["d_w2"]), _vp(g["d_wq"]),
                                 _vp(g["d_bn"]), _vp(g["d_keys"]), _vp(ws), ws_bytes, _vp(err),
                                 _events(stage_events), _stream(dev)),
          "ethos_layer_backward")
    return g


# ----------------------------------------------------------- fp32 path --
def expert_backward(latents, w1, ids, weights, xp, dot, dhacc, dims, htab=None, gtab=None):
    """Backward of ``expert_forward`` (ethos_expert_backward): the expert
    half of the layer's backward, for a host that routes with its own router.
    ``dot`` is ``expert_forward(..., save_dot=True)``'s second output and
    ``dhacc`` fp32 ``[T, dh]`` the gradient of hacc.  Returns a dict of fp32
    ``dxp [T, dh]``, ``d_weights [T, H, k]`` (the routing weights' gradient,
    the router backward's input), ``d_latents [N, dl]`` and ``d_w1 [dh, dl]``."""
    _require_cuda(ids, "ids")
    if (htab is None) != (gtab is None):
        raise ValueError("htab and gtab go together")
    T = ids.shape[0]
    dev = ids.device
    ed = make_dims(T, dims)
    L = lib()
    ws_bytes = L.ethos_expert_backward_workspace_size(ctypes.byref(ed))
    if ws_bytes == 0:
        check(L.ethos_check_dims(ctypes.byref(ed)), "ethos_check_dims")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    f32 = dict(dtype=torch.float32, device=dev)
    out = {"dxp": torch.empty((T, dims["d_hidden"]), **f32),
           "d_weights": torch.empty((T, dims["num_heads"], dims["top_k"]), **f32),
           "d_latents": torch.empty((dims["num_experts"], dims["d_latent"]), **f32),
           "d_w1": torch.empty((dims["d_hidden"], dims["d_latent"]), **f32)}
    err = device_error_word(dev)
    check(L.ethos_expert_backward(ctypes.byref(ed), _vp(latents), _vp(w1), _vp(ids.contiguous()),
                                  _vp(weights.contiguous()), _vp(xp.contiguous()), _vp(dot.contiguous()),
                                  _vp(dhacc.contiguous().float()), _vp(htab), _vp(gtab), _vp(out["dxp"]),
                                  _vp(out["d_weights"]), _vp(out["d_latents"]), _vp(out["d_w1"]), _vp(ws),
                                  ws_bytes, _vp(err), _stream(dev)), "ethos_expert_backward")
    return out


def router_backward(d_weights, x2d, pw, ids, weights, save_qpre, bn_training, eps, save_bn=None, dx=None):
    """Backward of ``router_forward`` (ethos_router_backward) given the routing
    weights' gradient ``d_weights`` fp32 ``[T, H, k]``; ``save_qpre`` /
    ``save_bn`` are the forward's save buffers.  With ``dx`` given (fp32
    ``[T, d]``) the router's share of dL/dx is added to it, else a new ``dx``
    is returned.  Returns a dict of fp32 ``dx``, ``d_wq [H*dq, d]``,
    ``d_bn [3, H*dq]`` (bias, gamma, beta) and ``d_keys [2, K, dq/2]``."""
    _require_cuda(x2d, "x")
    d = pw.dims
    T = x2d.shape[0]
    dev = x2d.device
    dims = make_dims(T, d)
    L = lib()
    ws_bytes = L.ethos_router_backward_workspace_size(ctypes.byref(dims))
    if ws_bytes == 0:
        check(L.ethos_check_dims(ctypes.byref(dims)), "ethos_check_dims")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    HQ = d["num_heads"] * d["d_query"]
    f32 = dict(dtype=torch.float32, device=dev)
    accumulate = dx is not None
    if dx is None:
        dx = torch.empty((T, d["d_model"]), **f32)
    elif dx.dtype != torch.float32 or not dx.is_contiguous() or tuple(dx.shape) != (T, d["d_model"]):
        raise ValueError("dx: a contiguous fp32 [T, d_model] tensor")
    out = {"dx": dx, "d_wq": torch.empty((HQ, d["d_model"]), **f32), "d_bn": torch.empty((3, HQ), **f32),
           "d_keys": torch.empty((2, d["num_sub_keys"], d["d_query"] // 2), **f32)}
    err = device_error_word(dev)
    check(L.ethos_router_backward(ctypes.byref(dims), 1 if bn_training else 0, float(eps), _vp(x2d), _vp(pw.w_cat),
                                  _vp(pw.bn), _vp(pw.key_cat), _vp(ids.contiguous()), _vp(weights.contiguous()),
                                  _vp(d_weights.contiguous().float()), _vp(save_qpre), _vp(save_bn), _vp(dx),
                                  1 if accumulate else 0, _vp(out["d_wq"]), _vp(out["d_bn"]), _vp(out["d_keys"]),
                                  _vp(ws), ws_bytes, _vp(err), _stream(dev)), "ethos_router_backward")
    return out


def _grad_layout(d):
    """Flat fp32 buffer for every parameter gradient (256-B aligned slices)."""
    HQ = d["num_heads"] * d["d_query"]
    shapes = [("d_latents", (d["num_experts"], d["d_latent"])), ("d_w1", (d["d_hidden"], d["d_latent"])),
              ("d_w2", (2 * d["d_model"], d["d_hidden"])), ("d_wq", (HQ, d["d_model"])), ("d_bn", (3, HQ)),
              ("d_keys", (2, d["num_sub_keys"], d["d_query"] // 2))]
    layout, off = [], 0
    for name, shp in shapes:
        layout.append((name, off, shp))
        off += (_numel(shp) + 63) // 64 * 64
    return layout, off


def layer_forward_f32(x2d, pw, bn_training, eps, momentum, save=False, router_only=False):
    """fp32 arithmetic (ethos_layer_forward_f32): fp32 ``x2d [T, d]`` and an
    fp32 ``PackedWeights``.  Returns ``y`` (fp32 [T, d]; absent with
    ``router_only``), ``ids``, ``weights`` and, when ``save``, the tensors the
    backward needs."""
    _require_cuda(x2d, "x")
    if not pw.fp32 or x2d.dtype != torch.float32:
        raise ValueError("layer_forward_f32 takes fp32 inputs and fp32 packed weights")
    d = pw.dims
    T = x2d.shape[0]
    dev = x2d.device
    dims = make_dims(T, d)
    L = lib()
    ws_bytes = L.ethos_forward_workspace_size_f32(ctypes.byref(dims), 1 if bn_training else 0)
    if ws_bytes == 0:
        st = L.ethos_check_dims(ctypes.byref(dims))
        check(st if st != 0 else 2, "ethos_forward_workspace_size_f32")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    H, k, dh, HQ, dq = d["num_heads"], d["top_k"], d["d_hidden"], d["num_heads"] * d["d_query"], d["d_query"]
    f32 = dict(dtype=torch.float32, device=dev)
    out = dict(ids=torch.empty((T, H, k), dtype=torch.int32, device=dev), weights=torch.empty((T, H, k), **f32))
    if not router_only:
        out["y"] = torch.empty((T, d["d_model"]), **f32)
    if save and not router_only:
        out["xp"] = torch.empty((T, dh), **f32)
        out["hacc"] = torch.empty((T, dh), **f32)
        out["dot"] = torch.empty((T, H * k), **f32)
        out["qpre"] = torch.empty((T, HQ), **f32)
        out["qhat"] = torch.empty((2, H, T, dq // 2), **f32)
        out["htab"] = torch.empty((d["num_experts"], dh), **f32)
        out["gtab"] = torch.empty((d["num_experts"], dh), **f32)
        if bn_training:
            out["bn_stats"] = torch.empty((2, HQ), **f32)
    g = out.get
    err = device_error_word(dev)
    check(L.ethos_layer_forward_f32(ctypes.byref(dims), _vp(x2d), _vp(pw.w_cat), _vp(pw.bn), float(eps),
                                    float(momentum), 1 if bn_training else 0, _vp(pw.key_cat), _vp(pw.latents),
                                    _vp(pw.w1), _vp(pw.wv), _vp(g("y")), _vp(out["ids"]), _vp(out["weights"]),
                                    _vp(g("xp")), _vp(g("hacc")), _vp(g("dot")), _vp(g("qpre")), _vp(g("bn_stats")),
                                    _vp(g("qhat")), _vp(g("htab")), _vp(g("gtab")), _vp(ws), ws_bytes, _vp(err),
                                    _stream(dev)), "ethos_layer_forward_f32")
    return out


def router_forward_f32(x2d, pw, bn_training, eps, momentum):
    """``(weights fp32 [T,H,k], ids int32 [T,H,k])`` in fp32 arithmetic."""
    out = layer_forward_f32(x2d, pw, bn_training, eps, momentum, router_only=True)
    return out["weights"], out["ids"]


def layer_backward_f32(dy, x32, pw, saved, bn_training, eps, stage_events=None):
    """Gradients of ``layer_forward_f32(save=True)`` (ethos_layer_backward_f32);
    the same dict as ``layer_backward``."""
    if stage_events is not None and len(stage_events) != 2:
        raise ValueError("stage_events: one event (or None) per ETHOS_BWD_STAGE_*")
    _require_cuda(dy, "dy")
    d = pw.dims
    T = dy.shape[0]
    dev = dy.device
    dims = make_dims(T, d)
    L = lib()
    ws_bytes = L.ethos_backward_workspace_size_f32(ctypes.byref(dims))
    if ws_bytes == 0:
        check(2, "ethos_backward_workspace_size_f32")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    layout, total = _grad_layout(d)
    flat = torch.empty(total, dtype=torch.float32, device=dev)
    g = {name: flat[o:o + _numel(shp)].view(shp) for name, o, shp in layout}
    g["dx"] = torch.empty((T, d["d_model"]), dtype=torch.float32, device=dev)
    g["flat"] = flat
    g["layout"] = layout
    dy = dy.contiguous().float()
    err = device_error_word(dev)
    check(L.ethos_layer_backward_f32(ctypes.byref(dims), 1 if bn_training else 0, float(eps), _vp(dy), _vp(x32),
                                     _vp(pw.w_cat), _vp(pw.bn), _vp(pw.key_cat), _vp(pw.latents), _vp(pw.w1),
                                     _vp(pw.wv), _vp(saved["ids"]), _vp(saved["weights"]), _vp(saved["xp"]),
                                     _vp(saved["hacc"]), _vp(saved["dot"]), _vp(saved["qpre"]),
                                     _vp(saved.get("bn_stats")), _vp(saved["qhat"]), _vp(saved.get("htab")),
                                     _vp(saved.get("gtab")), _vp(g["dx"]), _vp(g["d_latents"]), _vp(g["d_w1"]),
                                     _vp(g["d_w2"]), _vp(g["d_wq"]), _vp(g["d_bn"]), _vp(g["d_keys"]), _vp(ws),
                                     ws_bytes, _vp(err), _events(stage_events), _stream(dev)),
          "ethos_layer_backward_f32")
    return g
