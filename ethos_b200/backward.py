"""Autograd backward of EthosExpertLayer (and, under
``ethos_b200.dist.overlap_grad_allreduce``, the data-parallel gradient
all-reduce overlapped with it).

Maps the gradients computed by ``ethos_layer_backward`` (one C-ABI call, see
include/ethos_b200.h) onto the inputs of ``_EthosLayerFunction``: x, the layer
and the need-grad flag (no gradients), then the parameters in the order of ``EthosExpertLayer._grad_params`` --
expert_latents, net.0, net.2, query_projs weights, query_projs biases,
query_norms weights, query_norms biases, sub_keys_1, sub_keys_2.
"""

import torch
import torch.distributed as dist

from . import ops


def _overlapped_allreduce(layer, g, events):
    """Averages the flat fp32 gradient buffer over the process group set by
    ``ethos_b200.dist.overlap_grad_allreduce``: the latent and W1 slice as soon
    as the backward marks them final (ETHOS_BWD_STAGE_EXPERTS), the rest at
    its end, both on a side stream so the first overlaps the router and
    BatchNorm gradient kernels; the current stream then waits for both.
    When the layer's ``_grad_comm["log"]`` is a list, each call appends its
    timing events to it (benchmarks: how much of the all-reduce is exposed)."""
    comm = layer._grad_comm
    flat = g["flat"]
    boundary = g["layout"][2][1]  # d_latents, d_w1 come first; d_w2 starts here
    if comm.get("stream") is None or comm["stream"].device != flat.device:
        comm["stream"] = torch.cuda.Stream(flat.device)
    side = comm["stream"]
    works = []
    timing = comm.get("log") is not None
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(2)] if timing else None
    with torch.cuda.stream(side):
        side.wait_event(events[0])
        if timing:
            marks[0].record(side)
        works.append(dist.all_reduce(flat[:boundary], op=dist.ReduceOp.AVG, group=comm["group"], async_op=True))
        side.wait_event(events[1])
        works.append(dist.all_reduce(flat[boundary:], op=dist.ReduceOp.AVG, group=comm["group"], async_op=True))
        if timing:
            marks[1].record(side)
    for w in works:
        w.wait()  # the current stream waits; the host does not block
    if timing:
        # (experts done, backward kernels done, all-reduce start, all-reduce
        # done): read after a synchronize by whoever set comm["log"]
        comm["log"].append((events[0], events[1], marks[0], marks[1]))


def layer_backward(ctx, gy):
    layer = ctx.layer
    sv = ctx.saved
    pw = sv["pw"]
    H = layer.num_heads
    dq = layer.router.d_query
    eps, _ = layer.router._bn_eps_momentum()
    comm = getattr(layer, "_grad_comm", None)
    overlap = comm is not None and dist.is_available() and dist.is_initialized() and \
        dist.get_world_size(comm["group"]) > 1
    timing = overlap and comm.get("log") is not None
    events = [torch.cuda.Event(enable_timing=timing), torch.cuda.Event(enable_timing=timing)] if overlap else None
    if pw.fp32:
        g = ops.layer_backward_f32(gy.reshape(-1, gy.shape[-1]), sv["xin"], pw, sv, ctx.training_bn, eps,
                                   stage_events=events)
    else:
        # a bf16 input gets its gradient from the dx GEMM directly in bf16
        dx_dtype = torch.bfloat16 if ctx.x_dtype == torch.bfloat16 else torch.float32
        g = ops.layer_backward(gy.reshape(-1, gy.shape[-1]), sv["xin"], pw, sv, ctx.training_bn, eps,
                               stage_events=events, dx_dtype=dx_dtype)
    if overlap:
        _overlapped_allreduce(layer, g, events)
    params = ctx.params
    grads = [g["dx"].to(ctx.x_dtype)]
    dtypes = {p.dtype for p in params}
    if len(dtypes) == 1 and torch.float32 not in dtypes:
        # one conversion kernel for every parameter gradient
        conv = g["flat"].to(dtypes.pop())
        g = dict(g, **{name: conv[o:o + g[name].numel()].view(shp) for name, o, shp in g["layout"]})
    flat = [g["d_latents"], g["d_w1"], g["d_w2"]]
    flat += [g["d_wq"][h * dq:(h + 1) * dq] for h in range(H)]
    flat += [g["d_bn"][0, h * dq:(h + 1) * dq] for h in range(H)]
    flat += [g["d_bn"][1, h * dq:(h + 1) * dq] for h in range(H)]
    flat += [g["d_bn"][2, h * dq:(h + 1) * dq] for h in range(H)]
    flat += [g["d_keys"][0], g["d_keys"][1]]
    out = [grads[0], None, None]  # x, layer, need_grad (not tensors)
    for p, gp, need in zip(params, flat, ctx.needs_input_grad[3:]):
        out.append(gp.to(p.dtype).view_as(p) if need else None)
    ctx.saved = None
    return tuple(out)
