"""Autograd backward of EthosExpertLayer.

Maps the gradients computed by ``ethos_layer_backward`` (one C-ABI call, see
include/ethos_b200.h) onto the inputs of ``_EthosLayerFunction``: x, the layer
and the need-grad flag (no gradients), then the parameters in the order of ``EthosExpertLayer._grad_params`` --
expert_latents, net.0, net.2, query_projs weights, query_projs biases,
query_norms weights, query_norms biases, sub_keys_1, sub_keys_2.
"""

import torch

from . import ops


def layer_backward(ctx, gy):
    layer = ctx.layer
    sv = ctx.saved
    pw = sv["pw"]
    H = layer.num_heads
    dq = layer.router.d_query
    eps, _ = layer.router._bn_eps_momentum()
    g = ops.layer_backward(gy.reshape(-1, gy.shape[-1]), sv["x16"], pw, sv, ctx.training_bn, eps)
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
