"""Drop-in ETHOS expert layer for B200.

``EthosExpertLayer`` has the constructor, forward signature, sub-module tree
and ``state_dict`` of the reference's ``SimplifiedHypernetMoE``
(model.py:267-343) and ``FusedLowRankMoE_Reordered`` (kernels.py:123-221):

    expert_latents.weight                      [N, dl]
    generation_network.net.0.weight            [dh, dl]
    generation_network.net.2.weight            [2d, dh]
    router.query_projs.{h}.{weight,bias}       [dq, d], [dq]
    router.query_norms.{h}.{weight,bias,running_mean,running_var,num_batches_tracked}
    router.sub_keys_1.weight, router.sub_keys_2.weight   [K, dq/2]

so reference checkpoints load unchanged.  Its forward runs entirely in the
sm_100a kernels of ``libethos_b200.so``; there is no CPU or eager fallback.
"""

import torch
import torch.nn as nn

from . import ops
from .config import layer_dims

__all__ = ["ExpertGenerationNetwork", "ProductKeyRouter", "EthosExpertLayer", "swap_expert_layers"]


class ExpertGenerationNetwork(nn.Module):
    """Hypernetwork parameters (model.py:168-179).  The expert layer slices
    ``net[0].weight`` and ``net[2].weight`` directly (model.py:297-300); this
    ``forward`` exists for API compatibility only."""

    def __init__(self, d_latent, d_model, d_intermediate):
        super().__init__()
        self.d_expert_params = 2 * d_model
        self.net = nn.Sequential(
            nn.Linear(d_latent, d_intermediate, bias=False),
            nn.GELU(),
            nn.Linear(d_intermediate, self.d_expert_params, bias=False),
        )

    def forward(self, latent_vector):
        return self.net(latent_vector)


class ProductKeyRouter(nn.Module):
    """Product-key router (model.py:182-254) with the reference parameters.

    ``forward(x_flat [T, d]) -> (scores [T, H, k] in x.dtype, indices [T, H, k]
    int64)``.  Scores are the fp32 softmax weights of the selected experts
    (model.py:234), cast to ``x.dtype`` as the reference does.  Called on its
    own the router is an inference op (its outputs carry no gradient); inside
    ``EthosExpertLayer`` the routing weights are differentiated through."""

    def __init__(self, config):
        super().__init__()
        dims = layer_dims(config)
        self.d_model = dims["d_model"]
        self.num_experts = dims["num_experts"]
        self.top_k = dims["top_k"]
        self.d_query = dims["d_query"]
        self.num_heads = dims["num_heads"]
        self.num_sub_keys = dims["num_sub_keys"]
        self.query_projs = nn.ModuleList([nn.Linear(self.d_model, self.d_query) for _ in range(self.num_heads)])
        self.query_norms = nn.ModuleList([nn.BatchNorm1d(self.d_query) for _ in range(self.num_heads)])
        self.sub_keys_1 = nn.Embedding(self.num_sub_keys, self.d_query // 2)
        self.sub_keys_2 = nn.Embedding(self.num_sub_keys, self.d_query // 2)

    # -- parameter packing ------------------------------------------------
    def _bn_block(self):
        """fp32 [5, H*dq]: bias, gamma, beta, running mean, running var."""
        parts = ([m.bias for m in self.query_projs] + [n.weight for n in self.query_norms]
                 + [n.bias for n in self.query_norms] + [n.running_mean for n in self.query_norms]
                 + [n.running_var for n in self.query_norms])
        return torch.cat([t.detach() for t in parts]).to(torch.float32).view(5, -1).contiguous()

    def _bn_eps_momentum(self):
        n0 = self.query_norms[0]
        for n in self.query_norms:
            if n.eps != n0.eps or n.momentum != n0.momentum:
                raise ValueError("all query_norms must share eps and momentum")
            if not (n.affine and n.track_running_stats):
                raise ValueError("query_norms must be affine with running statistics")
        if n0.momentum is None:
            raise ValueError("BatchNorm momentum=None (cumulative average) is not supported")
        return float(n0.eps), float(n0.momentum)

    def _bn_training(self):
        return self.training

    def _write_back_running(self, bn):
        """Copy the kernel-updated running statistics back into the buffers
        and count the batch, as BatchNorm1d.forward does in training mode."""
        dq = self.d_query
        H = self.num_heads
        with torch.no_grad():
            dst = [n.running_mean for n in self.query_norms] + [n.running_var for n in self.query_norms]
            src = [bn[3, h * dq:(h + 1) * dq] for h in range(H)] + [bn[4, h * dq:(h + 1) * dq] for h in range(H)]
            torch._foreach_copy_(dst, src)
            torch._foreach_add_([n.num_batches_tracked for n in self.query_norms], 1)

    def forward(self, x_flat):
        ops._require_cuda(x_flat, "x_flat")
        _check_token_count(x_flat.shape[0], self._bn_training(), self.d_query)
        layer = _RouterOnly(self)
        pw = layer.packed(x_flat.device)
        eps, mom = self._bn_eps_momentum()
        training = self._bn_training()
        if pw.fp32:
            x32 = x_flat.detach().to(torch.float32).contiguous()
            w, ids = ops.router_forward_f32(x32, pw, training, eps, mom)
        else:
            x16 = x_flat.detach().to(torch.bfloat16).contiguous()
            w, ids = ops.router_forward(x16, pw, training, eps, mom)
        if training:
            self._write_back_running(pw.bn)
        return w.to(x_flat.dtype), ids.to(torch.int64)


def _bf16(t):
    return t.detach().to(torch.bfloat16).contiguous()


def _f32(t):
    return t.detach().to(torch.float32).contiguous()


def _fp32_arithmetic(module):
    """The layer computes in fp32 when its parameters are fp32 (the
    reference's model.py:208-343 then runs in fp32 too); bf16 or fp16
    parameters select the bf16 tensor-core path."""
    return next(module.parameters()).dtype == torch.float32


def _check_token_count(tokens, bn_training, dq):
    """The reference's own failures for degenerate batches: an empty batch
    fails its ``view(T, -1)`` of the routing scores (model.py:222), and
    BatchNorm1d in training mode rejects a single token (model.py:216)."""
    if tokens == 0:
        raise RuntimeError("cannot route an empty batch (0 tokens)")
    if bn_training and tokens == 1:
        raise ValueError(f"Expected more than 1 value per channel when training, got input size "
                         f"torch.Size([1, {dq}])")


class _RouterOnly:
    """Packs just the router's weights (for ProductKeyRouter.forward)."""

    def __init__(self, router):
        self.router = router

    def packed(self, device):
        r = self.router
        dims = dict(d_model=r.d_model, num_experts=r.num_experts, num_sub_keys=r.num_sub_keys,
                    top_k=r.top_k, num_heads=r.num_heads, d_latent=128, d_hidden=512,
                    d_query=r.d_query)
        if _fp32_arithmetic(r):
            w_cat = torch.cat([_f32(m.weight) for m in r.query_projs], 0)
            return ops.PackedWeights(w_cat=w_cat, key_cat=_keys_f32(r), latents=None, w1=None, wv=None,
                                     bn=r._bn_block(), dims=dims, fp32=True)
        w_cat = torch.cat([_bf16(m.weight) for m in r.query_projs], 0)
        return ops.PackedWeights(w_cat=w_cat, key_cat=_key_cat(r), latents=None, w1=None, wv=None,
                                 bn=r._bn_block(), dims=dims)


def _keys_f32(router):
    """fp32 [2, K, dq/2]: sub_keys_1.weight, sub_keys_2.weight."""
    return torch.stack([_f32(router.sub_keys_1.weight), _f32(router.sub_keys_2.weight)]).contiguous()


def _key_cat(router):
    k1 = _bf16(router.sub_keys_1.weight)
    k2 = _bf16(router.sub_keys_2.weight)
    return torch.stack([torch.cat([k1, k1], 1), torch.cat([k2, k2], 1)]).contiguous()


class _EthosLayerFunction(torch.autograd.Function):
    """Autograd boundary around the fused forward (and backward) kernels."""

    @staticmethod
    def forward(ctx, x2d, layer, need_grad, *params):
        # need_grad is decided by the caller: inside Function.forward grad
        # mode is always off and needs_input_grad ignores torch.no_grad()
        pw = layer._packed(x2d.device, fresh=need_grad)
        eps, mom = layer.router._bn_eps_momentum()
        training = layer.router._bn_training()
        if pw.fp32:
            # fp32 arithmetic throughout (no expert-path choice, no cached table)
            xin = x2d.to(torch.float32).contiguous()
            out = ops.layer_forward_f32(xin, pw, training, eps, mom, save=need_grad)
        else:
            xin = x2d.to(torch.bfloat16).contiguous()
            htab = layer._expert_table() if (layer.cache_expert_table and not need_grad) else None
            out = ops.layer_forward(xin, pw, training, eps, mom, save=need_grad, path=layer.expert_path, htab=htab)
        if training:
            layer.router._write_back_running(pw.bn)
        ctx.layer = layer
        ctx.training_bn = training
        ctx.x_dtype = x2d.dtype
        ctx.params = params
        if need_grad:
            ctx.saved = dict(out, xin=xin, pw=pw)
        return out["y"].to(x2d.dtype)

    @staticmethod
    def backward(ctx, gy):
        from . import backward as bwd  # noqa: WPS433 (kept local: built after the forward)
        return bwd.layer_backward(ctx, gy)


class EthosExpertLayer(nn.Module):
    """B200 ETHOS expert layer; drop-in for ``SimplifiedHypernetMoE`` /
    ``FusedLowRankMoE_Reordered`` (same ``__init__(config)``, same
    ``forward(x [B, S, d_model]) -> [B, S, d_model]``, same state_dict)."""

    def __init__(self, config):
        super().__init__()
        dims = layer_dims(config)
        self.dims = dims
        self.d_model = dims["d_model"]
        self.num_experts = dims["num_experts"]
        self.top_k = dims["top_k"]
        self.num_heads = dims["num_heads"]
        self.d_latent = dims["d_latent"]
        self.d_hidden = dims["d_hidden"]
        self.expert_latents = nn.Embedding(dims["num_experts"], dims["d_latent"])
        self.generation_network = ExpertGenerationNetwork(dims["d_latent"], dims["d_model"], dims["d_hidden"])
        self.router = ProductKeyRouter(config)
        # expert execution path (ops.EXPERT_AUTO / EXPERT_FUSED / EXPERT_TABLE):
        # AUTO evaluates gelu(E @ W1^T) once per expert when a step makes at
        # least one selection per expert on average, else per selection
        self.expert_path = ops.EXPERT_AUTO
        # inference with frozen parameters: keep the expert table H =
        # gelu(E @ W1^T) (N x dh fp16, 256 MiB at 262 144 experts) across
        # forwards and gather from it; rebuilt whenever a weight changes
        # (storage or version counter), never used when gradients are needed
        self.cache_expert_table = False
        self._cache_key = None
        self._cache = None

    def _weight_params(self):
        r = self.router
        ps = [self.expert_latents.weight, self.generation_network.net[0].weight,
              self.generation_network.net[2].weight]
        ps += [m.weight for m in r.query_projs] + [r.sub_keys_1.weight, r.sub_keys_2.weight]
        return ps

    def invalidate_weight_cache(self):
        """Drop the derived kernel-layout weights (and the cached expert
        table).  Inference forwards reuse them while every parameter keeps its
        storage and version counter; a write through ``param.data`` (as
        DeepSpeed's optimizers do) bumps neither, so a caller that updates the
        parameters that way must call this before the next inference forward.
        Forwards that need gradients always re-pack and are unaffected."""
        self._cache_key = None
        self._cache = None

    def _packed(self, device, fresh=False):
        """Derived kernel-layout weights, cached while the parameters are
        unchanged (same storage and version counters).  ``fresh`` rebuilds
        them unconditionally (training forwards: the optimizer may have
        written the parameters in a way the version counters do not see)."""
        ps = self._weight_params()
        key = (str(device),) + tuple((p.data_ptr(), p._version, p.dtype) for p in ps)
        if fresh or key != self._cache_key:
            d = self.d_model
            r = self.router
            W2 = self.generation_network.net[2].weight
            if _fp32_arithmetic(self):
                w_cat = torch.cat([_f32(m.weight) for m in r.query_projs] + [_f32(W2[:d].t())], 0)
                self._cache = dict(w_cat=w_cat, key_cat=_keys_f32(r), latents=_f32(self.expert_latents.weight),
                                   w1=_f32(self.generation_network.net[0].weight), wv=_f32(W2[d:]), fp32=True)
            else:
                w_cat = torch.cat([_bf16(m.weight) for m in r.query_projs] + [_bf16(W2[:d].t())], 0)
                self._cache = dict(w_cat=w_cat, key_cat=_key_cat(r), latents=_bf16(self.expert_latents.weight),
                                   w1=_bf16(self.generation_network.net[0].weight), wv=_bf16(W2[d:]), fp32=False)
            self._cache_key = None if fresh else key
        c = self._cache
        r = self.router
        bn_src = [m.bias for m in r.query_projs]
        for n in r.query_norms:
            bn_src += [n.weight, n.bias, n.running_mean, n.running_var]
        bn_key = (str(device),) + tuple((t.data_ptr(), t._version) for t in bn_src)
        if fresh or r.training or c.get("bn_key") != bn_key:
            # training mode always gets a fresh block: the kernels update its
            # running-statistics rows in place
            c["bn"] = r._bn_block()
            c["bn_key"] = None if (fresh or r.training) else bn_key
        return ops.PackedWeights(w_cat=c["w_cat"], key_cat=c["key_cat"], latents=c["latents"], w1=c["w1"],
                                 wv=c["wv"], bn=c["bn"], dims=self.dims, fp32=c["fp32"])

    def _expert_table(self):
        """The cached expert table for the weights ``_packed`` last saw (its
        cache entry is replaced, and the table with it, when they change)."""
        c = self._cache
        if c.get("htab") is None:
            c["htab"], _ = ops.expert_table_build(c["latents"], c["w1"], self.dims)
        return c["htab"]

    def _grad_params(self):
        r = self.router
        ps = [self.expert_latents.weight, self.generation_network.net[0].weight,
              self.generation_network.net[2].weight]
        ps += [m.weight for m in r.query_projs] + [m.bias for m in r.query_projs]
        ps += [n.weight for n in r.query_norms] + [n.bias for n in r.query_norms]
        ps += [r.sub_keys_1.weight, r.sub_keys_2.weight]
        return ps

    def forward(self, x):
        ops._require_cuda(x, "x")
        batch_size, seq_len, d_model = x.shape
        x2d = x.reshape(-1, d_model)
        _check_token_count(x2d.shape[0], self.router._bn_training(), self.router.d_query)
        params = self._grad_params()
        need_grad = torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in params))
        y = _EthosLayerFunction.apply(x2d, self, need_grad, *params)
        return y.view(batch_size, seq_len, d_model)


def swap_expert_layers(model, config=None):
    """Replace every reference expert layer inside ``model`` (modules with
    ``expert_latents``, ``generation_network`` and ``router`` children, i.e.
    ``SimplifiedHypernetMoE`` / ``FusedLowRankMoE_Reordered``, the choice made
    at model.py:350-355) by an ``EthosExpertLayer`` carrying the same
    state_dict.  Returns the number of layers swapped."""
    swapped = 0
    for name, child in list(model.named_children()):
        if isinstance(child, EthosExpertLayer):
            continue
        if all(hasattr(child, a) for a in ("expert_latents", "generation_network", "router")):
            cfg = config or _config_from_layer(child)
            new = EthosExpertLayer(cfg)
            new.load_state_dict(child.state_dict())
            p = next(child.parameters())
            new.to(device=p.device, dtype=p.dtype)
            new.train(child.training)
            setattr(model, name, new)
            swapped += 1
        else:
            swapped += swap_expert_layers(child, config)
    return swapped


def _config_from_layer(layer):
    from .config import EthosConfig
    r = layer.router
    return EthosConfig(d_model=layer.d_model, num_experts=layer.num_experts, top_k=layer.top_k,
                       num_routing_heads=layer.num_heads, d_latent=layer.d_latent,
                       d_intermediate_hypernet=layer.d_hidden, d_query=r.d_query)
