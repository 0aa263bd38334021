"""GPU parity of the backward kernels against autograd through the CPU oracle.

The oracle runs the reference math in fp32 on the bf16-rounded parameters and
inputs, with the expert selection fixed to the ids the kernels chose (near-tie
ids are excluded from parity by the margin rule; fixing them keeps gradient
comparisons independent of that choice).  Bar: every gradient tensor within
1e-2 relative error (bf16), plus the ids themselves under the margin rule."""

import pytest
import torch

from ethos_b200 import EthosConfig, EthosExpertLayer, ops
from ethos_b200.init import seeded_input, seeded_state_dict, tensor_generator
from helpers import dims_of, oracle_grads, rel_err
from oracle import ethos_oracle as orc

pytestmark = pytest.mark.gpu

CFG1 = dict(d_model=512, num_experts=4096, top_k=16, num_routing_heads=8, d_latent=128,
            d_intermediate_hypernet=512, d_query=512)
CFG2 = dict(d_model=1024, num_experts=512 * 512, top_k=16, num_routing_heads=8, d_latent=128,
            d_intermediate_hypernet=512, d_query=512)
# few selections per token: R = 4 runs the double-buffered backward gather,
# R = 8 the single-buffered one at its smallest safe batch count
CFG_R4 = dict(CFG1, top_k=4, num_routing_heads=1)
CFG_R8 = dict(CFG1, top_k=4, num_routing_heads=2)


def _bf(t):
    return t.to(torch.bfloat16).to(torch.float32)


def _stats_state(sd, seed=11):
    g = torch.Generator().manual_seed(seed)
    for k in sd:
        if k.endswith("running_mean"):
            sd[k] = 0.1 * torch.randn(sd[k].shape, generator=g)
        elif k.endswith("running_var"):
            sd[k] = 0.5 + torch.rand(sd[k].shape, generator=g)
        elif ".query_norms." in k and k.endswith(".weight"):
            sd[k] = 1.0 + 0.1 * torch.randn(sd[k].shape, generator=g)
        elif ".query_norms." in k and k.endswith(".bias"):
            sd[k] = 0.1 * torch.randn(sd[k].shape, generator=g)
        elif ".query_projs." in k and k.endswith(".bias"):
            sd[k] = 0.1 * torch.randn(sd[k].shape, generator=g)
    return sd


def _grad_tol(name):
    return 1e-2


@pytest.mark.parametrize("cfg,T,training", [(CFG1, 256, False), (CFG1, 256, True), (CFG2, 512, True),
                                            (CFG2, 1024, False), (CFG2, 2048, True), (CFG_R4, 300, True),
                                            (CFG_R8, 300, False),
                                            # ragged token counts (fused path below N / (H k) tokens,
                                            # the table path above) and the smallest training batches
                                            (CFG1, 1, False), (CFG1, 7, False), (CFG1, 2, True),
                                            (CFG1, 3, True), (CFG1, 131, True)])
def test_layer_backward_matches_oracle(cfg, T, training):
    layer = EthosExpertLayer(EthosConfig(**cfg))
    sd = _stats_state(seeded_state_dict(layer, seed=3))
    layer.load_state_dict(sd)
    layer = layer.to("cuda", torch.bfloat16).train(training)
    dims = dims_of(cfg)
    p = orc.params_from_state_dict(sd, dims, round_bf16=True)
    x = _bf(seeded_input(T, cfg["d_model"], seed=21))
    gy = _bf(torch.randn((T, cfg["d_model"]), generator=tensor_generator(5, "gy")))

    # the kernels' routing decisions for this input (same deterministic kernels)
    pw = layer._packed(torch.device("cuda"))
    eps, mom = layer.router._bn_eps_momentum()
    ids = ops.layer_forward(x.to("cuda", torch.bfloat16), pw, training, eps, mom)["ids"].cpu().to(torch.int64)
    layer.load_state_dict({k: v.to(torch.bfloat16) if v.is_floating_point() else v for k, v in sd.items()})

    xg = x.to("cuda", torch.bfloat16).requires_grad_(True)
    y = layer(xg.view(1, T, -1)).view(T, -1)
    y.backward(gy.to("cuda", torch.bfloat16))
    torch.cuda.synchronize()
    ops.check_device_error("cuda")

    # ids parity under the margin rule
    qn, _ = orc.router_queries(x, p, training)
    mask = orc.id_match_mask(orc.grid_top_scores(qn, p.K1, p.K2, cfg["top_k"] + 1), cfg["top_k"])
    _, ids_ref, _ = orc.router_forward(x, p, cfg["top_k"], training)
    assert torch.equal(ids[mask], ids_ref[mask])

    p.requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    y_ref, _, _ = orc.layer_forward_given_ids(xr, p, ids, training)
    assert rel_err(y.detach().float().cpu(), y_ref.detach()) <= 1e-2
    (y_ref * gy).sum().backward()

    assert rel_err(xg.grad.float().cpu(), xr.grad) <= 1e-2, "x"
    ref = oracle_grads(p, dims["num_heads"])
    named = dict(layer.named_parameters())
    for n, g_ref in ref.items():
        g = named[n].grad
        assert g is not None, n
        g = g.float().cpu()
        scale = g_ref.double().norm().item()
        err = (g.double() - g_ref.double()).norm().item()
        if training and n.endswith(".bias") and "query_projs" in n:
            # exactly zero in training-mode BatchNorm (the batch mean absorbs it)
            assert g.abs().max().item() <= 1e-6, n
            continue
        assert err <= _grad_tol(n) * scale + 1e-6, (n, err / max(scale, 1e-30))


def test_backward_training_step_changes_loss():
    """One SGD step with the kernel gradients lowers a quadratic loss."""
    cfg = CFG1
    layer = EthosExpertLayer(EthosConfig(**cfg))
    layer.load_state_dict(seeded_state_dict(layer, seed=9))
    layer = layer.to("cuda", torch.float32).train()
    T = 512
    x = seeded_input(T, cfg["d_model"], seed=2).to("cuda")
    target = torch.zeros(T, cfg["d_model"], device="cuda")

    def loss_fn():
        return ((layer(x.view(1, T, -1)).view(T, -1) - target) ** 2).mean()

    l0 = loss_fn()
    l0.backward()
    with torch.no_grad():
        for prm in layer.parameters():
            if prm.grad is not None:
                prm -= 50.0 * prm.grad
    l1 = loss_fn()
    assert l1.item() < l0.item()
