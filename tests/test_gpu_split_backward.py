"""GPU parity of the separate backward calls (ethos_expert_backward,
ethos_router_backward) -- the two halves of the layer's backward for a host
that routes with its own router, or runs only the router from this library.

Three checks: the two calls composed give what ethos_layer_backward gives; the
expert half alone matches autograd through the oracle's expert loop with the
routing weights as a leaf (model.py:306-336); the router half alone, after
ethos_router_forward, matches autograd through the oracle's router for a
given gradient of the routing weights (model.py:208-254).  Bar: 1e-2 relative
error (bf16), as for the whole layer."""

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
TOL = 1e-2


def _bf(t):
    return t.to(torch.bfloat16).to(torch.float32)


def _stats_state(sd, seed=11):
    g = torch.Generator().manual_seed(seed)
    for k in sd:
        if k.endswith("running_mean"):
            sd[k] = 0.1 * torch.randn(sd[k].shape, generator=g)
        elif k.endswith("running_var"):
            sd[k] = 0.5 + torch.rand(sd[k].shape, generator=g)
        elif ".query_norms." in k and k.endswith((".weight", ".bias")):
            sd[k] = (1.0 if k.endswith(".weight") else 0.0) + 0.1 * torch.randn(sd[k].shape, generator=g)
        elif ".query_projs." in k and k.endswith(".bias"):
            sd[k] = 0.1 * torch.randn(sd[k].shape, generator=g)
    return sd


def _setup(cfg, T, training, seed=3):
    layer = EthosExpertLayer(EthosConfig(**cfg))
    sd = _stats_state(seeded_state_dict(layer, seed=seed))
    layer.load_state_dict(sd)
    layer = layer.to("cuda", torch.bfloat16).train(training)
    pw = layer._packed(torch.device("cuda"))
    eps, mom = layer.router._bn_eps_momentum()
    x = _bf(seeded_input(T, cfg["d_model"], seed=21))
    gy = _bf(torch.randn((T, cfg["d_model"]), generator=tensor_generator(5, "gy")))
    return layer, sd, pw, eps, mom, x, gy


def _dhacc(gy16, pw, H):
    """dL/dhacc for y = hacc W_v^T / H (model.py:341)."""
    return (gy16.float() @ pw.wv.float()) / H


@pytest.mark.parametrize("cfg,T,training", [(CFG1, 256, False), (CFG1, 256, True), (CFG2, 1024, True)])
def test_split_backward_composes_to_layer_backward(cfg, T, training):
    _, _, pw, eps, mom, x, gy = _setup(cfg, T, training)
    d = pw.dims
    HQ = d["num_heads"] * d["d_query"]
    x16, gy16 = x.to("cuda", torch.bfloat16), gy.to("cuda", torch.bfloat16)
    sv = ops.layer_forward(x16, pw, training, eps, mom, save=True)
    whole = ops.layer_backward(gy16, x16, pw, sv, training, eps)

    e = ops.expert_backward(pw.latents, pw.w1, sv["ids"], sv["weights"], sv["xp"], sv["dot"],
                            _dhacc(gy16, pw, d["num_heads"]), d, sv.get("htab"), sv.get("gtab"))
    dx = e["dxp"] @ pw.w_cat[HQ:].float()
    r = ops.router_backward(e["d_weights"], x16, pw, sv["ids"], sv["weights"], sv["qpre"], training, eps,
                            save_bn=sv.get("bn_stats"), dx=dx)
    torch.cuda.synchronize()
    ops.check_device_error("cuda")
    assert r["dx"] is dx
    for name, got in (("d_latents", e["d_latents"]), ("d_w1", e["d_w1"]), ("d_wq", r["d_wq"]),
                      ("d_keys", r["d_keys"]), ("dx", r["dx"])):
        assert rel_err(got.cpu(), whole[name].cpu()) <= 2e-3, name
    # gamma and beta (the bias gradient is zero under batch statistics)
    rows = slice(0, 3) if not training else slice(1, 3)
    assert rel_err(r["d_bn"][rows].cpu(), whole["d_bn"][rows].cpu()) <= 2e-3
    if training:
        assert r["d_bn"][0].abs().max().item() <= 1e-6


@pytest.mark.parametrize("cfg,T", [(CFG1, 256), (CFG2, 1024)])
def test_expert_backward_matches_oracle(cfg, T):
    """Experts alone on the kernels' routing decisions, the routing weights a
    leaf: dL/d(weight), dE, dW1 and the experts' share of dx."""
    _, sd, pw, eps, mom, x, gy = _setup(cfg, T, False)
    d = pw.dims
    HQ = d["num_heads"] * d["d_query"]
    x16, gy16 = x.to("cuda", torch.bfloat16), gy.to("cuda", torch.bfloat16)
    sv = ops.layer_forward(x16, pw, False, eps, mom, save=True)
    hacc, dot = ops.expert_forward(pw.latents, pw.w1, sv["ids"], sv["weights"], sv["xp"], d, save_dot=True)
    e = ops.expert_backward(pw.latents, pw.w1, sv["ids"], sv["weights"], sv["xp"], dot,
                            _dhacc(gy16, pw, d["num_heads"]), d)
    dx_e = e["dxp"] @ pw.w_cat[HQ:].float()
    torch.cuda.synchronize()
    ops.check_device_error("cuda")

    p = orc.params_from_state_dict(sd, dims_of(cfg), round_bf16=True)
    p.requires_grad_(True)
    ids = sv["ids"].cpu().to(torch.int64)
    w = sv["weights"].cpu().clone().requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    y = orc.expert_forward(xr, w, ids, p)
    (y * gy).sum().backward()
    assert rel_err(e["d_weights"].cpu(), w.grad) <= TOL
    assert rel_err(e["d_latents"].cpu(), p.E.grad) <= TOL
    assert rel_err(e["d_w1"].cpu(), p.W1.grad) <= TOL
    assert rel_err(dx_e.cpu(), xr.grad) <= TOL


@pytest.mark.parametrize("cfg,T,training", [(CFG1, 256, False), (CFG1, 256, True), (CFG2, 1024, True)])
def test_router_backward_matches_oracle(cfg, T, training):
    """ethos_router_forward then ethos_router_backward for a seeded gradient
    of the routing weights: dx and every router parameter gradient."""
    layer, sd, pw, eps, mom, x, _ = _setup(cfg, T, training)
    d = pw.dims
    H, k, HQ = d["num_heads"], d["top_k"], d["num_heads"] * d["d_query"]
    x16 = x.to("cuda", torch.bfloat16)
    qpre = torch.empty((T, HQ), dtype=torch.float32, device="cuda")
    bn_stats = torch.empty((2, HQ), dtype=torch.float32, device="cuda") if training else None
    w16, ids16 = ops.router_forward(x16, pw, training, eps, mom, save_qpre=qpre, save_bn=bn_stats)
    dw = torch.randn((T, H, k), generator=tensor_generator(7, "dw"))
    r = ops.router_backward(dw.to("cuda"), x16, pw, ids16, w16, qpre, training, eps, save_bn=bn_stats)
    torch.cuda.synchronize()
    ops.check_device_error("cuda")

    p = orc.params_from_state_dict(sd, dims_of(cfg), round_bf16=True)
    ids = ids16.cpu().to(torch.int64)
    mask = orc.id_match_mask(orc.grid_top_scores(orc.router_queries(x, p, training)[0], p.K1, p.K2, k + 1), k)
    _, ids_ref, _ = orc.router_forward(x, p, k, training)
    assert torch.equal(ids[mask], ids_ref[mask])
    p.requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    w_ref, _ = orc.router_weights_given_ids(xr, p, ids, training)
    assert (w16.cpu() - w_ref.detach()).abs().max().item() <= 1e-5
    (w_ref * dw).sum().backward()
    assert rel_err(r["dx"].cpu(), xr.grad) <= TOL
    ref = oracle_grads(p, H)
    got = {}
    for h in range(H):
        got[f"router.query_projs.{h}.weight"] = r["d_wq"][h * d["d_query"]:(h + 1) * d["d_query"]]
        got[f"router.query_projs.{h}.bias"] = r["d_bn"][0, h * d["d_query"]:(h + 1) * d["d_query"]]
        got[f"router.query_norms.{h}.weight"] = r["d_bn"][1, h * d["d_query"]:(h + 1) * d["d_query"]]
        got[f"router.query_norms.{h}.bias"] = r["d_bn"][2, h * d["d_query"]:(h + 1) * d["d_query"]]
    got["router.sub_keys_1.weight"] = r["d_keys"][0]
    got["router.sub_keys_2.weight"] = r["d_keys"][1]
    for n, g in got.items():
        g_ref = ref[n]
        if training and "query_projs" in n and n.endswith(".bias"):
            assert g.abs().max().item() <= 1e-6, n  # the batch mean absorbs the bias
            continue
        assert rel_err(g.cpu(), g_ref) <= TOL, (n, rel_err(g.cpu(), g_ref))


@pytest.mark.parametrize("cfg,T,training", [(CFG1, 256, True), (CFG2, 1024, False)])
def test_layer_backward_bf16_dx_is_rounded_fp32_dx(cfg, T, training):
    """dx straight from the dx GEMM in bf16 (what the module uses for a bf16
    input) equals the fp32 dx rounded to bf16, bit for bit: the same GEMM and
    accumulation order, only the epilogue's store differs; the parameter
    gradients do not depend on dx's dtype (equal to fp32 rounding: the
    split-K weight-gradient GEMMs add their partials with fp32 atomics, whose
    order varies from run to run)."""
    _, _, pw, eps, mom, x, gy = _setup(cfg, T, training)
    x16, gy16 = x.to("cuda", torch.bfloat16), gy.to("cuda", torch.bfloat16)
    sv = ops.layer_forward(x16, pw, training, eps, mom, save=True)
    g32 = ops.layer_backward(gy16, x16, pw, sv, training, eps)
    g16 = ops.layer_backward(gy16, x16, pw, sv, training, eps, dx_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    ops.check_device_error("cuda")
    assert g16["dx"].dtype == torch.bfloat16
    assert torch.equal(g16["dx"], g32["dx"].to(torch.bfloat16))
    assert rel_err(g16["flat"], g32["flat"]) <= 1e-5
