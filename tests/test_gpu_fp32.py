"""fp32 arithmetic: a layer whose parameters are fp32 computes in fp32 (split-
bf16 tensor-core products, fp32 everywhere else) and meets the 1e-4 bar.

Against the oracle in fp32 on the SAME (unrounded) fp32 parameters and inputs,
and against the reference's own fp32 outputs and gradients recorded in
tests/golden/golden_cfg1.pt (SimplifiedHypernetMoE, model.py:208-343):
outputs and every gradient within 1e-4 relative error (norm-wise); routing
weights within 2e-5; ids identical wherever the top-k margin exceeds 1e-3."""

import pytest
import torch

from ethos_b200 import EthosConfig, EthosExpertLayer, ops
from ethos_b200.init import seeded_input, seeded_state_dict, tensor_generator
from golden.make_golden import sample_idx
from helpers import dims_of, golden_input, load_golden, margin_mask, oracle_grads, reference_state_dict, rel_err
from oracle import ethos_oracle as orc

pytestmark = pytest.mark.gpu

CFG1 = dict(d_model=512, num_experts=4096, top_k=16, num_routing_heads=8, d_latent=128,
            d_intermediate_hypernet=512, d_query=512)
CFG2 = dict(d_model=1024, num_experts=512 * 512, top_k=16, num_routing_heads=8, d_latent=128,
            d_intermediate_hypernet=512, d_query=512)
TOL = 1e-4


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


def _layer(cfg, sd, training):
    layer = EthosExpertLayer(EthosConfig(**cfg))
    layer.load_state_dict(sd)
    return layer.to("cuda", torch.float32).train(training)


def _run(layer, x, gy):
    T = x.shape[0]
    xg = x.to("cuda").requires_grad_(True)
    y = layer(xg.view(1, T, -1)).view(T, -1)
    assert y.dtype == torch.float32
    y.backward(gy.to("cuda"))
    torch.cuda.synchronize()
    ops.check_device_error("cuda")
    grads = {n: p.grad.detach().cpu() for n, p in layer.named_parameters()}
    return y.detach().cpu(), xg.grad.detach().cpu(), grads


def _kernel_ids(layer, x, training):
    pw = layer._packed(torch.device("cuda"), fresh=True)
    eps, mom = layer.router._bn_eps_momentum()
    out = ops.layer_forward_f32(x.to("cuda"), pw, training, eps, mom)
    return out["ids"].cpu().to(torch.int64), out["weights"].cpu()


@pytest.mark.parametrize("cfg,T,training", [(CFG1, 256, False), (CFG1, 256, True), (CFG2, 512, True)])
def test_fp32_layer_matches_oracle(cfg, T, training):
    sd = _stats_state(seeded_state_dict(EthosExpertLayer(EthosConfig(**cfg)), seed=3))
    dims = dims_of(cfg)
    p = orc.params_from_state_dict(sd, dims)
    x = seeded_input(T, cfg["d_model"], seed=21)
    gy = torch.randn((T, cfg["d_model"]), generator=tensor_generator(5, "gy"))
    ids, w = _kernel_ids(_layer(cfg, sd, training), x, training)
    layer = _layer(cfg, sd, training)
    y, dx, grads = _run(layer, x, gy)

    # routing: ids under the margin rule, fp32 weights on rows with equal ids
    w_ref, ids_ref, stats = orc.router_forward(x, p, cfg["top_k"], training)
    mask = margin_mask(x, p, cfg["top_k"], training)
    assert torch.equal(ids[mask], ids_ref[mask])
    row_ok = (ids == ids_ref).all(-1)
    assert row_ok.float().mean().item() > 0.99
    assert (w[row_ok] - w_ref[row_ok]).abs().max().item() <= 2e-5
    if training:  # running statistics written back into the buffers
        rm = torch.stack([n.running_mean.cpu() for n in layer.router.query_norms])
        rv = torch.stack([n.running_var.cpu() for n in layer.router.query_norms])
        assert rel_err(rm, stats[0]) <= TOL and rel_err(rv, stats[1]) <= TOL

    # output and every gradient, on the kernels' routing decisions
    p.requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    y_ref, _, _ = orc.layer_forward_given_ids(xr, p, ids, training)
    assert rel_err(y, y_ref.detach()) <= TOL
    (y_ref * gy).sum().backward()
    assert rel_err(dx, xr.grad) <= TOL, "x"
    for n, g_ref in oracle_grads(p, dims["num_heads"]).items():
        if training and "query_projs" in n and n.endswith(".bias"):
            assert grads[n].abs().max().item() <= 1e-6, n  # exactly zero under batch statistics
            continue
        assert rel_err(grads[n], g_ref) <= TOL, (n, rel_err(grads[n], g_ref))


def test_fp32_router_alone_matches_oracle():
    cfg = CFG1
    sd = _stats_state(seeded_state_dict(EthosExpertLayer(EthosConfig(**cfg)), seed=4))
    p = orc.params_from_state_dict(sd, dims_of(cfg))
    layer = _layer(cfg, sd, False)
    x = seeded_input(300, cfg["d_model"], seed=8)
    with torch.no_grad():
        scores, ids = layer.router(x.cuda())
    assert scores.dtype == torch.float32 and ids.dtype == torch.int64
    w_ref, ids_ref, _ = orc.router_forward(x, p, cfg["top_k"], False)
    mask = margin_mask(x, p, cfg["top_k"])
    ids = ids.cpu()
    assert torch.equal(ids[mask], ids_ref[mask])
    row_ok = (ids == ids_ref).all(-1)
    assert (scores.cpu()[row_ok] - w_ref[row_ok]).abs().max().item() <= 2e-5


def test_fp32_layer_matches_reference_golden_config1():
    """The reference's own fp32 forward (256 tokens, eval) and gradients
    (32 tokens, BatchNorm in training and in eval mode)."""
    rec = load_golden("cfg1")
    cfg = rec["cfg"]
    sd = reference_state_dict(rec)
    p = orc.params_from_state_dict(sd, dims_of(cfg))
    x = golden_input(rec)
    layer = _layer(cfg, sd, False)
    with torch.no_grad():
        y = layer(x.cuda().view(2, -1, cfg["d_model"])).view(rec["tokens"], -1).cpu()
        scores, ids = layer.router(x.cuda())
    ref = rec["eval"]
    ids = ids.cpu().to(torch.int32)
    mask = margin_mask(x, p, cfg["top_k"])
    assert torch.equal(ids[mask], ref["ids"][mask])
    rows = (ids == ref["ids"]).all(-1).all(-1)
    assert rows.float().mean().item() > 0.95
    assert rel_err(y[rows], ref["y"][rows]) <= TOL
    row_h = (ids == ref["ids"]).all(-1)
    assert (scores.cpu()[row_h] - ref["scores"][row_h]).abs().max().item() <= 2e-5

    compared = 0
    for mode in ("train", "eval_bwd"):
        e = rec[mode]
        Tb = e["tokens"]
        training = mode == "train"
        layer = _layer(cfg, sd, training)
        kids, _ = _kernel_ids(_layer(cfg, sd, training), x[:Tb], training)
        yb, dx, grads = _run(layer, x[:Tb], e["upstream"])
        _, ref_ids, _ = orc.router_forward(x[:Tb], p, cfg["top_k"], training)
        if not torch.equal(kids, ref_ids):
            # a near-tie decided differently: the reference's gradients belong
            # to other ids; check the decided positions and move on
            assert torch.equal(kids[margin_mask(x[:Tb], p, cfg["top_k"], training)],
                               ref_ids[margin_mask(x[:Tb], p, cfg["top_k"], training)])
            continue
        assert rel_err(yb, e["y"]) <= TOL, mode
        assert rel_err(dx, e["x_grad"]) <= TOL, mode
        for n, g_ref in e["grads"].items():
            if training and "query_projs" in n and n.endswith(".bias"):
                continue  # zero up to rounding under batch statistics
            assert rel_err(grads[n], g_ref) <= TOL, (mode, n)
        for n, s in e["grads_sampled"].items():
            g = grads[n]
            assert abs(g.double().norm().item() - s["norm"]) <= TOL * s["norm"], (mode, n)
            idx = sample_idx(g.numel(), n)
            assert rel_err(g.flatten()[idx], s["vals"]) <= 5 * TOL, (mode, n)
        compared += 1
    assert compared >= 1, "both backward cases met a near-tie; nothing was compared"


@pytest.mark.parametrize("T,training", [(1, False), (7, False), (131, False), (2, True), (3, True), (131, True)])
def test_fp32_ragged_token_counts(T, training):
    """Token counts that fill no tile (1, 7, 131) and the smallest batches
    training-mode BatchNorm accepts (2, 3): output and every gradient at 1e-4.

    The small training batches are the ill-conditioned case: a column whose
    tokens nearly agree normalises through their difference, which amplifies
    an error in the projection by up to 1 / (2 sqrt(eps)).  A hi/lo split
    projection (error near 2^-16) misses the bar there by 10x (dx 1.0e-3 at
    T = 2, 1.2e-4 at T = 3); the six-product projection holds fp32's own
    error (1.6e-5 and 7e-7 against an fp64 evaluation)."""
    cfg = CFG1
    sd = _stats_state(seeded_state_dict(EthosExpertLayer(EthosConfig(**cfg)), seed=6))
    dims = dims_of(cfg)
    p = orc.params_from_state_dict(sd, dims)
    x = seeded_input(T, cfg["d_model"], seed=40 + T)
    gy = torch.randn((T, cfg["d_model"]), generator=tensor_generator(T, "gy"))
    ids, _ = _kernel_ids(_layer(cfg, sd, training), x, training)
    y, dx, grads = _run(_layer(cfg, sd, training), x, gy)
    p.requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    y_ref, _, _ = orc.layer_forward_given_ids(xr, p, ids, training)
    assert rel_err(y, y_ref.detach()) <= TOL
    (y_ref * gy).sum().backward()
    assert rel_err(dx, xr.grad) <= TOL, rel_err(dx, xr.grad)
    for n, g_ref in oracle_grads(p, dims["num_heads"]).items():
        if training and "query_projs" in n and n.endswith(".bias"):
            continue  # zero up to rounding under batch statistics
        assert rel_err(grads[n], g_ref) <= TOL, (n, rel_err(grads[n], g_ref))
