"""Shared test helpers: golden-fixture loading, oracle parameter building and
the parity comparators (relative-norm error, margin-aware id matching)."""

import os

import torch

from ethos_b200.config import EthosConfig, layer_dims
from ethos_b200.init import seeded_input, seeded_state_dict
from oracle import ethos_oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# state_dict name of each oracle parameter gradient
def grad_names(H):
    names = {"E": "expert_latents.weight", "W1": "generation_network.net.0.weight",
             "W2": "generation_network.net.2.weight", "K1": "router.sub_keys_1.weight",
             "K2": "router.sub_keys_2.weight"}
    for h in range(H):
        names[("Wq", h)] = f"router.query_projs.{h}.weight"
        names[("bq", h)] = f"router.query_projs.{h}.bias"
        names[("gamma", h)] = f"router.query_norms.{h}.weight"
        names[("beta", h)] = f"router.query_norms.{h}.bias"
    return names


def oracle_grads(p, H):
    """Map oracle parameter .grad tensors to state_dict names."""
    out = {}
    for key, name in grad_names(H).items():
        if isinstance(key, tuple):
            attr, h = key
            g = getattr(p, attr).grad
            out[name] = None if g is None else g[h]
        else:
            out[name] = getattr(p, key).grad
    return out


def load_golden(case):
    return torch.load(os.path.join(GOLDEN, f"golden_{case}.pt"), weights_only=False)


def reference_state_dict(rec):
    """State dict of a golden case: stored (small cases) or regenerated from
    the seed (checked against the stored checksum)."""
    if rec.get("full"):
        return rec["state_dict"]
    from ethos_b200.layer import EthosExpertLayer
    layer = EthosExpertLayer(EthosConfig(**rec["cfg"]))
    sd = seeded_state_dict(layer, seed=0)
    if rec.get("round_bf16"):
        sd = {k: (v.to(torch.bfloat16).float() if v.is_floating_point() else v) for k, v in sd.items()}
    for k, (s, ss) in rec["checksum"].items():
        v = sd[k].double()
        assert abs(v.sum().item() - s.item()) <= 1e-9 * max(1.0, abs(s.item())) + 1e-9, k
        assert abs((v * v).sum().item() - ss.item()) <= 1e-9 * max(1.0, ss.item()), k
    return sd


def golden_input(rec):
    if "x" in rec:
        return rec["x"]
    x = seeded_input(rec["tokens"], rec["cfg"]["d_model"], seed=0)
    if rec.get("round_bf16"):
        x = x.to(torch.bfloat16).float()
    return x


def dims_of(cfg):
    return layer_dims(EthosConfig(**cfg))


def rel_err(a, b):
    a = a.double()
    b = b.double()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def max_rel(a, b):
    """max |a-b| / max |b| (elementwise, normalised by the reference scale)."""
    a = a.double()
    b = b.double()
    den = b.abs().max().item()
    return (a - b).abs().max().item() / (den if den > 0 else 1.0)


def margin_mask(x, p, top_k, training=False, margin=1e-3):
    """Which (t, h, j) positions are decided by more than `margin` in the fp32
    oracle (the id parity rule: positions decided by a margin above 1e-3)."""
    qn, _ = orc.router_queries(x, p, training)
    v = orc.grid_top_scores(qn, p.K1, p.K2, top_k + 1)
    return orc.id_match_mask(v, top_k, margin)
