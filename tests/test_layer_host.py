"""Host-side checks of the drop-in module: constructor arguments, sub-module
tree and state_dict identical to the reference (model.py:267-286,
kernels.py:130-143), reference checkpoints load, layer swapping, and no
silent CPU path."""

import os
import sys

import pytest
import torch

from ethos_b200 import EthosConfig, EthosExpertLayer, swap_expert_layers
from ethos_b200.init import seeded_state_dict
from helpers import load_golden

TINY = dict(d_model=256, num_experts=64 * 64, top_k=16, num_routing_heads=8, d_latent=128,
            d_intermediate_hypernet=512, d_query=64)


def _expected_keys(cfg):
    H = cfg["num_routing_heads"]
    keys = {"expert_latents.weight": (cfg["num_experts"], cfg["d_latent"]),
            "generation_network.net.0.weight": (cfg["d_intermediate_hypernet"], cfg["d_latent"]),
            "generation_network.net.2.weight": (2 * cfg["d_model"], cfg["d_intermediate_hypernet"]),
            "router.sub_keys_1.weight": (int(cfg["num_experts"] ** 0.5), cfg["d_query"] // 2),
            "router.sub_keys_2.weight": (int(cfg["num_experts"] ** 0.5), cfg["d_query"] // 2)}
    for h in range(H):
        keys[f"router.query_projs.{h}.weight"] = (cfg["d_query"], cfg["d_model"])
        keys[f"router.query_projs.{h}.bias"] = (cfg["d_query"],)
        for n in ("weight", "bias", "running_mean", "running_var"):
            keys[f"router.query_norms.{h}.{n}"] = (cfg["d_query"],)
        keys[f"router.query_norms.{h}.num_batches_tracked"] = ()
    return keys


def test_state_dict_layout_matches_reference():
    layer = EthosExpertLayer(EthosConfig(**TINY))
    sd = layer.state_dict()
    exp = _expected_keys(TINY)
    assert set(sd) == set(exp)
    for k, shape in exp.items():
        assert tuple(sd[k].shape) == shape, k


def test_reads_reference_config_object():
    class Cfg:  # attribute bag like train.Config
        pass
    c = Cfg()
    for k, v in TINY.items():
        setattr(c, k, v)
    layer = EthosExpertLayer(c)
    assert layer.router.num_sub_keys == 64 and layer.top_k == 16 and layer.num_heads == 8


def test_rejects_non_square_experts():
    with pytest.raises(ValueError):
        EthosExpertLayer(EthosConfig(**dict(TINY, num_experts=1000)))


def test_golden_state_dict_loads():
    rec = load_golden("small")
    layer = EthosExpertLayer(EthosConfig(**rec["cfg"]))
    layer.load_state_dict(rec["state_dict"])
    for k, v in rec["state_dict"].items():
        assert torch.equal(layer.state_dict()[k], v)


def test_seeded_init_matches_reference_module_when_available():
    ref_dir = os.environ.get("ETHOS_REFERENCE")
    if not ref_dir or not os.path.exists(os.path.join(ref_dir, "model.py")):
        pytest.skip("ETHOS_REFERENCE does not name a reference checkout")
    sys.path.insert(0, ref_dir)
    try:
        import model as ref_model
    finally:
        sys.path.remove(ref_dir)
    cfg = EthosConfig(**TINY)
    ref = ref_model.SimplifiedHypernetMoE(cfg)
    ours = EthosExpertLayer(cfg)
    assert set(ref.state_dict()) == set(ours.state_dict())
    for k, v in ref.state_dict().items():
        assert tuple(v.shape) == tuple(ours.state_dict()[k].shape), k
    a, b = seeded_state_dict(ref), seeded_state_dict(ours)
    for k in a:
        assert torch.equal(a[k], b[k])


def test_swap_expert_layers_moves_state():
    class FakeRefLayer(torch.nn.Module):  # same children as SimplifiedHypernetMoE
        def __init__(self, cfg):
            super().__init__()
            src = EthosExpertLayer(cfg)
            self.expert_latents = src.expert_latents
            self.generation_network = src.generation_network
            self.router = src.router
            self.d_model, self.num_experts, self.top_k = src.d_model, src.num_experts, src.top_k
            self.num_heads, self.d_latent, self.d_hidden = src.num_heads, src.d_latent, src.d_hidden

    cfg = EthosConfig(**TINY)
    block = torch.nn.Module()
    block.mlp = FakeRefLayer(cfg)
    before = {k: v.clone() for k, v in block.mlp.state_dict().items()}
    assert swap_expert_layers(block) == 1
    assert isinstance(block.mlp, EthosExpertLayer)
    for k, v in block.mlp.state_dict().items():
        assert torch.equal(v, before[k])


def test_forward_refuses_cpu_tensors():
    layer = EthosExpertLayer(EthosConfig(**TINY))
    with pytest.raises(RuntimeError, match="no CPU path"):
        layer(torch.zeros(1, 4, TINY["d_model"]))
    with pytest.raises(RuntimeError, match="no CPU path"):
        layer.router(torch.zeros(4, TINY["d_model"]))


def test_degenerate_batches_fail_like_the_reference():
    """An empty batch and a single token under training-mode BatchNorm are
    errors in the reference (its view(T, -1) and BatchNorm1d); the layer
    raises the same exception types before any kernel runs."""
    from ethos_b200.layer import _check_token_count
    with pytest.raises(RuntimeError):
        _check_token_count(0, False, 512)
    with pytest.raises(RuntimeError):
        _check_token_count(0, True, 512)
    with pytest.raises(ValueError, match="Expected more than 1 value per channel when training"):
        _check_token_count(1, True, 512)
    _check_token_count(1, False, 512)
    _check_token_count(2, True, 512)
