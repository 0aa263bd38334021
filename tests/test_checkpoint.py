"""Checkpoint round trips: reference-format state dicts (pytorch_model.bin and
DeepSpeed directories) load into models with swapped Ethos layers and come back
out key for key and bit for bit."""

import os

import torch

from ethos_b200 import EthosConfig, EthosExpertLayer, swap_expert_layers
from ethos_b200.checkpoint import (expert_layer_prefixes, expert_layer_state, load_reference_state_dict,
                                   save_state_dict)
from ethos_b200.init import seeded_state_dict

TINY = dict(d_model=256, num_experts=64 * 64, top_k=16, num_routing_heads=8, d_latent=128,
            d_intermediate_hypernet=512, d_query=64)


class _RefLikeLayer(torch.nn.Module):
    """Same children as the reference SimplifiedHypernetMoE."""

    def __init__(self, cfg):
        super().__init__()
        src = EthosExpertLayer(cfg)
        self.expert_latents, self.generation_network, self.router = (src.expert_latents, src.generation_network,
                                                                     src.router)
        self.d_model, self.num_experts, self.top_k = src.d_model, src.num_experts, src.top_k
        self.num_heads, self.d_latent, self.d_hidden = src.num_heads, src.d_latent, src.d_hidden


def _decoder(cfg, layers=2):
    """A stand-in for CompressedMoEModel's module tree: layers.{i}.mlp + extras."""
    m = torch.nn.Module()
    m.embed = torch.nn.Embedding(11, cfg.d_model)
    m.layers = torch.nn.ModuleList()
    for _ in range(layers):
        blk = torch.nn.Module()
        blk.norm = torch.nn.LayerNorm(cfg.d_model)
        blk.mlp = _RefLikeLayer(cfg)
        m.layers.append(blk)
    return m


def _seeded(model, seed):
    sd = model.state_dict()
    for i, blk in enumerate(model.layers):
        for k, v in seeded_state_dict(EthosExpertLayer(EthosConfig(**TINY)), seed=seed + i).items():
            sd[f"layers.{i}.mlp.{k}"] = v
    model.load_state_dict(sd)
    return sd


def test_pytorch_model_bin_round_trip(tmp_path):
    cfg = EthosConfig(**TINY)
    ref = _decoder(cfg)
    sd = _seeded(ref, 5)
    path = os.path.join(tmp_path, "pytorch_model.bin")
    torch.save(sd, path)

    ours = _decoder(cfg)
    assert swap_expert_layers(ours) == 2
    ours.load_state_dict(load_reference_state_dict(path))
    assert all(isinstance(b.mlp, EthosExpertLayer) for b in ours.layers)
    out = os.path.join(tmp_path, "out.bin")
    save_state_dict(ours, out)
    back = torch.load(out, weights_only=True)
    assert set(back) == set(sd)
    for k in sd:
        assert torch.equal(back[k], sd[k]), k
    # and the saved file loads into the reference-shaped model again
    again = _decoder(cfg)
    again.load_state_dict(back)


def test_deepspeed_directory(tmp_path):
    cfg = EthosConfig(**TINY)
    ref = _decoder(cfg, layers=1)
    sd = _seeded(ref, 9)
    tag_dir = os.path.join(tmp_path, "global_step7")
    os.makedirs(tag_dir)
    torch.save({"module": sd, "global_steps": 7}, os.path.join(tag_dir, "mp_rank_00_model_states.pt"))
    with open(os.path.join(tmp_path, "latest"), "w") as f:
        f.write("global_step7")
    got = load_reference_state_dict(str(tmp_path))
    assert set(got) == set(sd)
    assert expert_layer_prefixes(got) == ["layers.0.mlp."]
    layer = EthosExpertLayer(cfg)
    layer.load_state_dict(expert_layer_state(got, "layers.0.mlp."))
    for k, v in layer.state_dict().items():
        assert torch.equal(v, sd["layers.0.mlp." + k])
