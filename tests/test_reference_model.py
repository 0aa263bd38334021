"""The plug point in the reference's own decoder (CompressedMoEModel,
model.py:345-395).

* Always (CPU): the oracle reproduces the expert-layer outputs recorded inside
  the reference decoder's forward (tests/golden/golden_model.pt, made by
  tests/golden/make_golden.py from the reference's model.py).
* With a reference checkout named by ETHOS_REFERENCE (CPU, skipped
  otherwise): ``swap_expert_layers`` on a real ``CompressedMoEModel`` replaces
  exactly its expert layers and keeps every state_dict entry, tied
  ``tok_embeddings`` / ``output`` weights included; the swapped model's
  checkpoints (``pytorch_model.bin`` and a DeepSpeed directory) load back into
  a fresh reference model and vice versa.
* GPU: the swapped layers, fed the recorded inputs, give the reference
  decoder's recorded expert-layer outputs (bf16 compute, 1e-2) and routing
  (margin rule)."""

import os
import sys

import pytest
import torch

from ethos_b200 import EthosConfig, EthosExpertLayer, swap_expert_layers
from ethos_b200.checkpoint import expert_layer_prefixes, expert_layer_state, load_reference_state_dict, \
    save_state_dict
from ethos_b200.init import seeded_state_dict
from helpers import dims_of, load_golden, rel_err
from oracle import ethos_oracle as orc

LAYER_KEYS = ("d_model", "num_experts", "top_k", "num_routing_heads", "d_latent", "d_intermediate_hypernet",
              "d_query")


def _layer_cfg(model_cfg):
    return {k: model_cfg[k] for k in LAYER_KEYS}


def _rounded_state(cfg, seed):
    layer = EthosExpertLayer(EthosConfig(**cfg))
    sd = seeded_state_dict(layer, seed=seed)
    return {k: (v.to(torch.bfloat16).float() if v.is_floating_point() else v) for k, v in sd.items()}


def test_oracle_matches_reference_decoder_golden():
    rec = load_golden("model")
    cfg = _layer_cfg(rec["model_cfg"])
    assert len(rec["layers"]) == rec["model_cfg"]["num_layers"] - rec["model_cfg"]["num_dense_layers"]
    for entry in rec["layers"]:
        p = orc.params_from_state_dict(_rounded_state(cfg, entry["seed"]), dims_of(cfg))
        y, w, ids, _ = orc.layer_forward(entry["x"], p, cfg["top_k"])
        mask = orc.id_match_mask(orc.grid_top_scores(orc.router_queries(entry["x"], p)[0], p.K1, p.K2,
                                                     cfg["top_k"] + 1), cfg["top_k"])
        assert torch.equal(ids[mask], entry["ids"].to(torch.int64)[mask]), entry["prefix"]
        assert rel_err(y, entry["y"]) <= 1e-5, entry["prefix"]
        assert (w - entry["scores"]).abs().max().item() <= 1e-5


# ------------------------------------------------ the reference's own model --
class _Cfg:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def _reference_model_module():
    ref_dir = os.environ.get("ETHOS_REFERENCE")
    if not ref_dir or not os.path.exists(os.path.join(ref_dir, "model.py")):
        pytest.skip("ETHOS_REFERENCE does not name a reference checkout")
    sys.path.insert(0, ref_dir)
    try:
        import model as ref_model
    finally:
        sys.path.remove(ref_dir)
    return ref_model


def _reference_decoder(ref_model, seed=0):
    cfg = _Cfg(**load_golden("model")["model_cfg"])
    torch.manual_seed(seed)
    return ref_model.CompressedMoEModel(cfg), cfg


def test_swap_expert_layers_in_reference_decoder():
    ref_model = _reference_model_module()
    model, cfg = _reference_decoder(ref_model)
    before = {k: v.detach().clone() for k, v in model.state_dict().items()}
    n = swap_expert_layers(model)
    assert n == cfg.num_layers - cfg.num_dense_layers
    for i, blk in enumerate(model.layers):
        if i < cfg.num_dense_layers:
            assert isinstance(blk.mlp, ref_model.FFN)
        else:
            assert isinstance(blk.mlp, EthosExpertLayer)
            assert isinstance(blk.self_attn, ref_model.DeepseekV3Attention)  # the rest is untouched
    after = model.state_dict()
    assert set(after) == set(before)
    for k, v in before.items():
        assert torch.equal(after[k], v), k
    # the embedding and the output head stay one tensor (model.py:382)
    assert model.tok_embeddings.weight is model.output.weight
    assert swap_expert_layers(model) == 0  # idempotent
    assert expert_layer_prefixes(after) == [f"layers.{i}.mlp." for i in range(cfg.num_dense_layers, cfg.num_layers)]


def test_checkpoints_cross_between_reference_and_swapped_decoder(tmp_path):
    ref_model = _reference_model_module()
    ours, cfg = _reference_decoder(ref_model, seed=1)
    swap_expert_layers(ours)
    with torch.no_grad():  # make the expert layers distinguishable from a fresh init
        for i, blk in enumerate(ours.layers):
            if i >= cfg.num_dense_layers:
                blk.mlp.load_state_dict(seeded_state_dict(blk.mlp, seed=100 + i))
        ours.output.weight.mul_(2.0)
    # swapped model -> pytorch_model.bin -> the reference model
    path = tmp_path / "pytorch_model.bin"
    save_state_dict(ours, str(path))
    fresh, _ = _reference_decoder(ref_model, seed=2)
    fresh.load_state_dict(load_reference_state_dict(str(path)))
    sd_ours, sd_fresh = ours.state_dict(), fresh.state_dict()
    for k, v in sd_ours.items():
        assert torch.equal(sd_fresh[k], v), k
    assert fresh.tok_embeddings.weight is fresh.output.weight
    assert torch.equal(fresh.tok_embeddings.weight, ours.output.weight)
    # a DeepSpeed checkpoint directory of the reference model -> a swapped model
    tag = tmp_path / "ds" / "global_step7"
    tag.mkdir(parents=True)
    torch.save({"module": fresh.state_dict()}, str(tag / "mp_rank_00_model_states.pt"))
    (tmp_path / "ds" / "latest").write_text("global_step7")
    back, _ = _reference_decoder(ref_model, seed=3)
    swap_expert_layers(back)
    back.load_state_dict(load_reference_state_dict(str(tmp_path / "ds")))
    for k, v in back.state_dict().items():
        assert torch.equal(sd_ours[k], v), k
    # one expert layer's entries, relative to the layer
    pre = f"layers.{cfg.num_dense_layers}.mlp."
    layer_sd = expert_layer_state(sd_ours, pre)
    assert set(layer_sd) == set(ours.layers[cfg.num_dense_layers].mlp.state_dict())


# ------------------------------------------------------------------- GPU --
@pytest.mark.gpu
def test_gpu_layers_match_reference_decoder_golden():
    from ethos_b200 import ops
    rec = load_golden("model")
    cfg = _layer_cfg(rec["model_cfg"])
    B, S = rec["batch"], rec["seq"]
    for entry in rec["layers"]:
        sd = _rounded_state(cfg, entry["seed"])
        layer = EthosExpertLayer(EthosConfig(**cfg))
        layer.load_state_dict(sd)
        layer = layer.to("cuda", torch.bfloat16).eval()
        x = entry["x"]
        xg = x.to("cuda", torch.bfloat16)
        with torch.no_grad():
            y = layer(xg.view(B, S, -1)).view(B * S, -1).float().cpu()
            scores, ids = layer.router(xg)
        torch.cuda.synchronize()
        ops.check_device_error("cuda")
        p = orc.params_from_state_dict(sd, dims_of(cfg))
        mask = orc.id_match_mask(orc.grid_top_scores(orc.router_queries(x, p)[0], p.K1, p.K2,
                                                     cfg["top_k"] + 1), cfg["top_k"])
        ref_ids = entry["ids"].to(torch.int64)
        ids = ids.cpu()
        assert torch.equal(ids[mask], ref_ids[mask]), entry["prefix"]
        rows = (ids == ref_ids).all(-1).all(-1)
        assert rows.float().mean().item() > 0.8
        assert rel_err(y[rows], entry["y"][rows]) <= 1e-2, entry["prefix"]
