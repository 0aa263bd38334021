"""EthosDecoder (ethos_b200/decoder.py) against the reference's whole
decoder, CompressedMoEModel (model.py:345-395).

* CPU, always: the decoder's state_dict has exactly the reference's keys and
  shapes (recorded in tests/golden/golden_decoder.pt by make_golden.py).
* CPU, with a reference checkout named by ETHOS_REFERENCE (skipped
  otherwise): a dense block (RMSNorms, latent attention with rotary
  embedding, SwiGLU FFN) gives the reference TransformerBlock's output on the
  same weights and input, and checkpoints load both ways.
* GPU: the whole decoder -- embedding, attention and dense FFN in torch, the
  expert layer on this repository's kernels -- reproduces the reference's
  recorded fp32 logits: within 1e-4 with fp32 parameters (the fp32 path), and
  within the bound below with bf16 parameters (every part of the model in
  bf16)."""

import os
import sys

import pytest
import torch

from ethos_b200.decoder import DecoderConfig, EthosDecoder
from ethos_b200.init import seeded_state_dict
from helpers import load_golden, rel_err


def _decoder(rec):
    cfg = DecoderConfig(**{k: v for k, v in rec["model_cfg"].items() if k not in ("num_moe_layers", "use_triton")})
    model = EthosDecoder(cfg)
    sd = seeded_state_dict(model, seed=rec["seed"])
    sd["tok_embeddings.weight"] = sd["output.weight"]
    model.load_state_dict(sd)
    return model


def test_state_dict_matches_reference_keys():
    rec = load_golden("decoder")
    model = _decoder(rec)
    keys = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    assert keys == rec["keys"]
    assert model.tok_embeddings.weight is model.output.weight  # tied, as in the reference


def _reference_model():
    ref = os.environ.get("ETHOS_REFERENCE")
    if not ref or not os.path.exists(os.path.join(ref, "model.py")):
        pytest.skip("ETHOS_REFERENCE (a reference checkout) not set")
    sys.path.insert(0, ref)
    try:
        import model as model_mod  # the reference's model.py
    finally:
        sys.path.remove(ref)
    return model_mod


class _Cfg:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def test_dense_block_matches_reference_block():
    model_mod = _reference_model()
    rec = load_golden("decoder")
    cfg = _Cfg(**rec["model_cfg"])
    ref_blk = model_mod.TransformerBlock(cfg, is_moe_layer=False).eval()
    from ethos_b200.decoder import DecoderBlock
    blk = DecoderBlock(DecoderConfig(**{k: v for k, v in rec["model_cfg"].items()
                                        if k not in ("num_moe_layers", "use_triton")}), expert=False).eval()
    sd = seeded_state_dict(ref_blk, seed=5)
    ref_blk.load_state_dict(sd)
    blk.load_state_dict(sd)  # same keys, strict
    S = 40
    x = torch.randn(2, S, cfg.d_model, generator=torch.Generator().manual_seed(3))
    mask = torch.triu(torch.full((S, S), float("-inf")), diagonal=1)
    pos = torch.arange(S)
    saved = sys.modules.get("flash_attn", "absent")
    sys.modules["flash_attn"] = None  # the reference's matmul attention (its CPU path)
    try:
        with torch.no_grad():
            want = ref_blk(x, mask, pos)
    finally:
        if saved == "absent":
            del sys.modules["flash_attn"]
        else:
            sys.modules["flash_attn"] = saved
    with torch.no_grad():
        got = blk(x)
    assert rel_err(got, want) <= 1e-5


def test_checkpoints_load_both_ways():
    model_mod = _reference_model()
    rec = load_golden("decoder")
    ref = model_mod.CompressedMoEModel(_Cfg(**rec["model_cfg"]))
    ours = _decoder(rec)
    ref.load_state_dict(ours.state_dict())
    ours2 = EthosDecoder(DecoderConfig(**{k: v for k, v in rec["model_cfg"].items()
                                          if k not in ("num_moe_layers", "use_triton")}))
    ours2.load_state_dict(ref.state_dict())
    for k, v in ours.state_dict().items():
        assert torch.equal(v, ours2.state_dict()[k]), k


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,bound", [(torch.float32, 1e-4), (torch.bfloat16, 3e-2)])
def test_decoder_matches_reference_logits(dtype, bound):
    rec = load_golden("decoder")
    model = _decoder(rec).to("cuda", dtype).eval()
    with torch.no_grad():
        logits = model(rec["input_ids"].cuda())
    torch.cuda.synchronize()
    err = rel_err(logits.float().cpu(), rec["logits"])
    print(f"decoder logits, {dtype}: relative error {err:.2e}")
    assert err <= bound


def test_attention_same_with_and_without_autograd():
    """The latent attention's in-place inference path and its differentiable
    path compute the same values, and the latter back-propagates."""
    from ethos_b200.decoder import LatentAttention
    rec = load_golden("decoder")
    cfg = DecoderConfig(**{k: v for k, v in rec["model_cfg"].items() if k not in ("num_moe_layers", "use_triton")})
    att = LatentAttention(cfg)
    att.load_state_dict(seeded_state_dict(att, seed=4))
    x = torch.randn(2, 24, cfg.d_model, generator=torch.Generator().manual_seed(6))
    with torch.no_grad():
        inf = att(x)
    xg = x.clone().requires_grad_(True)
    trn = att(xg)
    trn.square().sum().backward()
    assert torch.allclose(inf, trn.detach(), rtol=1e-6, atol=1e-6)
    assert xg.grad is not None and torch.isfinite(xg.grad).all()
