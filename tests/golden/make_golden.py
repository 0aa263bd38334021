"""Generate the golden fixtures by running the REFERENCE itself.

Run in a container where the reference checkout exists (it is not needed
afterwards; the fixtures are committed):

    python tests/golden/make_golden.py --reference /path/to/ETHOS

It imports the reference's ``model.py`` and runs ``SimplifiedHypernetMoE``
(the non-Triton path, ``model.py:267-343``, with ``ProductKeyRouter``,
``model.py:182-254``) in fp32 on CPU, with the seeded initialisation of
``ethos_b200.init`` and seeded inputs / upstream gradients, and stores inputs,
outputs, router decisions, BatchNorm running-stat updates and autograd
gradients of every parameter and of ``x``.

The "model" case builds the reference's whole decoder (``CompressedMoEModel``,
``model.py:368-395``: 1 dense and 2 expert layers at a small size), runs its
forward on CPU and records what each expert layer received and returned,
with its routing; ``tests/test_reference_model.py`` replays those inputs
through the oracle and through the GPU layers.  The "decoder" case records
the same decoder's final logits with every parameter seeded by name, for
``tests/test_decoder.py``.

Small cases store every tensor.  The config-1 case (d_model 512, 4096
experts, 256 tokens) stores the forward outputs in full and, for a 32-token
backward, the full gradients of the small parameters plus norms and a fixed
sample of entries of the large ones (to keep the fixture small); the
parameters themselves are regenerated from the seed and checked against a
stored checksum.
"""

import argparse
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from ethos_b200.config import EthosConfig  # noqa: E402
from ethos_b200.init import seeded_init_, seeded_input, tensor_generator  # noqa: E402

CASES = {
    "tiny": dict(cfg=dict(d_model=64, num_experts=64, top_k=4, num_routing_heads=2,
                          d_latent=16, d_intermediate_hypernet=32, d_query=32),
                 tokens=10, batch=2, full=True, bwd_tokens=10),
    "small": dict(cfg=dict(d_model=128, num_experts=256, top_k=8, num_routing_heads=4,
                           d_latent=32, d_intermediate_hypernet=64, d_query=64),
                  tokens=24, batch=2, full=True, bwd_tokens=24),
    "cfg1": dict(cfg=dict(d_model=512, num_experts=4096, top_k=16, num_routing_heads=8,
                          d_latent=128, d_intermediate_hypernet=512, d_query=512),
                 tokens=256, batch=2, full=False, bwd_tokens=32),
    # the GPU parity protocol: the reference in fp32 on bf16-ROUNDED params
    # and inputs (what the bf16 kernels consume); forward only
    "cfg1_bf16r": dict(cfg=dict(d_model=512, num_experts=4096, top_k=16, num_routing_heads=8,
                                d_latent=128, d_intermediate_hypernet=512, d_query=512),
                       tokens=256, batch=2, full=False, bwd_tokens=32, round_bf16=True, fwd_only=True),
}

SAMPLE = 4096

# The reference's whole decoder (CompressedMoEModel, model.py:368-395) at a
# small size: 1 dense + 2 expert layers, the rest of train.Config's fields
# (train.py:28-58) scaled down.  Each expert layer gets the seeded
# initialisation (seed 100 + layer index) rounded to bf16, and a forward
# pre-hook rounds the layer's input to bf16, so the recorded outputs are the
# reference's fp32 arithmetic on the values the bf16 kernels consume.
MODEL_CASE = dict(vocab_size=1024, d_model=512, num_layers=3, num_heads=4, num_dense_layers=1,
                  num_moe_layers=2, q_lora_rank=64, kv_lora_rank=32, v_head_dim=32, qk_nope_head_dim=32,
                  qk_rope_head_dim=32, num_experts=4096, d_latent=128, d_intermediate_hypernet=512, top_k=16,
                  num_routing_heads=8, d_query=512, d_ffn_intermediate=512, max_seq_len=64, rms_norm_eps=1e-6,
                  rope_theta=10000.0, use_triton=False)
MODEL_BATCH, MODEL_SEQ = 2, 32

# The reference's whole decoder again, for an end-to-end check of
# ethos_b200.decoder.EthosDecoder: every parameter seeded by name (seed 21;
# the tied tok_embeddings / output weight takes output.weight's values), fp32
# throughout (no bf16 rounding: the GPU side runs the fp32 path), and the
# final logits recorded.
DECODER_CASE = dict(MODEL_CASE, vocab_size=512, num_layers=2, num_dense_layers=1, num_moe_layers=1)
DECODER_BATCH, DECODER_SEQ, DECODER_SEED = 2, 48, 21


def checksum(sd):
    out = {}
    for k, v in sd.items():
        v = v.double()
        out[k] = torch.tensor([v.sum().item(), (v * v).sum().item()], dtype=torch.float64)
    return out


def sample_idx(numel, name):
    g = tensor_generator(7, "sample." + name)
    return torch.randint(0, numel, (min(SAMPLE, numel),), generator=g)


def run_case(model_mod, name, spec):
    cfg = EthosConfig(**spec["cfg"])
    torch.manual_seed(0)
    ref = model_mod.SimplifiedHypernetMoE(cfg)
    seeded_init_(ref, seed=0)
    rnd = spec.get("round_bf16", False)
    if rnd:
        with torch.no_grad():
            for v in ref.state_dict().values():
                if v.is_floating_point():
                    v.copy_(v.to(torch.bfloat16).float())
    sd0 = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    T, B = spec["tokens"], spec["batch"]
    x = seeded_input(T, cfg.d_model, seed=0)
    if rnd:
        x = x.to(torch.bfloat16).float()
    rec = dict(cfg=spec["cfg"], tokens=T, full=spec["full"], checksum=checksum(sd0), round_bf16=rnd)
    if spec["full"]:
        rec["state_dict"] = sd0
        rec["x"] = x.clone()

    # ---- eval-mode forward over all tokens -------------------------------
    ref.eval()
    t0 = time.time()
    with torch.no_grad():
        scores, ids = ref.router(x)
        y = ref(x.view(B, T // B, cfg.d_model)).reshape(T, cfg.d_model)
    rec["eval"] = dict(y=y.clone(), scores=scores.clone(), ids=ids.to(torch.int32).clone())
    print(f"[{name}] eval forward {time.time() - t0:.1f}s")

    # ---- train-mode forward + backward on a token prefix -----------------
    for mode in (() if spec.get("fwd_only") else ("train", "eval_bwd")):
        ref.load_state_dict(sd0)
        ref.train(mode == "train")
        Tb = spec["bwd_tokens"]
        xb = x[:Tb].clone().requires_grad_(True)
        ref.zero_grad(set_to_none=True)
        t0 = time.time()
        yb = ref(xb.view(1, Tb, cfg.d_model)).reshape(Tb, cfg.d_model)
        g = torch.randn(yb.shape, generator=tensor_generator(0, "upstream." + mode))
        (yb * g).sum().backward()
        print(f"[{name}] {mode} fwd+bwd {time.time() - t0:.1f}s")
        grads = {n: p.grad.detach().clone() for n, p in ref.named_parameters() if p.grad is not None}
        entry = dict(tokens=Tb, y=yb.detach().clone(), upstream=g, x_grad=xb.grad.detach().clone())
        if mode == "train":
            entry["running"] = {k: v.detach().clone() for k, v in ref.state_dict().items()
                                if "running" in k or "num_batches" in k}
        if spec["full"]:
            entry["grads"] = grads
        else:
            small, big = {}, {}
            for n, gr in grads.items():
                if gr.numel() <= 65536 * 2:
                    small[n] = gr
                else:
                    idx = sample_idx(gr.numel(), n)
                    big[n] = dict(norm=gr.double().norm().item(),
                                  vals=gr.flatten()[idx].clone(), shape=tuple(gr.shape))
            entry["grads"] = small
            entry["grads_sampled"] = big
        rec[mode] = entry
    return rec


class _Cfg:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def run_model_case(model_mod):
    """Expert-layer inputs, outputs and routing inside the reference's own
    decoder forward (eval mode, CPU, fp32)."""
    cfg = _Cfg(**MODEL_CASE)
    torch.manual_seed(0)
    model = model_mod.CompressedMoEModel(cfg).eval()
    layers = []
    for i, blk in enumerate(model.layers):
        if i < cfg.num_dense_layers:
            continue
        seed = 100 + i
        seeded_init_(blk.mlp, seed=seed)
        with torch.no_grad():
            for v in blk.mlp.state_dict().values():
                if v.is_floating_point():
                    v.copy_(v.to(torch.bfloat16).float())
        entry = dict(prefix=f"layers.{i}.mlp.", seed=seed)
        blk.mlp.register_forward_pre_hook(lambda m, a: (a[0].to(torch.bfloat16).float(),))

        def keep(m, a, out, entry=entry):
            entry["x"] = a[0].detach().reshape(-1, a[0].shape[-1]).clone()
            entry["y"] = out.detach().reshape(-1, out.shape[-1]).clone()

        def keep_route(m, a, out, entry=entry):
            entry["scores"] = out[0].detach().float().clone()
            entry["ids"] = out[1].detach().to(torch.int32).clone()

        blk.mlp.register_forward_hook(keep)
        blk.mlp.router.register_forward_hook(keep_route)
        layers.append(entry)
    g = torch.Generator().manual_seed(5)
    input_ids = torch.randint(0, cfg.vocab_size, (MODEL_BATCH, MODEL_SEQ), generator=g)
    t0 = time.time()
    with torch.no_grad():
        logits = model(input_ids)
    print(f"[model] decoder forward {time.time() - t0:.1f}s, logits {tuple(logits.shape)}")
    return dict(model_cfg=dict(MODEL_CASE), batch=MODEL_BATCH, seq=MODEL_SEQ, input_ids=input_ids, layers=layers)


def run_decoder_case(model_mod):
    """Logits of the reference decoder (eval mode, CPU, fp32) with every
    parameter seeded by name."""
    from ethos_b200.init import seeded_state_dict
    cfg = _Cfg(**DECODER_CASE)
    model = model_mod.CompressedMoEModel(cfg).eval()
    sd = seeded_state_dict(model, seed=DECODER_SEED)
    sd["tok_embeddings.weight"] = sd["output.weight"]
    model.load_state_dict(sd)
    g = torch.Generator().manual_seed(9)
    input_ids = torch.randint(0, cfg.vocab_size, (DECODER_BATCH, DECODER_SEQ), generator=g)
    t0 = time.time()
    with torch.no_grad():
        logits = model(input_ids)
    print(f"[decoder] forward {time.time() - t0:.1f}s, logits {tuple(logits.shape)}")
    keys = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    return dict(model_cfg=dict(DECODER_CASE), seed=DECODER_SEED, input_ids=input_ids, logits=logits, keys=keys)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ETHOS_REFERENCE"),
                    help="reference checkout holding model.py (default: $ETHOS_REFERENCE)")
    ap.add_argument("--cases", default=",".join(list(CASES) + ["model", "decoder"]))
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or ETHOS_REFERENCE")
    sys.path.insert(0, args.reference)
    # the reference's attention uses flash_attn when it imports (a GPU-only
    # kernel); hiding the module selects its own matmul fallback
    # (model.py:156-163), which runs on the CPU
    sys.modules["flash_attn"] = None
    import model as model_mod  # the reference's model.py
    torch.set_num_threads(os.cpu_count() or 1)
    for name in args.cases.split(","):
        if name == "model":
            rec = run_model_case(model_mod)
        elif name == "decoder":
            rec = run_decoder_case(model_mod)
        else:
            rec = run_case(model_mod, name, CASES[name])
        path = os.path.join(HERE, f"golden_{name}.pt")
        torch.save(rec, path)
        print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
