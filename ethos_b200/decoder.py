"""The ETHOS decoder around the expert layer: the reference's
``CompressedMoEModel`` (model.py:345-395) rebuilt with ``EthosExpertLayer`` as
its expert FFN, for end-to-end runs of the whole model on the GPU.

Same constructor attributes and ``state_dict`` keys as the reference, so a
checkpoint of either loads into the other:

* ``tok_embeddings`` [vocab, d] tied to ``output`` (model.py:374,385);
* ``layers.{i}``: ``input_layernorm`` and ``post_attention_layernorm``
  (RMSNorm, model.py:19-29), ``self_attn`` (multi-head latent attention,
  model.py:76-166: a low-rank query path ``q_a_proj`` -> ``q_a_layernorm`` ->
  ``q_b_proj``, a compressed key/value path ``kv_a_proj_with_mqa`` ->
  ``kv_a_layernorm`` -> ``kv_b_proj`` plus one shared rotary key per token,
  rotary position embedding on the rope part of queries and keys, causal
  softmax attention with scale 1/sqrt(qk_nope + qk_rope), ``o_proj``), and
  ``mlp``: ``EthosExpertLayer`` from layer ``num_dense_layers`` on, the SwiGLU
  ``FFN`` (``w1``, ``w2``, ``w3``, model.py:255-263) before it;
* ``norm`` (RMSNorm) and ``output`` [vocab, d].

Only the expert layers run on this repository's kernels; attention, norms,
projections and the head are torch: cuBLAS, and for the attention core torch's
scaled_dot_product_attention, which on a B200 runs cuDNN's sm100 attention
kernel (0.12 ms per layer at config 4, where flash_attn 2.8, which the
reference calls, runs its sm80 kernel in 0.42 ms; ``use_flash_attn = True`` on
a ``LatentAttention`` selects it).  Queries, keys and values stay in
[batch, seq, heads, dim] layout and reach the kernel as transposed views, and
the output head's GEMM runs with the vocabulary padded to a multiple of 8
(an odd row length of the logits otherwise sends cuBLAS to an unaligned
kernel: 30 ms instead of 2-3 ms at config 4); the logits returned are a view
of the unpadded columns.
"""

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layer import EthosExpertLayer

__all__ = ["DecoderConfig", "RMSNorm", "LatentAttention", "SwiGLU", "DecoderBlock", "EthosDecoder"]


class DecoderConfig:
    """Attributes the decoder reads, named as the reference's training config
    (train.py:28-57) names them; any object with these attributes works."""

    def __init__(self, **kw):
        defaults = dict(vocab_size=100277, d_model=1024, num_layers=12, num_dense_layers=0, num_heads=16,
                        q_lora_rank=768, kv_lora_rank=256, qk_nope_head_dim=64, qk_rope_head_dim=64,
                        v_head_dim=64, d_ffn_intermediate=4096, max_seq_len=4096, rms_norm_eps=1e-6,
                        rope_theta=10000.0, num_experts=262144, top_k=16, num_routing_heads=8, d_latent=128,
                        d_intermediate_hypernet=512, d_query=512)
        defaults.update(kw)
        for k, v in defaults.items():
            setattr(self, k, v)


class RMSNorm(nn.Module):
    """y = weight * (x / sqrt(mean(x^2) + eps)), the mean and the scaling in
    fp32 and the result cast back to x's dtype before the weight."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        # torch's fused kernel normalises in fp32 and returns x's dtype; the
        # weight multiplies the rounded result, as in the reference
        return self.weight * F.rms_norm(x, (x.shape[-1],), None, self.eps)


class LatentAttention(nn.Module):
    """Multi-head latent attention with the reference's projections and
    rotary embedding (see the module docstring)."""

    def __init__(self, config):
        super().__init__()
        d, H = config.d_model, config.num_heads
        self.num_heads = H
        self.nope = config.qk_nope_head_dim
        self.rope = config.qk_rope_head_dim
        self.v_dim = config.v_head_dim
        self.kv_rank = config.kv_lora_rank
        self.q_dim = self.nope + self.rope
        self.scale = self.q_dim ** -0.5
        self.q_a_proj = nn.Linear(d, config.q_lora_rank, bias=False)
        self.q_a_layernorm = RMSNorm(config.q_lora_rank, config.rms_norm_eps)
        self.q_b_proj = nn.Linear(config.q_lora_rank, H * self.q_dim, bias=False)
        self.kv_a_proj_with_mqa = nn.Linear(d, self.kv_rank + self.rope, bias=False)
        self.kv_a_layernorm = RMSNorm(self.kv_rank, config.rms_norm_eps)
        self.kv_b_proj = nn.Linear(self.kv_rank, H * (self.nope + self.v_dim), bias=False)
        self.o_proj = nn.Linear(H * self.v_dim, d, bias=False)
        # rotary frequencies (not part of the state_dict, as in the reference)
        inv = 1.0 / (config.rope_theta ** (torch.arange(0, self.rope, 2, dtype=torch.float32) / self.rope))
        self.register_buffer("inv_freq", inv, persistent=False)
        self.use_flash_attn = False  # True: flash_attn's kernel (when it runs here) instead of torch's
        self._tables = {}

    def _cos_sin(self, S, dtype, device):
        """cos and sin of the first half of the rotary angles, [S, 1, rope/2]
        (the second half repeats them), kept per (length, dtype, device)."""
        key = (S, dtype, str(device))
        hit = self._tables.get(key)
        if hit is None:
            # angles in fp32 from fp32 positions, then rounded to the
            # activations' dtype, as the reference's cached tables are
            pos = torch.arange(S, device=device, dtype=torch.float32)
            ang = torch.outer(pos, self.inv_freq.to(device))
            hit = (ang.cos().to(dtype).view(S, 1, -1), ang.sin().to(dtype).view(S, 1, -1))
            self._tables = {key: hit}
        return hit

    def _rotary_into(self, out, t, cos, sin):
        """out <- t cos + rotate(t) sin, for t = [a, b] halves:
        out = [a cos - b sin, b cos + a sin], written into the view `out`."""
        r2 = self.rope // 2
        a, b = t[..., :r2], t[..., r2:]
        lo, hi = out[..., :r2], out[..., r2:]
        torch.mul(a, cos, out=lo)
        lo.addcmul_(b, sin, value=-1.0)
        torch.mul(b, cos, out=hi)
        hi.addcmul_(a, sin)

    def _core(self, q, k, v):
        """Causal attention on [B, S, H, dim] tensors -> [B, S, H*v_dim]."""
        B, S, H, _ = q.shape
        if self.use_flash_attn and q.is_cuda and q.dtype in (torch.bfloat16, torch.float16):
            try:
                from flash_attn import flash_attn_func
                vp = F.pad(v, (0, self.q_dim - self.v_dim)) if self.q_dim != self.v_dim else v
                o = flash_attn_func(q, k, vp, softmax_scale=self.scale, causal=True)
                return o[..., :self.v_dim].reshape(B, S, H * self.v_dim)
            except (ImportError, RuntimeError):
                self.use_flash_attn = False  # not available for this device: torch's kernel from now on
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                           scale=self.scale)
        return o.transpose(1, 2).reshape(B, S, H * self.v_dim)

    def forward(self, x):
        B, S, _ = x.shape
        H = self.num_heads
        q = self.q_b_proj(self.q_a_layernorm(self.q_a_proj(x))).view(B, S, H, self.q_dim)
        q_nope, q_rot = q.split([self.nope, self.rope], dim=-1)
        ckv = self.kv_a_proj_with_mqa(x)
        latent, k_rot = ckv.split([self.kv_rank, self.rope], dim=-1)
        kv = self.kv_b_proj(self.kv_a_layernorm(latent)).view(B, S, H, self.nope + self.v_dim)
        k_nope, v = kv.split([self.nope, self.v_dim], dim=-1)
        cos, sin = self._cos_sin(S, v.dtype, x.device)  # [S, 1, rope/2], over [.., S, H, rope/2]
        if torch.is_grad_enabled():
            # the same values by differentiable ops (out= writes record no graph)
            def rot(t):
                a, b = t[..., :self.rope // 2], t[..., self.rope // 2:]
                return torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)
            qf = torch.cat((q_nope, rot(q_rot)), dim=-1)
            kf = torch.cat((k_nope, rot(k_rot.unsqueeze(2)).expand(B, S, H, self.rope)), dim=-1)
            return self.o_proj(self._core(qf, kf, v))
        # inference: queries and keys assembled in place, [B, S, H, nope | rope]
        qf = torch.empty((B, S, H, self.q_dim), dtype=q.dtype, device=q.device)
        qf[..., :self.nope].copy_(q_nope)
        self._rotary_into(qf[..., self.nope:], q_rot, cos, sin)
        kr = torch.empty((B, S, 1, self.rope), dtype=k_rot.dtype, device=k_rot.device)
        self._rotary_into(kr, k_rot.unsqueeze(2), cos, sin)  # one rotary key per token, shared by the heads
        kf = torch.empty((B, S, H, self.q_dim), dtype=kv.dtype, device=kv.device)
        kf[..., :self.nope].copy_(k_nope)
        kf[..., self.nope:].copy_(kr.expand(B, S, H, self.rope))
        return self.o_proj(self._core(qf, kf, v))


class SwiGLU(nn.Module):
    """The reference's dense FFN: w2(silu(w1 x) * w3 x)."""

    def __init__(self, config):
        super().__init__()
        self.w1 = nn.Linear(config.d_model, config.d_ffn_intermediate, bias=False)
        self.w2 = nn.Linear(config.d_ffn_intermediate, config.d_model, bias=False)
        self.w3 = nn.Linear(config.d_model, config.d_ffn_intermediate, bias=False)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class DecoderBlock(nn.Module):
    def __init__(self, config, expert):
        super().__init__()
        self.self_attn = LatentAttention(config)
        self.mlp = EthosExpertLayer(config) if expert else SwiGLU(config)
        self.input_layernorm = RMSNorm(config.d_model, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.d_model, config.rms_norm_eps)

    def forward(self, x):
        h = x + self.self_attn(self.input_layernorm(x))
        return h + self.mlp(self.post_attention_layernorm(h))


class EthosDecoder(nn.Module):
    """``CompressedMoEModel`` with the B200 expert layers: ``forward(input_ids
    [B, S]) -> logits [B, S, vocab]`` (causal, positions 0..S-1)."""

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.tok_embeddings = nn.Embedding(config.vocab_size, config.d_model)
        self.layers = nn.ModuleList(
            [DecoderBlock(config, i >= config.num_dense_layers) for i in range(config.num_layers)])
        self.norm = RMSNorm(config.d_model, config.rms_norm_eps)
        self.output = nn.Linear(config.d_model, config.vocab_size, bias=False)
        self.tok_embeddings.weight = self.output.weight  # tied, as in the reference

    def expert_layers(self):
        return [b.mlp for b in self.layers if isinstance(b.mlp, EthosExpertLayer)]

    def forward(self, input_ids):
        h = self.tok_embeddings(input_ids)
        for blk in self.layers:
            h = blk(h)
        h = self.norm(h)
        w = self.output.weight
        pad = (-w.shape[0]) % 8
        if pad == 0 or not h.is_cuda:
            return F.linear(h, w)
        # aligned rows for cuBLAS; the extra columns are dropped by the view
        return F.linear(h, F.pad(w, (0, 0, 0, pad)))[..., :w.shape[0]]

