"""Seeded synthetic initialisation for benchmarks and parity tests.

Convention (the benchmark configs say "N(0, 1/sqrt(fan_in))"):

* every 2-D weight ``W[rows, cols]`` -- ``nn.Linear`` weights ``[out, in]`` as
  well as the embedding tables (latent codes, sub-keys) ``[rows, dim]`` -- is
  drawn N(0, 1) and scaled by ``1/sqrt(cols)``;
* biases are 0; BatchNorm gamma = 1, beta = 0, running mean 0, running var 1,
  ``num_batches_tracked`` 0; other 1-D weights (the decoder's RMSNorm gains)
  are 1;
* inputs ``x`` are N(0, 1).

Each tensor draws from its own ``torch.Generator`` seeded from ``seed`` and the
CRC32 of its ``state_dict`` key, so the values do not depend on module
construction order and the reference module (``model.SimplifiedHypernetMoE``)
and :class:`ethos_b200.EthosExpertLayer` receive identical values.
"""

import zlib

import torch

__all__ = ["seeded_state_dict", "seeded_init_", "seeded_input", "tensor_generator"]


def tensor_generator(seed, name):
    key = (int(seed) * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFFFFFF
    return torch.Generator().manual_seed(key)


def _value_for(name, like, seed):
    shape = tuple(like.shape)
    if name.endswith("num_batches_tracked"):
        return torch.zeros((), dtype=torch.int64)
    if ".query_norms." in name:
        if name.endswith(".weight") or name.endswith(".running_var"):
            return torch.ones(shape)
        return torch.zeros(shape)
    if name.endswith(".bias"):
        return torch.zeros(shape)
    if len(shape) == 1 and name.endswith("weight"):
        return torch.ones(shape)
    if len(shape) != 2:
        raise ValueError(f"unexpected parameter {name} with shape {shape}")
    g = tensor_generator(seed, name)
    return torch.randn(shape, generator=g, dtype=torch.float32) * (1.0 / shape[1] ** 0.5)


def seeded_state_dict(module, seed=0):
    """Return a CPU fp32 state_dict (int64 counters) with the seeded values."""
    out = {}
    for name, t in module.state_dict().items():
        out[name] = _value_for(name, t, seed)
    return out


@torch.no_grad()
def seeded_init_(module, seed=0):
    """Overwrite every entry of ``module.state_dict()`` in place."""
    for name, t in module.state_dict().items():
        t.copy_(_value_for(name, t, seed).to(dtype=t.dtype))
    return module


def seeded_input(tokens, d_model, seed=0, dtype=torch.float32):
    g = tensor_generator(seed, "input.x")
    return torch.randn((tokens, d_model), generator=g, dtype=torch.float32).to(dtype)
