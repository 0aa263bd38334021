"""The layer's derived kernel-layout weights (packed query/W_u block, doubled
sub-keys, BatchNorm block, cached expert table) must follow every parameter
update.  FusedAdamW writes the parameters through raw device pointers, so it
bumps their version counters; forwards that need gradients always re-pack.

After two optimizer steps the trained layer is compared with a fresh layer
loaded from the trained state_dict: forward outputs, routing and every
parameter gradient must agree, in training mode, in eval mode, and with the
expert table cached across forwards.  Both layers run the same kernels on the
same inputs, so the only differences left are the summation order of the
split-K fp32 atomics in the weight-gradient GEMMs (~1e-7 relative); a stale
cache would be off by the optimizer's step (~1e-1 relative at lr 1e-2).
"""

import pytest
import torch

from ethos_b200 import EthosConfig, EthosExpertLayer, ops
from ethos_b200.init import seeded_input, seeded_state_dict, tensor_generator
from ethos_b200.optim import FusedAdamW
from helpers import rel_err

pytestmark = pytest.mark.gpu

CFG = dict(d_model=512, num_experts=4096, top_k=16, num_routing_heads=8, d_latent=128,
           d_intermediate_hypernet=512, d_query=512)
T = 512


def _fresh_like(layer):
    fresh = EthosExpertLayer(EthosConfig(**CFG))
    fresh.load_state_dict({k: v.detach().cpu() for k, v in layer.state_dict().items()})
    return fresh.to("cuda", torch.bfloat16).train(layer.training)


def _step(layer, x, gy):
    for p in layer.parameters():
        p.grad = None
    y = layer(x.view(1, T, -1))
    y.backward(gy.view(1, T, -1))
    return y.detach(), {n: p.grad.detach().clone() for n, p in layer.named_parameters()}


def test_packed_weights_follow_fused_adamw_updates():
    layer = EthosExpertLayer(EthosConfig(**CFG))
    layer.load_state_dict(seeded_state_dict(layer, seed=3))
    layer = layer.to("cuda", torch.bfloat16).train()
    x = seeded_input(T, CFG["d_model"], seed=5).to("cuda", torch.bfloat16)
    gy = (torch.randn((T, CFG["d_model"]), generator=tensor_generator(6, "gy"))).to("cuda", torch.bfloat16)
    opt = FusedAdamW(layer.parameters(), lr=1e-2, weight_decay=0.01)

    # warm the inference caches first, so stale entries would be visible
    layer.eval()
    with torch.no_grad():
        layer(x.view(1, T, -1))
        layer.cache_expert_table = True
        layer(x.view(1, T, -1))
        layer.cache_expert_table = False
    layer.train()
    versions = [p._version for p in layer.parameters()]
    for _ in range(2):
        _step(layer, x, gy)
        opt.step()
    assert all(p._version > v for p, v in zip(layer.parameters(), versions))

    # training mode: forward and all gradients against a fresh layer
    fresh = _fresh_like(layer)
    y1, g1 = _step(layer, x, gy)
    y2, g2 = _step(fresh, x, gy)
    torch.cuda.synchronize()
    ops.check_device_error("cuda")
    assert rel_err(y1.float(), y2.float()) <= 1e-5
    for n in g1:
        assert rel_err(g1[n].float(), g2[n].float()) <= 1e-4, n

    # eval mode (cached BatchNorm block and packed weights), then the cached
    # expert table path
    layer.eval()
    fresh.eval()
    with torch.no_grad():
        ye1 = layer(x.view(1, T, -1))
        ye2 = fresh(x.view(1, T, -1))
        assert rel_err(ye1.float(), ye2.float()) <= 1e-5
        s1, i1 = layer.router(x)
        s2, i2 = fresh.router(x)
        assert (i1 == i2).float().mean().item() >= 0.999
        layer.cache_expert_table = True
        fresh.cache_expert_table = True
        assert rel_err(layer(x.view(1, T, -1)).float(), fresh(x.view(1, T, -1)).float()) <= 1e-5

        # a write through .data bumps no version counter: the documented
        # invalidation makes the next inference forward see it
        w = layer.generation_network.net[2].weight
        w.data.mul_(0.5)
        fresh.generation_network.net[2].weight.data.mul_(0.5)
        layer.invalidate_weight_cache()
        fresh.invalidate_weight_cache()
        assert rel_err(layer(x.view(1, T, -1)).float(), fresh(x.view(1, T, -1)).float()) <= 1e-5
    torch.cuda.synchronize()
    ops.check_device_error("cuda")
