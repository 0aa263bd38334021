"""FusedAdamW (ethos_adamw_step) against torch.optim.AdamW.

CPU: construction rules and argument checks of the C entry point (no compute).
GPU: several steps on fp32 parameters match torch.optim.AdamW to fp32
rounding; bf16 parameters with fp32 master weights match AdamW run on fp32
copies fed the same gradients, and the bf16 parameter is the rounded master."""

import ctypes

import pytest
import torch

from ethos_b200 import _lib


def test_rejects_cpu_parameters():
    from ethos_b200.optim import FusedAdamW
    with pytest.raises(ValueError):
        FusedAdamW([torch.nn.Parameter(torch.zeros(4))])


def test_entry_point_argument_checks():
    L = _lib.lib()
    # nothing to do: OK without touching a device
    assert L.ethos_adamw_step(None, 0, 0, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, None, None, None) == 0
    # null table, bad step, bad betas
    assert L.ethos_adamw_step(None, 2, 16, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, None, None, None) == 1
    assert L.ethos_adamw_step(ctypes.c_void_p(16), 1, 16, 1e-3, 0.9, 0.999, 1e-8, 0.0, 0, None, None, None) == 1
    assert L.ethos_adamw_step(ctypes.c_void_p(16), 1, 16, 1e-3, 1.0, 0.999, 1e-8, 0.0, 1, None, None, None) == 1


def _params(seed, dtype, shapes=((1000, 33), (7,), (4096,), (3, 5))):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(s, generator=g).to(dtype) for s in shapes]


@pytest.mark.gpu
@pytest.mark.parametrize("wd", [0.0, 0.01])
def test_fp32_matches_torch_adamw(wd):
    from ethos_b200.optim import FusedAdamW
    base = _params(1, torch.float32)
    ours = [torch.nn.Parameter(t.clone().cuda()) for t in base]
    ref = [torch.nn.Parameter(t.clone().cuda()) for t in base]
    o1 = FusedAdamW(ours, lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=wd)
    o2 = torch.optim.AdamW(ref, lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=wd, foreach=False)
    g = torch.Generator(device="cuda").manual_seed(2)
    for _ in range(5):
        for a, b in zip(ours, ref):
            gr = torch.randn(a.shape, device="cuda", generator=g)
            a.grad = gr.clone()
            b.grad = gr.clone()
        o1.step()
        o2.step()
    torch.cuda.synchronize()
    for a, b in zip(ours, ref):
        torch.testing.assert_close(a.detach(), b.detach(), rtol=2e-6, atol=2e-7)
        sa, sb = o1.state[a], o2.state[b]
        torch.testing.assert_close(sa["exp_avg"], sb["exp_avg"], rtol=1e-6, atol=1e-7)
        torch.testing.assert_close(sa["exp_avg_sq"], sb["exp_avg_sq"], rtol=1e-6, atol=1e-9)


@pytest.mark.gpu
def test_bf16_master_weights():
    from ethos_b200.optim import FusedAdamW
    base = _params(3, torch.float32)
    ours = [torch.nn.Parameter(t.to(torch.bfloat16).cuda()) for t in base]
    ref = [torch.nn.Parameter(t.to(torch.bfloat16).float().cuda()) for t in base]
    o1 = FusedAdamW(ours, lr=1e-2, weight_decay=0.1)
    o2 = torch.optim.AdamW(ref, lr=1e-2, weight_decay=0.1, foreach=False)
    g = torch.Generator(device="cuda").manual_seed(4)
    for _ in range(4):
        for a, b in zip(ours, ref):
            gr = torch.randn(a.shape, device="cuda", generator=g).to(torch.bfloat16)
            a.grad = gr.clone()
            b.grad = gr.float()
        o1.step()
        o2.step()
    torch.cuda.synchronize()
    for a, b in zip(ours, ref):
        master = o1.state[a]["master"]
        torch.testing.assert_close(master, b.detach(), rtol=2e-6, atol=2e-7)
        assert torch.equal(a.detach(), master.to(torch.bfloat16))


def test_clip_entry_point_argument_checks():
    L = _lib.lib()
    assert L.ethos_grad_clip_workspace_size() >= 8
    v = ctypes.c_void_p(256)
    # null table, non-positive max_norm, then a missing or short workspace
    # (all rejected before any device work)
    assert L.ethos_grad_clip_coef(None, 2, 1.0, v, 1 << 20, v, None, None) == 1
    assert L.ethos_grad_clip_coef(v, 2, 0.0, v, 1 << 20, v, None, None) == 1
    assert L.ethos_grad_clip_coef(v, 2, 1.0, None, 1 << 20, v, None, None) == 4
    assert L.ethos_grad_clip_coef(v, 2, 1.0, v, 8, v, None, None) == 4


def test_rejects_non_positive_max_grad_norm():
    from ethos_b200.optim import FusedAdamW
    with pytest.raises(ValueError):
        FusedAdamW([torch.nn.Parameter(torch.zeros(4))], max_grad_norm=0.0)


def _clip_run(dtype, max_norm, grad_scale, seed):
    """Three steps of FusedAdamW(max_grad_norm) and of clip_grad_norm_ +
    torch.optim.AdamW on fp32 copies fed the same gradients."""
    from ethos_b200.optim import FusedAdamW
    base = _params(seed, torch.float32)
    ours = [torch.nn.Parameter(t.to(dtype).cuda()) for t in base]
    ref = [torch.nn.Parameter(t.to(dtype).float().cuda()) for t in base]
    o1 = FusedAdamW(ours, lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, max_grad_norm=max_norm)
    o2 = torch.optim.AdamW(ref, lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, foreach=False)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    norms = []
    for _ in range(3):
        for a, b in zip(ours, ref):
            gr = (torch.randn(a.shape, device="cuda", generator=g) * grad_scale).to(dtype)
            a.grad = gr.clone()
            b.grad = gr.float()
        o1.step()
        norms.append((o1.last_grad_norm.item(), torch.nn.utils.clip_grad_norm_(ref, max_norm).item()))
        o2.step()
    torch.cuda.synchronize()
    return ours, ref, o1, norms


@pytest.mark.gpu
@pytest.mark.parametrize("grad_scale", [1.0, 1e-3])  # clipped (norm ~ 150), and below the limit
def test_clipping_matches_clip_grad_norm_fp32(grad_scale):
    ours, ref, _, norms = _clip_run(torch.float32, 1.0, grad_scale, 5)
    for mine, theirs in norms:
        assert abs(mine - theirs) <= 2e-6 * theirs
    for a, b in zip(ours, ref):
        torch.testing.assert_close(a.detach(), b.detach(), rtol=2e-6, atol=2e-7)


@pytest.mark.gpu
def test_clipping_bf16_master_weights_and_determinism():
    ours, ref, o1, norms = _clip_run(torch.bfloat16, 1.0, 1.0, 7)
    for mine, theirs in norms:
        assert abs(mine - theirs) <= 2e-6 * theirs
    for a, b in zip(ours, ref):
        torch.testing.assert_close(o1.state[a]["master"], b.detach(), rtol=2e-6, atol=2e-7)
    # the fixed-order norm: a second run from the same state and gradients
    # lands on bit-identical parameters
    again, _, _, norms2 = _clip_run(torch.bfloat16, 1.0, 1.0, 7)
    assert [m for m, _ in norms] == [m for m, _ in norms2]
    for a, b in zip(ours, again):
        assert torch.equal(a.detach(), b.detach())


@pytest.mark.gpu
def test_clipping_across_param_groups():
    """Two parameter groups with their own lr and weight decay: one clip norm
    over both (as clip_grad_norm_ over every parameter), each group updated
    with its own hyper-parameters from its slice of the descriptor table."""
    from ethos_b200.optim import FusedAdamW
    base = _params(11, torch.float32)
    ours = [torch.nn.Parameter(t.clone().cuda()) for t in base]
    ref = [torch.nn.Parameter(t.clone().cuda()) for t in base]
    groups = lambda ps: [dict(params=ps[:2], lr=3e-3, weight_decay=0.0), dict(params=ps[2:], lr=1e-2,
                                                                            weight_decay=0.1)]
    o1 = FusedAdamW(groups(ours), max_grad_norm=0.5)
    o2 = torch.optim.AdamW(groups(ref), foreach=False)
    g = torch.Generator(device="cuda").manual_seed(12)
    for _ in range(3):
        for a, b in zip(ours, ref):
            gr = torch.randn(a.shape, device="cuda", generator=g)
            a.grad = gr.clone()
            b.grad = gr.clone()
        o1.step()
        theirs = torch.nn.utils.clip_grad_norm_(ref, 0.5).item()
        o2.step()
        assert abs(o1.last_grad_norm.item() - theirs) <= 2e-6 * theirs
    torch.cuda.synchronize()
    for a, b in zip(ours, ref):
        torch.testing.assert_close(a.detach(), b.detach(), rtol=2e-6, atol=2e-7)
