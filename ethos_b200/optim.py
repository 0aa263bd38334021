"""Fused AdamW for the expert layer's parameters: the optimizer step the
reference runs through DeepSpeed (train.py:68-104).

``FusedAdamW`` follows ``torch.optim.AdamW`` exactly (decoupled weight decay,
bias-corrected moments, the same per-element order of operations) and updates
every parameter of a group in ONE kernel launch (``ethos_adamw_step``), reading
each gradient once.  bf16 / fp16 parameters keep an fp32 master copy by default
(``master_weights=True``, as DeepSpeed's bf16 optimizer does): the update runs
on the master and the parameter receives its rounded value.  CUDA tensors only;
there is no CPU path.
"""

import ctypes

import torch
from torch.autograd.graph import increment_version

from ._lib import check, lib
from .ops import _stream, device_error_word

__all__ = ["FusedAdamW"]



class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, master_weights=True):
        if lr < 0.0 or eps <= 0.0 or not (0.0 <= betas[0] < 1.0) or not (0.0 <= betas[1] < 1.0):
            raise ValueError("invalid AdamW hyper-parameters")
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay,
                                      master_weights=master_weights))
        for group in self.param_groups:
            for p in group["params"]:
                if not p.is_cuda:
                    raise ValueError("FusedAdamW runs on CUDA tensors only (no CPU path)")
                if p.dtype not in (torch.float32, torch.bfloat16):
                    raise ValueError(f"unsupported parameter dtype {p.dtype}")

    def _state_for(self, p, group):
        st = self.state[p]
        if not st:
            st["step"] = 0
            st["exp_avg"] = torch.zeros(p.shape, dtype=torch.float32, device=p.device)
            st["exp_avg_sq"] = torch.zeros(p.shape, dtype=torch.float32, device=p.device)
            if group["master_weights"] and p.dtype != torch.float32:
                st["master"] = p.detach().float().clone()
        return st

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            live = [p for p in group["params"] if p.grad is not None]
            if not live:
                continue
            dev = live[0].device
            rows, max_n, step = [], 0, None
            keep = []
            for p in live:
                st = self._state_for(p, group)
                st["step"] += 1
                if step is None:
                    step = st["step"]
                elif st["step"] != step:
                    raise RuntimeError("parameters of one group must share the step count")
                g = p.grad
                if g.dtype not in (torch.float32, torch.bfloat16) or g.is_sparse:
                    raise ValueError(f"unsupported gradient {g.dtype}")
                g = g.contiguous()
                pd = p.data
                if not pd.is_contiguous():
                    raise ValueError("FusedAdamW needs contiguous parameters")
                keep.append(g)
                master = st.get("master")
                n = pd.numel()
                max_n = max(max_n, n)
                rows.append([pd.data_ptr(), g.data_ptr(), st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr(),
                             master.data_ptr() if master is not None else 0, n,
                             (1 if pd.dtype == torch.bfloat16 else 0) | ((1 if g.dtype == torch.bfloat16 else 0) << 32)])
            # one 56-byte ethos_adam_tensor per row: 5 pointers, n, then the two
            # int32 flags packed little-endian into the last int64 word
            host = torch.tensor(rows, dtype=torch.int64).pin_memory()
            dtab = host.to(dev, non_blocking=True)
            beta1, beta2 = group["betas"]
            err = device_error_word(dev)
            check(lib().ethos_adamw_step(ctypes.c_void_p(dtab.data_ptr()), len(rows), max_n, group["lr"], beta1,
                                         beta2, group["eps"], group["weight_decay"], step,
                                         ctypes.c_void_p(err.data_ptr()), _stream(dev)),
                  "ethos_adamw_step")
            # the kernel wrote the parameters through raw pointers: bump their
            # version counters so that caches keyed on them (the expert
            # layer's packed weights and expert table) see the update
            increment_version(live)
            # the caching allocators order the reuse of these buffers after the
            # kernel; holding them until the next step is belt and braces
            self._inflight = (host, dtab, keep)
        return loss
