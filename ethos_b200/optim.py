"""Fused AdamW for the expert layer's parameters: the optimizer step the
reference runs through DeepSpeed (train.py:68-104).

``FusedAdamW`` follows ``torch.optim.AdamW`` exactly (decoupled weight decay,
bias-corrected moments, the same per-element order of operations) and updates
every parameter of a group in ONE kernel launch (``ethos_adamw_step``), reading
each gradient once.  bf16 / fp16 parameters keep an fp32 master copy by default
(``master_weights=True``, as DeepSpeed's bf16 optimizer does): the update runs
on the master and the parameter receives its rounded value.

``max_grad_norm`` adds the reference's global-norm gradient clipping
(``gradient_clipping: 1.0``, train.py:100) with the rule of
``torch.nn.utils.clip_grad_norm_`` over every parameter of every group: the
norm is computed on the device (``ethos_grad_clip_coef``, a fixed-order sum,
so data-parallel ranks holding the same gradients get the same coefficient)
and the AdamW kernel scales each gradient by the coefficient as it reads it;
no host synchronisation, and ``p.grad`` itself is left unscaled.
``last_grad_norm`` then holds the norm before clipping as a device scalar.
CUDA tensors only; there is no CPU path.
"""

import ctypes

import torch
from torch.autograd.graph import increment_version

from ._lib import check, lib
from .ops import _stream, device_error_word

__all__ = ["FusedAdamW"]



class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, master_weights=True,
                 max_grad_norm=None):
        if lr < 0.0 or eps <= 0.0 or not (0.0 <= betas[0] < 1.0) or not (0.0 <= betas[1] < 1.0):
            raise ValueError("invalid AdamW hyper-parameters")
        if max_grad_norm is not None and not max_grad_norm > 0.0:
            raise ValueError("max_grad_norm must be positive (or None for no clipping)")
        self.max_grad_norm = max_grad_norm
        self.last_grad_norm = None
        self._clip_bufs = None
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

    def _clip_buffers(self, dev):
        """Workspace and {norm, coef} output of the clip pass, kept across
        steps (alternate pairs, so a step never overwrites the norm that the
        previous step reported while it may still be read)."""
        if self._clip_bufs is None or self._clip_bufs[0].device != dev:
            ws = torch.empty(max(8, lib().ethos_grad_clip_workspace_size()), dtype=torch.uint8, device=dev)
            self._clip_bufs = (ws, torch.empty((2, 2), dtype=torch.float32, device=dev), [0])
        ws, out, turn = self._clip_bufs
        turn[0] ^= 1
        return ws, out[turn[0]]

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        plans, keep = [], []
        for group in self.param_groups:
            live = [p for p in group["params"] if p.grad is not None]
            if not live:
                continue
            rows, max_n, step = [], 0, None
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
            plans.append((group, live, rows, max_n, step))
        if not plans:
            return loss
        dev = plans[0][1][0].device
        if any(p.device != dev for _, live, _, _, _ in plans for p in live):
            raise ValueError("FusedAdamW updates the parameters of one device")
        L = lib()
        err = ctypes.c_void_p(device_error_word(dev).data_ptr())
        stream = _stream(dev)
        # one 56-byte ethos_adam_tensor per row: 5 pointers, n, then the two
        # int32 flags packed little-endian into the last int64 word; the
        # groups' rows are contiguous in one table
        all_rows = [r for _, _, rows, _, _ in plans for r in rows]
        host = torch.tensor(all_rows, dtype=torch.int64).pin_memory()
        dtab = host.to(dev, non_blocking=True)
        keep += [host, dtab]
        scale = None
        if self.max_grad_norm is not None:
            ws, out = self._clip_buffers(dev)
            check(L.ethos_grad_clip_coef(ctypes.c_void_p(dtab.data_ptr()), len(all_rows), float(self.max_grad_norm),
                                         ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(out.data_ptr()),
                                         err, stream),
                  "ethos_grad_clip_coef")
            self.last_grad_norm = out[0]
            scale = ctypes.c_void_p(out.data_ptr() + 4)
        row0 = 0
        for group, live, rows, max_n, step in plans:
            beta1, beta2 = group["betas"]
            check(L.ethos_adamw_step(ctypes.c_void_p(dtab.data_ptr() + 56 * row0), len(rows), max_n, group["lr"],
                                     beta1, beta2, group["eps"], group["weight_decay"], step, scale, err, stream),
                  "ethos_adamw_step")
            row0 += len(rows)
            # the kernel wrote the parameters through raw pointers: bump their
            # version counters so that caches keyed on them (the expert
            # layer's packed weights and expert table) see the update
            increment_version(live)
        # the caching allocators order the reuse of these buffers after the
        # kernels; holding them until the next step is belt and braces
        self._inflight = keep
        return loss
