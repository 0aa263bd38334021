"""Data parallelism for the expert layer: token shards, replicated parameters.

The reference trains under DeepSpeed ZeRO-2 over NCCL (train.py:93-99, 156),
i.e. data parallelism with the gradients reduced across ranks.  Here:

* the forward needs no communication: every rank runs its own token shard
  against the full (replicated) latent table, hypernetwork and router;
* the gradients of the latent table, hypernetwork, query projections,
  BatchNorm affine and sub-keys are averaged over the ranks in fp32 (NCCL over
  NVLink on B200): either by ``overlap_grad_allreduce`` inside the layer's
  backward, overlapped with it, or after the backward by ``GradAllReducer``
  in flat fp32 buckets (any ``torch.distributed`` backend; gloo in the CPU
  tests);
* BatchNorm uses each rank's batch statistics, as the reference does (no
  SyncBN); ``average_running_stats`` optionally averages the running
  statistics so that ranks evaluate identically.
"""

import torch
import torch.distributed as dist

__all__ = ["shard_range", "shard_tokens", "GradAllReducer", "average_running_stats", "overlap_grad_allreduce"]


def shard_range(total, rank, world):
    """Contiguous [start, stop) of ``total`` tokens owned by ``rank``."""
    base, rem = divmod(int(total), int(world))
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_tokens(x, rank, world, dim=0):
    start, stop = shard_range(x.shape[dim], rank, world)
    return x.narrow(dim, start, stop - start)


def overlap_grad_allreduce(module, group=None):
    """Let every EthosExpertLayer in ``module`` average its parameter gradients
    over ``group`` inside its own backward: the backward's flat fp32 gradient
    buffer is all-reduced (NCCL ``AVG``) in two slices, the latent table and
    W1 while the router and BatchNorm gradients are still being computed, the
    rest at the end, and the parameter gradients are formed from the reduced
    buffer -- no separate pack / unpack pass.  ``GradAllReducer`` skips these
    parameters.  Every rank must run the same backward.  Returns the layers."""
    from .layer import EthosExpertLayer
    layers = [m for m in module.modules() if isinstance(m, EthosExpertLayer)]
    for layer in layers:
        layer._grad_comm = dict(group=group, stream=None)
        for p in layer.parameters():
            p._ethos_allreduced = True
    return layers


class GradAllReducer:
    """Sums the ``.grad`` of ``params`` over the process group in flat fp32
    buckets of about ``bucket_bytes`` and divides by the world size.

    Every rank must call it after the same backward (the buckets are built
    from the parameter list, so all ranks issue identical collectives in the
    same order).  A parameter without a gradient contributes zeros."""

    def __init__(self, params, group=None, bucket_bytes=64 << 20, average=True):
        # parameters whose layer reduces them in its backward are left alone
        self.params = [p for p in params if p.requires_grad and not getattr(p, "_ethos_allreduced", False)]
        self.group = group
        self.average = average
        self.buckets = []
        cur, size = [], 0
        for p in self.params:
            n = p.numel() * 4
            if cur and size + n > bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
            cur.append(p)
            size += n
        if cur:
            self.buckets.append(cur)

    def __call__(self):
        if not self.buckets:
            return
        world = dist.get_world_size(self.group)
        handles = []
        flats = []
        for bucket in self.buckets:
            dev = bucket[0].device
            flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1).float()
                              for p in bucket]).to(dev)
            handles.append(dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True))
            flats.append(flat)
        for bucket, flat, h in zip(self.buckets, flats, handles):
            h.wait()
            if self.average and world > 1:
                flat.div_(world)
            off = 0
            for p in bucket:
                n = p.numel()
                g = flat[off:off + n].view_as(p).to(p.dtype)
                if p.grad is None:
                    p.grad = g.clone()
                else:
                    p.grad.copy_(g)
                off += n


@torch.no_grad()
def average_running_stats(module, group=None):
    """Average every BatchNorm running mean / variance over the group."""
    world = dist.get_world_size(group)
    for m in module.modules():
        if isinstance(m, torch.nn.modules.batchnorm._BatchNorm) and m.track_running_stats:
            for buf in (m.running_mean, m.running_var):
                t = buf.float().clone()
                dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
                buf.copy_((t / world).to(buf.dtype))
