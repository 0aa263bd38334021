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
  statistics so that ranks evaluate identically;
* ``bind_to_device_numa`` keeps each rank's host work and pinned staging
  buffers on its GPU's NUMA node.
"""

import os

import torch
import torch.distributed as dist

__all__ = ["shard_range", "shard_tokens", "GradAllReducer", "average_running_stats", "overlap_grad_allreduce",
           "bind_to_device_numa"]


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


def _affinity_cpus(words):
    """CPU ids set in an NVML CPU-affinity mask (64-bit words, CPU 64 i + b is
    bit b of word i)."""
    return {64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1}


def bind_to_device_numa(device=None, nvml=None, uuid=None):
    """Restricts this process to the CPUs that NVML reports as close to the
    GPU (its NUMA node), so that host memory the process touches first after
    the call -- the pinned buffers of host <-> device copies in particular --
    is placed in that node's memory and its copies do not cross the socket
    interconnect.  Call it once per rank, before allocating pinned buffers.

    Only the process's own CPU affinity changes (within the CPUs it may
    already use); no GPU setting is read-modify-written.  Returns the CPU set
    in effect afterwards, or None when NVML is missing or reports nothing
    usable (the affinity is then left as it was).  ``nvml`` and ``uuid``
    (the device UUID without its "GPU-" prefix) are for tests."""
    if nvml is None:
        try:
            import pynvml as nvml
        except ImportError:
            return None
    if uuid is None:
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    try:
        nvml.nvmlInit()
    except Exception:
        return None
    try:
        handle = nvml.nvmlDeviceGetHandleByUUID("GPU-" + uuid)
        words = nvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
    except Exception:
        return None
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:
            pass
    cpus = _affinity_cpus(words) & os.sched_getaffinity(0)
    if not cpus:
        return None
    os.sched_setaffinity(0, cpus)
    return cpus
