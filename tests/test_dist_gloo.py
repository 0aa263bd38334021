"""Multi-process data parallelism on CPU (gloo, world size 2).

The per-rank compute is the CPU oracle (the host-side sharding and gradient
all-reduce are what is under test): the all-reduced gradients of the token
shards must equal the single-process gradients of the whole batch (eval-mode
BatchNorm, so the shards are independent), and a rank that dies makes the
survivor's collective fail instead of hang."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

CFG = dict(d_model=64, num_experts=64, top_k=4, num_routing_heads=2, d_latent=16,
           d_intermediate_hypernet=32, d_query=32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _OracleModule(nn.Module):
    """The oracle parameters as nn.Parameters (so GradAllReducer sees them)."""

    def __init__(self):
        super().__init__()
        from ethos_b200.config import EthosConfig, layer_dims
        from ethos_b200.init import seeded_state_dict
        from ethos_b200.layer import EthosExpertLayer
        from oracle import ethos_oracle as orc
        cfg = EthosConfig(**CFG)
        self.dims = layer_dims(cfg)
        self.p = orc.params_from_state_dict(seeded_state_dict(EthosExpertLayer(cfg), seed=1), self.dims)
        self.names = ["E", "W1", "W2", "Wq", "bq", "gamma", "beta", "K1", "K2"]
        for n in self.names:
            setattr(self, "_" + n, nn.Parameter(getattr(self.p, n).clone()))

    def forward(self, x):
        from oracle import ethos_oracle as orc
        for n in self.names:
            setattr(self.p, n, getattr(self, "_" + n))
        y, _, _, _ = orc.layer_forward(x, self.p, self.dims["top_k"], training=False)
        return y


def _inputs(T=24):
    g = torch.Generator().manual_seed(3)
    return torch.randn(T, CFG["d_model"], generator=g), torch.randn(T, CFG["d_model"], generator=g)


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from ethos_b200.dist import GradAllReducer, shard_tokens
        torch.manual_seed(0)
        m = _OracleModule()
        x, gy = _inputs()
        xs, gs = shard_tokens(x, rank, world), shard_tokens(gy, rank, world)
        y = m(xs)
        # local mean over the shard; averaging over equal shards = global mean
        (y * gs).sum().div(xs.shape[0]).backward()
        GradAllReducer(m.parameters(), bucket_bytes=4096)()
        out[rank] = {n: p.grad.clone() for n, p in m.named_parameters()}
    finally:
        dist.destroy_process_group()


def test_sharded_allreduce_matches_full_batch():
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    m = _OracleModule()
    x, gy = _inputs()
    (m(x) * gy).sum().div(x.shape[0]).backward()
    for n, p in m.named_parameters():
        for r in range(world):
            torch.testing.assert_close(out[r][n], p.grad, rtol=1e-5, atol=1e-6)


def _dying_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # the rank leaves between steps, with nothing in flight
    from ethos_b200.dist import GradAllReducer
    p = nn.Parameter(torch.ones(8))
    p.grad = torch.ones(8)
    try:
        GradAllReducer([p])()
        q.put("completed")
    except Exception as e:  # noqa: BLE001 -- any collective error is the expected outcome
        q.put("error: " + type(e).__name__)


def test_dead_rank_fails_the_collective():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung instead of failing")
    assert q.get(timeout=5).startswith("error")


def test_shard_range_covers_tokens():
    from ethos_b200.dist import shard_range
    for total in (0, 1, 7, 16384):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


class _FakeNvml:
    """Stands in for pynvml: one device whose CPU-affinity mask is `words`."""

    def __init__(self, words, fail_handle=False):
        self.words, self.fail_handle, self.calls = words, fail_handle, []

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlShutdown(self):
        self.calls.append("shutdown")

    def nvmlDeviceGetHandleByUUID(self, uuid):
        self.calls.append(uuid)
        if self.fail_handle:
            raise RuntimeError("no such device")
        return 7

    def nvmlDeviceGetCpuAffinity(self, handle, n):
        assert handle == 7 and n >= 1
        return self.words


def test_bind_to_device_numa_with_fake_nvml():
    """The process is restricted to the CPUs of the GPU's affinity mask that
    it may already use; a failing NVML leaves the affinity alone."""
    import os
    from ethos_b200.dist import _affinity_cpus, bind_to_device_numa
    assert _affinity_cpus([0b1011, 1]) == {0, 1, 3, 64}
    before = os.sched_getaffinity(0)
    try:
        first = min(before)
        words = [0] * (first // 64 + 1)
        words[first // 64] = 1 << (first % 64)
        fake = _FakeNvml(words)
        got = bind_to_device_numa(nvml=fake, uuid="abc")
        assert got == {first} and os.sched_getaffinity(0) == {first}
        assert fake.calls[:2] == ["init", "GPU-abc"] and fake.calls[-1] == "shutdown"
        os.sched_setaffinity(0, before)
        # a mask outside the allowed CPUs, or an NVML error: nothing changes
        assert bind_to_device_numa(nvml=_FakeNvml([0]), uuid="abc") is None
        assert bind_to_device_numa(nvml=_FakeNvml([1], fail_handle=True), uuid="abc") is None
        assert os.sched_getaffinity(0) == before
    finally:
        os.sched_setaffinity(0, before)
