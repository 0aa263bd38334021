"""Data parallelism on 2 GPUs (skipped with fewer): the gradient all-reduce
that runs inside the layer's backward (overlap_grad_allreduce, NCCL AVG of the
flat fp32 gradient buffer) gives the same parameter gradients as
GradAllReducer after a plain backward, on the same token shards."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

CFG = dict(d_model=512, num_experts=4096, top_k=16, num_routing_heads=8, d_latent=128,
           d_intermediate_hypernet=512, d_query=512)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from ethos_b200 import EthosConfig, EthosExpertLayer, ops
        from ethos_b200.dist import GradAllReducer, overlap_grad_allreduce
        from ethos_b200.init import seeded_input, seeded_state_dict, tensor_generator
        T = 1024
        grads = []
        for mode in ("after", "overlap"):
            layer = EthosExpertLayer(EthosConfig(**CFG))
            layer.load_state_dict(seeded_state_dict(layer, seed=4))
            layer = layer.to(dev, torch.bfloat16).train()
            x = seeded_input(T, CFG["d_model"], seed=10 + rank).to(dev, torch.bfloat16)
            gy = torch.randn((T, CFG["d_model"]), generator=tensor_generator(20 + rank, "gy")).to(dev, torch.bfloat16)
            if mode == "overlap":
                overlap_grad_allreduce(layer)
            y = layer(x.view(1, T, -1))
            y.backward(gy.view(1, T, -1))
            if mode == "after":
                GradAllReducer(list(layer.parameters()))()
            torch.cuda.synchronize()
            ops.check_device_error(dev)
            grads.append({n: p.grad.float().cpu() for n, p in layer.named_parameters()})
        worst = 0.0
        for n in grads[0]:
            a, b = grads[0][n], grads[1][n]
            scale = a.norm().item()
            if scale > 0:
                worst = max(worst, (a - b).norm().item() / scale)
        out[rank] = worst
    finally:
        dist.destroy_process_group()


def test_overlapped_allreduce_matches_after_backward():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    # the "after" path rounds each rank's gradient to bf16 before summing, the
    # overlapped one sums in fp32: agreement to bf16 rounding
    for r in range(world):
        assert out[r] <= 1e-2, out[r]
