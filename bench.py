#!/usr/bin/env python
"""Benchmark of the ETHOS expert layer on B200 (one process per GPU).

Headline metric: expert-layer tokens/s at the default size -- config 2: 16384
tokens per GPU (batch 8 x seq 2048), d_model 1024, 262144 experts (two
512-entry sub-key tables), d_latent 128, d_hidden 512, 8 heads, top_k 16, bf16
forward with BatchNorm in eval mode, seeded synthetic N(0,1) inputs and
N(0, 1/sqrt(fan_in)) parameters (no dataset is used).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ethos|reference]

For N > 1 run it under torchrun (one rank per GPU): tokens shard across ranks
with the parameters replicated and no collective in the forward (weak scaling,
16384 tokens per GPU).  ``value`` = all ranks' tokens / max-over-ranks time.

The same line carries a ``train`` block (config 5): the training step --
forward with BatchNorm on batch statistics, backward through all parameters,
the NCCL all-reduce of every gradient overlapped with the backward (N > 1) and
a fused AdamW update -- timed at the same N, with the all-reduce time left
exposed and a cross-rank checksum of the reduced gradients and updated
parameters (the run exits non-zero if the ranks disagree) -- and short
``router`` (config 3, the routing microbenchmark) and ``decoder`` (config 4:
the whole 12-layer decoder forward with the ETHOS expert layers) blocks.

``--impl reference`` times the reference path's CPU implementation on the
host cores (the vectorised fp32 restatement in oracle/ethos_oracle.py of
SimplifiedHypernetMoE.forward, model.py:288-343; the reference's own code does
not travel to the GPU box) on a bounded token sample.
"""

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG1 = dict(d_model=512, num_experts=4096, top_k=16, num_routing_heads=8, d_latent=128,
            d_intermediate_hypernet=512, d_query=512)
CFG2 = dict(d_model=1024, num_experts=512 * 512, top_k=16, num_routing_heads=8, d_latent=128,
            d_intermediate_hypernet=512, d_query=512)
TOKENS = 16384
METRIC = "expert-layer tokens/s (262K experts, k=16x8 heads)"
UNIT = "tokens/s"
L2_FLUSH_BYTES = 256 << 20

# Algorithmic work at config 2 (router + experts forward), per token:
#   MACs: q-proj 8*512*1024, scoring 8*2*512*256, x_proj 1024*512,
#         expansion 128*128*512, dot + weighted sum 2*128*512, W_v 512*1024
FLOP_PER_TOKEN = 2 * (8 * 512 * 1024 + 8 * 2 * 512 * 256 + 1024 * 512 + 128 * 128 * 512
                      + 2 * 128 * 512 + 512 * 1024)
# Algorithmic HBM bytes per token of the whole forward: x in (2 KiB bf16),
# y out (2 KiB), the 128 selected latent rows (128 x 256 B), plus the weights
# (11.2 MB per step) spread over the step's tokens
HBM_BYTES_PER_TOKEN = 2048 + 2048 + 128 * 256
WEIGHT_BYTES = 11.2e6
N_EXPERTS = 512 * 512
# per-stage algorithmic work for the kernel roofline (kind, amount per step as
# a function of T): GEMM stages in FLOPs, the expert stage in HBM bytes
#   projection   x @ [Wq_0..Wq_7 | W_u]       2 * 1024 * 4608 per token
#   topk         sub-key scores q . K          2 * 8 * 2 * 512 * 256 per token
#   expert_table gelu(E @ W1^T), once per expert  2 * N * 128 * 512 per step
#   experts      the layer's HBM-gather term: the token's 128 selected latent
#                rows of 256 B (bf16 x 128).  This kernel reads 1 KB fp16 rows
#                of the expert table instead (4x the bytes, in exchange for
#                evaluating each expert's hidden row once per step rather than
#                once per selection), so its fraction of this roof is at most
#                about 1/4; its DRAM rate against the copy peak is reported
#                beside it as "dram".
#   end          hacc @ W_v                     2 * 512 * 1024 per token
STAGE_WORK = {
    "projection": ("tensor", lambda T: 2.0 * 1024 * 4608 * T),
    "topk": ("tensor", lambda T: 2.0 * 8 * 2 * 512 * 256 * T),
    "expert_table": ("tensor", lambda T: 2.0 * N_EXPERTS * 128 * 512),
    "experts": ("hbm", lambda T: 128 * 256 * float(T)),
    "end": ("tensor", lambda T: 2.0 * 512 * 1024 * T),
}
STAGE_KERNEL = {"projection": "k_gemm2sm<EpiProj> (2-SM pairs)", "topk": "k_score_topk<16>",
                "expert_table": "k_gemm_bf16_tn<EpiGeluF16>", "experts": "k_expert_gather",
                "end": "k_gemm_bf16_tn<EpiStoreBF16>"}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return dict(hbm_gbs=float(p["hbm_gbs"]), bf16_tflops=float(p["bf16_tflops"]),
                    bf16_tflops_sustained=float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                    source="measured")
    except (OSError, KeyError, ValueError):
        return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, source="fallback")


def load_traffic(stage):
    """Per-launch DRAM bytes of a stage's kernel from its committed ncu summary
    (profiles/<stage>_config2.md, line 'dram_bytes_per_launch: <bytes>')."""
    path = os.path.join(ROOT, "profiles", f"{stage}_config2.md")
    try:
        with open(path) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


def launches():
    """Kernels libethos_b200 has launched so far in this process."""
    from ethos_b200._lib import lib
    return int(lib().ethos_launch_count())


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed loop runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


def build_layer(device, dtype=torch.bfloat16):
    from ethos_b200 import EthosConfig, EthosExpertLayer
    from ethos_b200.init import seeded_init_
    layer = EthosExpertLayer(EthosConfig(**CFG2))
    seeded_init_(layer, seed=0)
    return layer.to(device=device, dtype=dtype).eval()


def _oracle_setup(cfg, tokens, round_bf16):
    from ethos_b200 import EthosConfig, EthosExpertLayer
    from ethos_b200.config import layer_dims
    from ethos_b200.init import seeded_input, seeded_state_dict
    from oracle import ethos_oracle as orc
    c = EthosConfig(**cfg)
    sd = seeded_state_dict(EthosExpertLayer(c), seed=0)
    p = orc.params_from_state_dict(sd, layer_dims(c), round_bf16=round_bf16)
    x = seeded_input(tokens, cfg["d_model"], seed=0)
    if round_bf16:
        x = x.to(torch.bfloat16).float()
    return orc, p, x


def _timed_loop(fn, tokens, budget_s):
    """Runs ``fn`` (which processes ``tokens`` tokens) until ``budget_s``
    seconds have passed; returns (tokens/s, tokens done, seconds)."""
    done, t0 = 0, time.perf_counter()
    while True:
        fn()
        done += tokens
        el = time.perf_counter() - t0
        if el >= budget_s:
            return done / el, done, el


def cpu_baseline(tokens_budget_s=12.0, sample_tokens=512):
    """Times the oracle restatement of the reference forward (fp32, all host
    threads) on repeated 512-token chunks of the config-2 workload for about
    `tokens_budget_s` seconds."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    orc, p, x = _oracle_setup(CFG2, sample_tokens, round_bf16=True)
    with torch.no_grad():
        orc.layer_forward(x[:64], p, CFG2["top_k"])  # warm-up
        val, done, el = _timed_loop(lambda: orc.layer_forward(x, p, CFG2["top_k"]), sample_tokens, tokens_budget_s)
    return dict(value=val, unit=UNIT, cores=cores, kind="port",
                sample=f"{done} tokens in {sample_tokens}-token chunks of config 2 (oracle fp32 restatement "
                       f"of model.py:288-343, torch CPU, {cores} threads), {el:.1f} s")


def cpu_baseline_config1(budget_s=2.0):
    """Config 1 in full: the 256-token fp32 forward at d_model 512 with 4096
    experts (the reference's own CPU-runnable case), repeated for ~budget_s."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    orc, p, x = _oracle_setup(CFG1, 256, round_bf16=False)
    with torch.no_grad():
        orc.layer_forward(x[:32], p, CFG1["top_k"])
        val, done, el = _timed_loop(lambda: orc.layer_forward(x, p, CFG1["top_k"]), 256, budget_s)
    return dict(value=val, unit=UNIT, cores=cores, kind="port",
                sample=f"config 1 in full (256 tokens, d_model 512, 4096 experts, fp32, BN eval), "
                       f"{done // 256} forwards in {el:.1f} s")


def cpu_baseline_train(budget_s=5.0, sample_tokens=256):
    """The training step's CPU counterpart: forward with BatchNorm on batch
    statistics and autograd backward through every parameter, on 256-token
    samples at config-2 dimensions (fp32 oracle restatement)."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    orc, p, x = _oracle_setup(CFG2, sample_tokens, round_bf16=True)
    p.requires_grad_(True)
    gy = torch.randn(x.shape, generator=torch.Generator().manual_seed(1))

    def step():
        for t in p.tensors():
            t.grad = None
        xr = x.clone().requires_grad_(True)
        y, _, _, _ = orc.layer_forward(xr, p, CFG2["top_k"], training=True)
        (y * gy).sum().backward()

    step()
    val, done, el = _timed_loop(step, sample_tokens, budget_s)
    return dict(value=val, unit=UNIT, cores=cores, kind="port",
                sample=f"{done} tokens in {sample_tokens}-token forward+backward samples at config-2 dims "
                       f"(oracle fp32 restatement, BN train, autograd through model.py:208-343), {el:.1f} s")


def run_reference(args, rank, world):
    if rank != 0:
        return
    steps = []
    cb = None
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(tokens_budget_s=args.ref_seconds, sample_tokens=512)
        if i >= args.warmup:
            steps.append(r["value"])
        cb = r
    val = sum(steps) / len(steps)
    line = dict(metric=METRIC, value=val, unit=UNIT, n_gpus=args.gpus, steps=args.steps, warmup=args.warmup,
                ms_per_step=1000.0 * 512 / val, higher_is_better=True, scaling="weak", vs_baseline=None,
                dtype="f32", data="synthetic", impl="reference",
                config=dict(workload="config 2: ETHOS expert layer forward, 262144 experts, k=16 x 8 heads, "
                                     "d_model 1024 (CPU sample)", tokens_per_sample=512),
                cpu_baseline=dict(value=val, unit=UNIT, cores=cb["cores"], kind=cb["kind"], sample=cb["sample"]),
                e2e=dict(value=val, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


def _bits_hash(t):
    """Order-dependent hash of a tensor's bit pattern (int64, on its device):
    equal tensors give equal hashes on every rank."""
    v = t.detach().contiguous().view(-1)
    if v.numel() == 0:
        return torch.zeros((), dtype=torch.int64, device=v.device)
    iv = v.view(torch.int16).to(torch.int64) & 0xFFFF
    w = torch.arange(iv.numel(), device=iv.device, dtype=torch.int64) % 65521 + 1
    return (iv * w).sum()


def train_block(args, rank, world, local, dev, layer=None, steps=None, sampler=True):
    """Config 5: the training step -- forward with BatchNorm on batch
    statistics, backward through every parameter, the NCCL AVG all-reduce of
    the flat fp32 gradient buffer overlapped with the backward (world > 1),
    then a fused AdamW update with fp32 master weights -- 16384 tokens per GPU.
    Returns the rank-0 report (every rank must call it: it runs collectives)."""
    import torch.distributed as dist
    from ethos_b200 import ops
    from ethos_b200.dist import overlap_grad_allreduce
    from ethos_b200.init import seeded_input, tensor_generator
    from ethos_b200.optim import FusedAdamW
    steps = steps or args.steps
    if layer is None:
        layer = build_layer(dev)
    layer.train()
    T = args.tokens
    x = seeded_input(T, CFG2["d_model"], seed=rank).to(device=dev, dtype=torch.bfloat16)
    gy = (torch.randn((T, CFG2["d_model"]), generator=tensor_generator(rank, "bench.gy")) * 1e-3).to(
        device=dev, dtype=torch.bfloat16)
    # AdamW as the reference's DeepSpeed config (train.py:74-79, with its
    # gradient clipping at global norm 1.0, train.py:100), fused over all of
    # the layer's parameters in one launch, fp32 master weights for bf16
    opt = FusedAdamW(layer.parameters(), lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                     max_grad_norm=1.0)
    comm = None
    if world > 1:
        overlap_grad_allreduce(layer)  # all-reduce inside the backward, overlapped
        comm = layer._grad_comm
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        opt.zero_grad(set_to_none=True)
        y = layer(x.view(1, T, -1))
        y.backward(gy.view(1, T, -1))
        opt.step()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    ops.check_device_error(dev)
    if comm is not None:
        comm["log"] = []
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    clk = ClockSampler(local) if sampler else None
    if clk:
        clk.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n_launch = launches()
    for s_, e_ in ev:
        flush.zero_()
        s_.record(stream)
        step()
        e_.record(stream)
    torch.cuda.synchronize()
    n_launch = launches() - n_launch
    if world > 1:
        dist.barrier()
    clocks = clk.stop() if clk else None
    ops.check_device_error(dev)
    ms = sum(s_.elapsed_time(e_) for s_, e_ in ev) / len(ev)
    ar = None
    if comm is not None:
        log = comm.pop("log")
        span = sum(a.elapsed_time(b) for _, _, a, b in log) / len(log)
        exposed = sum(max(0.0, end.elapsed_time(b)) for _, end, _, b in log) / len(log)
        tail = sum(e0.elapsed_time(end) for e0, end, _, _ in log) / len(log)
        ar = [span, exposed, tail]
    # cross-rank agreement: the reduced gradients of the last step and the
    # parameters after its update must be bit-identical on every rank
    params = list(layer.parameters())
    hashes = torch.stack([_bits_hash(p.grad) for p in params] + [_bits_hash(p) for p in params])
    if world > 1:
        t = torch.tensor([ms] + (ar or [0.0, 0.0, 0.0]), dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ar = t[0].item(), t[1:].tolist()
        gathered = [torch.empty_like(hashes) for _ in range(world)]
        dist.all_gather(gathered, hashes)
        identical = all(torch.equal(g_, gathered[0]) for g_ in gathered)
    else:
        identical = True
    grad_bytes = sum(p.numel() for p in params) * 4
    out = dict(metric="expert-layer training tokens/s (262K experts, k=16x8 heads)",
               value=T * world / (ms / 1e3), unit=UNIT, ms_per_step=ms, steps=steps, tokens_per_gpu=T,
               global_batch=T * world, parallelism=f"dp{world}", dtype="bf16 (fp32 gradients and master weights)",
               workload="config 5: forward (BN on batch statistics), backward through all 37 parameters, "
                        "NCCL AVG all-reduce of the fp32 gradients overlapped with the backward (N > 1), "
                        "global-norm gradient clipping at 1.0 and fused AdamW with fp32 master weights",
               l2="flushed between timed steps (256 MiB write)", gpu_launches=n_launch,
               allreduce=dict(bytes_per_step=grad_bytes if world > 1 else 0,
                              span_ms=ar[0] if ar else 0.0, exposed_ms=ar[1] if ar else 0.0,
                              overlap_window_ms=ar[2] if ar else 0.0,
                              note="span: first all-reduce start to last end on the side stream; exposed: "
                                   "after the backward's last kernel; overlap window: backward time after "
                                   "the latent-table gradient is final (max over ranks)"),
               grads_and_params_identical_across_ranks=identical)
    if clocks is not None:
        out["clocks"] = clocks
    if comm is not None:
        del layer._grad_comm
        for p in params:
            p._ethos_allreduced = False
    del opt
    return out


def run_train(args, rank, world, local, dev):
    """--mode train: config 5 alone, as its own JSON line."""
    tr = train_block(args, rank, world, local, dev)
    if rank == 0:
        line = dict(metric=tr["metric"], value=tr["value"], unit=UNIT, n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=tr["ms_per_step"], higher_is_better=True, scaling="weak",
                    vs_baseline=None, dtype="bf16", data="synthetic",
                    config=dict(workload=tr["workload"], tokens_per_gpu=tr["tokens_per_gpu"],
                                global_batch=tr["global_batch"], parallelism=tr["parallelism"], l2=tr["l2"]),
                    allreduce=tr["allreduce"], gpu_launches=tr["gpu_launches"],
                    grads_and_params_identical_across_ranks=tr["grads_and_params_identical_across_ranks"],
                    clocks=tr.get("clocks"))
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_train()
        print(json.dumps(line), flush=True)
    if not tr["grads_and_params_identical_across_ranks"]:
        raise SystemExit("ranks disagree on the reduced gradients / updated parameters")


def router_block(args, rank, world, local, dev, steps=None, sampler=True):
    """Config 3: product-key routing micro-benchmark -- 65 536 normalised
    queries per head for 8 heads (N(0,1), bf16, d_key 256), two 512 x 128
    sub-key tables, top-16 per half, top-16 of the candidate sums, int32 ids
    and fp32 softmax weights (ethos_product_key_topk).  Unit: query-heads.
    Returns the report (every rank must call it)."""
    import torch.distributed as dist
    from ethos_b200 import ops
    from ethos_b200.init import tensor_generator
    steps = steps or args.steps
    H, Q, dk, K, k = 8, 65536, 256, 512, 16
    g = tensor_generator(rank, "bench.router")
    q = torch.randn((H, Q, dk), generator=g).to(device=dev, dtype=torch.bfloat16)
    keys = (torch.randn((2, K, dk // 2), generator=g) / (dk // 2) ** 0.5).to(device=dev, dtype=torch.bfloat16)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        ops.product_key_topk(q, keys, k)
    torch.cuda.synchronize()
    ops.check_device_error(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    n_launch = launches()
    clk = ClockSampler(local) if sampler else None
    if clk:
        clk.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for s_, e_ in ev:
        flush.zero_()
        s_.record(stream)
        ops.product_key_topk(q, keys, k)
        e_.record(stream)
    torch.cuda.synchronize()
    n_launch = launches() - n_launch
    if world > 1:
        dist.barrier()
    clocks = clk.stop() if clk else None
    ms = sum(s_.elapsed_time(e_) for s_, e_ in ev) / len(ev)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    peaks = load_peaks()
    flops = 2.0 * 2 * K * (dk // 2) * H * Q
    tf = flops / (ms / 1e3) / 1e12
    out = dict(metric="product-key routing query-heads/s (2 x 512 sub-keys, d_key 256, top-16)",
               value=H * Q * world / (ms / 1e3), unit="query-heads/s", ms_per_step=ms, steps=steps,
               workload="config 3: product-key routing microbenchmark, 65536 queries x 8 heads, "
                        "bf16 queries, fp32 scores, int32 ids + fp32 weights",
               queries_per_head=Q, heads=H, parallelism=f"dp{world}",
               l2="flushed between timed steps (256 MiB write)",
               roofline=dict(bound="tensor", kernel="k_score_topk<16>", achieved=tf, peak=peaks["bf16_tflops"],
                             unit="TFLOP/s", frac=tf / peaks["bf16_tflops"], traffic=None,
                             peak_source=peaks["source"] + " bf16 burst"),
               gpu_launches=n_launch)
    if clocks is not None:
        out["clocks"] = clocks
    return out


def run_router(args, rank, world, local, dev):
    """--mode router: config 3 alone, as its own JSON line."""
    r = router_block(args, rank, world, local, dev)
    if rank == 0:
        line = dict(metric=r["metric"], value=r["value"], unit=r["unit"], n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=r["ms_per_step"], higher_is_better=True, scaling="weak",
                    vs_baseline=None, dtype="bf16", data="synthetic",
                    config=dict(workload=r["workload"], queries_per_head=r["queries_per_head"], heads=r["heads"],
                                parallelism=r["parallelism"], l2=r["l2"]),
                    roofline=r["roofline"], gpu_launches=r["gpu_launches"], clocks=r.get("clocks"))
        print(json.dumps(line), flush=True)


def fp32_block(args, rank, world, local, dev, steps=None):
    """The fp32 arithmetic path (fp32 parameters, the split-bf16 contractions):
    config 2 with 16 384 tokens per GPU, the forward with BatchNorm on running
    statistics and the forward + backward with batch statistics.  Returns the
    report (every rank must call it)."""
    import torch.distributed as dist
    from ethos_b200 import ops
    from ethos_b200.init import seeded_input, tensor_generator
    steps = steps or args.steps
    layer = build_layer(dev, dtype=torch.float32)
    T = args.tokens
    x = seeded_input(T, CFG2["d_model"], seed=rank).to(dev)
    gy = (torch.randn((T, CFG2["d_model"]), generator=tensor_generator(rank, "bench.gy32")) * 1e-3).to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def fwd():
        with torch.no_grad():
            layer(x.view(1, T, -1))

    def fwd_bwd():
        for q in layer.parameters():
            q.grad = None
        layer(x.view(1, T, -1)).backward(gy.view(1, T, -1))

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        ops.check_device_error(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for s_, e_ in ev:
            flush.zero_()
            s_.record(stream)
            fn()
            e_.record(stream)
        torch.cuda.synchronize()
        ops.check_device_error(dev)
        ms = sum(s_.elapsed_time(e_) for s_, e_ in ev) / len(ev)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms

    layer.eval()
    fwd_ms = timed(fwd)
    layer.train()
    train_ms = timed(fwd_bwd)
    del layer
    return dict(workload="config 2 with fp32 parameters: fp32 arithmetic path (split-bf16 tcgen05 "
                         "contractions, everything between them in fp32), 16384 tokens per GPU",
                forward_ms=fwd_ms, forward_tokens_per_s=T * world / (fwd_ms / 1e3),
                forward_backward_ms=train_ms, forward_backward_tokens_per_s=T * world / (train_ms / 1e3),
                batchnorm="running statistics in the forward line, batch statistics in forward + backward",
                l2="flushed between timed steps (256 MiB write)", steps=steps)


def decoder_block(args, rank, world, local, dev, steps=None, sampler=True):
    """Config 4: the whole ETHOS decoder forward (ethos_b200.decoder.EthosDecoder,
    the reference CompressedMoEModel's architecture, model.py:345-395): 12
    layers of RMSNorm + multi-head latent attention (16 heads, latent KV 256,
    rotary) + RMSNorm + ETHOS expert layer (config-2 dimensions), the final
    RMSNorm and the tied output head over a 100 277-entry vocabulary, on
    batch 8 x sequence 2048 token ids drawn Zipf(1.1), every parameter seeded
    by name, bf16.  Only the expert layers run on this repository's kernels;
    attention is torch's scaled_dot_product_attention (cuDNN's sm100 kernel on
    a B200; the reference calls flash_attn, whose sm80 kernel is slower here).
    A second,
    untimed pass records CUDA events around every expert layer for their share
    of the forward.  Every rank must call it."""
    import numpy as np
    import torch.distributed as dist
    from ethos_b200 import ops
    from ethos_b200.decoder import DecoderConfig, EthosDecoder
    from ethos_b200.init import seeded_state_dict
    steps = steps or args.steps
    seq = 2048
    T = args.tokens
    if T % seq != 0:
        raise SystemExit("--tokens must be a multiple of the sequence length 2048 for the decoder")
    cfg = DecoderConfig(num_layers=12, num_dense_layers=0, vocab_size=100277, **CFG2)
    model = EthosDecoder(cfg)
    sd = seeded_state_dict(model, seed=0)
    sd["tok_embeddings.weight"] = sd["output.weight"]
    model.load_state_dict(sd)
    del sd
    model = model.to(device=dev, dtype=torch.bfloat16).eval()
    rng = np.random.default_rng(1000 + rank)
    ids = rng.zipf(1.1, size=4 * T)
    ids = torch.from_numpy(ids[ids <= cfg.vocab_size][:T] - 1).to(dev).view(T // seq, seq)
    assert ids.numel() == T
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):
            model(ids)
        torch.cuda.synchronize()
        ops.check_device_error(dev)
        attn_impl = "flash_attn" if model.layers[0].self_attn.use_flash_attn else \
            "torch scaled_dot_product_attention"
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        n_launch = launches()
        clk = ClockSampler(local) if sampler else None
        if clk:
            clk.start()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for s_, e_ in ev:
            flush.zero_()
            s_.record(stream)
            model(ids)
            e_.record(stream)
        torch.cuda.synchronize()
        n_launch = launches() - n_launch
        if world > 1:
            dist.barrier()
        clocks = clk.stop() if clk else None
        ops.check_device_error(dev)
        # untimed: events around every expert layer
        marks = []
        hooks = []
        for layer in model.expert_layers():
            hooks.append(layer.register_forward_pre_hook(
                lambda m, a: marks.append(torch.cuda.Event(enable_timing=True)) or marks[-1].record(stream)))
            hooks.append(layer.register_forward_hook(
                lambda m, a, o: marks.append(torch.cuda.Event(enable_timing=True)) or marks[-1].record(stream)))
        totals = []
        for _ in range(3):
            marks.clear()
            flush.zero_()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            model(ids)
            e0.record(stream)
            torch.cuda.synchronize()
            expert = sum(marks[2 * i].elapsed_time(marks[2 * i + 1]) for i in range(len(marks) // 2))
            totals.append((expert, s0.elapsed_time(e0)))
        for h in hooks:
            h.remove()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in ev) / len(ev)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    expert_ms = sum(a for a, _ in totals) / len(totals)
    whole_ms = sum(b for _, b in totals) / len(totals)
    out = dict(metric="ETHOS decoder forward tokens/s (12 layers: MLA attention + ETHOS expert layer, "
                      "262K experts, k=16x8; vocab 100277)",
               value=T * world / (ms / 1e3), unit="tokens/s", ms_per_step=ms, steps=steps,
               data="synthetic (Zipf(1.1) token ids), random init",
               workload="config 4: embedding, 12 x (RMSNorm, MLA attention 16 heads / latent KV 256 / rotary, "
                        "RMSNorm, ETHOS expert layer), RMSNorm, tied output head; batch 8 x seq 2048",
               attention=attn_impl, expert_layers_ms=expert_ms, expert_share=expert_ms / whole_ms,
               tokens_per_gpu=T, batch=T // seq, seq_len=seq, layers=cfg.num_layers, vocab=cfg.vocab_size,
               parallelism=f"dp{world}", l2="flushed between timed steps (256 MiB write)", gpu_launches=n_launch)
    if clocks is not None:
        out["clocks"] = clocks
    del model
    return out


def run_decoder(args, rank, world, local, dev):
    """--mode decoder: config 4, the whole decoder forward, as its own JSON line."""
    r = decoder_block(args, rank, world, local, dev)
    if rank == 0:
        line = dict(metric=r["metric"], value=r["value"], unit=r["unit"], n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=r["ms_per_step"], higher_is_better=True, scaling="weak",
                    vs_baseline=None, dtype="bf16", data=r["data"],
                    config=dict(workload=r["workload"], tokens_per_gpu=r["tokens_per_gpu"], batch=r["batch"],
                                seq_len=r["seq_len"], layers=r["layers"], vocab=r["vocab"],
                                parallelism=r["parallelism"], l2=r["l2"], attention=r["attention"]),
                    expert_layers_ms=r["expert_layers_ms"], expert_share=r["expert_share"],
                    gpu_launches=r["gpu_launches"], clocks=r.get("clocks"))
        print(json.dumps(line), flush=True)

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ethos", choices=["ethos", "reference"])
    ap.add_argument("--tokens", type=int, default=TOKENS, help="tokens per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-train", action="store_true", help="leave the training block out of the forward line")
    ap.add_argument("--train-steps", type=int, default=20, help="timed training steps in the train block")
    ap.add_argument("--no-extra", action="store_true",
                    help="leave the config-3 router and config-4 decoder blocks out of the forward line")
    ap.add_argument("--ref-seconds", type=float, default=3.0,
                    help="CPU seconds per reference-arm step (a bounded sample of the workload)")
    ap.add_argument("--no-numa-bind", action="store_true",
                    help="with several ranks, leave each rank's CPU affinity alone instead of binding it to its "
                         "GPU's NUMA node (pinned staging buffers then land wherever the process first runs)")
    ap.add_argument("--mode", default="forward", choices=["forward", "train", "router", "decoder", "stack"],
                    help="forward: config 2 (headline, with the config-5 train block); train: config 5 alone; "
                         "router: config 3 routing microbenchmark; decoder (or stack): config 4, the whole "
                         "decoder forward")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    args.warmup = max(args.warmup, 3)

    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    args.host_cpus = None
    if world > 1 and not args.no_numa_bind:
        # each rank's pinned host buffers on its GPU's NUMA node (one rank per
        # GPU shares the host links; the single-rank run keeps every core for
        # its CPU baseline)
        from ethos_b200.dist import bind_to_device_numa
        cpus = bind_to_device_numa(dev)
        args.host_cpus = len(cpus) if cpus else None
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    ok = True
    try:
        if args.mode in ("train", "router", "decoder", "stack"):
            {"train": run_train, "router": run_router, "decoder": run_decoder,
             "stack": run_decoder}[args.mode](args, rank, world, local, dev)
        else:
            ok = run_forward(args, rank, world, local, dev)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    if not ok:
        raise SystemExit("ranks disagree on the reduced gradients / updated parameters")


def run_forward(args, rank, world, local, dev):
    """Config 2 (the headline) plus the config-5 train block; returns False if
    the ranks' reduced gradients or updated parameters differ."""
    import torch.distributed as dist
    from ethos_b200 import ops
    from ethos_b200.init import seeded_input
    layer = build_layer(dev)
    T = args.tokens
    x_host = seeded_input(T, CFG2["d_model"], seed=rank).to(torch.bfloat16).pin_memory()
    x_dev = x_host.to(dev)
    y_host = torch.empty((T, CFG2["d_model"]), dtype=torch.bfloat16).pin_memory()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    with torch.no_grad():
        # ---------------- device-resident forward (value) -----------------
        for _ in range(args.warmup):
            layer(x_dev.view(1, T, -1))
        torch.cuda.synchronize()
        ops.check_device_error(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        sampler = ClockSampler(local)
        sampler.start()
        barrier()
        torch.cuda.synchronize()
        n_launch = launches()
        for s, e in ev:
            flush.zero_()  # L2 flush between timed steps (outside the events)
            s.record(stream)
            layer(x_dev.view(1, T, -1))
            e.record(stream)
        torch.cuda.synchronize()
        n_launch = launches() - n_launch
        barrier()
        clocks = sampler.stop()
        ms = sum(s.elapsed_time(e) for s, e in ev) / len(ev)
        ms = max_over_ranks(ms)

        # ---------------- per-kernel stage timing (roofline) ---------------
        pw = layer._packed(dev)
        n_ev = len(ops.STAGES)
        sev = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(max(5, min(args.steps, 20)))]
        for _ in range(2):
            ops.layer_forward(x_dev, pw, False, 1e-5, 0.1, path=layer.expert_path)
        for evs in sev:
            flush.zero_()
            ops.layer_forward(x_dev, pw, False, 1e-5, 0.1, path=layer.expert_path, stage_events=evs)
        torch.cuda.synchronize()
        ops.check_device_error(dev)
        stage_ms = {}
        for i in range(1, n_ev):
            name = ops.STAGES[i]
            v = sum(evs[i - 1].elapsed_time(evs[i]) for evs in sev) / len(sev)
            stage_ms[name] = max_over_ranks(v)
        # the fused per-token expert path on the same routing, for comparison
        out = ops.layer_forward(x_dev, pw, False, 1e-5, 0.1, save=True)
        fev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(3)]
        ops.expert_forward(pw.latents, pw.w1, out["ids"], out["weights"], out["xp"], pw.dims, path=ops.EXPERT_FUSED)
        for s_, e_ in fev:
            flush.zero_()
            s_.record(stream)
            ops.expert_forward(pw.latents, pw.w1, out["ids"], out["weights"], out["xp"], pw.dims,
                               path=ops.EXPERT_FUSED)
            e_.record(stream)
        torch.cuda.synchronize()
        fused_ms = max_over_ranks(sum(s_.elapsed_time(e_) for s_, e_ in fev) / len(fev))
        del out

        # ---------------- end to end through the public API ---------------
        # Serving pipeline over three streams: the upload of step i+1 and the
        # download of step i-1 overlap the layer call of step i.  Every step
        # still uploads its input from pinned host memory, runs the layer
        # (after a 256 MiB L2 flush on the compute stream, inside the timed
        # region) and downloads its output; the timed span runs from before
        # the first upload to after the last download.  With compute=False
        # the same copies run alone (the host-link floor of the pipeline).
        e2e_steps = max(4, args.steps)  # the pipeline fills and drains once per run
        s_in = torch.cuda.Stream(dev)
        s_out = torch.cuda.Stream(dev)
        xd = [torch.empty_like(x_dev) for _ in range(2)]
        yh = [y_host, torch.empty_like(y_host).pin_memory()]
        y_stub = torch.zeros((T, CFG2["d_model"]), dtype=torch.bfloat16, device=dev)

        def pipeline(n, t0=None, t1=None, compute=True):
            up = [torch.cuda.Event() for _ in range(n)]
            used = [torch.cuda.Event() for _ in range(n)]
            done = [torch.cuda.Event() for _ in range(n)]
            down = [torch.cuda.Event() for _ in range(n)]
            if t0 is not None:
                t0.record(s_in)
            for i in range(n):
                b = i & 1
                with torch.cuda.stream(s_in):
                    if i >= 2:
                        s_in.wait_event(used[i - 2])  # the layer of step i-2 has read xd[b]
                    xd[b].copy_(x_host, non_blocking=True)
                    up[i].record(s_in)
                stream.wait_event(up[i])
                if compute:
                    flush.zero_()
                    y = layer(xd[b].view(1, T, -1)).view(T, -1)
                else:
                    y = y_stub
                used[i].record(stream)
                done[i].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(done[i])
                    if i >= 2:
                        s_out.wait_event(down[i - 2])  # yh[b] was read back by step i-2
                    yh[b].copy_(y, non_blocking=True)
                    y.record_stream(s_out)
                    down[i].record(s_out)
            if t1 is not None:
                s_in.wait_stream(s_out)
                t1.record(s_in)

        pipeline(3)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        pipeline(e2e_steps, t0, t1)
        torch.cuda.synchronize()
        barrier()
        ems = max_over_ranks(t0.elapsed_time(t1) / e2e_steps)
        ops.check_device_error(dev)
        # the same copies alone, concurrently on every rank
        pipeline(3, compute=False)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        pipeline(e2e_steps, t0, t1, compute=False)
        torch.cuda.synchronize()
        barrier()
        copy_ms = max_over_ranks(t0.elapsed_time(t1) / e2e_steps)

        # the same steps strictly one after another on one stream, for reference
        sev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(5)]
        for s, e in sev2:
            flush.zero_()
            s.record(stream)
            xs = x_host.to(dev, non_blocking=True)
            y = layer(xs.view(1, T, -1))
            y_host.copy_(y.view(T, -1), non_blocking=True)
            e.record(stream)
        torch.cuda.synchronize()
        serial_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in sev2) / len(sev2))

        # serving with frozen parameters: the expert table cached across
        # forwards (built once, outside the timed steps), L2 flushed per step
        layer.cache_expert_table = True
        for _ in range(2):
            layer(x_dev.view(1, T, -1))
        cev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(10)]
        for s, e in cev:
            flush.zero_()
            s.record(stream)
            layer(x_dev.view(1, T, -1))
            e.record(stream)
        torch.cuda.synchronize()
        layer.cache_expert_table = False
        cached_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in cev) / len(cev))
        ops.check_device_error(dev)
        del xd, yh, y_stub

    # ---------------- config 5: the training step at the same N --------------
    train = None
    if not args.no_train:
        train = train_block(args, rank, world, local, dev, layer=layer, steps=args.train_steps, sampler=False)
    del layer
    # configs 3 and 4 in the same run (short blocks; their own modes print
    # full lines): the routing microbenchmark and the 12 expert layers
    extra = {}
    if not args.no_extra and args.tokens == TOKENS:
        torch.cuda.empty_cache()
        extra["router"] = router_block(args, rank, world, local, dev, steps=20, sampler=False)
        extra["decoder"] = decoder_block(args, rank, world, local, dev, steps=5, sampler=False)
        torch.cuda.empty_cache()
        extra["fp32"] = fp32_block(args, rank, world, local, dev, steps=5)

    peaks = load_peaks()
    total_tokens = T * world
    value = total_tokens / (ms / 1e3)
    # roofline of the dominant kernel (largest stage of the step)
    stages = {k: v for k, v in stage_ms.items() if k in STAGE_WORK and v > 0}
    dom = max(stages, key=stages.get)
    kind, work = STAGE_WORK[dom]
    amount = work(T)
    if kind == "tensor":
        achieved, peak, unit = amount / (stages[dom] / 1e3) / 1e12, peaks["bf16_tflops"], "TFLOP/s"
    else:
        achieved, peak, unit = amount / (stages[dom] / 1e3) / 1e9, peaks["hbm_gbs"], "GB/s"
    traffic = load_traffic(dom)
    stage_report = {}
    for k, v in stages.items():
        kk, ww = STAGE_WORK[k]
        a = ww(T) / (v / 1e3)
        rep = dict(ms=v, kernel=STAGE_KERNEL[k], achieved=a / (1e12 if kk == "tensor" else 1e9),
                   unit="TFLOP/s" if kk == "tensor" else "GB/s",
                   frac=(a / 1e12 / peaks["bf16_tflops"]) if kk == "tensor" else (a / 1e9 / peaks["hbm_gbs"]))
        tr_k = load_traffic(k)
        if tr_k is not None:
            rep["dram_gbs"] = tr_k / (v / 1e3) / 1e9
            rep["dram_frac"] = rep["dram_gbs"] / peaks["hbm_gbs"]
        stage_report[k] = rep
    roofline = dict(bound=kind, kernel=STAGE_KERNEL[dom], stage=dom, achieved=achieved, peak=peak, unit=unit,
                    frac=achieved / peak, traffic=traffic,
                    peak_source=peaks["source"] + (" bf16 burst" if kind == "tensor" else " HBM copy"))
    if kind == "hbm":
        roofline["algorithmic_bytes_per_launch"] = amount
        roofline["note"] = ("achieved = the layer's HBM-gather term (128 selected latent rows x 256 B per token) "
                            "/ launch time; the kernel reads 1 KB fp16 expert-table rows per selection instead, "
                            "see dram")
        if traffic is not None:
            roofline["dram"] = dict(achieved=traffic / (stages[dom] / 1e3) / 1e9, unit="GB/s",
                                    frac=traffic / (stages[dom] / 1e3) / 1e9 / peak,
                                    source="dram_bytes_per_launch of profiles/experts_config2.md / launch time")
    layer_bytes = HBM_BYTES_PER_TOKEN * T + WEIGHT_BYTES
    line = dict(
        metric=METRIC, value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
        ms_per_step=ms, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="bf16",
        data="synthetic",
        config=dict(workload="config 2: ETHOS expert layer forward (router + experts), 262144 experts, "
                             "k=16 x 8 heads, d_model 1024, d_latent 128, d_hidden 512, BN eval",
                    tokens_per_gpu=T, global_batch=total_tokens, parallelism=f"dp{world} (token shards)",
                    l2="flushed between timed steps (256 MiB write)", expert_path="auto (table at this size)"),
        layer_tflops=FLOP_PER_TOKEN * T / (ms / 1e3) / 1e12,
        layer_roof=dict(tensor_frac=FLOP_PER_TOKEN * T / (ms / 1e3) / 1e12 / peaks["bf16_tflops"],
                        hbm_frac=layer_bytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                        note="whole forward: algorithmic FLOPs / bf16 burst peak and algorithmic HBM bytes "
                             "(x, y, 128 latent rows per token, weights) / copy peak"),
        roofline=roofline,
        stages=stage_report,
        fused_expert_path_ms=fused_ms,
        cached_table_serving=dict(value=total_tokens / (cached_ms / 1e3), unit=UNIT, ms_per_step=cached_ms,
                                  note="frozen parameters: expert table built once and reused, not the headline"),
        e2e=dict(value=total_tokens / (ems / 1e3), unit=UNIT, h2d_bytes_per_step=x_host.numel() * 2,
                 d2h_bytes_per_step=y_host.numel() * 2, ms_per_step=ems, steps=e2e_steps,
                 pipeline="upload / layer / download on three streams, L2 flush per step inside the span",
                 serial_ms_per_step=serial_ms, copy_only_ms_per_step=copy_ms,
                 copy_only_note="the same uploads and downloads without the layer, concurrently on every rank "
                                "(max over ranks)",
                 host_binding=(f"each rank bound to the {args.host_cpus} CPUs of its GPU's NUMA node before its "
                               "pinned buffers were allocated" if args.host_cpus else "process CPU affinity as "
                               "started")),
        gpu_launches=n_launch,
        clocks=clocks,
    )
    if train is not None:
        line["train"] = train
    line.update(extra)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
        line["cpu_baseline"]["config1"] = cpu_baseline_config1()
        if train is not None:
            train["cpu_baseline"] = cpu_baseline_train()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return train is None or train["grads_and_params_identical_across_ranks"]


if __name__ == "__main__":
    main()
