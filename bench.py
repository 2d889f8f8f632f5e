#!/usr/bin/env python
"""Throughput of turt's GPU-resident GPT train step on B200 (fwd + bwd + clip + AdamW).

Default workload: the 6-layer / 384-d "modern" GPT (6 heads, SwiGLU 1024, RMSNorm, RoPE,
tied 8192 vocab, block 256, batch 32 sequences per GPU), synthetic uniform tokens and
N(0, 0.02) weights.  One process per GPU (torchrun for N > 1); data parallel with per-layer
NCCL gradient all-reduce inside the backward pass; per-GPU batch is fixed (weak scaling).

Prints one JSON line (rank 0).  `value` is whole-job tokens/s with the token batches
already resident in HBM; `e2e` is the same step through the public C ABI with host token
arrays copied in and the loss copied out every step.  `--impl reference` times the
reference's CPU data-parallel worker pool (a C restatement, see oracle/) on this host.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: vocab, block, layers, heads, embd, arch, hidden, seqs per GPU, micro-batch seqs
    "gpt-6L-384d": dict(V=8192, T=256, L=6, H=6, E=384, arch="modern", hidden=1024, batch=32, micro=32),
    "gpt2-12L-768d": dict(V=8192, T=512, L=12, H=12, E=768, arch="gpt2", hidden=3072, batch=16, micro=16),
    "gpt-12L-768d-dp": dict(V=8192, T=1024, L=12, H=12, E=768, arch="modern", hidden=2048, batch=256, micro=16,
                            global_batch=True),
    "gpt-tiny-4L-128d": dict(V=8192, T=128, L=4, H=4, E=128, arch="modern", hidden=352, batch=8, micro=8),
    # two layers of the gpt2 workload: a small case of its kernels for profiler captures
    "gpt2-2L-768d": dict(V=8192, T=512, L=2, H=12, E=768, arch="gpt2", hidden=3072, batch=16, micro=16),
}
# turt_model_set_attention modes
ATTENTION_MODES = {"auto": 0, "tensor": 1, "flash": 2, "online": 3}
CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def flops_per_token(w) -> int:
    """Algorithmic FLOPs per trained token: 3 * [2L(4E^2 + kEh) + 2EV + 2LTE], k = 3 (SwiGLU) or 2 (GELU);
    causal attention counted at half."""
    k = 3 if w["arch"] == "modern" else 2
    L, E, h, V, T = w["L"], w["E"], w["hidden"], w["V"], w["T"]
    return 3 * (2 * L * (4 * E * E + k * E * h) + 2 * E * V + 2 * L * T * E)


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- reference arm
def cpu_pool_sample(w, workers: int, seed: int):
    """One step of the reference's CPU data-parallel pool (scripts/train-gpt.ts:200-242, C
    restatement in oracle/) over a bounded sample: one full sequence per worker."""
    import numpy as np

    from oracle.oracle import Oracle
    orc = Oracle()
    cfg = orc.cfg(w["V"], w["T"], w["L"], w["H"], w["E"], w["arch"], w["hidden"])
    params = orc.init(cfg, 7)
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    rng = np.random.default_rng(seed)
    n = workers * w["T"]
    ids = rng.integers(0, w["V"], n).astype(np.int32)
    tgt = rng.integers(0, w["V"], n).astype(np.int32)

    def step(k):
        t0 = time.perf_counter()
        orc.dp_step(cfg, params, m, v, k, ids, tgt, workers, w["T"], workers, 3e-4, 0.9, 0.95, 1e-8, 0.1, 1.0)
        return time.perf_counter() - t0

    return step, n


def cpu_info():
    """Host CPU as the CPU baselines report it: logical cores (nproc) and the model name."""
    model = None
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "cpu_model": model}


def pool_workers(w) -> int:
    """W = host cores - 2 worker threads, capped at the batch (scripts/train-gpt.ts:162)."""
    return max(1, min((os.cpu_count() or 4) - 2, w["batch"]))


def run_reference(args, w, rank: int) -> None:
    if rank != 0:
        return
    workers = pool_workers(w)
    step, tokens = cpu_pool_sample(w, workers, 1)
    for k in range(args.warmup):
        step(k + 1)
    secs = [step(args.warmup + k + 1) for k in range(args.steps)]
    total = sum(secs)
    value = tokens * args.steps / total
    line = {
        "impl": "reference", "metric": "train tokens/sec (fwd+bwd+clip+AdamW)", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "model": args.workload, "global_batch": workers, "seq_len": w["T"],
                   "parallelism": f"cpu-dp{workers}"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": workers, "kind": "port",
                         "workers": workers, **cpu_info(),
                         "sample": f"{workers} sequences x {w['T']} tokens per step (one per worker thread), "
                                   f"C restatement of the reference worker pool",
                         "batch_note": "the pool trains one sequence per worker thread per step, the GPU arm "
                                       f"{w['batch']} per GPU; tokens/s normalises the batch size"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def init_weights(model, w, seed: int):
    """N(0, 0.02) weights, residual projections scaled by 1/sqrt(2L), unit gains, zero biases
    (src/models/gpt.ts:97-102,154-155,182-184)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    parts = []
    res = 0.02 / math.sqrt(2 * w["L"])
    for name, shp in zip(model.names, model.shapes):
        n = int(np.prod(shp))
        base = name.split(".")[-1]
        if len(shp) == 1:
            parts.append(np.ones(n, np.float32) if base.endswith("g") else np.zeros(n, np.float32))
        else:
            std = res if base in ("projW", "downW", "mpW") else 0.02
            parts.append((rng.standard_normal(n) * std).astype(np.float32))
    model.load_flat(np.concatenate(parts))


def time_gemm(ctx, M, N, K, reps, precision):
    """Average device time of one TF32 tensor-core GEMM launch (A [M,K], B [N,K] K-major),
    the head-projection shape of the step, timed with CUDA events on the library's stream."""
    import numpy as np
    import torch

    from turt_b200._lib import check, lib
    a, b, c = ctx.buffer(M * K), ctx.buffer(N * K), ctx.buffer(M * N)
    rng = np.random.default_rng(0)
    ctx.upload(a, rng.standard_normal(M * K).astype(np.float32))
    ctx.upload(b, rng.standard_normal(N * K).astype(np.float32))
    stream = torch.cuda.current_stream()
    for _ in range(3):
        check(lib().turt_matmul_into(ctx.handle, a, b, c, M, K, N, 1, 0, 1, 0))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        check(lib().turt_matmul_into(ctx.handle, a, b, c, M, K, N, 1, 0, 1, 0))
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    for p in (a, b, c):
        ctx.free(p)
    ctx.reclaim()
    return ms


def train_throughput(name: str, steps: int, warmup: int, attention: str = "auto"):
    """Device-resident train steps (fwd + bwd + clip + AdamW) of workload `name` on this
    process's current GPU, the whole batch of one GPU per step (micro-batches accumulated):
    tokens/s and ms per step from CUDA events on the library's stream."""
    import numpy as np
    import torch

    from turt_b200.runtime import Context, Model, make_config
    w = WORKLOADS[name]
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = Context(torch.cuda.current_device())
    ctx.set_stream(stream.cuda_stream)
    model = Model(ctx, make_config(w["V"], w["T"], w["L"], w["H"], w["E"], w["arch"], w["hidden"]))
    model.set_attention(ATTENTION_MODES[attention])
    init_weights(model, w, 1234)
    seqs, micro, T = w["batch"], w["micro"], w["T"]
    rng = np.random.default_rng(7)
    ids = torch.from_numpy(rng.integers(0, w["V"], seqs * T).astype(np.int32)).cuda()
    tgt = torch.from_numpy(rng.integers(0, w["V"], seqs * T).astype(np.int32)).cuda()
    k = [0]

    def step():
        model.zero_grad()
        for j in range(seqs // micro):
            off = j * micro * T * 4
            model.forward_backward_device(ids.data_ptr() + off, tgt.data_ptr() + off, micro, T, loss_scale=micro / seqs)
        k[0] += 1
        model.adamw_step(3e-4, 0.9, 0.95, 1e-8, 0.1, 1 - 0.9 ** k[0], 1 - 0.95 ** k[0], clip=1.0)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    loss = model.read_loss()
    model.close()
    ctx.close()
    del ids, tgt
    torch.cuda.empty_cache()
    tok = seqs * T / (ms / 1000.0)
    peaks = measured_peaks()
    tflops = flops_per_token(w) * tok / 1e12
    return {"value": tok, "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "warmup": warmup,
            "global_batch": seqs, "micro_batch": micro, "seq_len": T, "attention": attention, "last_loss": loss,
            "achieved_tflops": tflops, "frac_of_sustained_tf32": tflops / (peaks["bf16_tflops_sustained"] / 2.0)}


def run_gpu(args, w, rank: int, world: int, local_rank: int) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from turt_b200.runtime import Context, Model, make_config

    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = Context(local_rank)
    ctx.set_stream(stream.cuda_stream)
    ctx.set_precision(args.precision)
    model = Model(ctx, make_config(w["V"], w["T"], w["L"], w["H"], w["E"], w["arch"], w["hidden"]))
    model.set_attention(ATTENTION_MODES[args.attention])
    init_weights(model, w, 1234)
    if world > 1:
        uid = [Model.dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        model.dp_init(rank, world, uid[0])

    seqs = w["batch"] // world if w.get("global_batch") else w["batch"]
    micro = min(w["micro"], seqs)
    assert seqs % micro == 0
    n_micro = seqs // micro
    T = w["T"]
    global_seqs = seqs * world
    rng = np.random.default_rng(100 + rank)
    pool = 4  # distinct resident token batches, cycled
    host_ids = [rng.integers(0, w["V"], seqs * T).astype(np.uint32) for _ in range(pool)]
    host_tgt = [rng.integers(0, w["V"], seqs * T).astype(np.uint32) for _ in range(pool)]
    dev_ids = [torch.from_numpy(a.view(np.int32)).cuda() for a in host_ids]
    dev_tgt = [torch.from_numpy(a.view(np.int32)).cuda() for a in host_tgt]
    torch.cuda.synchronize()

    lr, b1, b2, eps, wd, clip = 3e-4, 0.9, 0.95, 1e-8, 0.1, 1.0
    step_no = [0]

    def adam():
        step_no[0] += 1
        k = step_no[0]
        model.adamw_step(lr, b1, b2, eps, wd, 1 - b1 ** k, 1 - b2 ** k, clip=clip, grad_scale=1.0 / world)

    def device_step(i):
        model.zero_grad()
        ids, tgt = dev_ids[i % pool], dev_tgt[i % pool]
        for j in range(n_micro):
            if world > 1:
                model.dp_defer(j < n_micro - 1)
            off = j * micro * T * 4
            model.forward_backward_device(ids.data_ptr() + off, tgt.data_ptr() + off, micro, T,
                                          loss_scale=micro / seqs)
        adam()

    def host_step(i):
        model.zero_grad()
        ids, tgt = host_ids[i % pool], host_tgt[i % pool]
        loss = None
        for j in range(n_micro):
            if world > 1:
                model.dp_defer(j < n_micro - 1)
            sl = slice(j * micro * T, (j + 1) * micro * T)
            loss = model.forward_backward(ids[sl], tgt[sl], micro, T, loss_scale=micro / seqs,
                                          want_loss=(j == n_micro - 1))
        adam()
        return loss

    def timed(fn, steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = torch.tensor([e0.elapsed_time(e1)], device="cuda")
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    for i in range(args.warmup):
        device_step(i)
    model.read_loss()
    launches0 = Context.launch_count()
    with ClockSampler(local_rank) as clk:
        ms = timed(device_step, args.steps)
    launches = Context.launch_count() - launches0
    clocks = clk.summary()
    last_loss = model.read_loss()

    # e2e: host token arrays in, loss out, every step
    for i in range(2):
        host_step(i)
    ms_e2e = timed(host_step, args.steps)

    tokens_per_step = global_seqs * T
    value = tokens_per_step * args.steps / (ms / 1000.0)
    e2e = tokens_per_step * args.steps / (ms_e2e / 1000.0)

    peaks = measured_peaks()
    tf32_peak = peaks["bf16_tflops"] / 2.0  # dense TF32 tensor rate is half the bf16 rate
    tf32_peak_sust = peaks["bf16_tflops_sustained"] / 2.0
    out = None
    if rank == 0:
        N_tok, V, E = micro * T, w["V"], w["E"]
        gemm_ms = time_gemm(ctx, N_tok, V, E, 20, args.precision)
        gemm_flops = 2.0 * N_tok * V * E
        achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12
        f_tok = flops_per_token(w)
        step_tflops = f_tok * value / world / 1e12
        out = {
            "metric": "train tokens/sec (fwd+bwd+clip+AdamW)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if w.get("global_batch") else "weak", "vs_baseline": None,
            "dtype": "tf32x3" if args.precision == 3 else "tf32", "data": "synthetic",
            "config": {"workload": args.workload, "model": args.workload, "global_batch": global_seqs, "seq_len": T,
                       "parallelism": f"dp{world}", "micro_batch": micro, "attention": args.attention,
                       "gemm_precision": "3xTF32 (error-compensated)" if args.precision == 3 else "TF32",
                       "l2": "no flush: each step touches >1 GB of activations and weights (L2 is 126 MB)",
                       "last_loss": last_loss},
            "roofline": {"bound": "tensor", "kernel": "k_gemm_tf32 (head projection %dx%dx%d)" % (N_tok, V, E),
                         "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s", "frac": achieved / tf32_peak,
                         "traffic": (read_profile_traffic("gemm_pair_head_fwd_8192x8192x384.md")
                                     if (N_tok, V, E) == (8192, 8192, 384) else None),
                         "peak_source": f"{peaks['source']} bf16 dense / 2",
                         "launch_ms": gemm_ms,
                         "mma_issue_factor": 3 if args.precision == 3 else 1,
                         "frac_of_precision_peak": achieved * (3 if args.precision == 3 else 1) / tf32_peak},
            "step_roofline": {"flops_per_token": f_tok, "achieved_tflops_per_gpu": step_tflops,
                              "peak_tflops": tf32_peak_sust, "frac": step_tflops / tf32_peak_sust,
                              "peak_source": f"{peaks['source']} bf16 sustained / 2"},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 2 * seqs * T * 4,
                    "d2h_bytes_per_step": 4},
            "gpu_launches": launches,
            "clocks": clocks,
        }
    model.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and world == 1 and args.extra_workloads:
        # the other configurations on the same box, device-resident (no e2e), after the headline run
        extra = {}
        for name, steps, warm in (("gpt2-12L-768d", 5, 3), ("gpt-12L-768d-dp", 2, 3)):
            if name != args.workload:
                extra[name] = train_throughput(name, steps, warm)
        kernels, total_ms, value_ops, _, _ = measure_backward_ops(10, 3)
        extra["backward-ops"] = {"value": value_ops, "unit": "GB/s", "kernels": kernels,
                                 "note": "each launch alone after an L2 flush; median of 10"}
        out["extra_workloads"] = extra
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        workers = pool_workers(w)
        step, tokens = cpu_pool_sample(w, workers, 2)
        secs = step(1)
        # the single-thread variant: one sequence on one core (the reference's CPU train step
        # without the worker pool)
        step1, tokens1 = cpu_pool_sample(w, 1, 3)
        secs1 = step1(1)
        tiny = WORKLOADS["gpt-tiny-4L-128d"]
        wt = pool_workers(tiny)
        step_t, tokens_t = cpu_pool_sample(tiny, wt, 4)
        secs_t = step_t(1)
        out["cpu_baseline"] = {"value": tokens / secs, "unit": "tokens/s", "cores": workers, "kind": "port",
                               "workers": workers, **cpu_info(),
                               "sample": f"one reference CPU data-parallel step over {workers} sequences x {w['T']} "
                                         f"tokens ({workers} worker threads, C restatement of "
                                         f"scripts/train-gpt.ts + train-worker.ts)",
                               "single_thread": {"value": tokens1 / secs1, "unit": "tokens/s", "cores": 1,
                                                 "sample": f"one sequence of {w['T']} tokens on one thread"},
                               "tiny_4L_128d": {"value": tokens_t / secs_t, "unit": "tokens/s", "cores": wt,
                                                "sample": f"one pool step over {wt} sequences x {tiny['T']} tokens "
                                                          "of the 4-layer / 128-d modern GPT"},
                               "batch_note": f"the pool trains {workers} sequences per step, the GPU {global_seqs}; "
                                             "tokens/s normalises the batch size"}
    if out is not None:
        print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------- backward-op workload
OP_ROWS = 8192


def op_bytes():
    """Algorithmic HBM bytes of the standalone backward kernels (each element read or written once)."""
    N, E, h, V, n_adam = OP_ROWS, 384, 1024, 8192, 10_000_000
    return {
        "rms_bwd [8192,384]": 3 * N * E * 4 + 4 * N + 8 * E,
        "swiglu_bwd [8192,1024]": 5 * N * h * 4,
        "softmax_ce_grad [8192,8192]": 2 * N * V * 4 + 2 * N * 4,
        "adamw_clip 10M": 8 * n_adam * 4,
    }


def read_profile_traffic(name: str, key: str = "traffic_bytes_per_launch"):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) recorded by an ncu
    capture summarised under profiles/ (a line `<key>: N`), or None."""
    import re
    path = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(path):
        return None
    m = re.search(re.escape(key) + r":\s*([0-9]+)", open(path).read())
    return int(m.group(1)) if m else None


def measure_backward_ops(steps: int, warmup: int):
    """Standalone timing of the train step's fused memory-bound backward kernels on seeded
    N(0, 1) inputs with 8192 rows; each launch timed alone with CUDA events after an L2 flush.
    Returns (per-kernel results, total ms, aggregate GB/s, launches, clock summary)."""
    import torch

    from turt_b200._lib import check, lib
    from turt_b200.runtime import Context
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = Context(0)
    ctx.set_stream(stream.cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(7)
    dev = "cuda"

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32)

    N, E, h, V, n_adam = OP_ROWS, 384, 1024, 8192, 10_000_000
    x, dy, gam = randn(N, E), randn(N, E), randn(E)
    rstd = torch.rsqrt((x * x).mean(dim=1) + 1e-5)
    dx, dg = torch.empty_like(x), torch.zeros(E, device=dev)
    ga, up, dact = randn(N, h), randn(N, h), randn(N, h)
    dga, dup = torch.empty_like(ga), torch.empty_like(up)
    logits = randn(N, V)
    tgt = torch.randint(0, V, (N,), generator=g, device=dev, dtype=torch.int32)
    loss_rows = torch.empty(N, device=dev)
    p, gr, m = randn(n_adam), randn(n_adam), randn(n_adam)
    v = randn(n_adam).abs()
    flush = torch.empty(64 * 1024 * 1024, device=dev)  # 256 MB > L2
    flush_rd = torch.ones(64 * 1024 * 1024, device=dev)
    P = lambda t: t.data_ptr()
    h_ = ctx.handle
    calls = {
        "rms_bwd [8192,384]": lambda: check(lib().turt_fused_rms_bwd(h_, P(x), P(dy), P(gam), P(rstd), None, P(dx),
                                                                     P(dg), N, E)),
        "swiglu_bwd [8192,1024]": lambda: check(lib().turt_fused_swiglu_bwd(h_, P(ga), P(up), P(dact), P(dga), P(dup),
                                                                            N * h)),
        "softmax_ce_grad [8192,8192]": lambda: check(lib().turt_fused_ce(h_, P(logits), P(tgt), P(loss_rows), N, V,
                                                                          1.0 / N)),
        "adamw_clip 10M": lambda: check(lib().turt_fused_adamw_clip(h_, P(p), P(gr), P(m), P(v), n_adam, 3e-4, 0.9,
                                                                    0.95, 1e-8, 0.1, 0.1, 0.0975, 1.0, None)),
    }
    nbytes = op_bytes()
    peaks = measured_peaks()
    kernels = {}
    launches0 = Context.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clk:
        for name, fn in calls.items():
            for _ in range(warmup):
                fn()
            times = []
            for _ in range(steps):
                flush.fill_(1.0)  # evict: 256 MB of writes
                flush_rd.sum()    # ... then 256 MB of reads, so no dirty line is written back inside the launch
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                e1.synchronize()
                times.append(e0.elapsed_time(e1))
            ms = statistics.median(times)
            gbs = nbytes[name] / (ms / 1000.0) / 1e9
            kernels[name] = {"ms": ms, "bytes": nbytes[name], "gbs": gbs, "frac": gbs / peaks["hbm_gbs"]}
    launches = Context.launch_count() - launches0
    total_ms = sum(k["ms"] for k in kernels.values())
    total_bytes = sum(nbytes.values())
    value = total_bytes / (total_ms / 1000.0) / 1e9
    ctx.close()
    return kernels, total_ms, value, launches, clk.summary()


def run_backward_ops(args, rank: int) -> None:
    if rank != 0:
        return
    kernels, total_ms, value, launches, clocks = measure_backward_ops(args.steps, args.warmup)
    peaks = measured_peaks()
    N = OP_ROWS
    top = "softmax_ce_grad [8192,8192]"
    out = {
        "metric": "standalone backward-op kernels: algorithmic HBM bytes / time", "value": value, "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "backward-ops", "rows": N, "inputs": "seeded N(0,1), uniform int targets",
                   "l2": "flushed before every timed launch (256 MB write, then 256 MB read of another buffer); "
                         "ms = median launch"},
        "kernels": kernels,
        "roofline": {"bound": "hbm", "kernel": "k_ce_fused " + top, "achieved": kernels[top]["gbs"],
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": kernels[top]["frac"],
                     "traffic": read_profile_traffic("backward_ops_8192rows.md", "k_ce_fused_traffic_bytes_per_launch"),
                     "peak_source": f"{peaks['source']} HBM copy"},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_ops_baseline()
    out["e2e"] = {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                  "note": "device-resident kernels: no host copies belong to this workload"}
    print(json.dumps(out), flush=True)


def step_gemm_shapes(w):
    """The tensor-core GEMMs of one train step of workload `w`, as turt_matmul_into calls:
    (name, M, N, K, transA, transB, accumulate, launches per step).  A is [M,K] (transA: stored
    [K,M]), B is [K,N] (transB: stored [N,K]); weight gradients accumulate."""
    N, E, h, V, L = w["micro"] * w["T"], w["E"], w["hidden"], w["V"], w["L"]
    W1 = 2 * h if w["arch"] == "modern" else h
    return [
        ("fwd qkv", N, 3 * E, E, 0, 0, 0, L), ("fwd proj", N, E, E, 0, 0, 0, L), ("fwd mlp up", N, W1, E, 0, 0, 0, L),
        ("fwd mlp down", N, E, h, 0, 0, 0, L), ("fwd head", N, V, E, 0, 1, 0, 1),
        ("dX head", N, E, V, 0, 0, 0, 1), ("dX mlp down (dact)", N, h, E, 0, 1, 0, L),
        ("dX mlp up", N, E, W1, 0, 1, 0, L), ("dX proj", N, E, E, 0, 1, 0, L), ("dX qkv", N, E, 3 * E, 0, 1, 0, L),
        ("dW head", V, E, N, 1, 0, 1, 1), ("dW mlp down", h, E, N, 1, 0, 1, L), ("dW mlp up", E, W1, N, 1, 0, 1, L),
        ("dW proj", E, E, N, 1, 0, 1, L), ("dW qkv", E, 3 * E, N, 1, 0, 1, L),
    ]


def run_gemm_table(args, rank: int) -> None:
    """Every tensor-core GEMM shape of the train step timed on its own (median of back-to-back
    launches on L2-warm operands, as in the step where each GEMM reads what the previous kernel
    wrote), with its algorithmic TFLOP/s and the fraction of the 3xTF32 ceiling (TF32 peak / 3)."""
    if rank != 0:
        return
    import torch

    from turt_b200._lib import check, lib
    from turt_b200.runtime import Context
    w = WORKLOADS[args.table_workload]
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = Context(0)
    ctx.set_stream(stream.cuda_stream)
    ctx.set_precision(args.precision)
    bn, pair = (int(x) for x in args.force_tile.split(","))
    check(lib().turt_gemm_set_tile(bn, pair))
    peaks = measured_peaks()
    tf32 = peaks["bf16_tflops"] / 2.0
    issue = 3 if args.precision == 3 else 1
    g = torch.Generator(device="cuda").manual_seed(7)
    rows, total_ms, total_flop = [], 0.0, 0.0
    launches0 = Context.launch_count()
    with ClockSampler(0) as clk:
        for (name, M, N, K, ta, tb, acc, per_step) in step_gemm_shapes(w):
            a = torch.randn(M * K, generator=g, device="cuda")
            b = torch.randn(K * N, generator=g, device="cuda")
            c = torch.zeros(M * N, device="cuda")

            def fn():
                check(lib().turt_matmul_into(ctx.handle, a.data_ptr(), b.data_ptr(), c.data_ptr(), M, K, N, 1, ta, tb,
                                             acc))

            for _ in range(args.warmup):
                fn()
            times = []
            for _ in range(args.steps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                e1.synchronize()
                times.append(e0.elapsed_time(e1))
            ms = statistics.median(times)
            tflops = 2.0 * M * N * K / (ms / 1000.0) / 1e12
            rows.append({"gemm": name, "M": M, "N": N, "K": K, "A": "MN-major" if ta else "K-major",
                         "B": "K-major" if tb else "MN-major", "us": ms * 1000.0, "tflops": tflops,
                         "frac_tf32": tflops / tf32, "frac_of_precision_peak": tflops * issue / tf32,
                         "per_step": per_step})
            total_ms += ms * per_step
            total_flop += 2.0 * M * N * K * per_step
            del a, b, c
    launches = Context.launch_count() - launches0
    ctx.close()
    agg = total_flop / (total_ms / 1000.0) / 1e12
    out = {"metric": "train-step GEMM throughput, every shape timed alone (algorithmic 2MNK FLOPs)", "value": agg,
           "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "tf32x3" if issue == 3 else "tf32", "data": "synthetic",
           "config": {"workload": "gemm-table", "model": args.table_workload, "tile": args.force_tile,
                      "l2": "not flushed: back-to-back launches on the same operands, median per shape"},
           "shapes": rows,
           "roofline": {"bound": "tensor", "kernel": "all step GEMM shapes", "achieved": agg, "peak": tf32,
                        "unit": "TFLOP/s", "frac": agg / tf32, "frac_of_precision_peak": agg * issue / tf32,
                        "mma_issue_factor": issue, "traffic": None, "peak_source": f"{peaks['source']} bf16 dense / 2"},
           "e2e": {"value": agg, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                   "note": "device-resident operands: no host copies belong to this workload"},
           "gpu_launches": launches, "clocks": clk.summary()}
    print(json.dumps(out), flush=True)


def run_gemm(args, rank: int) -> None:
    """One tensor-core GEMM C[M,N] = A[M,K] B[N,K]^T (both K-major, the head-projection
    layout) repeated: algorithmic 2MNK FLOPs over the median CUDA-event launch time."""
    if rank != 0:
        return
    import torch

    from turt_b200._lib import check, lib
    from turt_b200.runtime import Context
    M, N, K = (int(t) for t in args.gemm.split(","))
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = Context(0)
    ctx.set_stream(stream.cuda_stream)
    ctx.set_precision(args.precision)
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(M, K, generator=g, device="cuda")
    b = torch.randn(N, K, generator=g, device="cuda")
    c = torch.empty(M, N, device="cuda")
    flush = torch.empty(64 * 1024 * 1024, device="cuda")
    flush_rd = torch.ones(64 * 1024 * 1024, device="cuda")

    def fn():
        check(lib().turt_matmul_into(ctx.handle, a.data_ptr(), b.data_ptr(), c.data_ptr(), M, K, N, 1, 0, 1, 0))

    for _ in range(args.warmup):
        fn()
    times = []
    launches0 = Context.launch_count()
    with ClockSampler(0) as clk:
        for _ in range(args.steps):
            flush.fill_(1.0)
            flush_rd.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
    launches = Context.launch_count() - launches0
    ms = statistics.median(times)
    peaks = measured_peaks()
    tf32 = peaks["bf16_tflops"] / 2.0
    achieved = 2.0 * M * N * K / (ms / 1000.0) / 1e12
    issue = 3 if args.precision == 3 else 1
    out = {"metric": "tensor-core GEMM throughput (algorithmic 2MNK FLOPs)", "value": achieved, "unit": "TFLOP/s",
           "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "tf32x3" if issue == 3 else "tf32", "data": "synthetic",
           "config": {"workload": "gemm", "M": M, "N": N, "K": K, "layout": "A [M,K], B [N,K], both K-major",
                      "l2": "flushed before every timed launch (256 MB write, then 256 MB read of another "
                            "buffer); ms = median launch"},
           "roofline": {"bound": "tensor", "kernel": "k_gemm_tf32 / k_gemm_tf32_pair", "achieved": achieved,
                        "peak": tf32, "unit": "TFLOP/s", "frac": achieved / tf32,
                        "frac_of_precision_peak": achieved * issue / tf32, "mma_issue_factor": issue,
                        "traffic": None, "peak_source": f"{peaks['source']} bf16 dense / 2"},
           "e2e": {"value": achieved, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                   "note": "device-resident operands"},
           "gpu_launches": launches, "clocks": clk.summary()}
    ctx.close()
    print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------- decode workload
DECODE_MODEL = "gpt-6L-384d"


def decode_cpu_sample(seconds: float = 10.0):
    """GPT.generate on the CPU (oracle C restatement of src/models/gpt.ts:291-341: one full forward
    over the context per new token), timed on new tokens at contexts 128..; 1 thread."""
    from oracle.oracle import Oracle
    w = WORKLOADS[DECODE_MODEL]
    orc = Oracle()
    cfg = orc.cfg(w["V"], w["T"], w["L"], w["H"], w["E"], w["arch"], w["hidden"])
    params = orc.init(cfg, 1)
    prompt = list(range(1, w["T"] // 2 + 1))
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and n < 16:
        orc.generate(cfg, params, prompt + [n % w["V"]] * n, 1, temperature=1.0, topk=0, rng_state=orc.rng(n))
        n += 1
    secs = time.perf_counter() - t0
    return {"value": n / secs, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{n} new tokens of {DECODE_MODEL} at contexts {w['T'] // 2}..{w['T'] // 2 + n - 1}, one full "
                      f"forward each (oracle C restatement of GPT.generate, 1 thread)"}


def run_decode(args, rank: int) -> None:
    """KV-cached generation on one GPU: prefill T/2 tokens, then T/2 decode steps, each the host
    call a user makes (token in, logits out).  value / e2e: new tokens per second over the K
    timed steps (CUDA events, 8-byte token copy in, 32 KB logits copy out per step included).
    Roofline: the bytes a step must read (every weight once + the cached keys / values) over
    the step time, against the HBM copy peak (the weights mostly sit in L2, so a fraction near
    or above 1 would be possible; a low one means the step is latency-bound)."""
    if rank != 0:
        return
    import numpy as np
    import torch

    from turt_b200.runtime import Context, Model, make_config
    w = WORKLOADS[DECODE_MODEL]
    V, T, L, E = w["V"], w["T"], w["L"], w["E"]
    ctx = Context(0)
    model = Model(ctx, make_config(V, T, L, w["H"], E, w["arch"], w["hidden"]))
    model.init_reference(1)
    ids = [int(x) for x in np.random.default_rng(0).integers(0, V, T)]
    n0 = T // 2
    steps = min(args.steps * 8, T - n0)
    warm = min(args.warmup, 8)
    model.generate_prefill(ids[:n0 - warm])
    for pos in range(n0 - warm, n0):  # warm-up steps (graph capture happens in the first)
        model.generate_step(ids[pos], pos)
    launches0 = Context.launch_count()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for pos in range(n0, n0 + steps):
            model.generate_step(ids[pos], pos)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    launches = Context.launch_count() - launches0
    value = steps / (ms / 1000.0)
    weight_bytes = model.num_params() * 4
    kv_bytes = 2 * L * E * 4 * (n0 + steps / 2)  # mean cached positions read per step
    achieved = (weight_bytes + kv_bytes) / (ms / 1000.0 / steps) / 1e9
    peaks = measured_peaks()
    line = {"metric": "decode tokens/sec (KV-cached generation, batch 1)", "value": value, "unit": "tokens/s",
            "n_gpus": 1, "steps": steps, "warmup": warm, "ms_per_step": ms / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "decode", "model": DECODE_MODEL, "context": f"{n0}..{n0 + steps}",
                       "l2": "no flush: a step re-reads the same weights (the L2 keeps them, as in use)"},
            "roofline": {"bound": "hbm", "kernel": "decode step (GEMVs, split attention, head)",
                         "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                         "bytes_per_step": weight_bytes + kv_bytes, "peak_source": f"{peaks['source']} HBM copy"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": V * 4},
            "gpu_launches": launches, "clocks": clk.summary()}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = decode_cpu_sample()
    model.close()
    ctx.close()
    print(json.dumps(line), flush=True)


def cpu_ops_baseline():
    """The oracle's restatement of the same four ops (single thread) on 1/8 of each workload."""
    import numpy as np

    from oracle.oracle import Oracle
    orc = Oracle()
    rng = np.random.default_rng(7)
    N, E, h, V, n = OP_ROWS // 8, 384, 1024, 8192, 10_000_000 // 8
    x, dy = rng.standard_normal((N, E)).astype(np.float32), rng.standard_normal((N, E)).astype(np.float32)
    gam = rng.standard_normal(E).astype(np.float32)
    a, u, d = (rng.standard_normal(N * h).astype(np.float32) for _ in range(3))
    logits = rng.standard_normal((N, V)).astype(np.float32)
    tgt = rng.integers(0, V, N).astype(np.int32)
    p, g, m = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
    v = np.abs(rng.standard_normal(n)).astype(np.float32)
    t0 = time.perf_counter()
    orc.rmsnorm(x, gam, dy)
    orc.silu_bwd(a, d * u)
    orc.cross_entropy(logits, tgt)
    orc.clip(g, 1.0)
    orc.adamw_bc(p, g, m, v, 3e-4, 0.9, 0.95, 1e-8, 0.1, 0.1, 0.0975)
    secs = time.perf_counter() - t0
    return {"value": sum(op_bytes().values()) / 8 / secs / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": "the four ops on 1/8 of each size (1024 rows, 1.25M AdamW elements), oracle C restatement"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="turt", choices=["turt", "reference"])
    ap.add_argument("--workload", default="gpt-6L-384d",
                    choices=sorted(WORKLOADS) + ["backward-ops", "gemm", "gemm-table", "decode"])
    ap.add_argument("--table-workload", default="gpt-6L-384d", choices=sorted(WORKLOADS),
                    help="model whose train-step GEMM shapes --workload gemm-table times")
    ap.add_argument("--force-tile", default="0,-1",
                    help="BN,PAIR for --workload gemm-table (turt_gemm_set_tile; 0,-1 = the planner's choice)")
    ap.add_argument("--gemm", default="8192,8192,384", help="M,N,K of the gemm workload")
    ap.add_argument("--precision", type=int, default=3, choices=[1, 3])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-workloads", dest="extra_workloads", action="store_false",
                    help="skip timing the gpt2-12L-768d, 12L-768d data-parallel (1 GPU) and backward-op "
                         "workloads after the headline run (N = 1 only)")
    ap.add_argument("--attention", default="auto", choices=sorted(ATTENTION_MODES),
                    help="attention kernels of the train step (turt_model_set_attention)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload in ("gemm", "gemm-table"):
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the gemm workloads are kernel microbenchmarks "
                                  "with no reference counterpart"}), flush=True)
            return
        (run_gemm if args.workload == "gemm" else run_gemm_table)(args, rank)
        return
    if args.workload == "decode":
        if args.impl == "reference":
            if rank == 0:
                line = decode_cpu_sample()
                print(json.dumps({"impl": "reference", "metric": "decode tokens/sec (KV-cached generation, batch 1)",
                                  "value": line["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": 1,
                                  "warmup": 0, "higher_is_better": True, "dtype": "f32", "data": "synthetic",
                                  "config": {"workload": "decode", "model": DECODE_MODEL}, "cpu_baseline": line,
                                  "e2e": {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}), flush=True)
            return
        run_decode(args, rank)
        return
    if args.workload == "backward-ops":
        if args.impl == "reference":
            if rank == 0:
                line = cpu_ops_baseline()
                print(json.dumps({"impl": "reference", "metric": "standalone backward-op kernels: algorithmic HBM "
                                  "bytes / time", "value": line["value"], "unit": "GB/s", "n_gpus": args.gpus,
                                  "steps": 1, "warmup": 0, "higher_is_better": True, "dtype": "f32",
                                  "data": "synthetic", "config": {"workload": "backward-ops"}, "cpu_baseline": line,
                                  "e2e": {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}), flush=True)
            return
        run_backward_ops(args, rank)
        return
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w, rank)
        return
    run_gpu(args, w, rank, world, local_rank)


if __name__ == "__main__":
    main()
