#!/usr/bin/env python3
"""Benchmark of the YOLO26 C2PSA PSA Attention forward (bf16, 1600 tokens).

Workload (configs[1] of the north star): per GPU a batch of 64 seeded N(0,1)
feature maps 128×40×40, weights N(0,0.02), BN folded; bf16 storage, f32
accumulation.  One step = one call of the fused op on the whole batch.
Multi-GPU: one process per GPU (torchrun), image shards with no collective on
the data path (weak scaling: every rank runs its own 64-image batch); the
timing is the max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the CPU restatement of the reference maths (the
reference has no CPU path) with all host threads on a bounded sample of the
same workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "attention images/sec (C2PSA PSA attention fwd, bf16, 1600 tokens)"
UNIT = "images/s"
B_PER_GPU, C, H, W, NH, KD = 64, 128, 40, 40, 2, 32
N_TOK = H * W
# algorithmic FLOPs per image (qkv + QK^T + PV + PE + proj), per the survey's count
FLOP_QKV = 2 * N_TOK * C * (NH * 4 * KD)
FLOP_QK = 2 * NH * N_TOK * N_TOK * KD
FLOP_PV = 2 * NH * N_TOK * N_TOK * 2 * KD
FLOP_PE = 2 * 9 * C * N_TOK
FLOP_PROJ = 2 * N_TOK * C * C
FLOP_IMG = FLOP_QKV + FLOP_QK + FLOP_PV + FLOP_PE + FLOP_PROJ
FLOP_ATTN_IMG = FLOP_QK + FLOP_PV
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# DRAM bytes (read + write) of one attention-kernel launch at the full workload, from the committed
# ncu capture in profiles/psa_fwd_kernels_cfg2_ncu_full.md (52.46 MB read + 4.88 MB written)
ATTN_TRAFFIC_BYTES = 57_345_024


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_sample(n_img: int, threads: int, seed: int = 1234):
    """Times the torch-CPU f32 restatement on ``n_img`` images; returns img/s."""
    import torch
    from oracle import psa_oracle as po
    torch.set_num_threads(threads)
    p = po.psa_synthetic(n_img, H, W, seed=seed)
    t = {k: torch.tensor(v) for k, v in p.items()}
    args = (t["x"], t["w_qkv"], t["b_qkv"], t["w_pe"], t["b_pe"], t["w_proj"], t["b_proj"], NH, KD)
    po.psa_attention_torch(*args)  # warm
    t0 = time.perf_counter()
    po.psa_attention_torch(*args)
    dt = time.perf_counter() - t0
    return n_img / dt, dt


def run_reference(args, ws, rank):
    """CPU reference arm: rank 0 only."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    n_img = B_PER_GPU  # one step = the whole 64-image batch of the workload
    vals = []
    for _ in range(args.warmup):
        cpu_sample(n_img, threads)
    for _ in range(args.steps):
        v, _ = cpu_sample(n_img, threads)
        vals.append(v)
    val = statistics.mean(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * n_img / val,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg2: C2PSA PSA attention fwd, 128x40x40 (1600 tokens), nh=2, kd=32, hd=64",
                   "global_batch": n_img, "seq_len": N_TOK, "parallelism": "host threads"},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{n_img} images of 128x40x40 per step, torch-CPU f32 restatement of the "
                                   "reference maths (the reference has no CPU path)"},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist
    from vision_rs_b200 import _lib
    from vision_rs_b200 import psa as vp

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    rng = np.random.default_rng(1000 + rank)
    B = args.batch
    f = lambda *s, std=1.0: torch.tensor((rng.standard_normal(s) * std).astype(np.float32))
    x = f(B, C, H, W).to(dev, torch.bfloat16)
    op = vp.PsaAttention(f(NH * 4 * KD, C, std=0.02), f(NH * 4 * KD, std=0.02), f(C, 1, 3, 3, std=0.02),
                         f(C, std=0.02), f(C, C, std=0.02), f(C, std=0.02), NH, KD, dtype=torch.bfloat16,
                         device=dev)
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)  # > L2 (126 MB)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clk = ClockSampler(local).__enter__()
    t_w = time.perf_counter()
    nw = 0
    while nw < args.warmup or time.perf_counter() - t_w < args.min_warm_s:
        op.forward_into(x, y)
        nw += 1
        if nw % 50 == 0:
            torch.cuda.synchronize()
    barrier()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    lc0 = _lib.lib().va_launch_count()
    barrier()
    for i in range(args.steps):
        flush.fill_(float(i))  # evict L2 between timed steps (outside the events)
        starts[i].record(stream)
        op.forward_into(x, y)
        ends[i].record(stream)
    barrier()
    clk.__exit__(None, None, None)
    launches = _lib.lib().va_launch_count() - lc0
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = statistics.mean(step_ms)

    # dominant kernel (flash attention) timed alone on the same stream
    dom = time_dominant(op, x, args, stream)

    if args.no_e2e:
        e2e_ms = float("nan")
    else:
        e2e_ms = time_e2e(op, x, y, args, stream, barrier)

    t = torch.tensor([ms, e2e_ms, dom["ms"]], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, dom_ms = t.tolist()

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample()

    if rank == 0:
        emit(args, ws, B, ms, e2e_ms, dom, dom_ms, launches, cpu, clk, x, y)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def time_e2e(op, x, y, args, stream, barrier):
    """Same metric through the public API with host buffers: every step copies
    the batch from pinned host memory, runs the op and copies y back."""
    import torch
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    for _ in range(max(1, args.warmup)):
        op.forward_into(x.copy_(xh, non_blocking=True), y)
        yh.copy_(y, non_blocking=True)
    barrier()
    e_s = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        e_s[i].record(stream)
        x.copy_(xh, non_blocking=True)
        op.forward_into(x, y)
        yh.copy_(y, non_blocking=True)
        e_e[i].record(stream)
    barrier()
    return statistics.mean(s.elapsed_time(e) for s, e in zip(e_s, e_e))


def cpu_baseline_sample():
    """The torch-CPU f32 restatement on this host's cores: whole 64-image
    batches, repeated until ≥10 s of CPU time."""
    threads = os.cpu_count() or 1
    tot_img, tot_s = 0, 0.0
    while tot_s < 10.0:
        v, dt = cpu_sample(B_PER_GPU, threads)
        tot_img += B_PER_GPU
        tot_s += dt
    return {"value": tot_img / tot_s, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{tot_img} images of 128x40x40 in {tot_s:.1f} s (64-image calls), torch-CPU f32 "
                      "restatement of the reference maths (the reference has no CPU path)"}


def emit(args, ws, B, ms, e2e_ms, dom, dom_ms, launches, cpu, clk, x, y):
    pk, src = peaks()
    achieved = dom["flop"] / (dom_ms * 1e-3) / 1e12
    peak = pk["bf16_tflops"]
    line = {
        "metric": METRIC, "value": B * ws / (ms * 1e-3), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "cfg2: C2PSA PSA attention fwd, 128x40x40 (1600 tokens), nh=2, kd=32, hd=64",
                   "global_batch": B * ws, "per_gpu_batch": B, "seq_len": N_TOK,
                   "parallelism": f"image shards x{ws}, no collective",
                   "l2": "flushed between timed steps (256 MB write)",
                   "precision": "bf16 I/O and qkv GEMM; f16 attention operands; f32 accumulation"},
        "e2e": None if math.isnan(e2e_ms) else {
            "value": B * ws / (e2e_ms * 1e-3), "unit": UNIT,
            "h2d_bytes_per_step": x.numel() * x.element_size(),
            "d2h_bytes_per_step": y.numel() * y.element_size()},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "kernel": dom["name"], "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": f"{src} bf16_tflops (burst)",
                     "traffic": ATTN_TRAFFIC_BYTES if B == B_PER_GPU else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                                       "(profiles/psa_fwd_kernels_cfg2_ncu_full.md)",
                     "flop_per_launch": dom["flop"], "ms_per_launch": dom_ms},
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
        "tflops_whole_op": FLOP_IMG * B / (ms * 1e-3) / 1e12,
    }
    print(json.dumps(line), flush=True)


def time_dominant(op, x, args, stream):
    """Average duration of the dominant kernel — the tcgen05 flash-attention
    kernel — timed alone with CUDA events on the launching stream, on the
    op's own intermediates (Q/K/V as the qkv kernel left them in the
    workspace)."""
    import torch
    from vision_rs_b200 import _lib
    B = x.shape[0]
    y = torch.empty_like(x)
    op.forward_into(x, y)  # fills the workspace: qk at offset 0, then v, then o
    ws = op.workspace(B, H, W, x.device)
    Np = (N_TOK + 7) // 8 * 8
    al = lambda n: (n + 255) // 256 * 256
    qk_off = 0
    v_off = qk_off + al(2 * B * NH * N_TOK * KD * 2)
    o_off = v_off + al(B * C * Np * 2)
    base = ws.data_ptr()
    st = stream.cuda_stream
    call = lambda: _lib.call("va_psa_flash_attention_fwd_f16", base + qk_off, base + v_off, base + o_off, None,
                             B, NH, H, W, st)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    n = max(5, args.steps)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=x.device)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for i in range(n):
        flush.fill_(float(i))
        evs[i][0].record(stream)
        call()
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    return {"name": "attn_kernel (tcgen05 flash attention, QK^T + PV, 64-wide V)", "ms": ms,
            "flop": B * FLOP_ATTN_IMG}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--min-warm-s", type=float, default=1.5,
                    help="keep warming up at least this long so the clock sampler sees the load")
    ap.add_argument("--batch", type=int, default=B_PER_GPU, help="per-GPU batch (profiling of smaller cases)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
