#!/usr/bin/env python3
"""Benchmarks of the B200 attention hot path of vision-rs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfg1|...|cfg5]

Configurations (the north star's configs; synthetic seeded inputs of the
named shapes and distributions, random-init weights):

* ``cfg1``: the same op in f32 on one 128×20×20 feature map (batch 1, 400
  tokens): the latency of the f32 path.
* ``cfg2`` (default, the headline): YOLO26 C2PSA PSA Attention forward, bf16,
  per GPU a batch of 64 feature maps 128×40×40 (1600 tokens).  Step = one
  call of the fused op on the batch.
* ``cfg3``: RF-DETR MSDeformAttn forward + backward, batch 8, 300 queries,
  16 heads × 16, levels 80²/40²/20², 4 points (``--dtype f32|bf16``).
* ``cfg4``: DINOv2-S attention (packed QKV Linear + attention, bf16), batch 16
  at 560×560 (1 + 40×40 tokens): one global layer + one 4×4-windowed layer.
* ``cfg5``: PSA Attention training step, bf16 with f32 master weights, 32
  images of 128×20×20 per GPU: forward + backward + NCCL all-reduce of the
  weight gradients + SGD.
* ``conv``: the convolutions around the block — every Conv+BN+SiLU of the
  YOLO26n backbone layers 1-8 at 640×640 input (18 convs, 1×1 and 3×3,
  stride 1 and 2, 8 to 384 channels), bf16 NHWC, batch 64; each conv runs on
  its own resident input.  Step = the 18 conv launches.

Multi-GPU: one process per GPU (torchrun), image shards (weak scaling); cfg2-4
have no collective, cfg5 all-reduces its gradients.  Timing: CUDA events on
the launching stream, L2 flushed between timed steps, max over ranks.
``--impl reference`` times the CPU restatement of the same maths (the
reference has no CPU path; for cfg3/cfg4 the reference has no such operator at
all) with all host threads on a bounded sample; under torchrun only rank 0 runs.
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

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}

# ── cfg1 constants ──────────────────────────────────────────────────────────
C, NH, KD = 128, 2, 32
P1_B, P1_H, P1_W = 1, 20, 20
N1 = P1_H * P1_W
# one flash_attention2_forward call (one V half, 32 wide): QK^T + PV FLOPs and q/k/v/o + LSE bytes
FLOP_FA_CALL1 = 2 * NH * N1 * N1 * KD * 2
BYTES_FA_CALL1 = 4 * NH * N1 * KD * 4 + NH * N1 * 4
FLOP_IMG1 = 2 * N1 * C * (NH * 4 * KD) + 2 * FLOP_FA_CALL1 + 2 * 9 * C * N1 + 2 * N1 * C * C

# ── cfg2 constants ──────────────────────────────────────────────────────────
P2_B, P2_H, P2_W = 64, 40, 40
N2 = P2_H * P2_W
FLOP_ATTN_IMG2 = 2 * NH * N2 * N2 * KD + 2 * NH * N2 * N2 * 2 * KD
FLOP_IMG2 = 2 * N2 * C * (NH * 4 * KD) + FLOP_ATTN_IMG2 + 2 * 9 * C * N2 + 2 * N2 * C * C
# DRAM bytes (read + write) of one attention-kernel launch at the full cfg2 workload, measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum of attn_kernel, one launch: 52.46 MB read + 4.88 MB written)
ATTN_TRAFFIC_BYTES = 57_345_024

# ── cfg3 constants (SURVEY per-unit bytes) ──────────────────────────────────
MS_B, MS_Q, MS_NH, MS_DH, MS_P = 8, 300, 16, 16, 4
MS_SHAPES = ((80, 80), (40, 40), (20, 20))
MS_FWD_BYTES = {"f32": 76_800_000, "bf16": 34_406_400 + 3_686_400 + 1_843_200 + 1_228_800}
MS_BWD_BYTES_F32 = 151_100_000

# ── cfg4 constants ──────────────────────────────────────────────────────────
DN_B, DN_HID, DN_HEADS, DN_GRID, DN_WIN = 16, 384, 6, 40, 10
DN_N = 1 + DN_GRID * DN_GRID
DN_NW = (DN_GRID // DN_WIN) ** 2
DN_NWIN = 1 + DN_WIN * DN_WIN
DN_FLOP_GLOBAL_ATTN_IMG = 2 * 2 * DN_HEADS * DN_N * DN_N * 64
DN_FLOP_IMG = (2 * DN_N * DN_HID * 3 * DN_HID + DN_FLOP_GLOBAL_ATTN_IMG
               + 2 * DN_NW * DN_NWIN * DN_HID * 3 * DN_HID + 2 * 2 * DN_HEADS * DN_NW * DN_NWIN * DN_NWIN * 64)

# ── conv stack: YOLO26n backbone layers 1-8 at 640 (name, C_in, C_out, k, stride, input H = W) ──
CONV_B = 64
CONV_LAYERS = [("l1", 16, 32, 3, 2, 320), ("l2.cv1", 32, 32, 1, 1, 160), ("l2.m.cv1", 16, 8, 3, 1, 160),
               ("l2.m.cv2", 8, 16, 3, 1, 160), ("l2.cv2", 48, 64, 1, 1, 160), ("l3", 64, 64, 3, 2, 160),
               ("l4.cv1", 64, 64, 1, 1, 80), ("l4.m.cv1", 32, 16, 3, 1, 80), ("l4.m.cv2", 16, 32, 3, 1, 80),
               ("l4.cv2", 96, 128, 1, 1, 80), ("l5", 128, 128, 3, 2, 80), ("l6.cv1", 128, 128, 1, 1, 40),
               ("l6.m.cv3x3", 32, 32, 3, 1, 40), ("l6.cv2", 192, 128, 1, 1, 40), ("l7", 128, 256, 3, 2, 40),
               ("l8.cv1", 256, 256, 1, 1, 20), ("l8.m.cv3x3", 64, 64, 3, 1, 20), ("l8.cv2", 384, 256, 1, 1, 20)]


def conv_out(h, k, s):
    return (h + 2 * (k // 2) - k) // s + 1


def conv_layer_work(ci, co, k, s, h):
    """(FLOP, bytes) of one image through one conv: MACs × 2; x in + y out (bf16) + weights."""
    ho = conv_out(h, k, s)
    return 2 * ho * ho * co * ci * k * k, 2 * (h * h * ci + ho * ho * co) + 2 * co * ci * k * k


# ── cfg5 constants ──────────────────────────────────────────────────────────
T5_B, T5_H, T5_W = 32, 20, 20
N5 = T5_H * T5_W
FLOP_FWD_IMG5 = 2 * N5 * C * 256 + 2 * NH * N5 * N5 * (KD + 2 * KD) + 2 * 9 * C * N5 + 2 * N5 * C * C


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def stop(self):
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
        for ln in self.lines:
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
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def evict_l2(flush, i):
    """Evict L2 (126 MB) with a 256 MB buffer: write it, then read it back, so
    the cache holds only clean lines of the buffer — the timed work neither
    finds its inputs cached nor pays for writing back the eviction's own
    dirty lines."""
    flush.fill_(float(i))
    flush.sum()


def event_time(fn, n, stream, flush=None):
    """Mean duration (ms) of ``fn`` over n launches, CUDA events on ``stream``,
    L2 evicted before each (outside the events)."""
    import torch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for i in range(n):
        if flush is not None:
            evict_l2(flush, i)
        evs[i][0].record(stream)
        fn()
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(b) for a, b in evs)


def pipelined_e2e_ms(steps, h2d, compute, d2h, nbuf=2):
    """Per-step time of a serving pipeline: step i's host→device copy, compute
    and device→host copy run on three streams, so the copies of one step
    overlap the compute of its neighbours (nbuf device buffers per direction).
    h2d(b, stream), compute(b, stream), d2h(b, stream) issue step work on
    buffer b; each runs with its stream current, so torch copies land on it.
    Timed with CUDA events from the first copy-in to the last copy-out."""
    import torch
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    in_done = [torch.cuda.Event() for _ in range(nbuf)]
    cmp_done = [torch.cuda.Event() for _ in range(nbuf)]
    out_done = [torch.cuda.Event() for _ in range(nbuf)]
    for e in cmp_done + out_done:
        e.record(torch.cuda.current_stream())
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    for i in range(steps):
        b = i % nbuf
        s_in.wait_event(cmp_done[b])       # the compute that read this input buffer is done
        with torch.cuda.stream(s_in):
            h2d(b, s_in)
        in_done[b].record(s_in)
        s_cmp.wait_event(in_done[b])
        s_cmp.wait_event(out_done[b])      # the copy-out that read this output buffer is done
        with torch.cuda.stream(s_cmp):
            compute(b, s_cmp)
        cmp_done[b].record(s_cmp)
        s_out.wait_event(cmp_done[b])
        with torch.cuda.stream(s_out):
            d2h(b, s_out)
        out_done[b].record(s_out)
    t1.record(s_out)
    s_in.wait_event(out_done[(steps - 1) % nbuf])
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / steps


# ═════════════════════════════ workloads ═════════════════════════════════════
class Cfg1:
    metric = "attention images/sec (C2PSA PSA attention fwd, f32, 400 tokens, batch 1)"
    unit, dtype, batch = "images/s", "f32", P1_B
    workload = "cfg1: C2PSA PSA attention fwd, f32, 1x128x20x20 (400 tokens), nh=2, kd=32, hd=64"

    def __init__(self, dev, rank, batch, args):
        import torch
        from vision_rs_b200 import psa as vp
        rng = np.random.default_rng(900 + rank)
        f = lambda *s, std=1.0: torch.tensor((rng.standard_normal(s) * std).astype(np.float32))
        self.B = batch
        self.x = f(batch, C, P1_H, P1_W).to(dev)
        self.op = vp.PsaAttention(f(NH * 4 * KD, C, std=0.02), f(NH * 4 * KD, std=0.02), f(C, 1, 3, 3, std=0.02),
                                  f(C, std=0.02), f(C, C, std=0.02), f(C, std=0.02), NH, KD, dtype=torch.float32,
                                  device=dev)
        self.y = torch.empty_like(self.x)
        self.xh = self.x.cpu().pin_memory()
        self.yh = torch.empty_like(self.xh).pin_memory()
        self.packed = f(4, batch * NH, N1, KD).to(dev)  # a packed Q|K|V_lo|V_hi buffer for the kernel alone

    def step(self):
        self.op.forward_into(self.x, self.y)

    def e2e_step(self):
        self.x.copy_(self.xh, non_blocking=True)
        self.op.forward_into(self.x, self.y)
        self.yh.copy_(self.y, non_blocking=True)

    def io_bytes(self):
        return self.x.numel() * 4, self.y.numel() * 4

    def dominant(self, args, stream, flush):
        """One flash_attention2_forward call (the FFMA flash attention, one
        32-wide V half; the op makes two) on a packed buffer of cfg1's size."""
        import torch
        from vision_rs_b200 import _lib
        BH = self.B * NH
        sec = BH * N1 * KD * 4
        base, st = self.packed.data_ptr(), stream.cuda_stream
        o = torch.empty(BH, N1, KD, device=self.x.device)
        lse = torch.empty(BH * N1, device=self.x.device)
        call = lambda: _lib.call("va_flash_attention2_forward_f32", base, base + sec, base + 2 * sec, o.data_ptr(),
                                 lse.data_ptr(), N1, N1, 1.0 / math.sqrt(KD), float("-inf"), BH, KD, st)
        for _ in range(args.warmup):
            call()
        ms = event_time(call, max(5, args.steps), stream, flush)
        pk, src = peaks()
        work = BYTES_FA_CALL1 * self.B
        ach = work / (ms * 1e-3) / 1e9
        return {"bound": "hbm", "kernel": "fa_fwd_simt_kernel (f32 FFMA flash attention, one V half)",
                "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                "peak_source": f"{src} hbm_gbs", "traffic": None, "bytes_per_launch": work,
                "flop_per_launch": FLOP_FA_CALL1 * self.B, "ms_per_launch": ms,
                "note": "latency-bound: one image is 800 query rows; neither HBM nor the FFMA pipe is the limit"}

    def extra(self, ms):
        return {"us_per_image": 1000.0 * ms / self.B, "gflops_whole_op": FLOP_IMG1 * self.B / (ms * 1e-3) / 1e9}

    config = {"seq_len": N1, "precision": "f32 throughout (FFMA kernels; the f32 bound max-abs 1e-5 rules out TF32)"}

    @staticmethod
    def cpu_sample(threads, n_img=1, seed=1234):
        import torch
        from oracle import psa_oracle as po
        torch.set_num_threads(threads)
        p = po.psa_synthetic(1, P1_H, P1_W, seed=seed)
        t = {k: torch.tensor(v) for k, v in p.items()}
        a = (t["x"], t["w_qkv"], t["b_qkv"], t["w_pe"], t["b_pe"], t["w_proj"], t["b_proj"], NH, KD)
        po.psa_attention_torch(*a)
        t0 = time.perf_counter()
        for _ in range(n_img):
            po.psa_attention_torch(*a)
        return n_img, time.perf_counter() - t0

    sample_desc = ("single images of 128x20x20 (batch 1), torch-CPU f32 restatement of the reference maths (the "
                   "reference has no CPU path)")


# YOLO26 widths of the C2PSA block (c2psa sets num_heads = c/64): n → 128, s/m/l → 256, x → 384
WIDTHS = {"n": 128, "s": 256, "x": 384}


class Cfg2:
    unit, dtype, batch = "images/s", "bf16", P2_B

    @staticmethod
    def names(width):
        """(metric, workload) of the config at a YOLO26 width."""
        Cw = WIDTHS[width]
        wtag = "" if width == "n" else f", width {width} (C={Cw})"
        return (f"attention images/sec (C2PSA PSA attention fwd, bf16, 1600 tokens{wtag})",
                f"cfg2: C2PSA PSA attention fwd, {Cw}x40x40 (1600 tokens), nh={Cw // 64}, kd=32, hd=64")

    def __init__(self, dev, rank, batch, args):
        import torch
        from vision_rs_b200 import psa as vp
        self.C = WIDTHS[args.width]
        self.nh = self.C // 64
        Cw, nh = self.C, self.nh
        self.metric, self.workload = self.names(args.width)
        self.flop_attn_img = FLOP_ATTN_IMG2 * nh // NH
        self.flop_img = 2 * N2 * Cw * (nh * 4 * KD) + self.flop_attn_img + 2 * 9 * Cw * N2 + 2 * N2 * Cw * Cw
        rng = np.random.default_rng(1000 + rank)
        f = lambda *s, std=1.0: torch.tensor((rng.standard_normal(s) * std).astype(np.float32))
        self.B = batch
        self.x = f(batch, Cw, P2_H, P2_W).to(dev, torch.bfloat16)
        self.op = vp.PsaAttention(f(nh * 4 * KD, Cw, std=0.02), f(nh * 4 * KD, std=0.02), f(Cw, 1, 3, 3, std=0.02),
                                  f(Cw, std=0.02), f(Cw, Cw, std=0.02), f(Cw, std=0.02), nh, KD,
                                  dtype=torch.bfloat16, device=dev)
        self.y = torch.empty_like(self.x)
        self.xh = self.x.cpu().pin_memory()
        self.yh = torch.empty_like(self.xh).pin_memory()

    def step(self):
        self.op.forward_into(self.x, self.y)

    def e2e_step(self):
        self.x.copy_(self.xh, non_blocking=True)
        self.op.forward_into(self.x, self.y)
        self.yh.copy_(self.y, non_blocking=True)

    def e2e_pipelined(self, steps):
        import torch
        xs = [self.x, torch.empty_like(self.x)]
        ys = [self.y, torch.empty_like(self.y)]
        return pipelined_e2e_ms(steps, lambda b, st: xs[b].copy_(self.xh, non_blocking=True),
                                lambda b, st: self.op.forward_into(xs[b], ys[b], stream=st),
                                lambda b, st: self.yh.copy_(ys[b], non_blocking=True))

    def io_bytes(self):
        return self.x.numel() * 2, self.y.numel() * 2

    def dominant(self, args, stream, flush):
        """The tcgen05 flash-attention kernel alone on the op's intermediates."""
        from vision_rs_b200 import _lib
        B = self.B
        self.op.forward_into(self.x, self.y)
        ws = self.op.workspace(B, P2_H, P2_W, self.x.device)
        Np = (N2 + 7) // 8 * 8
        al = lambda n: (n + 255) // 256 * 256
        Cw, nh = self.C, self.nh
        # workspace offsets of Q/K, V and O: the C = 128 kernels' layout, or the general one (after qkv)
        qk_off = 0 if Cw == C else al(B * 2 * Cw * Np * 2)
        v_off = qk_off + al(2 * B * nh * N2 * KD * 2)
        o_off = v_off + al(B * Cw * Np * 2)
        base, st = ws.data_ptr(), stream.cuda_stream
        call = lambda: _lib.call("va_psa_flash_attention_fwd_f16", base + qk_off, base + v_off, base + o_off, None,
                                 B, nh, P2_H, P2_W, st)
        for _ in range(args.warmup):
            call()
        ms = event_time(call, max(5, args.steps), stream, flush)
        pk, src = peaks()
        work = B * self.flop_attn_img
        ach = work / (ms * 1e-3) / 1e12
        return {"bound": "tensor", "kernel": "attn_kernel (tcgen05 flash attention, QK^T + PV, 64-wide V)",
                "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": ach / pk["bf16_tflops"],
                "peak_source": f"{src} bf16_tflops (burst)",
                "traffic": ATTN_TRAFFIC_BYTES if (B == P2_B and Cw == C) else None,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at this workload",
                "flop_per_launch": work, "ms_per_launch": ms}

    def extra(self, ms):
        return {"tflops_whole_op": self.flop_img * self.B / (ms * 1e-3) / 1e12}

    @property
    def config(self):
        return {"seq_len": N2, "channels": self.C, "heads": self.nh,
                "precision": "bf16 I/O and qkv GEMM; f16 attention operands; f32 accumulation"}

    def cpu_sample(self, threads, n_img=P2_B, seed=1234):
        import torch
        from oracle import psa_oracle as po
        torch.set_num_threads(threads)
        Cw = WIDTHS[getattr(self, "width", "n")]
        p = po.psa_synthetic(n_img, P2_H, P2_W, C=Cw, num_heads=Cw // 64, seed=seed)
        t = {k: torch.tensor(v) for k, v in p.items()}
        a = (t["x"], t["w_qkv"], t["b_qkv"], t["w_pe"], t["b_pe"], t["w_proj"], t["b_proj"], Cw // 64, KD)
        po.psa_attention_torch(*a)
        t0 = time.perf_counter()
        po.psa_attention_torch(*a)
        return n_img, time.perf_counter() - t0

    sample_desc = "images of Cx40x40, torch-CPU f32 restatement of the reference maths (the reference has no CPU path)"


class Cfg3:
    unit, batch = "images/s", MS_B
    workload = "cfg3: RF-DETR MSDeformAttn fwd+bwd, Q=300, 16 heads x 16, levels 80x80/40x40/20x20, P=4"

    def __init__(self, dev, rank, batch, args):
        import torch
        from oracle import msdeform_oracle as mo
        from vision_rs_b200 import msdeform as ms
        self.dtype = args.dtype
        self.metric = f"attention images/sec (RF-DETR MSDeformAttn fwd+bwd, {self.dtype})"
        self.ms, self.B = ms, batch
        p = mo.msdeform_synthetic(B=batch, Q=MS_Q, nh=MS_NH, dh=MS_DH, shapes=MS_SHAPES, P=MS_P, seed=100 + rank)
        tdt = torch.float32 if self.dtype == "f32" else torch.bfloat16
        self.d = {k: torch.as_tensor(v).to(dev, tdt if k in ("value", "grad_out") else None) for k, v in p.items()}
        self.ws = torch.empty(ms.msdeform_attn_workspace_bytes(batch, MS_NH, 3, MS_Q, MS_P), dtype=torch.uint8,
                              device=dev)
        self.args = (self.d["value"], self.d["spatial_shapes"], self.d["level_start"], self.d["loc"], self.d["attn"])
        self.h = {k: self.d[k].cpu().pin_memory() for k in ("value", "loc", "attn", "grad_out")}
        self.out = None
        S = sum(h * w for h, w in MS_SHAPES)
        self.touched = self._touched(p, S)

    @staticmethod
    def _touched(p, S):
        """Distinct (b, pixel, head) value rows any sample reads (host count)."""
        loc, shapes = p["loc"], np.asarray(MS_SHAPES)
        B, Q, nh, L, P, _ = loc.shape
        rows = set()
        for l, (H, W) in enumerate(shapes):
            s0 = int(sum(h * w for h, w in MS_SHAPES[:l]))
            x = loc[..., l, :, 0] * W - 0.5
            y = loc[..., l, :, 1] * H - 0.5
            x0, y0 = np.floor(x).astype(np.int64), np.floor(y).astype(np.int64)
            bi = np.broadcast_to(np.arange(B)[:, None, None, None], x0.shape)
            hi = np.broadcast_to(np.arange(nh)[None, None, :, None], x0.shape)
            for dy in (0, 1):
                for dx in (0, 1):
                    xi, yi = x0 + dx, y0 + dy
                    ok = (xi >= 0) & (xi < W) & (yi >= 0) & (yi < H)
                    key = (bi[ok] * S + s0 + yi[ok] * W + xi[ok]) * nh + hi[ok]
                    rows.update(np.unique(key).tolist())
        return len(rows)

    def _run(self):
        self.out = self.ms.msdeform_attn_forward(*self.args)
        self.g = self.ms.msdeform_attn_backward(*self.args, self.d["grad_out"], workspace=self.ws)

    def step(self):
        self._run()

    def e2e_step(self):
        for k, v in self.h.items():
            self.d[k].copy_(v, non_blocking=True)
        self._run()
        outs = (self.out,) + tuple(self.g)
        if not hasattr(self, "oh"):
            self.oh = [o.cpu().pin_memory() for o in outs]
        for o, h in zip(outs, self.oh):
            h.copy_(o, non_blocking=True)

    def e2e_pipelined(self, steps):
        import torch
        keys = ("value", "loc", "attn", "grad_out")
        dev = [{k: self.d[k] for k in keys}, {k: torch.empty_like(self.d[k]) for k in keys}]
        self._run()
        outs = [[torch.empty_like(self.out)] + [torch.empty_like(g) for g in self.g] for _ in range(2)]
        if not hasattr(self, "oh"):
            self.oh = [o.cpu().pin_memory() for o in outs[0]]

        def h2d(b, st):
            for k in keys:
                dev[b][k].copy_(self.h[k], non_blocking=True)

        def compute(b, st):
            d = dev[b]
            a = (d["value"], self.d["spatial_shapes"], self.d["level_start"], d["loc"], d["attn"])
            self.ms.msdeform_attn_forward(*a, out=outs[b][0], stream=st)
            self.ms.msdeform_attn_backward(*a, d["grad_out"], workspace=self.ws, stream=st, out=tuple(outs[b][1:]))

        def d2h(b, st):
            for o, h in zip(outs[b], self.oh):
                h.copy_(o, non_blocking=True)

        return pipelined_e2e_ms(steps, h2d, compute, d2h)

    def io_bytes(self):
        h2d = sum(v.numel() * v.element_size() for v in self.h.values())
        self._run()
        d2h = sum(o.numel() * o.element_size() for o in (self.out,) + tuple(self.g))
        return h2d, d2h

    def dominant(self, args, stream, flush):
        """The forward gather kernel alone (HBM roofline on the full-map bytes)."""
        call = lambda: self.ms.msdeform_attn_forward(*self.args, out=self.out)
        self._run()
        for _ in range(args.warmup):
            call()
        ms = event_time(call, max(5, args.steps), stream, flush)
        bwd = lambda: self.ms.msdeform_attn_backward(*self.args, self.d["grad_out"], workspace=self.ws)
        ms_b = event_time(bwd, max(5, args.steps), stream, flush)
        pk, src = peaks()
        work = MS_FWD_BYTES[self.dtype] * self.B // MS_B
        ach = work / (ms * 1e-3) / 1e9
        load = "16-byte (4 x f32)" if self.dtype == "f32" else "8-byte (4 x bf16)"
        r = {"bound": "hbm", "kernel": f"msda_fwd_kernel (bilinear gather, {load} corner loads)", "achieved": ach,
             "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"], "peak_source": f"{src} hbm_gbs",
             "traffic": None, "bytes_per_launch": work, "ms_per_launch": ms,
             "backward": {"ms": ms_b, "bytes": MS_BWD_BYTES_F32 * self.B // MS_B if self.dtype == "f32" else None,
                          "frac": (MS_BWD_BYTES_F32 * self.B // MS_B / (ms_b * 1e-3) / 1e9 / pk["hbm_gbs"])
                          if self.dtype == "f32" else None}}
        return r

    def extra(self, ms):
        return {"touched_value_rows": self.touched}

    @property
    def config(self):
        return {"seq_len": MS_Q, "precision": f"{self.dtype} value/out/grads, f32 loc/attn, f32 accumulation; "
                                              "deterministic backward (no atomics)"}

    def cpu_sample(self, threads, n_img=MS_B):
        import torch
        from oracle import msdeform_oracle as mo
        torch.set_num_threads(threads)
        p = mo.msdeform_synthetic(B=n_img, Q=MS_Q, nh=MS_NH, dh=MS_DH, shapes=MS_SHAPES, P=MS_P, seed=5)
        t = {k: torch.as_tensor(v) for k, v in p.items()}
        v = t["value"].requires_grad_(True)
        loc = t["loc"].requires_grad_(True)
        at = t["attn"].requires_grad_(True)
        t0 = time.perf_counter()
        out = mo.msdeform_attn_torch(v, t["spatial_shapes"], t["level_start"], loc, at)
        out.backward(t["grad_out"])
        return n_img, time.perf_counter() - t0

    sample_desc = ("images (8 x 300 queries) fwd+bwd through torch-CPU f32 grid_sample + autograd (the reference "
                   "has no deformable attention)")


class Cfg4:
    metric = "attention images/sec (DINOv2-S attention, global + 4x4-windowed layer, bf16, 1601 tokens)"
    unit, dtype, batch = "images/s", "bf16", DN_B
    workload = ("cfg4: DINOv2-S attention at 560x560 (1601 tokens), hidden 384, 6x64 heads, packed QKV Linear; "
                "one global layer + one layer over 16 windows of 10x10 patches (+cls per window)")

    def __init__(self, dev, rank, batch, args):
        import torch
        from oracle import dinov2_oracle as do
        from vision_rs_b200 import dinov2
        self.dn, self.B = dinov2, batch
        x, w, b = do.dinov2_synthetic(S=batch, n=DN_N, hidden=DN_HID, seed=200 + rank)
        self.x = torch.as_tensor(x).to(dev, torch.bfloat16)
        self.op = dinov2.DinoV2Attention(torch.as_tensor(w).to(dev, torch.bfloat16), torch.as_tensor(b).to(dev),
                                         DN_HEADS)
        self.opw = dinov2.DinoV2Attention(self.op.w_qkv, self.op.b_qkv, DN_HEADS)
        self.og = torch.empty_like(self.x)
        self.xw = dinov2.window_partition(self.x, DN_GRID, DN_GRID, DN_WIN)
        self.ow = torch.empty_like(self.xw)
        self.o2 = torch.empty_like(self.x)
        self.xh = self.x.cpu().pin_memory()
        self.oh = torch.empty_like(self.xh).pin_memory()
        self.oh2 = torch.empty_like(self.xh).pin_memory()

    def _run(self):
        self.op.forward_into(self.x, self.og)
        self.dn.window_partition(self.x, DN_GRID, DN_GRID, DN_WIN, out=self.xw)
        self.opw.forward_into(self.xw, self.ow)
        self.dn.window_unpartition(self.ow, self.B, DN_GRID, DN_GRID, DN_WIN, out=self.o2)

    def step(self):
        self._run()

    def e2e_step(self):
        self.x.copy_(self.xh, non_blocking=True)
        self._run()
        self.oh.copy_(self.og, non_blocking=True)
        self.oh2.copy_(self.o2, non_blocking=True)

    def e2e_pipelined(self, steps):
        import torch
        xs = [self.x, torch.empty_like(self.x)]
        og = [self.og, torch.empty_like(self.og)]
        o2 = [self.o2, torch.empty_like(self.o2)]
        xw = [self.xw, torch.empty_like(self.xw)]
        ow = [self.ow, torch.empty_like(self.ow)]
        op2 = self.dn.DinoV2Attention(self.op.w_qkv, self.op.b_qkv, DN_HEADS)  # own workspace on the compute stream
        opw2 = self.dn.DinoV2Attention(self.op.w_qkv, self.op.b_qkv, DN_HEADS)

        def compute(b, st):
            op2.forward_into(xs[b], og[b], stream=st)
            self.dn.window_partition(xs[b], DN_GRID, DN_GRID, DN_WIN, out=xw[b], stream=st)
            opw2.forward_into(xw[b], ow[b], stream=st)
            self.dn.window_unpartition(ow[b], self.B, DN_GRID, DN_GRID, DN_WIN, out=o2[b], stream=st)

        def d2h(b, st):
            self.oh.copy_(og[b], non_blocking=True)
            self.oh2.copy_(o2[b], non_blocking=True)

        return pipelined_e2e_ms(steps, lambda b, st: xs[b].copy_(self.xh, non_blocking=True), compute, d2h)

    def io_bytes(self):
        return self.x.numel() * 2, 2 * self.x.numel() * 2

    def dominant(self, args, stream, flush):
        """The global layer's attention kernel alone (head dim 64, 1601 tokens)
        on the Q/K/V the op's QKV GEMM left in its workspace."""
        from vision_rs_b200 import _lib
        self.op.forward_into(self.x, self.og)
        base, st = self.op._ws.data_ptr(), stream.cuda_stream
        v_off = (2 * self.B * DN_HEADS * DN_N * 64 * 2 + 255) // 256 * 256
        call = lambda: _lib.call("va_dinov2_flash_attention_fwd_f16", base, base + v_off, self.og.data_ptr(), self.B,
                                 DN_N, DN_HEADS, st)
        for _ in range(args.warmup):
            call()
        ms = event_time(call, max(5, args.steps), stream, flush)
        qkv = torch_empty_like_qkv(self.x)
        lin = lambda: self.dn.qkv_linear(self.x, self.op.w_qkv, self.op.b_qkv, out=qkv)
        ms_lin = event_time(lin, max(5, args.steps), stream, flush)
        # the whole global layer (QKV Linear + attention) through the op, and torch's own
        # F.linear + scaled_dot_product_attention on the same bf16 inputs, for comparison
        import torch
        import torch.nn.functional as F
        ours = lambda: self.op.forward_into(self.x, self.og)
        wt, bt = self.op.w_qkv, self.op.b_qkv.to(torch.bfloat16)
        B_, n_ = self.x.shape[0], self.x.shape[1]

        def torch_global():
            q, k, v = F.linear(self.x, wt, bt).view(B_, n_, 3, DN_HEADS, 64).permute(2, 0, 3, 1, 4)
            return F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B_, n_, DN_HID)
        for _ in range(args.warmup):
            ours()
            torch_global()
        self.global_ms = event_time(ours, max(5, args.steps), stream, flush)
        self.torch_global_ms = event_time(torch_global, max(5, args.steps), stream, flush)
        pk, src = peaks()
        work = self.B * DN_FLOP_GLOBAL_ATTN_IMG
        ach = work / (ms * 1e-3) / 1e12
        return {"bound": "tensor", "kernel": "attn_kernel<64> (tcgen05 flash attention, global layer, 1601 tokens)",
                "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": ach / pk["bf16_tflops"],
                "peak_source": f"{src} bf16_tflops (burst)", "traffic": None, "flop_per_launch": work,
                "ms_per_launch": ms, "qkv_linear_ms": ms_lin,
                "qkv_linear_tflops": 2 * self.B * DN_N * DN_HID * 3 * DN_HID / (ms_lin * 1e-3) / 1e12}

    def extra(self, ms):
        return {"tflops_whole_step": DN_FLOP_IMG * self.B / (ms * 1e-3) / 1e12,
                "global_layer_ms": getattr(self, "global_ms", None),
                "torch_global_layer_ms": getattr(self, "torch_global_ms", None),
                "torch_global_layer": "torch F.linear + F.scaled_dot_product_attention, bf16, same inputs "
                                      "(a measurement beside ours, not a path of this library)"}

    config = {"seq_len": DN_N, "window_seq_len": DN_NWIN,
              "precision": "bf16 I/O, weights and QKV GEMM; f16 Q/K/V/P; f32 accumulation",
              "cls_in_windows": "cls token prepended to every window; un-partition averages the windows' cls"}

    @staticmethod
    def cpu_sample(threads, n_img=2):
        import torch
        from oracle import dinov2_oracle as do
        torch.set_num_threads(threads)
        x, w, b = do.dinov2_synthetic(S=n_img, n=DN_N, hidden=DN_HID, seed=9)
        xt, wt, bt = torch.as_tensor(x), torch.as_tensor(w), torch.as_tensor(b)
        xw = torch.as_tensor(do.window_partition(x, DN_GRID, DN_GRID, DN_WIN))
        t0 = time.perf_counter()
        do.dinov2_attention_torch(xt, wt, bt, DN_HEADS)
        do.dinov2_attention_torch(xw, wt, bt, DN_HEADS)
        return n_img, time.perf_counter() - t0

    sample_desc = ("images (one global + one windowed layer) through torch-CPU f32 Linear + SDPA (the reference has "
                   "no DINOv2 code)")


def torch_empty_like_qkv(x):
    import torch
    return torch.empty(*x.shape[:-1], 3 * x.shape[-1], device=x.device, dtype=x.dtype)


class Cfg5:
    metric = "training images/sec (C2PSA PSA attention fwd+bwd+allreduce+SGD, bf16, 400 tokens)"
    unit, dtype, batch = "images/s", "bf16", T5_B
    workload = ("cfg5: C2PSA PSA attention training step, 32 x 128x20x20 per GPU, MSE loss, all-reduce of "
                "the 50,816 f32 weight gradients, SGD on f32 master weights")

    def __init__(self, dev, rank, batch, args):
        import torch
        from oracle import psa_oracle as po
        from vision_rs_b200 import train
        self.train, self.B = train, batch
        s = po.psa_synthetic(batch, T5_H, T5_W, seed=300 + rank)
        wseed = po.psa_synthetic(1, T5_H, T5_W, seed=77)  # identical weights on every rank
        rng = np.random.default_rng(400 + rank)
        bf = lambda a: torch.as_tensor(np.asarray(a, np.float32)).to(dev, torch.bfloat16)
        self.x = bf(s["x"])
        self.t = bf(rng.standard_normal(self.x.shape))
        self.params = {k: bf(wseed[k]) for k in ("w_qkv", "w_pe", "w_proj")}
        self.params.update({k: torch.as_tensor(wseed[k]).to(dev) for k in ("b_qkv", "b_pe", "b_proj")})
        # the local step replays from a CUDA graph (one host launch instead of ≈15)
        self.step_obj = train.PsaTrainStep(B=batch, H=T5_H, W=T5_W, device=dev, graph=True)
        self.master = train.PsaTrainStep.master_from(self.params)
        self.lr = 1e-3
        self.xh = self.x.cpu().pin_memory()
        self.th = self.t.cpu().pin_memory()
        self.lh = torch.empty(1, dtype=torch.float32).pin_memory()
        # several ranks: the all-reduce + SGD is one peer-memory kernel per rank
        # (PeerGradComm), or NCCL all-reduce + the SGD kernel with --allreduce nccl
        import torch.distributed as dist
        multi = dist.is_initialized() and dist.get_world_size() > 1
        self.comm = train.PeerGradComm() if multi and args.allreduce == "peer" else None
        # with the peer comm the whole step (fwd + bwd + all-reduce + SGD) replays from one graph
        self.graph_step = train.DpStepGraph(self.step_obj, self.comm) if self.comm is not None else None
        self.allreduce = ("none (one rank)" if not multi else
                          "peer-memory all-reduce fused with SGD (one kernel), whole step replayed from one CUDA "
                          "graph" if self.comm else "NCCL all-reduce")

    def step(self):
        if self.graph_step is not None:
            self.loss = self.graph_step(self.x, self.t, self.params, self.master, self.lr)
            return
        self.loss = self.train.dp_train_step(self.step_obj, self.x, self.t, self.params, self.master, self.lr,
                                             comm=self.comm)

    def close(self):
        if self.comm is not None:
            self.comm.close()

    def e2e_step(self):
        self.x.copy_(self.xh, non_blocking=True)
        self.t.copy_(self.th, non_blocking=True)
        self.step()
        self.lh.copy_(self.loss, non_blocking=True)

    def io_bytes(self):
        return 2 * self.x.numel() * 2, 4

    def dominant(self, args, stream, flush):
        """The local forward+backward alone (no collective), and the all-reduce alone."""
        import torch
        import torch.distributed as dist
        fb = lambda: self.step_obj.forward_backward(self.x, self.t, self.params)
        for _ in range(args.warmup):
            fb()
        ms = event_time(fb, max(5, args.steps), stream, flush)
        ar_ms = nccl_ms = None
        if dist.is_initialized():
            g = self.step_obj.grads
            nccl = lambda: dist.all_reduce(g)
            for _ in range(3):
                nccl()
            nccl_ms = event_time(nccl, max(5, args.steps), stream, None)
            ar_ms = nccl_ms
            if self.comm is not None:
                g.zero_()  # repeated in-place sums stay finite; lr 0 leaves the weights as they are
                peer = lambda: self.comm.allreduce_sgd(g, self.master, self.params, 0.0)
                for _ in range(3):
                    peer()
                torch.cuda.synchronize()
                dist.barrier()  # ranks start the timed launches together
                ar_ms = event_time(peer, max(5, args.steps), stream, None)
        pk, src = peaks()
        work = 3 * FLOP_FWD_IMG5 * self.B
        ach = work / (ms * 1e-3) / 1e12
        peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
        return {"bound": "tensor", "kernel": "local fwd+bwd (all kernels of one shard's step, no collective)",
                "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "peak_source": f"{src} bf16_tflops_sustained", "traffic": None,
                "flop_per_launch": work, "flop_count": "3 x forward FLOPs (backward ~ 2 x forward)",
                "ms_per_launch": ms, "allreduce": self.allreduce,
                "allreduce_us": None if ar_ms is None else 1000 * ar_ms,
                "allreduce_us_note": "back-to-back launches per rank after a barrier; includes the ranks' "
                                     "timeline skew (each launch waits for every peer's flag)",
                "nccl_allreduce_us": None if nccl_ms is None else 1000 * nccl_ms,
                "allreduce_bytes": 4 * self.train.GRAD_COUNT}

    def extra(self, ms):
        if self.comm is not None and self.comm.status() != 0:
            raise RuntimeError(f"peer all-reduce: a device-side wait gave up (status {self.comm.status()})")
        return {}

    config = {"seq_len": N5, "precision": "bf16 activations/weights, f16 GEMM operands, f32 attention backward, "
                                          "f32 gradients and master weights"}

    @staticmethod
    def cpu_sample(threads, n_img=T5_B):
        import torch
        from oracle import psa_oracle as po
        torch.set_num_threads(threads)
        s = po.psa_synthetic(n_img, T5_H, T5_W, seed=3)
        t = {k: torch.tensor(v).requires_grad_(k.startswith(("w_", "b_"))) for k, v in s.items()}
        tgt = torch.randn(n_img, C, T5_H, T5_W)
        t0 = time.perf_counter()
        y = po.psa_attention_torch(t["x"], t["w_qkv"], t["b_qkv"], t["w_pe"], t["b_pe"], t["w_proj"], t["b_proj"],
                                   NH, KD)
        ((y - tgt) ** 2).mean().backward()
        return n_img, time.perf_counter() - t0

    sample_desc = "images of 128x20x20 fwd+bwd, torch-CPU f32 autograd restatement (the reference has no CPU path)"


class ConvStack:
    metric = "conv images/sec (YOLO26n backbone Conv+BN+SiLU layers 1-8, bf16 NHWC, 640x640)"
    unit, dtype, batch = "images/s", "bf16", CONV_B
    workload = ("conv: the 18 Conv+BN(+SiLU) of YOLO26n backbone layers 1-8 at 640x640 input, batch 64, bf16 "
                "NHWC, BN folded, each conv on its own resident input")

    def __init__(self, dev, rank, batch, args):
        import torch
        from vision_rs_b200 import conv
        g = torch.Generator(device="cpu").manual_seed(700 + rank)
        self.B, self.layers = batch, []
        for name, ci, co, k, s, h in CONV_LAYERS:
            w = torch.randn(co, ci, k, k, generator=g) / math.sqrt(ci * k * k)
            b = torch.randn(co, generator=g) * 0.1
            x = torch.randn(batch, h, h, ci, generator=g).to(dev, torch.bfloat16)
            op = conv.ConvBnAct(w.numpy(), b.numpy(), s, True, device=dev)
            y = torch.empty(batch, conv_out(h, k, s), conv_out(h, k, s), co, dtype=torch.bfloat16, device=dev)
            self.layers.append((name, op, x, y))
        self.xh = [x.cpu().pin_memory() for _, _, x, _ in self.layers]
        self.yh = [torch.empty(y.shape, dtype=y.dtype).pin_memory() for _, _, _, y in self.layers]
        work = [conv_layer_work(ci, co, k, s, h) for _, ci, co, k, s, h in CONV_LAYERS]
        self.flop_img = sum(f for f, _ in work)
        self.bytes_img = sum(b for _, b in work)

    def step(self):
        for _, op, x, y in self.layers:
            op(x, out=y)

    def e2e_step(self):
        """Each conv called as a host-buffer op: its input copied in, its output copied out."""
        for (_, op, x, y), xh, yh in zip(self.layers, self.xh, self.yh):
            x.copy_(xh, non_blocking=True)
            op(x, out=y)
            yh.copy_(y, non_blocking=True)

    def io_bytes(self):
        return (sum(x.numel() * 2 for _, _, x, _ in self.layers), sum(y.numel() * 2 for _, _, _, y in self.layers))

    def dominant(self, args, stream, flush):
        """The whole stack against the roofline its arithmetic intensity picks
        (every launch is the same conv kernel), plus the per-layer times."""
        pk, src = peaks()
        per = {}
        for (name, op, x, y), (_, ci, co, k, s, h) in zip(self.layers, CONV_LAYERS):
            call = lambda: op(x, out=y)
            for _ in range(3):
                call()
            per[name] = event_time(call, max(5, args.steps), stream, flush) * 1e3
        ms = sum(per.values()) / 1e3
        flop, byts = self.flop_img * self.B, self.bytes_img * self.B
        ridge = pk["bf16_tflops"] * 1e12 / (pk["hbm_gbs"] * 1e9)
        if flop / byts >= ridge:
            ach = flop / (ms * 1e-3) / 1e12
            r = {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                 "peak_source": f"{src} bf16_tflops"}
        else:
            ach = byts / (ms * 1e-3) / 1e9
            r = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                 "peak_source": f"{src} hbm_gbs"}
        r.update({"kernel": "conv_nhwc_kernel (tcgen05 implicit GEMM, 18 launches: per-layer sum)",
                  "frac": r["achieved"] / r["peak"], "traffic": None, "flop_per_launch": flop,
                  "bytes_per_launch": byts, "ms_per_launch": ms, "intensity_flop_per_byte": flop / byts,
                  "us_per_layer": per})
        return r

    def extra(self, ms):
        return {"tflops": self.flop_img * self.B / (ms * 1e-3) / 1e12}

    config = {"layers": len(CONV_LAYERS), "input": "640x640 (layer 1 input 320x320x16)"}

    @staticmethod
    def cpu_sample(threads, n_img=1, seed=1234):
        """One image through every layer: torch-CPU f32 conv2d + bias + SiLU, NCHW."""
        import torch
        torch.set_num_threads(threads)
        g = torch.Generator().manual_seed(seed)
        t = 0.0
        for _, ci, co, k, s, h in CONV_LAYERS:
            x = torch.randn(n_img, ci, h, h, generator=g)
            w = torch.randn(co, ci, k, k, generator=g) / math.sqrt(ci * k * k)
            b = torch.randn(co, generator=g) * 0.1
            t0 = time.perf_counter()
            torch.nn.functional.silu(torch.nn.functional.conv2d(x, w, b, stride=s, padding=k // 2))
            t += time.perf_counter() - t0
        return n_img, t

    sample_desc = ("single images through the 18 convs, torch-CPU f32 conv2d + bias + SiLU (NCHW); the reference "
                   "runs its convs on the GPU only")


CONFIGS = {"cfg1": Cfg1, "cfg2": Cfg2, "cfg3": Cfg3, "cfg4": Cfg4, "cfg5": Cfg5, "conv": ConvStack}


# ═════════════════════════════ arms ══════════════════════════════════════════
def cpu_baseline(cfg_cls, args, min_s=10.0):
    """The CPU restatement on this host's cores, repeated until ≥ min_s."""
    threads = os.cpu_count() or 1
    inst = cfg_cls.__new__(cfg_cls)
    inst.dtype = getattr(args, "dtype", "f32")
    inst.width = getattr(args, "width", "n")
    tot_img, tot_s = 0, 0.0
    while tot_s < min_s:
        n, dt = inst.cpu_sample(threads)
        tot_img += n
        tot_s += dt
    return {"value": tot_img / tot_s, "unit": "images/s", "cores": threads, "kind": "port",
            "sample": f"{tot_img} {cfg_cls.sample_desc}; {tot_s:.1f} s"}


def run_reference(args, ws, rank):
    """CPU reference arm: rank 0 only."""
    if rank != 0:
        return
    cls = CONFIGS[args.config]
    threads = os.cpu_count() or 1
    inst = cls.__new__(cls)
    inst.dtype = args.dtype
    inst.width = args.width
    for _ in range(args.warmup):
        inst.cpu_sample(threads)
    n_tot, t_tot, ns = 0, 0.0, []
    for _ in range(args.steps):
        n, dt = inst.cpu_sample(threads)
        n_tot, t_tot = n_tot + n, t_tot + dt
        ns.append(n)
    val = n_tot / t_tot
    metric, workload = (cls.names(args.width) if hasattr(cls, "names")
                        else (getattr(cls, "metric", None)
                              or f"attention images/sec (RF-DETR MSDeformAttn fwd+bwd, {args.dtype})", cls.workload))
    line = {
        "impl": "reference", "metric": metric, "value": val, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * t_tot / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload, "global_batch": cls.batch * args.gpus, "per_gpu_batch": cls.batch,
                   "parallelism": "host threads", "sample_images_per_step": ns[0]},
        "cpu_baseline": {"value": val, "unit": "images/s", "cores": threads, "kind": "port",
                         "sample": f"per step: {cls.sample_desc}"},
        "e2e": {"value": val, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def timed_steps(wl, steps, warmup, min_warm_s, flush, dev, ws, barrier, counter=lambda: 0):
    """Warm up, then time ``steps`` steps (CUDA events per step on the current
    stream, L2 evicted before each, outside the events).  Returns the mean ms
    per step and how far ``counter()`` advanced over the timed steps."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream()
    # Warm up in chunks of `warmup` steps until both the step count and the
    # minimum duration are reached; with several ranks they agree (MAX) after
    # every chunk, so all run the same number of steps — a step may hold a
    # collective (cfg5), and ranks that disagreed on the count would hang.
    t_w = time.perf_counter()
    while True:
        for _ in range(warmup):
            wl.step()
        torch.cuda.synchronize()
        more = torch.tensor([1.0 if time.perf_counter() - t_w < min_warm_s else 0.0], device=dev)
        if ws > 1:
            dist.all_reduce(more, op=dist.ReduceOp.MAX)
        if more.item() == 0.0:
            break
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    c0 = counter()
    barrier()
    for i in range(steps):
        evict_l2(flush, i)  # between timed steps, outside the events
        starts[i].record(stream)
        wl.step()
        ends[i].record(stream)
    barrier()
    return statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends)), counter() - c0


# Configurations the default (cfg2) run also measures, briefly, so that one
# run covers every BASELINE configuration at the run's GPU count.
SIDE_CONFIGS = (("cfg1", {}), ("cfg3", {"dtype": "f32"}), ("cfg3_bf16", {"dtype": "bf16"}), ("cfg4", {}),
                ("cfg5", {}))


def measure_side(name, overrides, args, ws, rank, dev, flush, barrier):
    """One side configuration: images/s over a short timed run (max over
    ranks) and its dominant kernel's roofline fraction; no e2e, no CPU leg."""
    import copy

    import torch
    import torch.distributed as dist
    a = copy.copy(args)
    for k, v in overrides.items():
        setattr(a, k, v)
    a.steps, a.warmup = 10, 3
    cls = CONFIGS[name.split("_")[0]]
    wl = cls(dev, rank, cls.batch, a)
    try:
        ms, _ = timed_steps(wl, a.steps, a.warmup, 0.3, flush, dev, ws, barrier)
        dom = wl.dominant(a, torch.cuda.current_stream(), flush)
        t = torch.tensor([ms, dom["ms_per_launch"]], device=dev, dtype=torch.float64)
        if ws > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, dom_ms = t.tolist()
    finally:
        if hasattr(wl, "close"):
            wl.close()
    out = {"workload": wl.workload, "value": cls.batch * ws / (ms * 1e-3), "unit": "images/s",
           "ms_per_step": ms, "per_gpu_batch": cls.batch, "global_batch": cls.batch * ws, "steps": a.steps,
           "dtype": getattr(wl, "dtype", "bf16"),
           "dominant": {"kernel": dom.get("kernel"), "bound": dom.get("bound"), "frac": dom.get("frac"),
                        "peak_source": dom.get("peak_source"), "ms_per_launch_max_over_ranks": dom_ms}}
    del wl
    torch.cuda.empty_cache()
    return out


def run_ours(args, ws, rank, local):
    import datetime

    import torch
    import torch.distributed as dist
    from vision_rs_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        dist.barrier()  # communicator created on every rank before any work
    cls = CONFIGS[args.config]
    B = args.batch or cls.batch
    wl = cls(dev, rank, B, args)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)  # > L2 (126 MB)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clk = ClockSampler(local).start()
    replayed = lambda: (getattr(getattr(wl, "step_obj", None), "replayed_kernels", 0)
                        + getattr(getattr(wl, "graph_step", None), "replayed_kernels", 0))
    # kernels launched directly or by graph replays inside the timed steps
    ms, launches = timed_steps(wl, args.steps, args.warmup, args.min_warm_s, flush, dev, ws, barrier,
                               counter=lambda: _lib.lib().va_launch_count() + replayed())
    clk.stop()

    dom = wl.dominant(args, stream, flush)
    e2e_ms = float("nan")
    e2e_mode = "serial: copy-in, compute, copy-out on one stream"
    if not args.no_e2e:
        h2d, d2h = wl.io_bytes()
        for _ in range(max(1, args.warmup)):
            wl.e2e_step()
        barrier()
        if hasattr(wl, "e2e_pipelined"):
            wl.e2e_pipelined(max(3, args.warmup))
            barrier()
            e2e_ms = wl.e2e_pipelined(args.steps)
            e2e_mode = ("pipelined: copy-in, compute and copy-out of consecutive steps on three streams, double-"
                        "buffered; every step still copies its whole input in and its whole result out")
        else:
            e2e_ms = event_time(wl.e2e_step, args.steps, stream)
    t = torch.tensor([ms, e2e_ms, dom["ms_per_launch"]], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, dom_ms = t.tolist()
    dom["ms_per_launch_max_over_ranks"] = dom_ms

    side = {}
    if args.config == "cfg2" and args.width == "n" and not args.batch and args.side_configs:
        for name, ov in SIDE_CONFIGS:
            if ws > 1:  # every rank takes the same collective steps: a failure must end the run on all of them
                side[name] = measure_side(name, ov, args, ws, rank, dev, flush, barrier)
                continue
            try:  # one process: a failing side configuration must not cost the headline line
                side[name] = measure_side(name, ov, args, ws, rank, dev, flush, barrier)
            except Exception as e:  # noqa: BLE001 — reported in the line, not hidden
                side[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cls, args)
    if rank == 0:
        metric = wl.metric
        line = {
            "metric": metric, "value": B * ws / (ms * 1e-3), "unit": "images/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": getattr(wl, "dtype", "bf16"), "data": "synthetic",
            "config": dict({"workload": wl.workload, "global_batch": B * ws, "per_gpu_batch": B,
                            "parallelism": (f"data parallel x{ws}, {wl.allreduce} of the weight gradients"
                                            if args.config == "cfg5" else f"image shards x{ws}, no collective"),
                            "l2": "evicted between timed steps (256 MB buffer written, then read back)"}, **wl.config),
            "e2e": None if math.isnan(e2e_ms) else {
                "value": B * ws / (e2e_ms * 1e-3), "unit": "images/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "mode": e2e_mode},
            "gpu_launches": int(launches),
            "roofline": dom,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
        }
        line.update(wl.extra(ms))
        if side:
            line["other_configs"] = side
        print(json.dumps(line), flush=True)
    if hasattr(wl, "close"):
        wl.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--dtype", default="f32", choices=["f32", "bf16"], help="cfg3 value/grad dtype")
    ap.add_argument("--width", default="n", choices=sorted(WIDTHS),
                    help="cfg2: YOLO26 width of the C2PSA block (n: C=128, s/m/l: 256, x: 384)")
    ap.add_argument("--allreduce", default="peer", choices=["peer", "nccl"],
                    help="cfg5 with several GPUs: peer-memory all-reduce + SGD kernel, or NCCL all-reduce + SGD")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--min-warm-s", type=float, default=1.5,
                    help="keep warming up at least this long so the clock sampler sees the load")
    ap.add_argument("--batch", type=int, default=0, help="per-GPU batch (default: the config's)")
    ap.add_argument("--no-side-configs", dest="side_configs", action="store_false",
                    help="cfg2 only: skip the short runs of cfg1, cfg3 (f32, bf16), cfg4 and cfg5 "
                         "reported under other_configs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    ws, rank, local = dist_env()
    if ws > 1:
        # NCCL prints its version line on stdout when its debug level asks for it; the bench's
        # stdout is one JSON line, so keep NCCL to warnings (read when NCCL initialises)
        os.environ["NCCL_DEBUG"] = "WARN"
    if args.impl == "reference":
        run_reference(args, ws, rank)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
