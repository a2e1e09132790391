"""Benchmark of the two attention hot paths on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
        --master-addr 127.0.0.1 --master-port P bench.py --gpus N --steps K --warmup W

Rank 0 prints one JSON line. The headline `value` is causal prefill TFLOP/s on
BASELINE config 2 (B=4, H=16, N=4096, d=128, fp16, FLOPs 4 B H N^2 d / 2, the
reference's convention, bench/bench.py:153) summed over all ranks, each rank
running its own config-2 batch (independent (batch, head) units: weak scaling,
no collective). Extra objects report paged decode on config 4 (KV GB/s,
bytes sum(ctx) H_kv d 2 2, bench/bench.py:199-200), the long-context configs 3
(head-sharded prefill, strong scaling) and 5 (context-range decode with an NCCL
merge of the partials, strong scaling), the roofline of each dominant kernel
against MEASURED_PEAKS.json, the end-to-end time through the public API with
host buffers, and the CPU oracle timed on this host.

Timing: W untimed warm-up steps, then exactly K steps between CUDA events on
the launching stream, with a barrier and a device synchronize on both sides;
the time is the max over ranks. Inputs are larger than L2 (126 MB) in every
timed case, so no flush is needed between steps. Data are synthetic (seeded
N(0, 1) fp16), no dataset is involved.

`--impl reference` times the reference's own CPU implementation of the path
(its fp32 PyTorch oracle attnkernels/reference.py, restated in oracle/) with all
host threads, on a bounded sample of the same workload, and prints the same
kind of line with "impl": "reference". Under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "flash-attention-from-scratch_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

BASELINE_METRIC = "prefill TFLOP/s & paged-decode KV GB/s per B200 at 1/2/4/8 GPUs vs roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# BASELINE configs (synthetic, seeded).
CFG2 = dict(batch=4, heads=16, seq=4096, head_dim=128, causal=True)
CFG3 = dict(batch=1, heads=32, seq=32768, head_dim=128, causal=True, input_scale=0.5)
CFG4 = dict(batch=64, heads=32, kv_heads=32, head_dim=128, block_size=16, ctx_lo=512,
            ctx_hi=8192, partition=512)
CFG5 = dict(batch=8, heads=32, kv_heads=32, head_dim=128, block_size=16, ctx=131072)


def prefill_flops(batch, heads, seq, head_dim, causal, **_):
    return 4.0 * batch * heads * seq * seq * head_dim * (0.5 if causal else 1.0)


def kv_bytes(ctx_lens, kv_heads, head_dim):
    return float(sum(ctx_lens)) * kv_heads * head_dim * 2 * 2


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return {k: float(p[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """Per-launch DRAM bytes from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            return {}
    return {}


# ------------------------------------------------------------------ plumbing


class Dist:
    """Rank/world from the torchrun environment; NCCL process group if world > 1."""

    def __init__(self, gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}")
        self.device = torch.device("cuda", self.local)
        torch.cuda.set_device(self.device)
        self.group = None
        if self.world > 1:
            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=self.device)
            self.dist = dist

    def barrier(self):
        if self.world > 1:
            self.dist.barrier(device_ids=[self.local])

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 200 ms while under load."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def timed(fn, steps, warmup, d: Dist, spin_s=0.0):
    """ms for exactly `steps` calls of fn (max over ranks), after `warmup` calls.

    spin_s: keep the GPU busy with untimed calls for about this long first, so
    the clock samples taken meanwhile reflect the loaded state."""
    stream = torch.cuda.current_stream(d.device)
    for _ in range(warmup):
        fn()
    if spin_s > 0:
        t_end = time.perf_counter() + spin_s
        while time.perf_counter() < t_end:
            fn()
            stream.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    d.barrier()
    torch.cuda.synchronize(d.device)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize(d.device)
    d.barrier()
    return d.max(start.elapsed_time(end))


def roofline(bound, work_per_launch, ms_per_launch, peaks, peak_src, traffic=None):
    unit = "TFLOP/s" if bound == "tensor" else "GB/s"
    scale = 1e12 if bound == "tensor" else 1e9
    achieved = work_per_launch / (ms_per_launch * 1e-3) / scale
    peak = peaks["bf16_tflops"] if bound == "tensor" else peaks["hbm_gbs"]
    return {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "peak_source": f"{peak_src} ({'dense bf16/fp16 burst' if bound == 'tensor' else 'HBM copy'})"}
