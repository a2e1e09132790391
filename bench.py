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
timed case, so no flush is needed between steps. SM clocks and clock-event
reasons are read through NVML every 1 ms during the warm-up and timed steps
(`clocks` in the line). Data are synthetic (seeded N(0, 1) fp16), no dataset is
involved.

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

# stdout carries only the one JSON line: NCCL's version banner (NCCL_DEBUG=VERSION, as
# the image sets it) is printed to stdout, so that level becomes WARN, and NCCL's log
# lines go to stderr. NCCL reads both when it first initialises.
if os.environ.get("NCCL_DEBUG") == "VERSION":
    os.environ["NCCL_DEBUG"] = "WARN"
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

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

    def sum(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def gather(self, x: float) -> list:
        if self.world == 1:
            return [x]
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        out = torch.empty(self.world, dtype=torch.float64, device=self.device)
        self.dist.all_gather_into_tensor(out, t)
        return [round(float(v), 4) for v in out.tolist()]

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


class NvmlClockSampler:
    """SM clock and clock-event reasons read through NVML every `period_s` on a
    background thread while the block runs, so that a timed region of a few
    milliseconds is itself sampled. Falls back to ClockSampler (nvidia-smi every
    200 ms) when NVML is not usable."""

    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40}

    def __init__(self, device: torch.device, period_s=0.001):
        self.device, self.period = device, period_s
        self.fallback = None
        self.sm, self.mx, self.reasons = [], [], set()

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            pr = torch.cuda.get_device_properties(self.device)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:  # noqa: BLE001  no NVML: nvidia-smi sampling instead
            self.fallback = ClockSampler(self.device.index or 0).__enter__()
            return self
        self.stop = threading.Event()
        try:
            self.mx.append(self.nvml.nvmlDeviceGetMaxClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001
            pass

        def run():
            nv, h = self.nvml, self.handle
            while not self.stop.is_set():
                try:
                    self.sm.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.reasons.update(n for n, b in self.BITS.items() if bits & b)
                except Exception:  # noqa: BLE001
                    break
                self.stop.wait(self.period)

        # A short interpreter switch interval lets the sampling thread take the GIL
        # between the main thread's launches, not only while it waits on the device.
        self.switch = sys.getswitchinterval()
        sys.setswitchinterval(2e-4)
        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.fallback is not None:
            return self.fallback.__exit__(*exc)
        self.stop.set()
        self.thread.join(timeout=5)
        sys.setswitchinterval(self.switch)
        try:
            self.nvml.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass
        return False

    def summary(self):
        if self.fallback is not None:
            return self.fallback.summary()
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.sm),
                "sm_max_mhz": max(self.mx) if self.mx else None,
                "reasons": sorted(self.reasons), "samples": len(self.sm),
                "source": f"NVML every {self.period * 1e3:.0f} ms during warm-up and timed steps"}


def timed(fn, steps, warmup, d: Dist, spin_s=0.0, per_rank=None):
    """ms for exactly `steps` calls of fn (max over ranks), after `warmup` calls.
    If `per_rank` is a list, every rank's own ms is appended to it.

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
    mine = start.elapsed_time(end)
    if per_rank is not None:
        per_rank.extend(d.gather(mine))
    return d.max(mine)


def timed_each(fn, reps, warmup=1, flush_bytes=256 << 20, device=None):
    """Per-call device times (ms) of `reps` calls of fn, each on a cold L2: a
    buffer larger than L2 (126 MB) is written before every call, outside the
    CUDA events that bracket the call on the current stream."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        fn()
    out = []
    for _ in range(reps):
        flush.zero_()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        fn()
        end.record(stream)
        end.synchronize()
        out.append(start.elapsed_time(end))
    del flush
    return out


class _E2EPipeline:
    """Pipelined end-to-end steps: host inputs -> device (stream 1), op (stream 2),
    output -> host (stream 3), with two device buffer sets so that consecutive
    steps overlap. timed() measures exactly `steps` steps on the device (CUDA
    events; max over ranks), after `warmup` untimed ones."""

    def __init__(self, device, host_inputs, host_outs, op):
        self.device, self.hin, self.hout, self.op = device, host_inputs, host_outs, op
        self.din = [[torch.empty_like(h, device=device) for h in host_inputs] for _ in range(2)]
        self.s_in, self.s_op, self.s_out = (torch.cuda.Stream(device) for _ in range(3))
        self.ev_in = [torch.cuda.Event() for _ in range(2)]
        self.ev_op = [torch.cuda.Event() for _ in range(2)]
        self.ev_out = [torch.cuda.Event() for _ in range(2)]
        self.used = [False, False]
        self.t = 0

    def _step(self, cur):
        b = self.t % 2
        self.t += 1
        if self.used[b]:
            self.s_in.wait_event(self.ev_op[b])    # the op of the buffers' last use is done
        with torch.cuda.stream(self.s_in):
            for dst, src in zip(self.din[b], self.hin):
                dst.copy_(src, non_blocking=True)
            self.ev_in[b].record(self.s_in)
        self.s_op.wait_event(self.ev_in[b])
        with torch.cuda.stream(self.s_op):
            out = self.op(*self.din[b])
            self.ev_op[b].record(self.s_op)
        self.s_out.wait_event(self.ev_op[b])
        if self.used[b]:
            self.s_out.wait_event(self.ev_out[b])
        with torch.cuda.stream(self.s_out):
            self.hout[b].copy_(out, non_blocking=True)
            out.record_stream(self.s_out)
            self.ev_out[b].record(self.s_out)
        self.used[b] = True
        cur.wait_event(self.ev_out[b])

    def timed(self, steps, warmup, d):
        cur = torch.cuda.current_stream(self.device)
        for _ in range(warmup):
            self._step(cur)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        d.barrier()
        torch.cuda.synchronize(self.device)
        start.record(cur)
        for s in (self.s_in, self.s_op, self.s_out):
            s.wait_stream(cur)
        for _ in range(steps):
            self._step(cur)
        end.record(cur)
        torch.cuda.synchronize(self.device)
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


# ----------------------------------------------------------------- workloads


def randn_half(shape, gen, device, scale=1.0):
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if scale != 1.0:
        t.mul_(scale)
    return t.half()


def synthetic_paged_cache(ctx_lens, kv_heads, head_dim, block_size, seed, device):
    """Seeded paged cache: block tables are one random permutation of the pool."""
    g = torch.Generator().manual_seed(seed)
    nblk = [-(-c // block_size) for c in ctx_lens]
    pool = sum(nblk)
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    tables = torch.zeros(len(ctx_lens), max(nblk), dtype=torch.int32)
    pos = 0
    for b, n in enumerate(nblk):
        tables[b, :n] = perm[pos:pos + n]
        pos += n
    gd = torch.Generator(device=device).manual_seed(seed)
    shape = (pool, kv_heads, block_size, head_dim)
    kc = randn_half(shape, gd, device)
    vc = randn_half(shape, gd, device)
    return kc, vc, tables.to(device), torch.tensor(ctx_lens, dtype=torch.int32, device=device)


def bench_prefill_cfg2(args, d: Dist, peaks, peak_src, traffic):
    """Headline: config 2 per rank (weak scaling); kernel roofline; e2e with host buffers."""
    import attnkernels as ak

    c = CFG2
    shape = (c["batch"], c["heads"], c["seq"], c["head_dim"])
    gen = torch.Generator(device=d.device).manual_seed(1000 + d.rank)
    q, k, v = (randn_half(shape, gen, d.device) for _ in range(3))
    fn = lambda: ak.flash_attention(q, k, v, causal=True)  # noqa: E731
    ranks_ms = []
    with NvmlClockSampler(d.device) as clk:
        ms = timed(fn, args.steps, args.warmup, d, spin_s=args.spin, per_rank=ranks_ms)
    flops = prefill_flops(**c)
    res = {
        "ms_per_step": ms / args.steps,
        "value": flops * d.world / (ms / args.steps * 1e-3) / 1e12,
        "roofline": roofline("tensor", flops, ms / args.steps, peaks, peak_src,
                             traffic.get("flash_tc_kernel_cfg2")),
        "clocks": clk.summary(),
        "gpu_launches": args.steps,  # one flash_tc_kernel launch per step
        "per_rank_ms_per_step": [round(x / args.steps, 4) for x in ranks_ms],
    }
    # End to end through the public API: every step copies pinned host q, k, v to
    # the device, runs attention and copies the output back to pinned host
    # memory. Steps are pipelined over three streams and two device buffer sets
    # (a serving loop): step t's input copy overlaps step t-1's kernel and output
    # copy; PCIe carries host->device and device->host at the same time.
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    ho = [torch.empty_like(hq).pin_memory() for _ in range(2)]
    del q, k, v
    pipe = _E2EPipeline(d.device, (hq, hk, hv), ho,
                        lambda dq, dk, dv: ak.flash_attention(dq, dk, dv, causal=True))
    ms_e2e = pipe.timed(args.steps, args.warmup, d)
    res["e2e"] = {"value": round(flops * d.world / (ms_e2e / args.steps * 1e-3) / 1e12, 3),
                  "unit": "TFLOP/s", "ms_per_step": round(ms_e2e / args.steps, 4),
                  "h2d_bytes_per_step": 3 * hq.numel() * 2, "d2h_bytes_per_step": ho[0].numel() * 2,
                  "pipeline": "3 streams, 2 device buffer sets: step t's host->device copy "
                              "overlaps step t-1's kernel and device->host copy"}
    return res


def bench_prefill_shapes(args, d: Dist, peaks, peak_src, traffic):
    """The other two shapes BASELINE config 2 names: d=64 and N=4095 (odd length,
    tail masking), same batch and heads, causal; one batch per rank, device-timed
    like the headline, each with its own clock record."""
    import attnkernels as ak

    out = {}
    for key, d_head, n in (("d64", 64, 4096), ("n4095", 128, 4095)):
        c = dict(CFG2, head_dim=d_head, seq=n)
        shape = (c["batch"], c["heads"], c["seq"], c["head_dim"])
        gen = torch.Generator(device=d.device).manual_seed(1100 + d.rank)
        q, k, v = (randn_half(shape, gen, d.device) for _ in range(3))
        fn = lambda: ak.flash_attention(q, k, v, causal=True)  # noqa: E731
        with NvmlClockSampler(d.device) as clk:
            ms = timed(fn, args.steps, args.warmup, d)
        flops = prefill_flops(**c)
        out[key] = {
            "workload": f"causal prefill B={c['batch']} H={c['heads']} N={n} d={d_head} "
                        "(BASELINE config 2 variant), one batch per GPU",
            "ms_per_step": round(ms / args.steps, 4),
            "value": round(flops * d.world / (ms / args.steps * 1e-3) / 1e12, 2),
            "unit": "TFLOP/s",
            "roofline": roofline("tensor", flops, ms / args.steps, peaks, peak_src,
                                 traffic.get(f"flash_tc_kernel_cfg2_{key}")),
            "clocks": clk.summary(),
            "gpu_launches": args.steps,
            "l2": "inputs larger than L2 (q, k, v %d MiB per step), no flush"
                  % (3 * q.numel() * 2 >> 20)}
        del q, k, v
    torch.cuda.empty_cache()
    return out


def bench_decode_cfg4(args, d: Dist, peaks, peak_src, traffic):
    """Config 4 per rank (independent sequences: weak scaling)."""
    import attnkernels as ak

    c = CFG4
    g = torch.Generator().manual_seed(4000 + d.rank)
    ctx = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (c["batch"],), generator=g).tolist()
    kc, vc, tables, lens = synthetic_paged_cache(ctx, c["kv_heads"], c["head_dim"],
                                                 c["block_size"], 4000 + d.rank, d.device)
    gq = torch.Generator(device=d.device).manual_seed(4100 + d.rank)
    q = randn_half((c["batch"], c["heads"], 1, c["head_dim"]), gq, d.device)
    max_ctx = max(ctx)
    fn = lambda: ak.paged_decode(q, kc, vc, tables, lens, max_ctx,  # noqa: E731
                                 partition_size=c["partition"])
    ranks_ms = []
    with NvmlClockSampler(d.device) as clk:
        ms = timed(fn, args.steps, args.warmup, d, spin_s=args.spin, per_rank=ranks_ms)
    nbytes = kv_bytes(ctx, c["kv_heads"], c["head_dim"])
    total_bytes = d.sum(nbytes)  # each rank decodes its own seeded batch
    res = {
        "config": {"workload": "paged decode, BASELINE config 4", "batch": c["batch"],
                   "heads": c["heads"], "kv_heads": c["kv_heads"], "head_dim": c["head_dim"],
                   "block_size": c["block_size"], "ctx_mean": sum(ctx) / len(ctx),
                   "ctx_max": max_ctx, "partition": c["partition"],
                   "l2": "inputs larger than L2 (KV %.2f GB)" % (nbytes / 1e9)},
        "metric": "paged-decode KV GB/s", "unit": "GB/s",
        "ms_per_step": ms / args.steps,
        "value": total_bytes / (ms / args.steps * 1e-3) / 1e9,
        "per_rank_ms_per_step": [round(x / args.steps, 4) for x in ranks_ms],
        # The timed op is memset + decode kernel + merge kernel: the kernel's own
        # time is lower, so this fraction is a lower bound.
        "roofline": roofline("hbm", nbytes, ms / args.steps, peaks, peak_src,
                             traffic.get("paged_decode_kernel_cfg4")),
        "clocks": clk.summary(),
        "gpu_launches": 2 * args.steps,  # decode + merge kernels (plus one memset node)
    }
    hq = q.cpu().pin_memory()
    htab, hlen = tables.cpu().pin_memory(), lens.cpu().pin_memory()
    ho = [torch.empty_like(hq).pin_memory() for _ in range(2)]
    pipe = _E2EPipeline(d.device, (hq, htab, hlen), ho,
                        lambda dq, dt, dl: ak.paged_decode(dq, kc, vc, dt, dl, max_ctx,
                                                           partition_size=c["partition"]))
    ms_e2e = pipe.timed(args.steps, args.warmup, d)
    res["e2e"] = {"value": round(total_bytes / (ms_e2e / args.steps * 1e-3) / 1e9, 1),
                  "unit": "GB/s", "ms_per_step": round(ms_e2e / args.steps, 4),
                  "h2d_bytes_per_step": hq.numel() * 2 + htab.numel() * 4 + hlen.numel() * 4,
                  "d2h_bytes_per_step": ho[0].numel() * 2,
                  "note": "the KV cache is resident state; per step the query, block tables "
                          "and lengths go up and the output comes back",
                  "pipeline": "3 streams, 2 device buffer sets: step t's host->device copy "
                              "overlaps step t-1's kernels and device->host copy"}
    return res


def torch_comparison(args, d: Dist, ours_prefill, ours_decode):
    """Library kernels on the same inputs, for context (not the product): torch
    SDPA backends on prefill config 2, and for decode config 4 the torch route
    the reference compares against (gather the paged K/V into a contiguous padded
    cache, then SDPA with a length mask)."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    steps, warmup = max(3, args.steps // 2), 3
    out = {"note": "library kernels on the same inputs, for context; value = the same "
                   "metric as the line above"}
    c = CFG2
    shape = (c["batch"], c["heads"], c["seq"], c["head_dim"])
    gen = torch.Generator(device=d.device).manual_seed(2000)
    q, k, v = (randn_half(shape, gen, d.device) for _ in range(3))
    flops = prefill_flops(**c)
    import attnkernels as ak

    pre = {"ours (headline)": round(ours_prefill, 1)}
    ours = lambda: ak.flash_attention(q, k, v, causal=True)  # noqa: E731
    ms = timed(ours, steps, warmup, d) / steps
    pre["ours"] = round(flops / (ms * 1e-3) / 1e12, 1)
    for name in ("FLASH_ATTENTION", "EFFICIENT_ATTENTION", "CUDNN_ATTENTION"):
        key = "sdpa_" + name.split("_")[0].lower()
        be = getattr(SDPBackend, name, None)
        if be is None:
            pre[key] = "unavailable: backend not in this torch"
            continue

        def fn(be=be):
            with sdpa_kernel([be]):
                return F.scaled_dot_product_attention(q, k, v, is_causal=True)

        try:
            fn()
            torch.cuda.synchronize(d.device)
            ms = timed(fn, steps, warmup, d) / steps
            pre[key] = round(flops / (ms * 1e-3) / 1e12, 1)
        except Exception as e:  # noqa: BLE001  a backend that does not run here
            pre[key] = "unavailable: " + str(e).splitlines()[0][:120]
    out["prefill_cfg2_tflops"] = pre
    del q, k, v

    c = CFG4
    g = torch.Generator().manual_seed(4000 + d.rank)
    ctx = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (c["batch"],), generator=g).tolist()
    kc, vc, tables, lens = synthetic_paged_cache(ctx, c["kv_heads"], c["head_dim"],
                                                 c["block_size"], 4000 + d.rank, d.device)
    gq = torch.Generator(device=d.device).manual_seed(4100 + d.rank)
    qd = randn_half((c["batch"], c["heads"], 1, c["head_dim"]), gq, d.device)
    nblk = -(-max(ctx) // c["block_size"])
    idx = torch.arange(nblk * c["block_size"], device=d.device)
    mask = (idx[None, :] < lens[:, None].long())[:, None, None, :]

    def gather(cache):
        x = cache[tables[:, :nblk].long()]  # [B, nblk, Hkv, bs, D]
        return x.permute(0, 2, 1, 3, 4).reshape(x.shape[0], x.shape[2], -1, x.shape[4])

    def gather_sdpa():
        return F.scaled_dot_product_attention(qd, gather(kc), gather(vc), attn_mask=mask)

    dec = {"ours": round(ours_decode, 1)}
    try:
        gather_sdpa()
        torch.cuda.synchronize(d.device)
        ms = timed(gather_sdpa, steps, warmup, d) / steps
        dec["torch_gather_sdpa"] = round(kv_bytes(ctx, c["kv_heads"], c["head_dim"]) /
                                         (ms * 1e-3) / 1e9, 1)
    except Exception as e:  # noqa: BLE001
        dec["torch_gather_sdpa"] = "unavailable: " + str(e).splitlines()[0][:120]
    out["decode_cfg4_gbps"] = dec
    del kc, vc, qd, mask
    torch.cuda.empty_cache()
    return out


def bench_long_context(args, d: Dist, peaks, peak_src, traffic):
    """Configs 3 and 5, total work fixed and split over the ranks (strong scaling).
    Each entry carries its own NVML clock record; `traffic` is the per-launch DRAM
    bytes of one rank's kernel, from a smaller ncu capture scaled by the units
    processed (profiles/traffic.json)."""
    import attnkernels as ak
    from attnkernels import parallel

    out = {}
    # Config 3: heads sharded, no collective.
    c = CFG3
    h0, h1 = parallel.head_range(c["heads"], d.world, d.rank)
    gen = torch.Generator(device=d.device).manual_seed(3000 + h0)
    shape = (c["batch"], h1 - h0, c["seq"], c["head_dim"])
    q, k, v = (randn_half(shape, gen, d.device, c["input_scale"]) for _ in range(3))
    with NvmlClockSampler(d.device) as clk:
        ms = timed(lambda: ak.flash_attention(q, k, v, causal=True), args.steps, args.warmup, d)
    flops = prefill_flops(**{x: c[x] for x in ("batch", "heads", "seq", "head_dim", "causal")})
    per_rank = prefill_flops(c["batch"], h1 - h0, c["seq"], c["head_dim"], True)
    t3 = traffic.get("flash_tc_kernel_cfg3_per_head")
    out["config3_prefill"] = {
        "workload": "causal prefill B=1 H=32 N=32768 d=128, heads sharded over ranks",
        "heads_per_rank": h1 - h0, "scaling": "strong", "ms_per_step": round(ms / args.steps, 4),
        "value": round(flops / (ms / args.steps * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
        "roofline": roofline("tensor", per_rank, ms / args.steps, peaks, peak_src,
                             None if t3 is None else int(t3 * (h1 - h0))),
        "clocks": clk.summary(),
        "gpu_launches": args.steps}
    del q, k, v
    torch.cuda.empty_cache()

    # Config 5: each sequence's context split into block-aligned ranges, one per
    # rank; partials merged across ranks (by default one kernel that pushes them to
    # every peer over NVLink and merges; --cp-exchange nccl: an NCCL all-gather).
    c = CFG5
    t0, t1 = parallel.context_range(c["ctx"], c["block_size"], d.world, d.rank)
    local = [t1 - t0] * c["batch"]
    kc, vc, tables, lens = synthetic_paged_cache(local, c["kv_heads"], c["head_dim"],
                                                 c["block_size"], 5000 + d.rank, d.device)
    gq = torch.Generator(device=d.device).manual_seed(5100)  # the same q on every rank
    q = randn_half((c["batch"], c["heads"], c["head_dim"]), gq, d.device)
    part = ak.decode_partition(c["batch"], c["kv_heads"], t1 - t0)
    if d.world == 1:
        fn = lambda: ak.paged_decode(q, kc, vc, tables, lens, t1 - t0,  # noqa: E731
                                     partition_size=part)
        launches = 2
    else:
        cp = (parallel.ContextParallelDecode(exchange="peer") if args.cp_exchange == "peer"
              else parallel.ContextParallelDecode(chunks=args.cp_chunks, exchange="nccl"))
        fn = lambda: cp(q, kc, vc, tables, lens, t1 - t0, partition_size=part)  # noqa: E731
        # per chunk: decode kernel + local split-K merge + the merge across ranks (the
        # peer exchange: decode + local merge + one exchange-and-merge kernel)
        launches = 3 if args.cp_exchange == "peer" else 3 * min(args.cp_chunks, c["batch"])
    with NvmlClockSampler(d.device) as clk:
        ms = timed(fn, args.steps, args.warmup, d)
    total = kv_bytes([c["ctx"]] * c["batch"], c["kv_heads"], c["head_dim"])
    t5 = traffic.get("paged_decode_kernel_cfg5_per_token")
    out["config5_decode"] = {
        "workload": "paged decode B=8 H=32 d=128 ctx=131072, context ranges over ranks, "
                    + ("(o, m, l) partials exchanged over NVLink peer memory and merged in one "
                       "kernel" if args.cp_exchange == "peer" and d.world > 1 else
                       "NCCL all-gather + merge of the (o, m, l) partials" if d.world > 1 else
                       "one rank: split-K decode + merge"),
        "tokens_per_rank": t1 - t0, "partition": part, "scaling": "strong",
        "ms_per_step": round(ms / args.steps, 4),
        "value": round(total / (ms / args.steps * 1e-3) / 1e9, 1), "unit": "GB/s",
        "roofline": roofline("hbm", total / d.world, ms / args.steps, peaks, peak_src,
                             None if t5 is None else int(t5 * (t1 - t0) * c["batch"])),
        "clocks": clk.summary(),
        "gpu_launches": launches * args.steps}
    if d.world > 1:
        # The same step without the exchange: this rank's partials alone (decode kernel +
        # local split-K merge), to name what the exchange and the merge across ranks add.
        # Three interleaved rounds of both, medians: one pair of runs is within the
        # run-to-run noise of the difference.
        partials = lambda: ak.paged_decode_partials(q, kc, vc, tables, lens, t1 - t0,  # noqa: E731
                                                    partition_size=part)
        full_r, local_r = [], []
        for _ in range(3):
            full_r.append(timed(fn, args.steps, args.warmup, d) / args.steps)
            local_r.append(timed(partials, args.steps, args.warmup, d) / args.steps)
        ms_full, ms_local = statistics.median(full_r), statistics.median(local_r)
        out["config5_decode"]["local_partials_ms_per_step"] = round(ms_local, 4)
        out["config5_decode"]["full_step_ms_median_of_3"] = round(ms_full, 4)
        out["config5_decode"]["exchange_and_merge_ms_per_step"] = round(ms_full - ms_local, 4)
        nbytes = c["batch"] * c["heads"] * (c["head_dim"] + 2) * 4
        out["config5_decode"]["exchange"] = (
            f"peer memory: each rank stores its {nbytes} bytes of partials into every peer over "
            f"NVLink and raises a flag there; one kernel waits for the peers' flags and merges"
            if args.cp_exchange == "peer" else
            f"NCCL all_gather_into_tensor of {nbytes} bytes per rank, then the merge kernel; "
            f"batch cut into {min(args.cp_chunks, c['batch'])} chunk(s) whose exchanges "
            f"overlap the next chunk's decode")
    return out


def _timed_cpu(fn, min_s=10.0, max_reps=100000):
    fn()  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if (el >= min_s and reps >= 3) or reps >= max_reps:
            return el, reps


def cpu_baseline(min_s=10.0):
    """The oracle (reference.py restated) on this host's cores, bounded samples."""
    from oracle import reference as ref

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    g = torch.Generator().manual_seed(7)
    c = CFG2
    q, k, v = (torch.randn(1, 1, c["seq"], c["head_dim"], generator=g).half() for _ in range(3))
    el, reps = _timed_cpu(lambda: ref.attention_fp32(q, k, v, causal=True), min_s)
    flops = prefill_flops(1, 1, c["seq"], c["head_dim"], True)
    pre = {"value": round(flops * reps / el / 1e12, 5), "unit": "TFLOP/s", "cores": cores,
           "kind": "port",
           "sample": f"1 of 64 (batch, head) pairs of config 2 (N=4096, d=128, causal) per "
                     f"call, {reps} calls in {el:.1f} s"}
    c = CFG4
    gen = torch.Generator().manual_seed(8)
    ctx = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (2,), generator=gen).tolist()
    kc, vc, tables, lens = synthetic_paged_cache(ctx, c["kv_heads"], c["head_dim"],
                                                 c["block_size"], 8, "cpu")
    qd = torch.randn(2, c["heads"], c["head_dim"], generator=gen).half()
    el, reps = _timed_cpu(lambda: ref.paged_decode_fp32(qd, kc, vc, tables, lens), min_s)
    dec = {"value": round(kv_bytes(ctx, c["kv_heads"], c["head_dim"]) * reps / el / 1e9, 4),
           "unit": "GB/s", "cores": cores, "kind": "port",
           "sample": f"2 of 64 sequences of config 4 (ctx {ctx}), {reps} calls in {el:.1f} s"}
    return pre, dec


def reference_arm(args):
    """The reference's CPU implementation (oracle port), K timed steps of a bounded sample."""
    from oracle import reference as ref

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    c = CFG2
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, 1, c["seq"], c["head_dim"], generator=g).half() for _ in range(3))
    step = lambda: ref.attention_fp32(q, k, v, causal=True)  # noqa: E731
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    flops = prefill_flops(1, 1, c["seq"], c["head_dim"], True)
    value = flops * args.steps / el / 1e12
    sample = ("each step: 1 of the 64 (batch, head) pairs of config 2 (B=4, H=16, N=4096, "
              "d=128, causal), fp32 on the host cores")
    return {
        "impl": "reference", "metric": BASELINE_METRIC, "value": round(value, 5),
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": "causal prefill, BASELINE config 2 (bounded sample per step)",
                   "batch": 1, "heads": 1, "seq_len": c["seq"], "head_dim": c["head_dim"],
                   "causal": True},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "oracle/reference.py restates the reference's attnkernels/reference.py "
                "(its fp32 PyTorch path); the reference itself is Python and cannot travel "
                "to this host",
    }


def profile_case(kind, d: Dist):
    """One small case for an ncu capture: inputs above L2, a few GB at most."""
    import attnkernels as ak

    if kind == "prefill":
        c = CFG2  # 192 MiB of q, k, v
        gen = torch.Generator(device=d.device).manual_seed(1000)
        shape = (c["batch"], c["heads"], c["seq"], c["head_dim"])
        q, k, v = (randn_half(shape, gen, d.device) for _ in range(3))
        fn = lambda: ak.flash_attention(q, k, v, causal=True)  # noqa: E731
    elif kind in ("prefill_d64", "prefill_n4095"):
        c = dict(CFG2, head_dim=64) if kind == "prefill_d64" else dict(CFG2, seq=4095)
        gen = torch.Generator(device=d.device).manual_seed(1100)
        shape = (c["batch"], c["heads"], c["seq"], c["head_dim"])
        q, k, v = (randn_half(shape, gen, d.device) for _ in range(3))
        fn = lambda: ak.flash_attention(q, k, v, causal=True)  # noqa: E731
    elif kind == "prefill_long":
        # 8 of config 3's 32 heads (q, k, v 192 MiB, above L2): its DRAM bytes per head
        # scale to a rank's share of config 3.
        c = CFG3
        gen = torch.Generator(device=d.device).manual_seed(3000)
        shape = (1, 8, c["seq"], c["head_dim"])
        q, k, v = (randn_half(shape, gen, d.device, c["input_scale"]) for _ in range(3))
        fn = lambda: ak.flash_attention(q, k, v, causal=True)  # noqa: E731
    elif kind == "decode_long":
        # One sequence of config 5's 131072 tokens, 32 heads (2.1 GB of K/V); DRAM bytes
        # per token scale to a rank's share of config 5.
        c = CFG5
        kc, vc, tables, lens = synthetic_paged_cache([c["ctx"]], c["kv_heads"], c["head_dim"],
                                                     c["block_size"], 5000, d.device)
        q = randn_half((1, c["heads"], c["head_dim"]),
                       torch.Generator(device=d.device).manual_seed(5100), d.device)
        part = ak.decode_partition(1, c["kv_heads"], c["ctx"])
        fn = lambda: ak.paged_decode(q, kc, vc, tables, lens, c["ctx"],  # noqa: E731
                                     partition_size=part)
    elif kind == "decode_d64":
        # head_dim 64 at the decode_gqa shape, one query head per kv head (8 and 8):
        # 1.07 GB of K/V, partition 512.
        ctx = [8192] * 64
        kc, vc, tables, lens = synthetic_paged_cache(ctx, 8, 64, 16, 4200, d.device)
        q = randn_half((64, 8, 64), torch.Generator(device=d.device).manual_seed(2), d.device)
        fn = lambda: ak.paged_decode(q, kc, vc, tables, lens, 8192,  # noqa: E731
                                     partition_size=512)
    elif kind == "decode_gqa":
        # The reference's results-table decode layer (32 query over 8 kv heads, d 128,
        # block 16) at 64 sequences of 8192 tokens: 2.1 GB of K/V, partition 512.
        ctx = [8192] * 64
        kc, vc, tables, lens = synthetic_paged_cache(ctx, 8, 128, 16, 4200, d.device)
        q = randn_half((64, 32, 128), torch.Generator(device=d.device).manual_seed(2),
                       d.device)
        fn = lambda: ak.paged_decode(q, kc, vc, tables, lens, 8192,  # noqa: E731
                                     partition_size=512)
    else:
        c = CFG4  # batch 16 of config 4: about 1.1 GB of K/V
        g = torch.Generator().manual_seed(4000)
        ctx = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (16,), generator=g).tolist()
        kc, vc, tables, lens = synthetic_paged_cache(ctx, c["kv_heads"], c["head_dim"],
                                                     c["block_size"], 4000, d.device)
        q = randn_half((16, c["heads"], c["head_dim"]),
                       torch.Generator(device=d.device).manual_seed(1), d.device)
        fn = lambda: ak.paged_decode(q, kc, vc, tables, lens, max(ctx),  # noqa: E731
                                     partition_size=c["partition"])
    for _ in range(5):
        fn()
    torch.cuda.synchronize(d.device)
    ak.check_device_status(d.device)


def split_ablation(args, d: Dist):
    """Decode GB/s versus partition size (the reference's split ablation,
    bench/bench.py:274-280, on B200 shapes): config 4, config 5 on one GPU, and
    one rank's share of config 5 at 8 GPUs (partials + local merge, no exchange)."""
    import attnkernels as ak
    from attnkernels import parallel

    rows = []
    cases = []
    c = CFG4
    g = torch.Generator().manual_seed(4000)
    ctx4 = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (c["batch"],), generator=g).tolist()
    cases.append(("config4", ctx4, False))
    c5 = CFG5
    cases.append(("config5_1gpu", [c5["ctx"]] * c5["batch"], False))
    t0, t1 = parallel.context_range(c5["ctx"], c5["block_size"], 8, 0)
    cases.append(("config5_rank_of_8", [t1 - t0] * c5["batch"], True))
    for name, ctx, partial in cases:
        kc, vc, tables, lens = synthetic_paged_cache(ctx, 32, 128, 16, 7, d.device)
        q = randn_half((len(ctx), 32, 128), torch.Generator(device=d.device).manual_seed(3), d.device)
        nbytes = kv_bytes(ctx, 32, 128)
        for part in [256, 512, 1024, 2048, 4096, None]:
            pp = part if part is not None else ak.decode_partition(len(ctx), 32, max(ctx))
            if partial:
                fn = lambda: ak.paged_decode_partials(q, kc, vc, tables, lens, max(ctx),  # noqa: E731
                                                      partition_size=pp)
            else:
                fn = lambda: ak.paged_decode(q, kc, vc, tables, lens, max(ctx),  # noqa: E731
                                             partition_size=pp)
            ms = timed(fn, args.steps, args.warmup, d) / args.steps
            rows.append({"case": name, "partition": pp, "auto": part is None,
                         "splits": -(-max(ctx) // pp), "ms": round(ms, 4),
                         "gbps": round(nbytes / (ms * 1e-3) / 1e9, 1)})
        del kc, vc
        torch.cuda.empty_cache()
    return rows


def main():
    ap = argparse.ArgumentParser(description="attention hot paths on B200")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-long", action="store_true", help="skip configs 3 and 5")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--only-prefill", action="store_true", help="headline kernel only")
    ap.add_argument("--no-compare", action="store_true",
                    help="skip the torch SDPA / gather+SDPA comparison rows")
    ap.add_argument("--spin", type=float, default=0.0,
                    help="seconds of untimed load before a timed region (default none: the "
                         "clocks are sampled during the timed steps themselves)")
    ap.add_argument("--cp-exchange", choices=["nccl", "peer"], default="peer",
                    help="how context-parallel decode exchanges its partials at N > 1: an NCCL "
                         "all-gather + merge kernel, or one kernel over peer memory")
    ap.add_argument("--cp-chunks", type=int, default=1,
                    help="batch chunks of the context-parallel decode at N > 1 (each "
                         "chunk's exchange overlaps the next chunk's decode)")
    ap.add_argument("--ablation", action="store_true",
                    help="print the decode split-size ablation (one JSON list) and exit")
    ap.add_argument("--profile", choices=["prefill", "prefill_d64", "prefill_n4095",
                                          "prefill_long", "decode", "decode_gqa", "decode_d64",
                                          "decode_long"],
                    help="run one small case of a kernel (3 + 2 launches) for ncu, no timing")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        print(json.dumps(reference_arm(args)), flush=True)
        return

    d = Dist(args.gpus)
    import attnkernels as ak

    ak.load_extension()  # fails loudly without the native library
    if args.profile:
        profile_case(args.profile, d)
        return
    if args.ablation:
        rows = split_ablation(args, d)
        if d.rank == 0:
            print(json.dumps({"split_ablation": rows}), flush=True)
        return
    peaks, peak_src = load_peaks()
    traffic = load_traffic()
    pre = bench_prefill_cfg2(args, d, peaks, peak_src, traffic)
    shapes = None if args.only_prefill else bench_prefill_shapes(args, d, peaks, peak_src,
                                                                 traffic)
    line = {
        "metric": BASELINE_METRIC,
        "value": round(pre["value"], 2),
        "unit": "TFLOP/s",
        "value_is": "causal prefill TFLOP/s, BASELINE config 2 per GPU, summed over GPUs",
        "n_gpus": d.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(pre["ms_per_step"], 4),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(pre["value"] / d.world / 13.94, 2),
        "vs_baseline_ref": "per GPU vs the reference's flash_wmma_bn32 on the same config on "
                           "a T4, 13.94 TFLOP/s (reference results/t4.md:44)",
        "dtype": "fp16", "data": "synthetic",
        "config": {"workload": "causal prefill, BASELINE config 2, one batch per GPU",
                   "batch": CFG2["batch"], "heads": CFG2["heads"], "seq_len": CFG2["seq"],
                   "head_dim": CFG2["head_dim"], "causal": True,
                   "parallelism": f"{d.world} GPU(s), independent (batch, head) units, "
                                  "no collective",
                   "l2": "inputs larger than L2 (q, k, v 192 MiB per step), no flush"},
        "roofline": pre["roofline"],
        "e2e": pre["e2e"],
        "gpu_launches": pre["gpu_launches"],
        "per_rank_ms_per_step": pre["per_rank_ms_per_step"],
        "clocks": pre["clocks"],
    }
    if shapes is not None:
        line["prefill_cfg2_shapes"] = shapes
    if not args.only_prefill:
        line["decode"] = bench_decode_cfg4(args, d, peaks, peak_src, traffic)
        if not args.no_long:
            line["long_context"] = bench_long_context(args, d, peaks, peak_src, traffic)
        if d.world == 1 and not args.no_compare:
            line["torch_comparison"] = torch_comparison(args, d, line["value"],
                                                        line["decode"]["value"])
    ak.check_device_status(d.device)
    if d.rank == 0 and d.world == 1 and not args.no_cpu:
        pre_cpu, dec_cpu = cpu_baseline()
        line["cpu_baseline"] = pre_cpu
        if "decode" in line:
            line["decode"]["cpu_baseline"] = dec_cpu
    if d.rank == 0:
        print(json.dumps(line), flush=True)
    d.close()


if __name__ == "__main__":
    main()
