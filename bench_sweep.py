"""Results sweep on one B200: the reference's results tables, measured with bench.py.

    python bench_sweep.py --out results/b200.json [--quick] [--only prefill decode ...]
    python bench_report.py results/b200.json > results/b200.md

What is swept is the reference's published results layout (its bench/bench.py
sections prefill, decode, split_ablation and ragged: the shapes, the
implementation names and the JSON row fields), so that its tables and these
compare line by line. How it is measured is this repository's: every call is
timed by bench.timed_each (CUDA events on the current stream, L2 written cold
before each call, outside the events), rows carry bench.roofline's fraction of
MEASURED_PEAKS.json (`frac`) and the median SM clock that bench.NvmlClockSampler
saw while the row was timed (`sm_mhz`), and inputs come from bench's seeded
generators.

Shapes: prefill at head_dim 64 and 128, causal and not, 16 heads, sequence
512..8192 with batch * sequence = 16384; decode with 32 query heads over 8 kv
heads (4 per kv head), head_dim 128, block size 16, batch 1..64 x context
1024..32768 (cases above 2.2 GB of K and V left out); every power-of-two
partition from 256 up for the split ablation; 16 ragged sequences of
U[512, 32768] tokens. `max_abs_err` is against fp32 attention computed here on
the GPU (prefill: batch 0, heads 0 and 1; decode: sequence 0).
"""
from __future__ import annotations

import argparse
import datetime as dt
import itertools
import json
import math
import platform
import statistics
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "flash-attention-from-scratch_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

import bench  # noqa: E402

SECTIONS = ("prefill", "decode", "split_ablation", "ragged")
PREFILL_HEADS = 16
PREFILL_TOKENS = 16384  # batch * sequence, every prefill row
DEC_HQ, DEC_HKV, DEC_D, DEC_BS = 32, 8, 128, 16
DECODE_KV_LIMIT = 2.2e9  # bytes of K + V above which a decode case is left out


def decode_kv_bytes(ctx_lens):
    """K and V bytes of the decode layer (fp16): the reference's byte convention."""
    return bench.kv_bytes(ctx_lens, DEC_HKV, DEC_D)


class Harness:
    """Timing, clocks and roofline fractions for the sweep's rows (one GPU)."""

    def __init__(self, budget_ms=300.0, max_reps=50):
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.peaks, self.peak_src = bench.load_peaks()
        self.budget_ms, self.max_reps = budget_ms, max_reps

    def time(self, fn):
        """(median ms of one call, median SM MHz while timing)."""
        probe = statistics.median(bench.timed_each(fn, reps=1, warmup=1, device=self.device))
        reps = int(min(self.max_reps, max(3, self.budget_ms / max(probe, 1e-3))))
        with bench.NvmlClockSampler(self.device) as clk:
            ms = statistics.median(bench.timed_each(fn, reps=reps, warmup=0, device=self.device))
        return ms, clk.summary().get("sm_mhz")

    def rate(self, bound, work, ms):
        """(throughput, fraction of the measured peak) from bench.roofline."""
        r = bench.roofline(bound, work, ms, self.peaks, self.peak_src)
        return r["achieved"], r["frac"]

    def extra_memory_mb(self, fn):
        """Peak device memory one call allocates beyond what is held (output included)."""
        torch.cuda.synchronize(self.device)
        torch.cuda.reset_peak_memory_stats(self.device)
        held = torch.cuda.memory_allocated(self.device)
        out = fn()
        torch.cuda.synchronize(self.device)
        extra = torch.cuda.max_memory_allocated(self.device) - held
        del out
        return round(extra / 2**20, 1)


# -------------------------------------------------------------- fp32 checks


def attention_fp32(q, k, v, causal):
    """Exact attention of fp16 inputs in fp32 (top-left causal mask)."""
    s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if causal:
        keep = torch.ones(s.shape[-2:], dtype=torch.bool, device=s.device).tril()
        s = s.masked_fill(~keep, float("-inf"))
    return torch.softmax(s, dim=-1) @ v.float()


def contiguous_kv(cache, tables, n_blocks):
    """Paged [blocks, H_kv, bs, D] -> [B, H_kv, n_blocks * bs, D] through the block table."""
    b = tables.shape[0]
    picked = cache[tables[:, :n_blocks].reshape(-1).long()]
    picked = picked.view(b, n_blocks, *cache.shape[1:])
    return picked.transpose(1, 2).flatten(2, 3)


def decode_fp32_first(q, kc, vc, tables, ctx0):
    """Sequence 0 of the decode in fp32: [H, D]."""
    n_blocks = -(-ctx0 // kc.shape[2])
    g = q.shape[1] // kc.shape[1]
    k = contiguous_kv(kc, tables[:1], n_blocks)[0, :, :ctx0].float().repeat_interleave(g, 0)
    v = contiguous_kv(vc, tables[:1], n_blocks)[0, :, :ctx0].float().repeat_interleave(g, 0)
    s = (k @ q[0].float().unsqueeze(-1)).squeeze(-1) / math.sqrt(q.shape[-1])
    return (torch.softmax(s, dim=-1).unsqueeze(1) @ v).squeeze(1)


def gather_then_sdpa(q, kc, vc, tables, n_blocks, lens=None):
    """Decode without a paged kernel (the reference's comparison route): copy the
    blocks into a padded contiguous cache, then SDPA with the query heads of a kv
    head as query rows and, for ragged batches, a length mask."""
    b, hq, d = q.shape
    k = contiguous_kv(kc, tables, n_blocks)
    v = contiguous_kv(vc, tables, n_blocks)
    mask = None
    if lens is not None:
        pos = torch.arange(k.shape[2], device=q.device)
        mask = (pos.unsqueeze(0) < lens.long().unsqueeze(1)).view(b, 1, 1, -1)
    o = F.scaled_dot_product_attention(q.view(b, kc.shape[1], hq // kc.shape[1], d), k, v,
                                       attn_mask=mask)
    return o.reshape(b, hq, d)


# ------------------------------------------------------------------ prefill


def sdpa_backends():
    """SDPA backends that run fp16 [B, H, N, 128] here: name -> "ok" or why not."""
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
    except ImportError:
        return {}
    q = torch.randn(1, 2, 256, 128, device="cuda", dtype=torch.float16)
    found = {}
    for name in ("FLASH_ATTENTION", "EFFICIENT_ATTENTION", "CUDNN_ATTENTION", "MATH"):
        backend = getattr(SDPBackend, name, None)
        if backend is None:
            continue
        try:
            with sdpa_kernel([backend]):
                F.scaled_dot_product_attention(q, q, q, is_causal=True)
            torch.cuda.synchronize()
            found[name] = "ok"
        except Exception as e:  # noqa: BLE001  a backend this GPU or build lacks
            found[name] = "unavailable: " + str(e).splitlines()[0][:200]
    return found


def prefill_impls(q, k, v, causal, backends):
    """The reference's prefill implementation names -> callables on these inputs."""
    import attnkernels as ak
    from torch.nn.attention import SDPBackend, sdpa_kernel

    def on_backend(name):
        def run():
            with sdpa_kernel([getattr(SDPBackend, name)]):
                return F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        return run

    impls = {"sdpa": lambda: F.scaled_dot_product_attention(q, k, v, is_causal=causal)}
    for backend, short in (("FLASH_ATTENTION", "flash"), ("EFFICIENT_ATTENTION", "efficient"),
                           ("CUDNN_ATTENTION", "cudnn")):
        if backends.get(backend) == "ok":
            impls["sdpa_" + short] = on_backend(backend)
    small = q.shape[2] <= 4096  # the N x N score matrix stays in reach
    if small and backends.get("MATH") == "ok":
        impls["sdpa_math"] = on_backend("MATH")
    if small:
        impls["naive"] = lambda: ak.naive_attention(q, k, v, causal=causal)
    impls["flash_simt"] = lambda: ak.flash_attention(q, k, v, causal, variant="simt")
    for bn in (32, 64):
        impls[f"flash_wmma_bn{bn}"] = (
            lambda bn=bn: ak.flash_attention(q, k, v, causal, variant="wmma", block_n=bn))
    return impls


def run_prefill(h, rows, quick, backends):
    seqs = (512, 1024) if quick else (512, 1024, 2048, 4096, 8192)
    tokens = 4096 if quick else PREFILL_TOKENS
    gen = torch.Generator(device=h.device).manual_seed(0)
    for d, causal, n in itertools.product((64, 128), (False, True), seqs):
        batch = max(1, tokens // n)
        q, k, v = (bench.randn_half((batch, PREFILL_HEADS, n, d), gen, h.device)
                   for _ in range(3))
        want = attention_fp32(q[:1, :2], k[:1, :2], v[:1, :2], causal)
        flops = bench.prefill_flops(batch, PREFILL_HEADS, n, d, causal)
        group = []
        for impl, fn in prefill_impls(q, k, v, causal, backends).items():
            try:
                err = (fn()[:1, :2].float() - want).abs().max().item()
                ms, mhz = h.time(fn)
                mem = h.extra_memory_mb(fn)
            except Exception as e:  # noqa: BLE001  e.g. a backend out of memory
                print(f"prefill {impl} d={d} N={n}: {str(e).splitlines()[0][:200]}", flush=True)
                torch.cuda.empty_cache()
                continue
            tflops, frac = h.rate("tensor", flops, ms)
            group.append(dict(section="prefill", impl=impl, batch=batch, heads=PREFILL_HEADS,
                              seq=n, head_dim=d, causal=causal, ms=round(ms, 4),
                              tflops=round(tflops, 3), frac=frac, n_gpus=1, sm_mhz=mhz,
                              peak_mem_mb=mem, max_abs_err=float(f"{err:.3g}")))
        sdpa_ms = {r["impl"]: r["ms"] for r in group}.get("sdpa")
        for r in group:
            r["speedup_vs_sdpa"] = round(sdpa_ms / r["ms"], 3) if sdpa_ms else None
            print(f"prefill d={d} causal={int(causal)} B={batch} N={n:5d} {r['impl']:16s} "
                  f"{r['ms']:9.3f} ms {r['tflops']:8.2f} TFLOP/s ({r['frac']:.3f}) "
                  f"err {r['max_abs_err']:.1e}", flush=True)
        rows.extend(group)
        del q, k, v, want
        torch.cuda.empty_cache()


# ------------------------------------------------------------------- decode


def decode_rows(h, section, seq_lens, impls_wanted, partition=None, seed=0, **extra):
    """Rows of one decode case (all requested implementations on the same cache); `extra`
    adds fields to every row (the ragged section records its `ctx_lens`)."""
    import attnkernels as ak

    b = len(seq_lens)
    kc, vc, tables, lens = bench.synthetic_paged_cache(seq_lens, DEC_HKV, DEC_D, DEC_BS, seed,
                                                       h.device)
    q = bench.randn_half((b, DEC_HQ, DEC_D),
                         torch.Generator(device=h.device).manual_seed(seed + 1), h.device)
    top = max(seq_lens)
    n_blocks = -(-top // DEC_BS)
    ragged = len(set(seq_lens)) > 1
    part = partition or ak.decode_partition(b, DEC_HKV, top, num_heads=DEC_HQ)
    impls = {
        "paged_split": lambda: ak.paged_decode(q, kc, vc, tables, lens, top,
                                               partition_size=partition),
        "paged_nosplit": lambda: ak.paged_decode(q, kc, vc, tables, lens, top,
                                                 partition_size=1 << 30),
        "torch_gather_sdpa": lambda: gather_then_sdpa(q, kc, vc, tables, n_blocks,
                                                      lens if ragged else None),
    }
    if not ragged:
        k_flat = contiguous_kv(kc, tables, n_blocks)
        v_flat = contiguous_kv(vc, tables, n_blocks)
        q_rows = q.view(b, DEC_HKV, DEC_HQ // DEC_HKV, DEC_D)
        impls["torch_sdpa_contiguous"] = lambda: F.scaled_dot_product_attention(q_rows, k_flat,
                                                                                v_flat)
    want = decode_fp32_first(q, kc, vc, tables, seq_lens[0])
    nbytes = decode_kv_bytes(seq_lens)
    out = []
    for impl in impls_wanted:
        fn = impls.get(impl)
        if fn is None:
            continue
        try:
            err = (fn()[:1].float().reshape(want.shape) - want).abs().max().item()
            ms, mhz = h.time(fn)
        except Exception as e:  # noqa: BLE001  e.g. the gather route out of memory
            print(f"{section} {impl} B={b} ctx={top}: {str(e).splitlines()[0][:200]}", flush=True)
            torch.cuda.empty_cache()
            continue
        gbps, frac = h.rate("hbm", nbytes, ms)
        row = dict(section=section, impl=impl, batch=b, ctx=top, ctx_mean=sum(seq_lens) / b,
                   heads=DEC_HQ, kv_heads=DEC_HKV, head_dim=DEC_D, block_size=DEC_BS,
                   ms=round(ms, 4), gbps=round(gbps, 1), frac=frac, n_gpus=1, sm_mhz=mhz,
                   max_abs_err=float(f"{err:.3g}"), **extra)
        if impl == "paged_split":
            row.update(partition=part, splits=-(-top // part))
        out.append(row)
    gather_ms = {r["impl"]: r["ms"] for r in out}.get("torch_gather_sdpa")
    for r in out:
        if gather_ms:
            r["speedup_vs_torch_gather"] = round(gather_ms / r["ms"], 3)
        print(f"{section} B={b:3d} ctx={top:6d} {r['impl']:22s} {r['ms']:8.4f} ms "
              f"{r['gbps']:7.1f} GB/s ({r['frac']:.3f}) err {r['max_abs_err']:.1e}", flush=True)
    del kc, vc, q
    torch.cuda.empty_cache()
    return out


def run_decode(h, rows, quick):
    batches = (1, 16) if quick else (1, 4, 16, 64)
    ctxs = (1024, 4096) if quick else (1024, 2048, 4096, 8192, 16384, 32768)
    impls = ("paged_split", "paged_nosplit", "torch_gather_sdpa", "torch_sdpa_contiguous")
    for b, c in itertools.product(batches, ctxs):
        if decode_kv_bytes([c] * b) <= DECODE_KV_LIMIT:
            rows.extend(decode_rows(h, "decode", [c] * b, impls, seed=b * 100000 + c))


def run_split_ablation(h, rows, quick):
    for b, c in ((1, 8192),) if quick else ((1, 32768), (4, 8192), (16, 4096)):
        part = 256
        while part <= c:
            rows.extend(decode_rows(h, "split_ablation", [c] * b, ("paged_split",),
                                    partition=part, seed=b * 100000 + c))
            part *= 2


def run_ragged(h, rows, quick):
    b, top = (8, 8192) if quick else (16, 32768)
    lens = torch.randint(512, top + 1, (b,), generator=torch.Generator().manual_seed(0)).tolist()
    rows.extend(decode_rows(h, "ragged", lens,
                            ("paged_split", "paged_nosplit", "torch_gather_sdpa"), seed=7,
                            ctx_lens=lens))


# --------------------------------------------------------------------- main


def environment(h):
    p = torch.cuda.get_device_properties(h.device)
    try:
        smi = subprocess.run(["nvidia-smi", "--query-gpu=name,driver_version,clocks.max.sm,"
                              "clocks.max.mem", "--format=csv,noheader",
                              "-i", str(h.device.index or 0)],
                             capture_output=True, text=True, timeout=30).stdout.strip()
    except Exception:  # noqa: BLE001
        smi = ""
    return dict(gpu=p.name, sm=f"{p.major}.{p.minor}", sm_count=p.multi_processor_count,
                memory_gb=round(p.total_memory / 2**30, 1), torch=torch.__version__,
                cuda=torch.version.cuda, nvidia_smi=smi, python=platform.python_version(),
                date=dt.datetime.now(dt.timezone.utc).strftime("%Y-%m-%d %H:%M UTC"),
                measured_peaks={"source": h.peak_src, "tflops": h.peaks["bf16_tflops"],
                                "hbm_gbs": h.peaks["hbm_gbs"]},
                timing="bench.timed_each: CUDA events per call, L2 written cold before each "
                       "call; median over ~0.3 s of calls; clocks from bench.NvmlClockSampler")


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default="results/b200.json")
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--only", nargs="*", default=list(SECTIONS), choices=SECTIONS)
    args = ap.parse_args()
    if not torch.cuda.is_available():
        sys.exit("bench_sweep.py needs a CUDA device")
    import attnkernels as ak

    ak.load_extension()  # fails loudly without the native library
    h = Harness()
    meta = environment(h)
    meta["sdpa_backends"] = sdpa_backends()
    print(json.dumps(meta, indent=1), flush=True)
    rows = []
    out = Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    runners = {"prefill": lambda: run_prefill(h, rows, args.quick, meta["sdpa_backends"]),
               "decode": lambda: run_decode(h, rows, args.quick),
               "split_ablation": lambda: run_split_ablation(h, rows, args.quick),
               "ragged": lambda: run_ragged(h, rows, args.quick)}
    for name in args.only:
        try:
            runners[name]()
        except Exception as e:  # noqa: BLE001  keep the sections already measured
            print(f"section {name} failed: {e!r}", flush=True)
            meta.setdefault("failed_sections", {})[name] = repr(e)[:500]
        out.write_text(json.dumps({"meta": meta, "results": rows}, indent=1))
    code, site = ak.device_status()
    meta["device_status"] = {"code": code, "site": site}
    out.write_text(json.dumps({"meta": meta, "results": rows}, indent=1))
    print("wrote", out, "device status", code, site)
    if code != 0:
        sys.exit(f"kernel error status {code} at site {site}")


if __name__ == "__main__":
    main()
