"""Results sweep of the attention kernels on B200 against PyTorch, written as JSON.

    python bench_sweep.py --out results/b200.json [--quick] [--only prefill decode ...]
    python bench_report.py results/b200.json > results/b200.md

The sections, shapes, implementation names and row fields are those of the
reference's results sweep (bench/bench.py:138-300), so the tables it makes
compare line by line with the reference's published ones:

* prefill: head_dim 64 and 128, causal and not, 16 heads, seq 512..8192 with
  batch * seq = 16384 tokens; torch SDPA (default and each backend that runs),
  naive (seq <= 4096), flash simt, flash wmma with block_n 32 and 64.
* decode: 32 query heads over 8 kv heads (G = 4), head_dim 128, block size 16,
  batch 1..64 x context 1024..32768 (cases above 2.2 GB of K+V skipped, as in
  the reference); paged split-K, paged without splits, torch gather + SDPA and
  SDPA on an already contiguous cache.
* split_ablation: paged decode at every partition size 256..context.
* ragged: 16 sequences with seeded contexts U[512, 32768].

B200 differences: the L2 flush before every timed call writes 256 MiB (L2 is
126 MB); every row carries `frac`, its throughput over the measured peak of
MEASURED_PEAKS.json (dense fp16/bf16 tensor peak for prefill, HBM copy
bandwidth for decode), and `n_gpus` (1). `max_abs_err` is against an fp32
PyTorch restatement of each op computed in this file (batch 0, heads 0-1 for
prefill; sequence 0 for decode). Timing: CUDA events around each call on the
current stream, after one warm-up call, median of 3..50 calls (enough for
about 0.3 s). Data are seeded N(0, 1) fp16.
"""
from __future__ import annotations

import argparse
import datetime as dt
import json
import math
import platform
import statistics
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "flash-attention-from-scratch_b200"))

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

import attnkernels as ak  # noqa: E402

try:
    from torch.nn.attention import SDPBackend, sdpa_kernel
except ImportError:  # older torch
    SDPBackend = sdpa_kernel = None

PREFILL_HEADS = 16
HQ, HKV, D, BS = 32, 8, 128, 16  # decode: grouped-query layer, 4 query heads per kv head
FLUSH_BYTES = 256 * 2**20
_FLUSH = None


def flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    _FLUSH.zero_()


def time_ms(fn, warmup=1, target_ms=300.0, min_reps=3, max_reps=50):
    """Median CUDA-event time of one call; L2 flushed before each, outside the events."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    times = []
    reps = max_reps
    while len(times) < reps:
        flush_l2()
        start.record()
        fn()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end))
        if len(times) == 1:
            reps = int(min(max_reps, max(min_reps, target_ms / max(times[0], 1e-3))))
    return statistics.median(times)


def peak_extra_mb(fn):
    """Peak device memory of one call above what was allocated before (output included)."""
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    out = fn()
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    del out
    return round(peak / 2**20, 1)


def kernel_names(fn):
    """Names of the CUDA kernels one call launches (which SDPA backend ran)."""
    from torch.profiler import ProfilerActivity, profile

    fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    names = []
    for e in prof.events():
        dev = getattr(e, "device_type", None)
        if dev is not None and "CUDA" in str(dev) and e.name not in names:
            names.append(e.name)
    return names


def sdpa_with(backend):
    def run(q, k, v, causal):
        with sdpa_kernel([backend]):
            return F.scaled_dot_product_attention(q, k, v, is_causal=causal)
    return run


def sdpa_backends():
    """Which SDPA backends run here for fp16 [B, H, N, 128]."""
    out = {}
    if sdpa_kernel is None:
        return out
    q = torch.randn(1, 2, 256, 128, device="cuda", dtype=torch.float16)
    for name in ["FLASH_ATTENTION", "EFFICIENT_ATTENTION", "CUDNN_ATTENTION", "MATH"]:
        be = getattr(SDPBackend, name, None)
        if be is None:
            continue
        try:
            sdpa_with(be)(q, q, q, True)
            torch.cuda.synchronize()
            out[name] = "ok"
        except Exception as e:  # noqa: BLE001  a backend that does not run here
            out[name] = "unavailable: " + str(e).splitlines()[0][:200]
    return out


def roofs():
    """Ceilings measured in this process: device copy and a cuBLAS fp16 GEMM 8192^3."""
    x = torch.empty(512 * 2**20, dtype=torch.uint8, device="cuda")
    y = torch.empty_like(x)
    ms = time_ms(lambda: y.copy_(x))
    copy_gbps = 2 * x.numel() / (ms * 1e-3) / 1e9
    del x, y
    a = torch.randn(8192, 8192, device="cuda", dtype=torch.float16)
    ms = time_ms(lambda: a @ a)
    mm_tflops = 2 * 8192**3 / (ms * 1e-3) / 1e12
    del a
    torch.cuda.empty_cache()
    return dict(copy_gbps=round(copy_gbps, 1), fp16_gemm_tflops=round(mm_tflops, 2))


def measured_peaks():
    """MEASURED_PEAKS.json (driver-written), else the pool's earlier measurement."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return {"hbm_gbs": float(j["hbm_gbs"]), "tflops": float(j["bf16_tflops"]),
                "source": "MEASURED_PEAKS.json"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "source": "fallback"}


# ----------------------------------------------------------- fp32 checks


def attention_fp32(q, k, v, causal, scale=None):
    """softmax(scale q k^T, top-left causal mask) v in fp32."""
    q, k, v = q.float(), k.float(), v.float()
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    if causal:
        n, m = s.shape[-2], s.shape[-1]
        s.masked_fill_(torch.ones(n, m, dtype=torch.bool, device=s.device).triu(1),
                       float("-inf"))
    return torch.matmul(torch.softmax(s, -1), v)


def prefill_err(out, q, k, v, causal):
    r = attention_fp32(q[:1, :2], k[:1, :2], v[:1, :2], causal)
    return (out[:1, :2].float() - r).abs().max().item()


def gather_kv(cache, tables, n_blocks):
    """[num_blocks, H_kv, bs, D] -> [B, H_kv, n_blocks * bs, D]."""
    g = cache[tables[:, :n_blocks].long()]
    b, nb, h, bs, d = g.shape
    return g.permute(0, 2, 1, 3, 4).reshape(b, h, nb * bs, d)


def decode_row0_fp32(q, kc, vc, tables, ctx0):
    """Sequence 0 of paged decode in fp32: [H, D]."""
    hq, hkv, bs = q.shape[1], kc.shape[1], kc.shape[2]
    k = gather_kv(kc, tables[:1], -(-ctx0 // bs))[0, :, :ctx0].float()
    v = gather_kv(vc, tables[:1], -(-ctx0 // bs))[0, :, :ctx0].float()
    k = k.repeat_interleave(hq // hkv, dim=0)
    v = v.repeat_interleave(hq // hkv, dim=0)
    s = torch.einsum("hd,hcd->hc", q[0].float(), k) / math.sqrt(q.shape[-1])
    return torch.einsum("hc,hcd->hd", torch.softmax(s, -1), v)


def gather_sdpa(q, kc, vc, tables, n_blocks, lens=None):
    """The route without a paged kernel: gather into a padded contiguous cache, then
    SDPA with the G query heads of a kv head folded into G query rows."""
    B, H, Dh = q.shape
    hkv = kc.shape[1]
    k = gather_kv(kc, tables, n_blocks)
    v = gather_kv(vc, tables, n_blocks)
    mask = None
    if lens is not None:
        idx = torch.arange(k.shape[2], device=q.device)
        mask = (idx[None, :] < lens[:, None].long())[:, None, None, :]
    o = F.scaled_dot_product_attention(q.view(B, hkv, H // hkv, Dh), k, v, attn_mask=mask)
    return o.reshape(B, H, Dh)


def paged_cache(ctx_lens, seed):
    """Seeded paged cache: block ids a random permutation of the pool, N(0, 1) K and V."""
    g = torch.Generator().manual_seed(seed)
    nblk = [-(-c // BS) for c in ctx_lens]
    pool = sum(nblk)
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    tables = torch.zeros(len(ctx_lens), max(nblk), dtype=torch.int32)
    pos = 0
    for b, n in enumerate(nblk):
        tables[b, :n] = perm[pos:pos + n]
        pos += n
    gd = torch.Generator(device="cuda").manual_seed(seed)
    shape = (pool, HKV, BS, D)
    kc = torch.randn(shape, generator=gd, device="cuda", dtype=torch.float16)
    vc = torch.randn(shape, generator=gd, device="cuda", dtype=torch.float16)
    lens = torch.tensor(ctx_lens, dtype=torch.int32, device="cuda")
    return kc, vc, tables.cuda(), lens


# ---------------------------------------------------------------- prefill


def bench_prefill(results, quick, backends, peaks):
    tokens = 4096 if quick else 16384  # batch * seq kept constant
    seqs = [512, 1024] if quick else [512, 1024, 2048, 4096, 8192]
    gen = torch.Generator(device="cuda").manual_seed(0)
    for d in [64, 128]:
        for causal in [False, True]:
            for n in seqs:
                b = max(1, tokens // n)
                shape = (b, PREFILL_HEADS, n, d)
                q, k, v = (torch.randn(shape, generator=gen, device="cuda",
                                       dtype=torch.float16) for _ in range(3))
                flops = 4.0 * b * PREFILL_HEADS * n * n * d * (0.5 if causal else 1.0)
                impls = {"sdpa": lambda: F.scaled_dot_product_attention(q, k, v,
                                                                        is_causal=causal)}
                for name in ["FLASH_ATTENTION", "EFFICIENT_ATTENTION", "CUDNN_ATTENTION"]:
                    if backends.get(name) == "ok":
                        impls["sdpa_" + name.split("_")[0].lower()] = (
                            lambda be=getattr(SDPBackend, name): sdpa_with(be)(q, k, v, causal))
                if n <= 4096 and backends.get("MATH") == "ok":
                    impls["sdpa_math"] = lambda: sdpa_with(SDPBackend.MATH)(q, k, v, causal)
                if n <= 4096:
                    impls["naive"] = lambda: ak.naive_attention(q, k, v, causal=causal)
                impls["flash_simt"] = lambda: ak.flash_attention(q, k, v, causal, variant="simt")
                for bn in (32, 64):
                    impls[f"flash_wmma_bn{bn}"] = (
                        lambda bn=bn: ak.flash_attention(q, k, v, causal, variant="wmma",
                                                         block_n=bn))
                rows = []
                for name, fn in impls.items():
                    try:
                        out = fn()
                        err = prefill_err(out, q, k, v, causal)
                        del out
                        ms = time_ms(fn)
                        mem = peak_extra_mb(fn)
                    except Exception as e:  # noqa: BLE001  e.g. out of memory
                        print(f"prefill {name} d={d} N={n} failed: {e!r}"[:300], flush=True)
                        torch.cuda.empty_cache()
                        continue
                    tflops = flops / (ms * 1e-3) / 1e12
                    rows.append(dict(section="prefill", impl=name, batch=b, heads=PREFILL_HEADS,
                                     seq=n, head_dim=d, causal=causal, ms=round(ms, 4),
                                     tflops=round(tflops, 3),
                                     frac=round(tflops / peaks["tflops"], 4), n_gpus=1,
                                     peak_mem_mb=mem, max_abs_err=float(f"{err:.3g}")))
                base = next((r["ms"] for r in rows if r["impl"] == "sdpa"), None)
                for r in rows:
                    r["speedup_vs_sdpa"] = round(base / r["ms"], 3) if base else None
                    results.append(r)
                    print(f"prefill d={d} causal={int(causal)} B={b} N={n:5d} {r['impl']:18s} "
                          f"{r['ms']:9.3f} ms {r['tflops']:8.2f} TFLOP/s "
                          f"{r['peak_mem_mb']:8.1f} MB err {r['max_abs_err']:.2e} "
                          f"x{r['speedup_vs_sdpa']}", flush=True)
                del q, k, v
                torch.cuda.empty_cache()


# ----------------------------------------------------------------- decode


def kv_bytes(ctx_lens):
    return sum(ctx_lens) * HKV * D * 2 * 2  # K and V, fp16


def decode_case(results, section, ctx_lens, wanted, peaks, partition=None, extra=None,
                seed=0):
    B = len(ctx_lens)
    kc, vc, tables, lens = paged_cache(ctx_lens, seed)
    q = torch.randn(B, HQ, D, generator=torch.Generator(device="cuda").manual_seed(seed + 1),
                    device="cuda", dtype=torch.float16)
    max_ctx = max(ctx_lens)
    nblk = -(-max_ctx // BS)
    uniform = len(set(ctx_lens)) == 1
    impls = {}
    if "paged_split" in wanted:
        impls["paged_split"] = lambda: ak.paged_decode(q, kc, vc, tables, lens, max_ctx,
                                                        partition_size=partition)
    if "paged_nosplit" in wanted:
        impls["paged_nosplit"] = lambda: ak.paged_decode(q, kc, vc, tables, lens, max_ctx,
                                                          partition_size=1 << 30)
    if "torch_gather_sdpa" in wanted:
        mask_lens = None if uniform else lens
        impls["torch_gather_sdpa"] = lambda: gather_sdpa(q, kc, vc, tables, nblk, mask_lens)
    kg = vg = None
    if "torch_sdpa_contiguous" in wanted and uniform:
        kg = gather_kv(kc, tables, nblk)
        vg = gather_kv(vc, tables, nblk)
        qg = q.view(B, HKV, HQ // HKV, D)
        impls["torch_sdpa_contiguous"] = lambda: F.scaled_dot_product_attention(qg, kg, vg)
    expect = decode_row0_fp32(q, kc, vc, tables, ctx_lens[0])
    nbytes = kv_bytes(ctx_lens)
    part = partition if partition is not None else ak.decode_partition(B, HKV, max_ctx, num_heads=HQ)
    rows = []
    for name, fn in impls.items():
        try:
            out = fn()
            err = (out[:1].float().reshape(expect.shape) - expect).abs().max().item()
            del out
            ms = time_ms(fn)
        except Exception as e:  # noqa: BLE001  e.g. out of memory
            print(f"{section} {name} B={B} ctx={max_ctx} failed: {e!r}"[:300], flush=True)
            torch.cuda.empty_cache()
            continue
        gbps = nbytes / (ms * 1e-3) / 1e9
        row = dict(section=section, impl=name, batch=B, ctx=max_ctx, ctx_mean=sum(ctx_lens) / B,
                   heads=HQ, kv_heads=HKV, head_dim=D, block_size=BS, ms=round(ms, 4),
                   gbps=round(gbps, 1), frac=round(gbps / peaks["hbm_gbs"], 4), n_gpus=1,
                   max_abs_err=float(f"{err:.3g}"))
        if name == "paged_split":
            row["partition"] = part
            row["splits"] = -(-max_ctx // part)
        if extra:
            row.update(extra)
        rows.append(row)
    base = next((x["ms"] for x in rows if x["impl"] == "torch_gather_sdpa"), None)
    for r in rows:
        if base:
            r["speedup_vs_torch_gather"] = round(base / r["ms"], 3)
        results.append(r)
        print(f"{section} B={B:3d} ctx={max_ctx:6d} {r['impl']:22s} {r['ms']:8.4f} ms "
              f"{r['gbps']:7.1f} GB/s err {r['max_abs_err']:.1e}"
              f"{'  part=' + str(r.get('partition')) if 'partition' in r else ''}", flush=True)
    del kc, vc, kg, vg, q
    torch.cuda.empty_cache()


def bench_decode(results, quick, peaks):
    batches = [1, 16] if quick else [1, 4, 16, 64]
    ctxs = [1024, 4096] if quick else [1024, 2048, 4096, 8192, 16384, 32768]
    wanted = ["paged_split", "paged_nosplit", "torch_gather_sdpa", "torch_sdpa_contiguous"]
    for B in batches:
        for c in ctxs:
            if kv_bytes([c] * B) > 2.2e9:
                continue
            decode_case(results, "decode", [c] * B, wanted, peaks, seed=B * 100000 + c)


def bench_split_ablation(results, quick, peaks):
    cases = [(1, 8192)] if quick else [(1, 32768), (4, 8192), (16, 4096)]
    for B, c in cases:
        p = 256
        while p <= c:
            decode_case(results, "split_ablation", [c] * B, ["paged_split"], peaks,
                        partition=p, seed=B * 100000 + c)
            p *= 2


def bench_ragged(results, quick, peaks):
    g = torch.Generator().manual_seed(0)
    B = 8 if quick else 16
    hi = 8192 if quick else 32768
    lens = torch.randint(512, hi + 1, (B,), generator=g).tolist()
    decode_case(results, "ragged", lens, ["paged_split", "paged_nosplit", "torch_gather_sdpa"],
                peaks, extra=dict(ctx_lens=lens), seed=7)


# ------------------------------------------------------------------- main


def meta():
    p = torch.cuda.get_device_properties(0)
    try:
        smi = subprocess.run(["nvidia-smi", "--query-gpu=name,driver_version,clocks.max.sm,"
                              "clocks.max.mem", "--format=csv,noheader", "-i", "0"],
                             capture_output=True, text=True, timeout=30).stdout.strip()
    except Exception:  # noqa: BLE001
        smi = ""
    return dict(gpu=p.name, sm=f"{p.major}.{p.minor}", sm_count=p.multi_processor_count,
                memory_gb=round(p.total_memory / 2**30, 1), torch=torch.__version__,
                cuda=torch.version.cuda, nvidia_smi=smi, python=platform.python_version(),
                date=dt.datetime.now(dt.timezone.utc).strftime("%Y-%m-%d %H:%M UTC"))


SECTIONS = ["prefill", "decode", "split_ablation", "ragged"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="results/b200.json")
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--only", nargs="*", default=SECTIONS, choices=SECTIONS)
    args = ap.parse_args()
    if not torch.cuda.is_available():
        sys.exit("bench_sweep.py needs a CUDA device")
    torch.manual_seed(0)
    ak.load_extension()
    info = meta()
    info["sdpa_backends"] = sdpa_backends()
    try:
        for d in (64, 128):
            q = torch.randn(4, 16, 2048, d, device="cuda", dtype=torch.float16)
            info[f"sdpa_default_kernels_prefill_d{d}"] = kernel_names(
                lambda: F.scaled_dot_product_attention(q, q, q, is_causal=True))
        qd = torch.randn(4, 8, 4, 128, device="cuda", dtype=torch.float16)
        kd = torch.randn(4, 8, 4096, 128, device="cuda", dtype=torch.float16)
        info["sdpa_default_kernels_decode"] = kernel_names(
            lambda: F.scaled_dot_product_attention(qd, kd, kd))
        del q, qd, kd
    except Exception as e:  # noqa: BLE001
        info["sdpa_default_kernels_error"] = repr(e)[:300]
    info["roofs"] = roofs()
    peaks = measured_peaks()
    info["measured_peaks"] = peaks
    info["flush_bytes"] = FLUSH_BYTES
    print(json.dumps(info, indent=1), flush=True)
    results = []
    for name in args.only:
        try:
            if name == "prefill":
                bench_prefill(results, args.quick, info["sdpa_backends"], peaks)
            else:
                globals()["bench_" + name](results, args.quick, peaks)
        except Exception as e:  # noqa: BLE001  keep what was measured
            print(f"section {name} failed: {e!r}", flush=True)
            info.setdefault("failed_sections", {})[name] = repr(e)[:500]
        Path(args.out).parent.mkdir(parents=True, exist_ok=True)
        Path(args.out).write_text(json.dumps(dict(meta=info, results=results), indent=1))
    code, site = ak.device_status()
    info["device_status"] = {"code": code, "site": site}
    Path(args.out).write_text(json.dumps(dict(meta=info, results=results), indent=1))
    print("wrote", args.out, "device status", code, site)
    if code != 0:
        sys.exit(f"kernel error status {code} at site {site}")


if __name__ == "__main__":
    main()
