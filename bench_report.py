"""Markdown tables from a bench_sweep.py JSON file (the reference's bench/report.py tables,
plus the fraction of the measured B200 peak for this build's kernels).

    python bench_report.py results/b200.json > results/b200.md
"""
from __future__ import annotations

import json
import sys

PREFILL_ORDER = ["sdpa", "sdpa_flash", "sdpa_efficient", "sdpa_cudnn", "sdpa_math", "naive",
                 "flash_simt", "flash_wmma_bn32", "flash_wmma_bn64"]
DECODE_ORDER = ["paged_split", "paged_nosplit", "torch_gather_sdpa", "torch_sdpa_contiguous"]


def cell(x, nd):
    return "" if x is None else f"{x:.{nd}f}"


def table(title, key_names, rows, key, col, value, order, nd):
    """One pivot: a line per key(row), a column per row[col] in `order`."""
    cols = [c for c in order if any(r[col] == c for r in rows)]
    lines = {}
    for r in rows:
        lines.setdefault(key(r), {})[r[col]] = r.get(value)
    out = [f"#### {title}", "", "| " + " | ".join(key_names + cols) + " |",
           "|" + "---|" * len(key_names) + "---:|" * len(cols)]
    for k, vals in lines.items():
        k = k if isinstance(k, tuple) else (k,)
        out.append("| " + " | ".join([str(x) for x in k] + [cell(vals.get(c), nd) for c in cols])
                   + " |")
    return "\n".join(out) + "\n"


def render(data) -> str:
    m = data["meta"]
    parts = []
    smi = m.get("nvidia_smi", "")
    driver = smi.split(",")[1].strip() if smi.count(",") >= 1 else "?"
    parts.append(f"GPU: {m['gpu']} (sm_{m['sm'].replace('.', '')}, {m['sm_count']} SMs, "
                 f"{m['memory_gb']} GB), driver {driver}, PyTorch {m['torch']}, CUDA {m['cuda']}, "
                 f"measured {m['date']}.\n")
    if "roofs" in m:
        parts.append(f"Ceilings measured in the sweep: device-to-device copy "
                     f"{m['roofs']['copy_gbps']} GB/s, fp16 GEMM 8192^3 (cuBLAS) "
                     f"{m['roofs']['fp16_gemm_tflops']} TFLOP/s.\n")
    if "measured_peaks" in m:
        p = m["measured_peaks"]
        parts.append(f"`frac` columns divide by {p['source']}: {p['tflops']} TFLOP/s dense "
                     f"tensor (prefill), {p['hbm_gbs']} GB/s HBM copy (decode).\n")
    if "sdpa_backends" in m:
        parts.append("SDPA backends here: " + ", ".join(
            f"{k}: {'ok' if v == 'ok' else 'unavailable'}"
            for k, v in m["sdpa_backends"].items()) + ".\n")
    res = data["results"]

    pre = [r for r in res if r["section"] == "prefill"]
    dims = sorted({r["head_dim"] for r in pre})
    for d in dims:
        for causal in (False, True):
            rows = [r for r in pre if r["head_dim"] == d and r["causal"] == causal]
            if rows:
                kind = "causal" if causal else "non-causal"
                parts.append(table(f"Prefill TFLOP/s, head_dim {d}, {kind}, 16 heads",
                                   ["seq", "batch"], rows, lambda r: (r["seq"], r["batch"]),
                                   "impl", "tflops", PREFILL_ORDER, 2))
    ours = [r for r in pre if r["impl"] == "flash_wmma_bn64" and "frac" in r]
    if ours:
        parts.append(table("flash_wmma (tcgen05 kernel): fraction of the measured tensor peak",
                           ["head_dim", "causal", "seq", "batch"], ours,
                           lambda r: (r["head_dim"], r["causal"], r["seq"], r["batch"]),
                           "impl", "frac", ["flash_wmma_bn64"], 3))
    for d in dims:
        rows = [r for r in pre if r["head_dim"] == d and not r["causal"]]
        if rows:
            parts.append(table(f"Prefill peak extra memory (MB), head_dim {d}, non-causal "
                               f"(includes the output)", ["seq", "batch"], rows,
                               lambda r: (r["seq"], r["batch"]), "impl", "peak_mem_mb",
                               PREFILL_ORDER, 0))
    if pre:
        lines = ["#### Prefill max abs error vs fp32 (worst case over all shapes)", "",
                 "| impl | max abs error |", "|---|---:|"]
        for c in PREFILL_ORDER:
            errs = [r["max_abs_err"] for r in pre if r["impl"] == c]
            if errs:
                lines.append(f"| {c} | {max(errs):.2e} |")
        parts.append("\n".join(lines) + "\n")

    dec = [r for r in res if r["section"] == "decode"]
    if dec:
        key = lambda r: (r["batch"], r["ctx"])  # noqa: E731
        parts.append(table("Decode GB/s (K+V bytes / time), 32 query heads, 8 kv heads, "
                           "head_dim 128", ["batch", "ctx"], dec, key, "impl", "gbps",
                           DECODE_ORDER, 1))
        parts.append(table("Decode time (ms)", ["batch", "ctx"], dec, key, "impl", "ms",
                           DECODE_ORDER, 4))
        parts.append(table("Decode: fraction of the measured HBM copy bandwidth",
                           ["batch", "ctx"], dec, key, "impl", "frac",
                           ["paged_split", "paged_nosplit"], 3))
    abl = [r for r in res if r["section"] == "split_ablation"]
    if abl:
        lines = ["#### Split-K partition size", "",
                 "| batch | ctx | partition | splits | work units | ms | GB/s |",
                 "|---|---|---:|---:|---:|---:|---:|"]
        for r in abl:
            lines.append(f"| {r['batch']} | {r['ctx']} | {r['partition']} | {r['splits']} | "
                         f"{r['splits'] * r['batch'] * r['kv_heads']} | {r['ms']:.4f} | "
                         f"{r['gbps']:.1f} |")
        parts.append("\n".join(lines) + "\n")
    rag = [r for r in res if r["section"] == "ragged"]
    if rag:
        lens = rag[0].get("ctx_lens", [])
        lines = [f"#### Ragged batch: {len(lens)} sequences, mean context "
                 f"{rag[0]['ctx_mean']:.0f}, max {rag[0]['ctx']}", "",
                 "| impl | ms | GB/s (useful bytes) |", "|---|---:|---:|"]
        for r in rag:
            lines.append(f"| {r['impl']} | {r['ms']:.4f} | {r['gbps']:.1f} |")
        parts.append("\n".join(lines) + "\n")
    return "\n".join(parts)


def main(path):
    with open(path) as f:
        sys.stdout.write(render(json.load(f)))


if __name__ == "__main__":
    main(sys.argv[1])
