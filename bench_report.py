"""Markdown tables of a bench_sweep.py JSON file.

    python bench_report.py results/b200.json > results/b200.md

The tables are the reference's results tables (one per prefill head_dim and
mask, decode throughput and time, the split-K ablation, the ragged batch, with
its implementation columns in its order), plus columns this build adds: the
fraction of the measured B200 peak (`frac`) and the median SM clock of each
row (`sm_mhz`).
"""
from __future__ import annotations

import json
import sys

PREFILL_COLUMNS = ("sdpa", "sdpa_flash", "sdpa_efficient", "sdpa_cudnn", "sdpa_math", "naive",
                   "flash_simt", "flash_wmma_bn32", "flash_wmma_bn64")
DECODE_COLUMNS = ("paged_split", "paged_nosplit", "torch_gather_sdpa", "torch_sdpa_contiguous")


class Grid:
    """A titled Markdown table: one line per key (in first-seen order), one column
    per name in `columns` that has at least one value."""

    def __init__(self, title, key_names, columns, digits):
        self.title, self.key_names, self.columns, self.digits = title, key_names, columns, digits
        self.cells: dict[tuple, dict[str, float]] = {}

    def put(self, key, column, value):
        self.cells.setdefault(tuple(key), {})[column] = value

    def markdown(self):
        used = [c for c in self.columns if any(c in line for line in self.cells.values())]
        head = "| " + " | ".join(list(self.key_names) + used) + " |"
        rule = "|" + "---|" * len(self.key_names) + "---:|" * len(used)
        body = []
        for key, line in self.cells.items():
            vals = ["" if line.get(c) is None else f"{line[c]:.{self.digits}f}" for c in used]
            body.append("| " + " | ".join([str(k) for k in key] + vals) + " |")
        return "\n".join([f"#### {self.title}", "", head, rule, *body]) + "\n"


def grid_of(rows, title, key_names, key, value, columns, digits, column="impl"):
    g = Grid(title, key_names, columns, digits)
    for r in rows:
        g.put(key(r), r[column], r.get(value))
    return g.markdown()


def preamble(meta):
    smi = [x.strip() for x in meta.get("nvidia_smi", "").split(",")]
    driver = smi[1] if len(smi) > 1 else "?"
    out = [f"GPU: {meta['gpu']} (sm_{meta['sm'].replace('.', '')}, {meta['sm_count']} SMs, "
           f"{meta['memory_gb']} GB), driver {driver}, PyTorch {meta['torch']}, CUDA "
           f"{meta['cuda']}, measured {meta['date']}.\n"]
    peaks = meta.get("measured_peaks")
    if peaks:
        out.append(f"`frac` = throughput / the measured peak ({peaks['source']}): "
                   f"{peaks['tflops']} TFLOP/s dense fp16/bf16 tensor for prefill, "
                   f"{peaks['hbm_gbs']} GB/s HBM copy for decode.\n")
    if "timing" in meta:
        out.append(f"Timing: {meta['timing']}.\n")
    if "sdpa_backends" in meta:
        states = ", ".join(f"{k}: {'ok' if v == 'ok' else 'unavailable'}"
                           for k, v in meta["sdpa_backends"].items())
        out.append(f"SDPA backends here: {states}.\n")
    return out


def prefill_tables(pre):
    out = []
    dims = sorted({r["head_dim"] for r in pre})
    by_shape = lambda r: (r["seq"], r["batch"])  # noqa: E731
    for d in dims:
        for causal in (False, True):
            rows = [r for r in pre if r["head_dim"] == d and r["causal"] == causal]
            if rows:
                mask = "causal" if causal else "non-causal"
                out.append(grid_of(rows, f"Prefill TFLOP/s, head_dim {d}, {mask}, "
                                   f"{rows[0]['heads']} heads", ["seq", "batch"], by_shape,
                                   "tflops", PREFILL_COLUMNS, 2))
    ours = [r for r in pre if r["impl"] == "flash_wmma_bn64"]
    if ours:
        g = Grid("flash_wmma (the tcgen05 kernel): fraction of the measured tensor peak, "
                 "and the SM clock", ["head_dim", "causal", "seq", "batch"],
                 ["frac", "sm_mhz"], 3)
        for r in ours:
            key = (r["head_dim"], r["causal"], r["seq"], r["batch"])
            g.put(key, "frac", r.get("frac"))
            g.put(key, "sm_mhz", r.get("sm_mhz"))
        out.append(g.markdown())
    for d in dims:
        rows = [r for r in pre if r["head_dim"] == d and not r["causal"]]
        if rows:
            out.append(grid_of(rows, f"Prefill peak extra memory (MB), head_dim {d}, "
                               "non-causal (includes the output)", ["seq", "batch"], by_shape,
                               "peak_mem_mb", PREFILL_COLUMNS, 0))
    worst = {}
    for r in pre:
        worst[r["impl"]] = max(worst.get(r["impl"], 0.0), r["max_abs_err"])
    lines = ["#### Prefill max abs error vs fp32 (worst case over all shapes)", "",
             "| impl | max abs error |", "|---|---:|"]
    lines += [f"| {c} | {worst[c]:.2e} |" for c in PREFILL_COLUMNS if c in worst]
    out.append("\n".join(lines) + "\n")
    return out


def decode_tables(dec):
    by_case = lambda r: (r["batch"], r["ctx"])  # noqa: E731
    r0 = dec[0]
    layer = (f"{r0['heads']} query heads, {r0['kv_heads']} kv heads, "
             f"head_dim {r0['head_dim']}")
    return [grid_of(dec, f"Decode GB/s (K+V bytes / time), {layer}", ["batch", "ctx"], by_case,
                    "gbps", DECODE_COLUMNS, 1),
            grid_of(dec, "Decode time (ms)", ["batch", "ctx"], by_case, "ms", DECODE_COLUMNS, 4),
            grid_of(dec, "Decode: fraction of the measured HBM copy bandwidth",
                    ["batch", "ctx"], by_case, "frac", ("paged_split", "paged_nosplit"), 3)]


def ablation_table(abl):
    lines = ["#### Split-K partition size", "",
             "| batch | ctx | partition | splits | work units | ms | GB/s | frac |",
             "|---|---|---:|---:|---:|---:|---:|---:|"]
    for r in abl:
        units = r["splits"] * r["batch"] * r["kv_heads"]
        lines.append(f"| {r['batch']} | {r['ctx']} | {r['partition']} | {r['splits']} | "
                     f"{units} | {r['ms']:.4f} | {r['gbps']:.1f} | {r.get('frac', 0):.3f} |")
    return "\n".join(lines) + "\n"


def ragged_table(rag):
    lens = rag[0].get("ctx_lens", [])
    lines = [f"#### Ragged batch: {len(lens)} sequences, mean context {rag[0]['ctx_mean']:.0f}, "
             f"max {rag[0]['ctx']}", "", "| impl | ms | GB/s (useful bytes) | frac |",
             "|---|---:|---:|---:|"]
    lines += [f"| {r['impl']} | {r['ms']:.4f} | {r['gbps']:.1f} | {r.get('frac', 0):.3f} |"
              for r in rag]
    return "\n".join(lines) + "\n"


def render(data) -> str:
    res = data["results"]
    section = lambda name: [r for r in res if r["section"] == name]  # noqa: E731
    parts = preamble(data["meta"])
    if section("prefill"):
        parts += prefill_tables(section("prefill"))
    if section("decode"):
        parts += decode_tables(section("decode"))
    if section("split_ablation"):
        parts.append(ablation_table(section("split_ablation")))
    if section("ragged"):
        parts.append(ragged_table(section("ragged")))
    return "\n".join(parts)


def main(path):
    with open(path) as f:
        sys.stdout.write(render(json.load(f)))


if __name__ == "__main__":
    main(sys.argv[1])
