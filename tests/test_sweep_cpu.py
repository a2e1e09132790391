"""The results sweep's own fp32 checks and its report, on CPU: the error columns of
bench_sweep.py are measured against restatements that must agree with the oracle,
and bench_report.py must render every section the sweep writes."""
import json

import torch

import bench_report
import bench_sweep
from oracle import reference as ref


def test_attention_fp32_matches_oracle():
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(1, 2, 96, 64, generator=g) for _ in range(3))
    for causal in (False, True):
        got = bench_sweep.attention_fp32(q, k, v, causal)
        want = ref.attention_fp32(q, k, v, causal)
        assert (got - want).abs().max().item() < 1e-5


def test_decode_checks_match_oracle():
    torch.manual_seed(3)
    ctx = [40, 17, 64]
    kc, vc, tables, lens = ref.make_paged_cache(ctx, 2, 32, block_size=16, dtype=torch.float32,
                                                device="cpu", extra_blocks=2)
    q = torch.randn(3, 8, 32)
    want = ref.paged_decode_fp32(q, kc, vc, tables, lens)
    row0 = bench_sweep.decode_fp32_first(q, kc, vc, tables, ctx[0])
    assert (row0 - want[0]).abs().max().item() < 1e-5
    nblk = -(-max(ctx) // 16)
    got = bench_sweep.gather_then_sdpa(q, kc, vc, tables, nblk, lens)
    assert (got - want).abs().max().item() < 1e-5
    assert torch.equal(bench_sweep.contiguous_kv(kc, tables, nblk),
                       ref.gather_kv(kc, tables, nblk))


def test_section_drivers_call_decode_rows_with_its_signature(monkeypatch):
    """Every decode section's call binds to decode_rows' parameters (the ragged
    section adds its ctx_lens field to the rows)."""
    import inspect

    sig = inspect.signature(bench_sweep.decode_rows)
    calls = []

    def fake(*args, **kwargs):
        calls.append(sig.bind(*args, **kwargs))
        return []

    monkeypatch.setattr(bench_sweep, "decode_rows", fake)
    rows = []
    for run in (bench_sweep.run_decode, bench_sweep.run_split_ablation, bench_sweep.run_ragged):
        run(None, rows, True)
    assert calls and calls[-1].arguments["extra"]["ctx_lens"] == calls[-1].arguments["seq_lens"]


def test_kv_bytes_convention():
    # K and V, fp16, 8 kv heads of 128: the reference's bench/bench.py:199-200.
    assert bench_sweep.decode_kv_bytes([1024, 2048]) == 3072 * 8 * 128 * 4


def test_report_renders_every_section():
    meta = {"gpu": "NVIDIA B200", "sm": "10.0", "sm_count": 148, "memory_gb": 178.4,
            "torch": "2.11", "cuda": "12.8", "nvidia_smi": "NVIDIA B200, 580.159, 1965, 3996",
            "date": "now", "timing": "events per call",
            "measured_peaks": {"hbm_gbs": 6536.0, "tflops": 1644.0, "source": "measured"},
            "sdpa_backends": {"FLASH_ATTENTION": "ok", "MATH": "unavailable: x"}}
    res = []
    for impl in ("sdpa", "flash_wmma_bn64"):
        res.append(dict(section="prefill", impl=impl, batch=4, heads=16, seq=4096, head_dim=128,
                        causal=True, ms=0.3, tflops=900.0, frac=0.55, n_gpus=1,
                        peak_mem_mb=64.0, max_abs_err=1e-3))
        res.append(dict(section="prefill", impl=impl, batch=4, heads=16, seq=4096, head_dim=128,
                        causal=False, ms=0.5, tflops=1000.0, frac=0.6, n_gpus=1,
                        peak_mem_mb=64.0, max_abs_err=1e-3))
    for impl in ("paged_split", "torch_gather_sdpa"):
        res.append(dict(section="decode", impl=impl, batch=16, ctx=4096, ctx_mean=4096, heads=32,
                        kv_heads=8, head_dim=128, block_size=16, ms=0.1, gbps=5000.0, frac=0.76,
                        n_gpus=1, max_abs_err=1e-4))
    res.append(dict(section="split_ablation", impl="paged_split", batch=1, ctx=32768,
                    ctx_mean=32768, heads=32, kv_heads=8, head_dim=128, block_size=16, ms=0.05,
                    gbps=3000.0, frac=0.4, n_gpus=1, max_abs_err=1e-4, partition=256,
                    splits=128))
    res.append(dict(section="ragged", impl="paged_split", batch=3, ctx=900, ctx_mean=700.0,
                    heads=32, kv_heads=8, head_dim=128, block_size=16, ms=0.02, gbps=900.0,
                    frac=0.1, n_gpus=1, max_abs_err=1e-4, ctx_lens=[500, 700, 900]))
    text = bench_report.render(json.loads(json.dumps({"meta": meta, "results": res})))
    for title in ("Prefill TFLOP/s, head_dim 128, causal", "Prefill TFLOP/s, head_dim 128, "
                  "non-causal", "fraction of the measured tensor peak", "peak extra memory",
                  "max abs error", "Decode GB/s", "Decode time", "HBM copy bandwidth",
                  "Split-K partition size", "Ragged batch: 3 sequences"):
        assert title in text, title
    assert "| 4096 | 4 | 900.00 | 900.00 |" in text
    assert "| 1 | 32768 | 256 | 128 | 1024 | 0.0500 | 3000.0 | 0.400 |" in text
    assert "| 128 | True | 4096 | 4 | 0.550 |" in text
