"""Generate the golden fixtures that pin the CPU oracle to the reference project.

Runs the reference project's own oracle module, attnkernels/reference.py of
sonhoang/flash-attention-from-scratch, on CPU and saves its inputs and outputs:

    python tests/golden/make_golden.py <path to the reference checkout>

Only this script reads the reference; the fixtures it writes (small .npz files
next to it) are what the tests use. Inputs are fp16 draws from fixed seeds;
outputs are the reference's fp32 results.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference(root: Path):
    path = root / "attnkernels" / "reference.py"
    spec = importlib.util.spec_from_file_location("upstream_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def qkv(seed, b, h, n, d, q_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(b, h, n, d, generator=g) * q_scale).half()
    k = torch.randn(b, h, n, d, generator=g).half()
    v = torch.randn(b, h, n, d, generator=g).half()
    return q, k, v


def prefill_cases(ref):
    cases = {
        # B=1, H=4, N=256, d=64, non-causal, seed 0.
        "prefill_config1": dict(seed=0, shape=(1, 4, 256, 64), causal=False, q_scale=1.0),
        "prefill_causal_d64_n17": dict(seed=1, shape=(2, 3, 17, 64), causal=True, q_scale=1.0),
        "prefill_causal_d128_n129": dict(seed=2, shape=(1, 2, 129, 128), causal=True, q_scale=1.0),
        "prefill_large_logits": dict(seed=3, shape=(1, 1, 100, 64), causal=True, q_scale=6.0),
    }
    for name, c in cases.items():
        q, k, v = qkv(c["seed"], *c["shape"], q_scale=c["q_scale"])
        out = ref.attention_fp32(q, k, v, c["causal"])
        np.savez_compressed(HERE / f"{name}.npz", q=q.numpy(), k=k.numpy(), v=v.numpy(),
                            out=out.numpy(), causal=np.array(c["causal"]))


def decode_cases(ref):
    cases = {
        # Ragged GQA batch, d=128, block 16 (the reference test's RAGGED lengths, shortened).
        "decode_gqa_d128": dict(seed=10, ctx=[1, 17, 100, 257, 33], hkv=2, hq=8, d=128, bs=16),
        "decode_mha_d64_bs8": dict(seed=11, ctx=[150, 5, 64], hkv=2, hq=2, d=64, bs=8),
    }
    for name, c in cases.items():
        torch.manual_seed(c["seed"])
        g = torch.Generator().manual_seed(c["seed"])
        kc, vc, tables, lens = ref.make_paged_cache(c["ctx"], c["hkv"], c["d"], block_size=c["bs"],
                                                    device="cpu", extra_blocks=3, generator=g)
        q = torch.randn(len(c["ctx"]), c["hq"], c["d"]).half()
        out = ref.paged_decode_fp32(q, kc, vc, tables, lens)
        nblk = -(-max(c["ctx"]) // c["bs"])
        gathered = ref.gather_kv(kc, tables[:1], nblk)  # first sequence only (size)
        sdpa = ref.paged_decode_torch(q.float(), kc.float(), vc.float(), tables, nblk,
                                      context_lens=lens)
        np.savez_compressed(HERE / f"{name}.npz", q=q.numpy(), k_cache=kc.numpy(),
                            v_cache=vc.numpy(), block_tables=tables.numpy(),
                            context_lens=lens.numpy(), out=out.numpy(),
                            gathered_k=gathered.numpy(), sdpa_out=sdpa.numpy(),
                            seed=np.array(c["seed"]), block_size=np.array(c["bs"]),
                            extra_blocks=np.array(3))


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <path to the reference checkout>")
    root = Path(sys.argv[1])
    ref = load_reference(root)
    torch.set_num_threads(1)  # deterministic reduction order
    prefill_cases(ref)
    decode_cases(ref)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
