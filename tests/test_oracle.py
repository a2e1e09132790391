"""The CPU oracle against golden fixtures produced by the reference itself.

tests/golden/*.npz were written by tests/golden/make_golden.py, which runs the
reference project's attnkernels/reference.py. These tests pin the restatement in
oracle/reference.py to it, so the GPU parity tests can trust the oracle.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reference as ref

GOLDEN = Path(__file__).resolve().parent / "golden"
PREFILL = sorted(GOLDEN.glob("prefill_*.npz"))
DECODE = sorted(GOLDEN.glob("decode_*.npz"))


def load(path):
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def test_fixtures_present():
    assert len(PREFILL) >= 4 and len(DECODE) >= 2


@pytest.mark.parametrize("path", PREFILL, ids=lambda p: p.stem)
def test_attention_matches_reference(path):
    z = load(path)
    q, k, v = (torch.from_numpy(z[n]) for n in "qkv")
    out = ref.attention_fp32(q, k, v, bool(z["causal"]))
    # Same fp32 arithmetic up to summation order inside the BLAS.
    np.testing.assert_allclose(out.numpy(), z["out"], rtol=0, atol=2e-6)


@pytest.mark.parametrize("path", PREFILL, ids=lambda p: p.stem)
def test_attention_row_blocks_are_exact(path):
    z = load(path)
    q, k, v = (torch.from_numpy(z[n]) for n in "qkv")
    a = ref.attention_fp32(q, k, v, bool(z["causal"]), row_block=7)
    b = ref.attention_fp32(q, k, v, bool(z["causal"]), row_block=1 << 20)
    np.testing.assert_allclose(a.numpy(), b.numpy(), rtol=0, atol=4e-6)


@pytest.mark.parametrize("path", DECODE, ids=lambda p: p.stem)
def test_paged_decode_matches_reference(path):
    z = load(path)
    q = torch.from_numpy(z["q"])
    kc, vc = torch.from_numpy(z["k_cache"]), torch.from_numpy(z["v_cache"])
    bt, lens = torch.from_numpy(z["block_tables"]), torch.from_numpy(z["context_lens"])
    out = ref.paged_decode_fp32(q, kc, vc, bt, lens)
    np.testing.assert_allclose(out.numpy(), z["out"], rtol=0, atol=2e-6)


@pytest.mark.parametrize("path", DECODE, ids=lambda p: p.stem)
def test_gather_and_sdpa_baseline_match_reference(path):
    z = load(path)
    kc, vc = torch.from_numpy(z["k_cache"]), torch.from_numpy(z["v_cache"])
    bt, lens = torch.from_numpy(z["block_tables"]), torch.from_numpy(z["context_lens"])
    bs = int(z["block_size"])
    nblk = -(-int(lens.max()) // bs)
    g = ref.gather_kv(kc, bt[:1], nblk)
    assert np.array_equal(g.numpy(), z["gathered_k"])
    q = torch.from_numpy(z["q"])
    sdpa = ref.paged_decode_torch(q.float(), kc.float(), vc.float(), bt, nblk, context_lens=lens)
    np.testing.assert_allclose(sdpa.numpy(), z["sdpa_out"], rtol=0, atol=2e-6)


@pytest.mark.parametrize("path", DECODE, ids=lambda p: p.stem)
def test_make_paged_cache_reproduces_reference(path):
    """Same seed, same RNG calls: identical block tables and caches."""
    z = load(path)
    seed, bs = int(z["seed"]), int(z["block_size"])
    lens = z["context_lens"].tolist()
    torch.manual_seed(seed)
    g = torch.Generator().manual_seed(seed)
    kc, vc, bt, ctx = ref.make_paged_cache(lens, z["k_cache"].shape[1], z["k_cache"].shape[3],
                                           block_size=bs, device="cpu",
                                           extra_blocks=int(z["extra_blocks"]), generator=g)
    assert np.array_equal(bt.numpy(), z["block_tables"])
    assert np.array_equal(kc.numpy(), z["k_cache"])
    assert np.array_equal(vc.numpy(), z["v_cache"])
    assert np.array_equal(ctx.numpy(), z["context_lens"])


@pytest.mark.parametrize("path", DECODE, ids=lambda p: p.stem)
@pytest.mark.parametrize("parts", [1, 2, 3])
def test_partials_merge_equals_full(path, parts):
    """Splitting each context into block-aligned ranges and merging is exact."""
    z = load(path)
    q = torch.from_numpy(z["q"])
    kc, vc = torch.from_numpy(z["k_cache"]), torch.from_numpy(z["v_cache"])
    bt, lens = torch.from_numpy(z["block_tables"]), torch.from_numpy(z["context_lens"])
    bs = int(z["block_size"])
    os_, ms, ls = [], [], []
    for r in range(parts):
        tabs, sub = [], []
        for b, c in enumerate(lens.tolist()):
            nb = -(-c // bs)
            b0, b1 = nb * r // parts, nb * (r + 1) // parts
            t0, t1 = min(c, b0 * bs), min(c, b1 * bs)
            row = torch.zeros(bt.shape[1], dtype=torch.int32)
            row[: b1 - b0] = bt[b, b0:b1]
            tabs.append(row)
            sub.append(t1 - t0)
        o, m, l = ref.paged_decode_partials_fp32(q, kc, vc, torch.stack(tabs),
                                                 torch.tensor(sub, dtype=torch.int32))
        os_.append(o), ms.append(m), ls.append(l)
    merged = ref.merge_partials_fp32(torch.stack(os_), torch.stack(ms), torch.stack(ls))
    np.testing.assert_allclose(merged.numpy(), z["out"], rtol=0, atol=2e-6)


def test_merge_of_empty_rows_is_zero():
    o = torch.zeros(2, 3, 4)
    m = torch.full((2, 3), float("-inf"))
    l = torch.zeros(2, 3)
    assert torch.equal(ref.merge_partials_fp32(o, m, l), torch.zeros(3, 4))


def test_causal_first_row_is_v0():
    """Known answer of the reference's tests/test_prefill.py:63-67 on the oracle."""
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 1, 128, 64, generator=g).half() for _ in range(3))
    out = ref.attention_fp32(q, k, v, causal=True)
    assert torch.allclose(out[0, 0, 0], v[0, 0, 0].float(), atol=1e-6)
