"""Paged decode on the GPU vs the per-sequence fp32 CPU oracle.

The reference's tests/test_decode.py cases (its ATOL) come first; then the
golden fixtures, BASELINE config 4 at full size and config 5's context length
(oracle on sampled sequences / heads), this build's tolerance, a 4-D q, the
partials + merge path that
context parallelism uses (ranks emulated on one GPU), and block ids outside the
cache being reported instead of read.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import attnkernels as ak
from attnkernels.parallel import context_range
from conftest import max_err, mean_err
from oracle.reference import make_paged_cache, paged_decode_fp32, paged_decode_torch

pytestmark = pytest.mark.gpu

ATOL = 3e-3  # the reference's decode tolerance (tests/test_decode.py:9)
MAX_ABS, MEAN_ABS = 2e-3, 1e-4
GOLDEN = Path(__file__).resolve().parent / "golden"


def cache(ctx, hkv, d, bs=16, extra=5, seed=None):
    g = None if seed is None else torch.Generator().manual_seed(seed)
    return make_paged_cache(ctx, hkv, d, block_size=bs, extra_blocks=extra, device="cuda",
                            generator=g)


def oracle(q, kc, vc, tables, lens):
    return paged_decode_fp32(q.cpu(), kc.cpu(), vc.cpu(), tables.cpu(), lens.cpu())


def run(ctx, hq, hkv, d, bs=16, partition=None):
    k_cache, v_cache, tables, lens = cache(ctx, hkv, d, bs)
    q = torch.randn(len(ctx), hq, d, device="cuda").half()
    out = ak.paged_decode(q, k_cache, v_cache, tables, lens, max(ctx), partition_size=partition)
    ref = oracle(q, k_cache, v_cache, tables, lens)
    assert out.shape == q.shape and out.dtype == torch.float16
    assert torch.isfinite(out).all()
    return max_err(out, ref), mean_err(out, ref)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("heads", [(8, 8), (8, 4), (32, 8), (16, 2)])
@pytest.mark.parametrize("ctx", [[1], [100], [256], [1000, 1000], [5000]])
def test_uniform(d, heads, ctx):
    mx, mean = run(ctx, heads[0], heads[1], d)
    assert mx < ATOL
    assert mx < MAX_ABS and mean < MEAN_ABS


RAGGED = [1, 17, 255, 256, 257, 999, 4097, 33]


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("partition", [None, 256, 1024, 1 << 20])
def test_ragged_batch(d, partition):
    """Different context lengths in one batch; partition 1<<20 means no split-K."""
    mx, mean = run(RAGGED, 32, 8, d, partition=partition)
    assert mx < ATOL
    assert mx < MAX_ABS and mean < MEAN_ABS


@pytest.mark.parametrize("bs", [8, 16, 32])
def test_block_sizes(bs):
    mx, mean = run([300, 2000, 17], 8, 2, 128, bs=bs)
    assert mx < ATOL
    assert mx < MAX_ABS and mean < MEAN_ABS


@pytest.mark.parametrize("bs", [1, 4, 24, 64])
def test_odd_block_sizes(bs):
    """Block sizes that do not divide the 16-token stage (pages split across stages)."""
    mx, mean = run([300, 50, 17], 4, 4, 64, bs=bs)
    assert mx < MAX_ABS and mean < MEAN_ABS


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("heads", [(8, 4), (16, 2)])
@pytest.mark.parametrize("bs", [1, 3, 4, 24, 64])
def test_grouped_odd_block_sizes(d, heads, bs):
    """G = 2 and 8 (the tensor-core consumer) with pages that split 4-token copy groups
    and 16-token stages, and partial last stages (17, 50, 300 tokens)."""
    mx, mean = run([300, 50, 17, 1], heads[0], heads[1], d, bs=bs)
    assert mx < MAX_ABS and mean < MEAN_ABS


@pytest.mark.parametrize("heads", [(8, 2), (8, 8)])
def test_partial_stages_never_read_other_units(heads):
    """Thousands of short units per launch, so every warp's ring is reused across
    units: sequences whose V holds +inf (their own outputs are not finite) next to
    sequences whose last stage is partial. The rows of a partial stage past its last
    token must not hold another unit's V, or P = 0 times inf would turn into NaN."""
    n = 2000
    ctx = [48 if b % 2 == 0 else 21 for b in range(n)]
    k_cache, v_cache, tables, lens = cache(ctx, heads[1], 64, seed=11)
    for b in range(0, n, 2):
        v_cache[tables[b, 0], :, 5, :] = float("inf")
    q = torch.randn(n, heads[0], 64, device="cuda").half()
    out = ak.paged_decode(q, k_cache, v_cache, tables, lens, 48)
    clean = torch.arange(1, n, 2, device="cuda")
    assert torch.isfinite(out[clean]).all()
    ref = oracle(q[clean], k_cache, v_cache, tables[clean], lens[clean])
    assert max_err(out[clean], ref) < MAX_ABS and mean_err(out[clean], ref) < MEAN_ABS


def test_long_context_split():
    mx, mean = run([32768], 32, 8, 128)
    assert mx < ATOL
    assert mx < MAX_ABS and mean < MEAN_ABS


def test_split_choice_does_not_change_result():
    k_cache, v_cache, tables, lens = cache([6000, 3000], 4, 128, extra=0)
    q = torch.randn(2, 16, 128, device="cuda").half()
    outs = [ak.paged_decode(q, k_cache, v_cache, tables, lens, 6000, partition_size=p)
            for p in (256, 768, 2048, 6144)]
    for o in outs[1:]:
        assert max_err(o, outs[0]) < 2e-3


def test_torch_baseline_matches():
    """The gather + SDPA baseline used in the benchmark is itself correct."""
    ctx = [512, 512, 300]
    k_cache, v_cache, tables, lens = cache(ctx, 8, 128, extra=0)
    q = torch.randn(3, 32, 128, device="cuda").half()
    out = paged_decode_torch(q, k_cache, v_cache, tables, 32, context_lens=lens)
    assert max_err(out, oracle(q, k_cache, v_cache, tables, lens)) < ATOL
    ours = ak.paged_decode(q, k_cache, v_cache, tables, lens, 512)
    ref = oracle(q, k_cache, v_cache, tables, lens)
    assert max_err(ours, ref) < MAX_ABS and mean_err(ours, ref) < MEAN_ABS


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("decode_*.npz")), ids=lambda p: p.stem)
@pytest.mark.parametrize("partition", [None, 256])
def test_golden_fixtures(path, partition):
    with np.load(path) as z:
        q = torch.from_numpy(z["q"]).cuda()
        kc, vc = torch.from_numpy(z["k_cache"]).cuda(), torch.from_numpy(z["v_cache"]).cuda()
        bt = torch.from_numpy(z["block_tables"]).cuda()
        lens = torch.from_numpy(z["context_lens"]).cuda()
        want = torch.from_numpy(z["out"])
    out = ak.paged_decode(q, kc, vc, bt, lens, int(lens.max()), partition_size=partition)
    assert max_err(out, want) < MAX_ABS and mean_err(out, want) < MEAN_ABS


def test_four_dim_query():
    """BASELINE config 4 writes q as [B, H, 1, D]."""
    k_cache, v_cache, tables, lens = cache([700, 90], 4, 128)
    q = torch.randn(2, 4, 1, 128, device="cuda").half()
    out = ak.paged_decode(q, k_cache, v_cache, tables, lens, 700)
    assert out.shape == q.shape
    ref = oracle(q[:, :, 0], k_cache, v_cache, tables, lens)
    assert max_err(out[:, :, 0], ref) < MAX_ABS and mean_err(out[:, :, 0], ref) < MEAN_ABS


def test_zero_length_sequence_gives_zero_row():
    k_cache, v_cache, tables, lens = cache([300, 5], 2, 64)
    lens[1] = 0
    q = torch.randn(2, 2, 64, device="cuda").half()
    for part in (256, 1024):
        out = ak.paged_decode(q, k_cache, v_cache, tables, lens, 300, partition_size=part)
        assert torch.equal(out[1], torch.zeros_like(out[1]))
        ref = oracle(q[:1], k_cache, v_cache, tables[:1], lens[:1])
        assert max_err(out[:1], ref) < MAX_ABS and mean_err(out[:1], ref) < MEAN_ABS


def test_config4_full_size():
    """B=64, H=Hkv=32, d=128, bs=16, ctx ~ U[512, 8192], partition 512."""
    g = torch.Generator().manual_seed(4)
    ctx = torch.randint(512, 8193, (64,), generator=g).tolist()
    k_cache, v_cache, tables, lens = cache(ctx, 32, 128, extra=0, seed=4)
    q = torch.randn(64, 32, 1, 128, device="cuda").half()
    out = ak.paged_decode(q, k_cache, v_cache, tables, lens, max(ctx), partition_size=512)
    assert torch.isfinite(out).all()
    kc_cpu, vc_cpu = k_cache.cpu(), v_cache.cpu()
    for b in (0, 17, 63):
        ref = oracle(q[b:b + 1, :, 0], kc_cpu, vc_cpu, tables[b:b + 1], lens[b:b + 1])
        assert max_err(out[b:b + 1, :, 0], ref) < MAX_ABS
        assert mean_err(out[b:b + 1, :, 0], ref) < MEAN_ABS
    ak.check_device_status()


def test_config5_context_length():
    """BASELINE config 5's 131072-token context (one sequence), oracle on two heads."""
    k_cache, v_cache, tables, lens = cache([131072], 32, 128, extra=0, seed=5)
    q = torch.randn(1, 32, 128, device="cuda").half()
    out = ak.paged_decode(q, k_cache, v_cache, tables, lens, 131072)
    for h in (0, 31):
        kc = k_cache[:, h:h + 1].cpu()
        vc = v_cache[:, h:h + 1].cpu()
        ref = paged_decode_fp32(q[:, h:h + 1].cpu(), kc, vc, tables.cpu(), lens.cpu())
        assert max_err(out[:, h:h + 1], ref) < MAX_ABS
        assert mean_err(out[:, h:h + 1], ref) < MEAN_ABS


def local_view(tables, lens, bs, world, rank):
    rows, sub = [], []
    for b, c in enumerate(lens.tolist()):
        t0, t1 = context_range(c, bs, world, rank)
        b0, nb = t0 // bs, -(-(t1 - t0) // bs)
        row = torch.zeros(tables.shape[1], dtype=torch.int32, device=tables.device)
        row[:nb] = tables[b, b0:b0 + nb]
        rows.append(row)
        sub.append(t1 - t0)
    return torch.stack(rows), torch.tensor(sub, dtype=torch.int32, device=tables.device)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_context_parallel_partials_and_merge(world):
    """Ranks emulated on one GPU: partials of each context range, merged by the
    merge kernel, equal the single-GPU decode (and the oracle)."""
    ctx = [3000, 17, 1024, 200]
    k_cache, v_cache, tables, lens = cache(ctx, 4, 128)
    q = torch.randn(4, 8, 128, device="cuda").half()
    rows = 4 * 8
    stride = -(-(rows * 130) // 4) * 4
    gathered = torch.empty(world, stride, device="cuda")
    for r in range(world):
        bt, ln = local_view(tables, lens, 16, world, r)
        buf = gathered[r]
        ak.paged_decode_partials(q, k_cache, v_cache, bt, ln, max(1, int(ln.max())),
                                 partition_size=512,
                                 out=(buf[: rows * 128].view(4, 8, 128),
                                      buf[rows * 128: rows * 129].view(4, 8),
                                      buf[rows * 129: rows * 130].view(4, 8)))
    out = ak.merge_partials(gathered[:, : rows * 128].view(world, 4, 8, 128),
                            gathered[:, rows * 128: rows * 129].view(world, 4, 8),
                            gathered[:, rows * 129: rows * 130].view(world, 4, 8))
    full = ak.paged_decode(q, k_cache, v_cache, tables, lens, 3000)
    ref = oracle(q, k_cache, v_cache, tables, lens)
    assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < MEAN_ABS
    assert max_err(out, full) < 2e-3


def test_partials_of_empty_rows():
    k_cache, v_cache, tables, lens = cache([40, 40], 2, 64)
    lens[0] = 0
    q = torch.randn(2, 2, 64, device="cuda").half()
    o, m, l = ak.paged_decode_partials(q, k_cache, v_cache, tables, lens, 40)
    assert torch.equal(o[0], torch.zeros_like(o[0]))
    assert torch.isinf(m[0]).all() and (m[0] < 0).all()
    assert torch.equal(l[0], torch.zeros_like(l[0]))
    assert (l[1] >= 1).all()


def test_out_of_range_block_id_is_reported():
    k_cache, v_cache, tables, lens = cache([64], 2, 64, extra=0)
    tables[0, 1] = k_cache.shape[0] + 7  # outside the cache
    q = torch.randn(1, 2, 64, device="cuda").half()
    ak.check_device_status()
    ak.paged_decode(q, k_cache, v_cache, tables, lens, 64)
    code, _ = ak.device_status()
    assert code == 2
    ak.check_device_status()  # cleared


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("heads", [(8, 4), (32, 8), (16, 2)])
@pytest.mark.parametrize("partition", [None, 256])
def test_grouped_heads_at_tolerance(d, heads, partition):
    """Query heads sharing a kv head (G = 2, 4, 8), ragged contexts, this build's tolerance."""
    mx, mean = run([3000, 17, 1100, 256, 5], heads[0], heads[1], d, partition=partition)
    assert mx < MAX_ABS and mean < MEAN_ABS


@pytest.mark.parametrize("heads", [(8, 8), (32, 8)])
def test_many_parts_per_row(heads):
    """36 splits of a 9000-token context next to rows of 2 and 1 splits: the merge
    with eight warps per row (32 parts and more), in both output forms."""
    ctx = [9000, 300, 200]
    k_cache, v_cache, tables, lens = cache(ctx, heads[1], 128)
    q = torch.randn(len(ctx), heads[0], 128, device="cuda").half()
    ref = oracle(q, k_cache, v_cache, tables, lens)
    out = ak.paged_decode(q, k_cache, v_cache, tables, lens, 9000, partition_size=256)
    assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < MEAN_ABS
    o, m, l = ak.paged_decode_partials(q, k_cache, v_cache, tables, lens, 9000,
                                       partition_size=256)
    assert max_err(o, ref) < MAX_ABS and mean_err(o, ref) < MEAN_ABS
    assert torch.isfinite(m).all() and (l >= 1).all()


def test_batch_beyond_one_launch():
    """More sequences than one launch takes (2048): the batch runs as several launches."""
    g = torch.Generator().manual_seed(5)
    ctx = torch.randint(1, 40, (2100,), generator=g).tolist()
    k_cache, v_cache, tables, lens = cache(ctx, 2, 64, seed=5)
    q = torch.randn(len(ctx), 8, 64, device="cuda").half()
    out = ak.paged_decode(q, k_cache, v_cache, tables, lens, max(ctx))
    ref = oracle(q, k_cache, v_cache, tables, lens)
    assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < MEAN_ABS
