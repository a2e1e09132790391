"""Prefill attention on the GPU vs the fp32 CPU oracle.

The first group restates the reference's tests/test_prefill.py cases (all four
variants); each case asserts the reference's own ATOL and this build's
tolerance, max-abs 2e-3 AND mean-abs 1e-4 on fp16 outputs. The second group
holds the kernels to that tolerance on the golden fixtures and on the BASELINE
shapes at full size, checked on sampled heads and rows (slicing the oracle by
head or by query rows is exact).

One case has a wider mean-abs bound, for a stated reason: with scores of std 6
(test_large_logits, the large-logit fixture) the outputs are close to single
rows of v, |o| up to ~4, and rounding the exact fp32 answer to fp16 alone
already leaves a mean-abs error of 1.02e-4 (1.04e-4 at d 64) on those inputs;
there the bound is 2e-3 max-abs and 2e-4 mean-abs.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import attnkernels as ak
from conftest import max_err, mean_err
from oracle.reference import attention_fp32

pytestmark = pytest.mark.gpu

ATOL = 5e-3          # the reference's prefill tolerance (tests/test_prefill.py:14)
MAX_ABS = 2e-3       # this build's tolerance, max-abs ...
MEAN_ABS = 1e-4      # ... and mean-abs, on fp16 outputs
LARGE_LOGIT_MEAN_ABS = 2e-4  # fp16 rounding of the exact answer alone is 1.0e-4 there
GOLDEN = Path(__file__).resolve().parent / "golden"

VARIANTS = {
    "naive": lambda q, k, v, c: ak.naive_attention(q, k, v, causal=c),
    "simt": lambda q, k, v, c: ak.flash_attention(q, k, v, causal=c, variant="simt"),
    "wmma32": lambda q, k, v, c: ak.flash_attention(q, k, v, causal=c, variant="wmma", block_n=32),
    "wmma64": lambda q, k, v, c: ak.flash_attention(q, k, v, causal=c, variant="wmma", block_n=64),
}


def rand_qkv(b, h, n, d, q_scale=1.0):
    q = (torch.randn(b, h, n, d, device="cuda") * q_scale).half()
    k = torch.randn(b, h, n, d, device="cuda").half()
    v = torch.randn(b, h, n, d, device="cuda").half()
    return q, k, v


def oracle(q, k, v, causal):
    return attention_fp32(q.cpu(), k.cpu(), v.cpu(), causal)


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("n", [1, 17, 64, 100, 129, 256, 333])
def test_matches_fp32(variant, causal, d, n):
    q, k, v = rand_qkv(2, 3, n, d)
    out = VARIANTS[variant](q, k, v, causal)
    ref = oracle(q, k, v, causal)
    assert out.shape == q.shape and out.dtype == torch.float16
    assert torch.isfinite(out).all()
    assert max_err(out, ref) < ATOL
    assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < MEAN_ABS


@pytest.mark.parametrize("variant", ["simt", "wmma32", "wmma64"])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d", [64, 128])
def test_long_sequence(variant, causal, d):
    q, k, v = rand_qkv(1, 2, 2048 + 7, d)
    out = VARIANTS[variant](q, k, v, causal)
    ref = oracle(q, k, v, causal)
    assert max_err(out, ref) < ATOL
    assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < MEAN_ABS


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("d", [64, 128])
def test_large_logits(variant, d):
    """Scores with a std of about 6: exp would overflow without the running max."""
    q, k, v = rand_qkv(1, 2, 300, d, q_scale=6.0)
    out = VARIANTS[variant](q, k, v, True)
    assert torch.isfinite(out).all()
    ref = oracle(q, k, v, True)
    assert max_err(out, ref) < 2 * ATOL
    assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < LARGE_LOGIT_MEAN_ABS


def test_causal_first_row_is_v0():
    q, k, v = rand_qkv(1, 1, 128, 64)
    for name, fn in VARIANTS.items():
        out = fn(q, k, v, True)
        assert max_err(out[0, 0, 0], v[0, 0, 0]) < 1e-3, name


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_matches_sdpa(variant):
    q, k, v = rand_qkv(2, 4, 512, 64)
    out = VARIANTS[variant](q, k, v, True)
    sdpa = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert max_err(out, sdpa) < ATOL
    ref = oracle(q, k, v, True)
    assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < MEAN_ABS


def test_rejects_bad_input():
    q, k, v = rand_qkv(1, 1, 16, 32)
    with pytest.raises(ValueError):
        ak.flash_attention(q, k, v)
    q, k, v = rand_qkv(1, 1, 16, 64)
    with pytest.raises(ValueError):
        ak.flash_attention(q, k, v, variant="tensor")
    with pytest.raises(RuntimeError, match="block_n"):
        ak.flash_attention(q, k, v, block_n=128)


# --------------------------------------------------- this build's tolerance


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("prefill_*.npz")), ids=lambda p: p.stem)
@pytest.mark.parametrize("variant", list(VARIANTS))
def test_golden_fixtures(path, variant):
    """Inputs and outputs produced by the reference's own oracle, every variant."""
    with np.load(path) as z:
        q, k, v = (torch.from_numpy(z[n]).cuda() for n in "qkv")
        want = torch.from_numpy(z["out"])
        causal = bool(z["causal"])
    out = VARIANTS[variant](q, k, v, causal)
    mean_tol = LARGE_LOGIT_MEAN_ABS if "large_logits" in path.stem else MEAN_ABS
    assert max_err(out, want) < MAX_ABS
    assert mean_err(out, want) < mean_tol


@pytest.mark.parametrize("d,n", [(128, 4096), (64, 4096), (128, 4095)])
def test_config2_full_size(d, n):
    """BASELINE config 2 (B=4, H=16, causal) at full size; oracle on sampled heads."""
    torch.manual_seed(2)
    q, k, v = rand_qkv(4, 16, n, d)
    out = ak.flash_attention(q, k, v, causal=True)
    assert torch.isfinite(out).all()
    for b, h in [(0, 0), (1, 7), (3, 15)]:
        ref = oracle(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], v[b:b + 1, h:h + 1], True)
        o = out[b:b + 1, h:h + 1]
        assert max_err(o, ref) < MAX_ABS, (b, h)
        assert mean_err(o, ref) < MEAN_ABS, (b, h)
    ak.check_device_status()


def test_config3_long_context_rows():
    """BASELINE config 3 (B=1, H=32, N=32768, causal, inputs x0.5): first and last
    rows of sampled heads against the oracle over the full key range."""
    torch.manual_seed(3)
    n = 32768
    q = (torch.randn(1, 32, n, 128, device="cuda") * 0.5).half()
    k = (torch.randn(1, 32, n, 128, device="cuda") * 0.5).half()
    v = (torch.randn(1, 32, n, 128, device="cuda") * 0.5).half()
    out = ak.flash_attention(q, k, v, causal=True)
    assert torch.isfinite(out).all()
    for h in (0, 31):
        kh, vh = k[:, h:h + 1].cpu(), v[:, h:h + 1].cpu()
        for r0, r1 in [(0, 256), (n - 256, n), (12345, 12345 + 128)]:
            ref = attention_fp32(q[:, h:h + 1, r0:r1].cpu(), kh, vh, True, q_start=r0)
            o = out[:, h:h + 1, r0:r1]
            assert max_err(o, ref) < MAX_ABS, (h, r0)
            assert mean_err(o, ref) < MEAN_ABS, (h, r0)


@pytest.mark.parametrize("b,h,n", [(3, 100, 384), (2, 97, 1280), (1, 1, 2304)])
def test_scheduling_groups(b, h, n):
    """Many (batch, head) pairs: the CTAs run in groups of pairs with a remainder
    group first. Every pair of every group must be computed exactly once (checked
    on heads from the first group, a middle one and the last)."""
    torch.manual_seed(11)
    q, k, v = rand_qkv(b, h, n, 128)
    out = ak.flash_attention(q, k, v, causal=True)
    assert torch.isfinite(out).all()
    pairs = sorted({0, (b * h) // 2, b * h - 1})
    for x in pairs:
        bi, hi = divmod(x, h)
        ref = oracle(q[bi:bi + 1, hi:hi + 1], k[bi:bi + 1, hi:hi + 1], v[bi:bi + 1, hi:hi + 1], True)
        o = out[bi:bi + 1, hi:hi + 1]
        assert max_err(o, ref) < MAX_ABS, (bi, hi)
        assert mean_err(o, ref) < MEAN_ABS, (bi, hi)
    ak.check_device_status()


@pytest.mark.parametrize("n", [1, 127, 128, 129, 255, 256, 257, 1000])
@pytest.mark.parametrize("causal", [False, True])
def test_tile_edges(n, causal):
    """Sequence lengths around the 128-row tiles and the 2-tile CTA."""
    q, k, v = rand_qkv(1, 3, n, 128)
    out = ak.flash_attention(q, k, v, causal=causal)
    ref = oracle(q, k, v, causal)
    assert max_err(out, ref) < MAX_ABS
    assert mean_err(out, ref) < MEAN_ABS


def test_scale_argument():
    q, k, v = rand_qkv(1, 2, 200, 64)
    for scale in (0.05, 0.3, -0.1):
        out = ak.flash_attention(q, k, v, causal=True, scale=scale)
        ref = attention_fp32(q.cpu(), k.cpu(), v.cpu(), True, scale=scale)
        assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < MEAN_ABS


def test_non_contiguous_inputs_are_made_contiguous():
    q, k, v = rand_qkv(2, 64, 4, 128)
    qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))  # [2, 4, 64, 128] views
    out = ak.flash_attention(qt, kt, vt, causal=True)
    ref = oracle(qt, kt, vt, True)
    assert max_err(out, ref) < MAX_ABS and mean_err(out, ref) < MEAN_ABS


def test_deterministic():
    q, k, v = rand_qkv(2, 4, 700, 128)
    a = ak.flash_attention(q, k, v, causal=True)
    b = ak.flash_attention(q, k, v, causal=True)
    assert torch.equal(a, b)


def test_linear_in_v():
    """Size-independent property: O(q, k, a v1 + b v2) = a O(v1) + b O(v2)."""
    q, k, v1 = rand_qkv(1, 4, 2048, 128)
    v2 = torch.randn_like(v1, dtype=torch.float32).half()
    mix = (0.5 * v1.float() + 0.25 * v2.float()).half()
    o1 = ak.flash_attention(q, k, v1, causal=True).float()
    o2 = ak.flash_attention(q, k, v2, causal=True).float()
    om = ak.flash_attention(q, k, mix, causal=True).float()
    assert (om - (0.5 * o1 + 0.25 * o2)).abs().max().item() < 4e-3
