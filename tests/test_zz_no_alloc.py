"""attn_paged_decode_noalloc: paged decode for callers that cannot allocate.

Some callers cannot allocate device memory where they run decode (a plugin in a
serving framework that owns the whole device-memory pool, or a latency-critical
loop where cudaMalloc / cudaFree may synchronise the device). This entry point
takes no workspace: its split-K scratch is a fixed 32 MiB array inside the
library. Called through the C ABI, it must give the same output as the
workspace-taking attn_paged_decode, on two calls in a row (the second call
reuses the array the first one left behind), and must refuse problems whose
scratch would not fit.

This file sorts last so that a run stopping at its first failure has run every
other test before it.
"""
import ctypes

import pytest
import torch

import attnkernels as ak
from attnkernels import _native
from conftest import max_err, mean_err
from oracle.reference import make_paged_cache

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-3, 1e-4  # the decode tests' tolerance on fp16 outputs
SCRATCH_BYTES = 32 << 20


def noalloc(q, kc, vc, tables, lens, max_ctx, partition):
    """Call attn_paged_decode_noalloc through the C ABI; returns (rc, out)."""
    lib = _native.library()
    out = torch.empty_like(q)
    B, H, D = q.shape
    with torch.cuda.device(q.device):
        rc = lib.attn_paged_decode_noalloc(
            ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()),
            ctypes.c_void_p(vc.data_ptr()), ctypes.c_void_p(tables.data_ptr()),
            ctypes.c_void_p(lens.data_ptr()), ctypes.c_void_p(out.data_ptr()), B, H, kc.shape[1],
            D, kc.shape[2], kc.shape[0], tables.shape[1], max_ctx, 1.0 / D ** 0.5, partition,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


def case(ctx, hq, hkv, d, seed):
    torch.manual_seed(seed)
    kc, vc, tables, lens = make_paged_cache(ctx, hkv, d, device="cuda")
    q = torch.randn(len(ctx), hq, d, device="cuda").half()
    return q, kc, vc, tables, lens


def test_matches_workspace_entry_on_two_calls_in_a_row():
    first = case([3000, 17, 1024, 700, 4100], 32, 8, 128, seed=11)
    second = case([256, 5000, 1], 8, 8, 64, seed=12)
    for (q, kc, vc, tables, lens), part in ((first, 512), (second, 256)):
        max_ctx = int(lens.max())
        want = ak.paged_decode(q, kc, vc, tables, lens, max_ctx, partition_size=part)
        rc, got = noalloc(q, kc, vc, tables, lens, max_ctx, part)
        assert rc == 0, _native.library().attn_last_error()
        torch.cuda.synchronize()
        assert max_err(got, want) < MAX_ABS and mean_err(got, want) < MEAN_ABS
    ak.check_device_status()


def test_rejects_problems_beyond_the_fixed_scratch():
    q, kc, vc, tables, lens = case([300], 32, 32, 128, seed=13)
    lib = _native.library()
    # 4096 sequences x 32 heads x ceil(1M / 256) splits of partials: far above 32 MiB.
    big = 1 << 20
    need = lib.attn_paged_decode_workspace_bytes(4096, 32, 128, big, 256)
    assert need > SCRATCH_BYTES
    out = torch.empty(4096, 32, 128, device="cuda", dtype=torch.float16)
    rc = lib.attn_paged_decode_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()),
        ctypes.c_void_p(vc.data_ptr()), ctypes.c_void_p(tables.data_ptr()),
        ctypes.c_void_p(lens.data_ptr()), ctypes.c_void_p(out.data_ptr()), 4096, 32, 32, 128,
        16, kc.shape[0], big // 16, big, 0.1, 256, None)
    assert rc == 4
    assert "32 MiB" in lib.attn_last_error().decode() or str(SCRATCH_BYTES) in \
        lib.attn_last_error().decode()
