"""The C ABI library on CPU: it loads, exports every declared symbol, and rejects
bad arguments (before touching a GPU) with the reference's error conditions."""
import ctypes
import re
from pathlib import Path

import pytest

from attnkernels import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "attn_b200.h"
P = ctypes.c_void_p(4096)  # a non-null, aligned stand-in pointer: never dereferenced here


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(attn_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    return _native.library()


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ["attn_flash_fwd", "attn_flash_simt_fwd", "attn_naive_fwd", "attn_paged_decode",
              "attn_paged_decode_partials", "attn_merge_partials", "attn_device_status"]:
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert set(declared_functions()) == set(_native.SIGNATURES)


def test_abi_version(lib):
    assert lib.attn_abi_version() == _native.ABI_VERSION


def err(lib):
    return lib.attn_last_error().decode()


def test_flash_rejects_head_dim(lib):
    rc = lib.attn_flash_fwd(P, P, P, P, 1, 1, 16, 32, 0, 1.0, 64, None)
    assert rc == 2 and "head_dim must be 64 or 128" in err(lib)


def test_flash_rejects_block_n(lib):
    rc = lib.attn_flash_fwd(P, P, P, P, 1, 1, 16, 64, 0, 1.0, 48, None)
    assert rc == 2 and "block_n 32 or 64" in err(lib)


def test_flash_rejects_null_and_misaligned(lib):
    assert lib.attn_flash_fwd(None, P, P, P, 1, 1, 16, 64, 0, 1.0, 64, None) == 1
    assert lib.attn_flash_fwd(ctypes.c_void_p(4098), P, P, P, 1, 1, 16, 64, 0, 1.0, 64, None) == 1
    assert "16-byte aligned" in err(lib)


def test_empty_prefill_is_a_no_op(lib):
    assert lib.attn_flash_fwd(P, P, P, P, 0, 4, 16, 64, 1, 1.0, 32, None) == 0
    assert lib.attn_flash_simt_fwd(P, P, P, P, 2, 4, 0, 128, 1, 1.0, None) == 0


def decode(lib, **kw):
    a = dict(batch=2, hq=8, hkv=8, d=128, bs=16, nblk=10, maxb=5, max_ctx=80, partition=256,
             ws=P, ws_bytes=1 << 30)
    a.update(kw)
    return lib.attn_paged_decode(P, P, P, P, P, P, a["batch"], a["hq"], a["hkv"], a["d"], a["bs"],
                                 a["nblk"], a["maxb"], a["max_ctx"], 0.1, a["partition"], a["ws"],
                                 a["ws_bytes"], None)


def test_decode_rejects_like_the_reference(lib):
    assert decode(lib, hq=6, hkv=4) == 1 and "multiple of num_kv_heads" in err(lib)
    assert decode(lib, partition=100) == 1 and "positive multiple of 256" in err(lib)
    assert decode(lib, partition=0) == 1
    assert decode(lib, hq=24, hkv=8) == 2 and "{1,2,4,8}" in err(lib)
    assert decode(lib, d=96) == 2
    assert decode(lib, max_ctx=81) == 1 and "max_blocks_per_seq" in err(lib)
    assert decode(lib, ws=None) == 4 and "workspace" in err(lib)
    assert decode(lib, ws_bytes=16) == 4


def test_decode_workspace_size(lib):
    # counters (256 per 512 sequences) + o [B*H*S*D] fp32 + m, l [B*H*S] fp32, each
    # 256-byte aligned; S = k * ceil(ctx / part), k = 4 or 2 while B*H*S <= 8192 rows.
    align = lambda x: -(-x // 256) * 256  # noqa: E731
    for b, h, d, ctx, part, k in [(3, 4, 128, 1000, 256, 4), (64, 32, 128, 8192, 512, 1),
                                  (1, 32, 64, 32768, 256, 2), (1, 32, 128, 32768, 1024, 4)]:
        s = -(-ctx // part) * k
        want = align(-(-b // 512) * 4) + align(b * h * s * d * 4) + 2 * align(b * h * s * 4)
        assert lib.attn_paged_decode_workspace_bytes(b, h, d, ctx, part) == want, (b, h, ctx)
    assert lib.attn_naive_workspace_bytes(2, 3, 100) == 2 * 3 * 100 * 100 * 4


def test_merge_rejects(lib):
    assert lib.attn_merge_partials(P, P, P, 2, 4, 96, 512, 4, P, None) == 2
    assert lib.attn_merge_partials(P, P, P, 2, 4, 128, 513, 4, P, None) == 1
    assert lib.attn_merge_partials(P, P, P, 2, 0, 128, 512, 4, P, None) == 0


def test_selftest_rejects_unbounded(lib):
    assert lib.attn_selftest_wait_timeout(0, None) == 1
