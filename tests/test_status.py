"""Failure detection without a GPU fault: every mbarrier wait in the kernels is
bounded. A kernel that waits on a barrier nothing arrives on must give up after
its limit, report ATTN_DEVICE_WAIT_TIMEOUT in the device status word, and leave
the CUDA context usable."""
import time

import pytest
import torch

import attnkernels as ak

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_survives(ext):
    ak.check_device_status()
    t0 = time.perf_counter()
    ext.selftest_wait_timeout(50_000_000)  # 50 ms limit
    code, site = ak.device_status()
    elapsed = time.perf_counter() - t0
    assert code == 1 and site == 301
    assert elapsed < 5.0
    # The context still runs kernels correctly afterwards.
    q = torch.randn(1, 2, 300, 64, device="cuda").half()
    out = ak.flash_attention(q, q, q, causal=True)
    assert torch.isfinite(out).all()
    assert ak.device_status() == (0, 0)


def test_status_is_clean_after_normal_work():
    q = torch.randn(2, 4, 513, 128, device="cuda").half()
    ak.flash_attention(q, q, q, causal=False)
    ak.flash_attention(q, q, q, causal=True, variant="simt")
    ak.check_device_status()
