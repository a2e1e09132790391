"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on CPU.

Mirrors the reference's tests/conftest.py: the native library is loaded once
per session (before the first GPU test), every test starts from
torch.manual_seed(0), and errors are measured as max-abs (plus mean-abs, the
second half of the tolerance this build is held to).
"""
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "flash-attention-from-scratch_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

HAS_CUDA = torch.cuda.is_available()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    if HAS_CUDA:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def ext():
    import attnkernels

    return attnkernels.load_extension()


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)


def max_err(out, ref):
    return (out.float().cpu() - ref.float().cpu()).abs().max().item()


def mean_err(out, ref):
    return (out.float().cpu() - ref.float().cpu()).abs().mean().item()
