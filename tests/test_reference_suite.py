"""The reference project's own GPU test files, unmodified, against this package.

The reference's tests/test_prefill.py and tests/test_decode.py (with its
conftest.py) import `attnkernels` and the fp32 oracle `attnkernels.reference`
(tests/test_prefill.py:10-12, tests/test_decode.py:5-7). This package is the
`attnkernels` they get. It ships no `attnkernels.reference`: the oracle is test
infrastructure and lives in oracle/reference.py. So the files run in a child
pytest process whose plugin (written below, in that process only) registers
oracle/reference.py as `attnkernels.reference`, with the reference's defaults
(make_paged_cache builds its cache on "cuda"). Nothing in the package imports
the oracle.

The reference's test directory is not part of this repository. Point the
ATTN_REFERENCE_TESTS environment variable at a copy of it (the directory that
holds conftest.py, test_prefill.py and test_decode.py); without it the test is
skipped. The files are copied to a temporary directory before the run, so the
reference's conftest (which puts its parent directory first on sys.path) finds
no other `attnkernels` than this one.
"""
import os
import shutil
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "flash-attention-from-scratch_b200"
FILES = ("conftest.py", "test_prefill.py", "test_decode.py")

SHIM = textwrap.dedent('''
    """pytest plugin: `attnkernels` is the B200 package, `attnkernels.reference`
    the restated oracle with the reference's default device."""
    import functools
    import sys
    import types

    sys.path[:0] = [{root!r}, {pkg!r}]

    import attnkernels
    from oracle import reference as _oracle

    ref = types.ModuleType("attnkernels.reference")
    ref.__doc__ = "oracle/reference.py under the reference's module name"
    for _name in ("attention_fp32", "gather_kv", "paged_decode_fp32", "paged_decode_torch"):
        setattr(ref, _name, getattr(_oracle, _name))
    ref.make_paged_cache = functools.partial(_oracle.make_paged_cache, device="cuda")
    sys.modules["attnkernels.reference"] = ref
    attnkernels.reference = ref
''')


def reference_tests():
    path = os.environ.get("ATTN_REFERENCE_TESTS")
    if not path:
        return None
    p = Path(path)
    return p if all((p / f).is_file() for f in FILES) else None


def test_reference_suite_passes_unmodified(tmp_path):
    src = reference_tests()
    if src is None:
        pytest.skip("ATTN_REFERENCE_TESTS does not name the reference's tests/ directory")
    tests = tmp_path / "ref" / "tests"
    tests.mkdir(parents=True)
    for f in FILES:
        shutil.copyfile(src / f, tests / f)
    (tmp_path / "_attn_ref_shim.py").write_text(SHIM.format(root=str(ROOT), pkg=str(PKG)))
    env = dict(os.environ, PYTHONPATH=str(tmp_path))
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-p", "_attn_ref_shim", "-p", "no:cacheprovider",
         str(tests)],
        cwd=tmp_path / "ref", env=env, capture_output=True, text=True, timeout=1800)
    tail = "\n".join((r.stdout + r.stderr).splitlines()[-30:])
    print(tail)
    assert r.returncode == 0, tail
    assert " passed" in r.stdout and " failed" not in r.stdout, tail
