"""Build the sm_100a attention library: csrc/*.cu -> attnkernels/libattn_b200.so.

The library is plain CUDA C++ behind the C ABI in include/attn_b200.h; it does
not link against torch. nvcc compiles each translation unit for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`) with line info for the profiler,
and links the CUDA runtime statically.

    python flash-attention-from-scratch_b200/build.py          # incremental
    python flash-attention-from-scratch_b200/build.py --force  # rebuild all

Environment: NVCC (default: nvcc on PATH, else /usr/local/cuda/bin/nvcc),
ATTN_PTXAS_VERBOSE=1 prints ptxas register/shared-memory reports (as the
reference's loader does, attnkernels/__init__.py:41-42).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "attnkernels" / "libattn_b200.so"
SOURCES = ["api.cu", "prefill_tc.cu", "prefill_simt.cu", "decode.cu", "exchange.cu"]
HEADERS = ["common.cuh", "launch.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    env = os.environ.get("NVCC")
    if env:
        return env
    found = shutil.which("nvcc")
    return found or "/usr/local/cuda/bin/nvcc"


def _flags() -> list[str]:
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                    f"-I{ROOT / 'include'}", f"-I{CSRC}"]
    if os.environ.get("ATTN_PTXAS_VERBOSE") == "1":
        flags.append("-Xptxas=-v")
    return flags


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "attn_b200.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def _compile(src: str, force: bool) -> Path:
    s = CSRC / src
    o = BUILD / (s.stem + ".o")
    if force or _stale(o, s):
        cmd = [nvcc(), *_flags(), "-c", str(s), "-o", str(o)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return o


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build(force=args.force, verbose=True)
