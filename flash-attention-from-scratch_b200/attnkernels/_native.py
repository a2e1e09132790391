"""ctypes binding of libattn_b200.so, the C ABI of include/attn_b200.h.

`Extension` mirrors the call surface of the reference's compiled extension
(attnkernels/csrc/ext.cpp:12-17: naive_attention, flash_simt, flash_wmma,
paged_decode, taking and returning torch tensors), so code written against
`load_extension()` keeps working. Tensors cross the boundary as raw device
pointers plus the current CUDA stream of their device; the library never
allocates, so outputs and workspaces are allocated here from torch's caching
allocator, as the reference's C++ launchers do (paged_decode.cu:227-235).

A non-zero return code from the library raises RuntimeError with its message,
as the reference's TORCH_CHECK does.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libattn_b200.so"

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_size = ctypes.c_size_t
_u32p = ctypes.POINTER(ctypes.c_uint32)

# Every entry point of include/attn_b200.h: name -> (restype, argtypes).
SIGNATURES = {
    "attn_abi_version": (_int, []),
    "attn_last_error": (ctypes.c_char_p, []),
    "attn_flash_fwd": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _f32, _i64, _vp]),
    "attn_flash_simt_fwd": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _f32, _vp]),
    "attn_naive_workspace_bytes": (_size, [_i64, _i64, _i64]),
    "attn_naive_fwd": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _f32, _vp, _size,
                              _vp]),
    "attn_paged_decode_workspace_bytes": (_size, [_i64, _i64, _i64, _i64, _i64]),
    "attn_paged_decode": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                 _i64, _i64, _f32, _i64, _vp, _size, _vp]),
    "attn_paged_decode_partials": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                          _i64, _i64, _i64, _i64, _i64, _f32, _i64, _vp, _size,
                                          _vp]),
    "attn_merge_partials": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "attn_paged_decode_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                         _i64, _i64, _i64, _i64, _f32, _i64, _vp]),
    "attn_device_status": (_int, [_u32p, _u32p]),
    "attn_selftest_wait_timeout": (_int, [ctypes.c_uint64, _vp]),
    "attn_selftest_exp2": (_int, [_vp, _vp, _vp, _vp, _i64, _vp]),
    "attn_exchange_merge_partials": (_int, [ctypes.POINTER(_vp), ctypes.POINTER(_vp), _int, _int,
                                            ctypes.c_uint32, _i64, _i64, _i64, _vp, _vp]),
}

ABI_VERSION = 1
DEVICE_OK, DEVICE_WAIT_TIMEOUT, DEVICE_BAD_BLOCK = 0, 1, 2

_lock = threading.Lock()
_lib = None


def library() -> ctypes.CDLL:
    """Load the shared library once (building it first if it is missing)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                import importlib.util

                spec = importlib.util.spec_from_file_location(
                    "_attn_build", LIB_PATH.parent.parent / "build.py")
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                mod.build()
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.attn_abi_version() != ABI_VERSION:
                raise RuntimeError(f"{LIB_PATH} has ABI {lib.attn_abi_version()}, "
                                   f"expected {ABI_VERSION}")
            _lib = lib
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(library().attn_last_error().decode(errors="replace"))


def _ptr(t: torch.Tensor | None):
    # ctypes turns a Python int into the c_void_p argument.
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device):
    """The current CUDA stream of `device` as an integer handle."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def _on(device: torch.device):
    """Make `device` current for the call (the C ABI works on the current device);
    no device switch when it already is."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if torch.cuda.current_device() == idx:
        return contextlib.nullcontext()
    return torch.cuda.device(idx)


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    # 256-byte aligned: torch's caching allocator aligns every block to >= 512 B.
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


class _StreamWorkspaces:
    """One decode scratch buffer per (device, stream), kept between calls and grown
    when a call needs more, like a BLAS library's workspace: calls on one stream
    run in order, so each may reuse the bytes of the one before. The buffer is
    allocated while its stream is current, so the caching allocator never hands
    its memory to another stream while a kernel may still use it."""

    def __init__(self):
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, nbytes: int, device: torch.device, stream: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            with self._lock:
                buf = self._bufs.get(key)
                if buf is None or buf.numel() < nbytes:
                    buf = _workspace(max(int(nbytes), 1 << 20), device)
                    self._bufs[key] = buf
        return buf

    def clear(self) -> None:
        with self._lock:
            self._bufs.clear()


_decode_ws = _StreamWorkspaces()


class Extension:
    """The reference extension's functions, running the sm_100a kernels."""

    def __init__(self):
        self.lib = library()

    # ------------------------------------------------------------- prefill
    def flash_wmma(self, q, k, v, causal, scale, block_n):
        o = torch.empty_like(q)
        B, H, N, D = q.shape
        with _on(q.device):
            _check(self.lib.attn_flash_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), B, H, N, D,
                                           int(bool(causal)), float(scale), int(block_n),
                                           _stream(q.device)))
        return o

    def flash_simt(self, q, k, v, causal, scale):
        o = torch.empty_like(q)
        B, H, N, D = q.shape
        with _on(q.device):
            _check(self.lib.attn_flash_simt_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), B, H, N, D,
                                                int(bool(causal)), float(scale),
                                                _stream(q.device)))
        return o

    def naive_attention(self, q, k, v, causal, scale):
        o = torch.empty_like(q)
        B, H, N, D = q.shape
        ws = _workspace(self.lib.attn_naive_workspace_bytes(B, H, N), q.device)
        with _on(q.device):
            _check(self.lib.attn_naive_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), B, H, N, D,
                                           int(bool(causal)), float(scale), _ptr(ws),
                                           ws.numel(), _stream(q.device)))
        return o

    # -------------------------------------------------------------- decode
    def _decode_sizes(self, q, kc, bt):
        B, H, D = q.shape
        return B, H, kc.shape[1], D, kc.shape[2], kc.shape[0], bt.shape[1]

    def paged_decode(self, q, kc, vc, bt, ctx, max_ctx, scale, partition):
        out = torch.empty_like(q)
        B, H, Hkv, D, bs, nblk, maxb = self._decode_sizes(q, kc, bt)
        with _on(q.device):
            stream = _stream(q.device)
            ws = _decode_ws.get(
                self.lib.attn_paged_decode_workspace_bytes(B, H, D, max_ctx, partition),
                q.device, stream)
            _check(self.lib.attn_paged_decode(
                _ptr(q), _ptr(kc), _ptr(vc), _ptr(bt), _ptr(ctx), _ptr(out), B, H, Hkv, D, bs,
                nblk, maxb, int(max_ctx), float(scale), int(partition), _ptr(ws), ws.numel(),
                stream))
        return out

    def paged_decode_partials(self, q, kc, vc, bt, ctx, max_ctx, scale, partition,
                              o=None, m=None, l=None):
        B, H, Hkv, D, bs, nblk, maxb = self._decode_sizes(q, kc, bt)
        f32 = dict(dtype=torch.float32, device=q.device)
        o = torch.empty(B, H, D, **f32) if o is None else o
        m = torch.empty(B, H, **f32) if m is None else m
        l = torch.empty(B, H, **f32) if l is None else l
        with _on(q.device):
            stream = _stream(q.device)
            ws = _decode_ws.get(
                self.lib.attn_paged_decode_workspace_bytes(B, H, D, max_ctx, partition),
                q.device, stream)
            _check(self.lib.attn_paged_decode_partials(
                _ptr(q), _ptr(kc), _ptr(vc), _ptr(bt), _ptr(ctx), _ptr(o), _ptr(m), _ptr(l), B, H,
                Hkv, D, bs, nblk, maxb, int(max_ctx), float(scale), int(partition), _ptr(ws),
                ws.numel(), stream))
        return o, m, l

    def merge_partials(self, o_parts, m_parts, l_parts, rows, head_dim, o_part_stride,
                       ml_part_stride, num_parts, out):
        with _on(out.device):
            _check(self.lib.attn_merge_partials(
                _ptr(o_parts), _ptr(m_parts), _ptr(l_parts), int(num_parts), int(rows),
                int(head_dim), int(o_part_stride), int(ml_part_stride), _ptr(out),
                _stream(out.device)))
        return out

    def exchange_merge_partials(self, slot_ptrs, flag_ptrs, rank, epoch, rows, head_dim,
                                slot_stride, out):
        """attn_exchange_merge_partials: slot_ptrs / flag_ptrs are the device addresses
        (ints) of every rank's receive area and flag words for this call."""
        world = len(slot_ptrs)
        slots = (_vp * world)(*slot_ptrs)
        flags = (_vp * world)(*flag_ptrs)
        with _on(out.device):
            _check(self.lib.attn_exchange_merge_partials(
                slots, flags, int(world), int(rank), int(epoch) & 0xFFFFFFFF, int(rows),
                int(head_dim), int(slot_stride), _ptr(out), _stream(out.device)))
        return out

    # -------------------------------------------------------------- status
    def device_status(self, device=None):
        code, site = ctypes.c_uint32(0), ctypes.c_uint32(0)
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        with torch.cuda.device(dev):
            _check(self.lib.attn_device_status(ctypes.byref(code), ctypes.byref(site)))
        return code.value, site.value

    def selftest_exp2(self, x):
        """(poly, mufu, exp2f) of fp32 CUDA tensor x: the prefill softmax's two
        exponentials and CUDA's exp2f, elementwise."""
        x = x.contiguous()
        if x.dtype != torch.float32 or not x.is_cuda:
            raise ValueError("x must be an fp32 CUDA tensor")
        ys = [torch.empty_like(x) for _ in range(3)]
        with _on(x.device):
            _check(self.lib.attn_selftest_exp2(_ptr(x), *(_ptr(y) for y in ys), x.numel(),
                                               _stream(x.device)))
        return tuple(ys)

    def selftest_wait_timeout(self, timeout_ns, device=None):
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        with torch.cuda.device(dev):
            _check(self.lib.attn_selftest_wait_timeout(int(timeout_ns), _stream(dev)))
