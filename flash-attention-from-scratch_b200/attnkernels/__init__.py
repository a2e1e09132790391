"""Attention kernels for LLM inference on B200 (sm_100a).

Drop-in replacement for the `attnkernels` package of
sonhoang/flash-attention-from-scratch (attnkernels/__init__.py): same
functions, arguments, defaults and ValueError conditions, running hand-written
Blackwell kernels through the C ABI of include/attn_b200.h.

Prefill (many query tokens per sequence):
    naive_attention   three kernels, materialises the N x N scores
    flash_attention   variant "wmma": tcgen05 tensor cores (TMEM accumulators,
                      TMA-staged tiles); variant "simt": CUDA cores

Decode (one query token per sequence) over a paged KV cache:
    paged_decode      split-K / flash-decoding with bulk-copy page streaming,
                      plus a merge kernel

Additions (no counterpart in the reference): paged_decode_partials and
merge_partials expose the split state for context parallelism across GPUs
(see attnkernels.parallel), device_status reads the kernels' error word, and
release_workspaces drops the decode scratch kept between calls.

There is no CPU fallback: every function needs a B200 and the native library
(built by flash-attention-from-scratch_b200/build.py, or on first use).
"""
from __future__ import annotations

import functools
import math

import torch

from . import _native

__all__ = ["naive_attention", "flash_attention", "paged_decode", "decode_partition",
           "load_extension", "paged_decode_partials", "merge_partials", "device_status",
           "check_device_status", "release_workspaces", "CHUNK", "WMMA_BLOCK_N"]

# Decode partitions are multiples of this many tokens (attnkernels/__init__.py:29).
CHUNK = 256

# Accepted key-tile widths of the tensor-core variant, per head dim
# (attnkernels/__init__.py:33). On sm_100a both 32 and 64 run the same kernel,
# whose key tile is 128 rows; the argument is kept for drop-in compatibility.
WMMA_BLOCK_N = {64: 64, 128: 64}

# Decode work units (sequence, kv head, split) to aim for per resident warp of
# the decode kernel, its resident warps per SM, and the most splits of one
# sequence per query head of a kv head (each split adds a part to that row's
# merge; a unit of G query heads costs about G times the arithmetic per byte, so
# grouped-query layers get more, shorter units). Chosen from the split ablation
# on B200 (bench.py --ablation, bench_sweep.py).
_UNITS_PER_WARP = 32
_DECODE_WARPS_PER_SM = 8
_MAX_SPLITS = 32


def _decode_warps_per_sm(group, head_dim=128):
    """Warps per CTA (one CTA per SM) of the decode kernel for G query heads per kv
    head: 16 at head_dim 64, whose 2 KB stages make each warp latency-bound, 8 at
    128, for every G (DecCfg in csrc/decode.cu)."""
    del group
    return 2 * _DECODE_WARPS_PER_SM if head_dim == 64 else _DECODE_WARPS_PER_SM


@functools.lru_cache(maxsize=None)
def load_extension():
    """The native kernels, with the reference extension's call surface."""
    return _native.Extension()


def _check_prefill(q, k, v):
    """attnkernels/__init__.py:53-61: fp16 CUDA [B, H, N, D], same shapes, D in {64, 128}."""
    for t in (q, k, v):
        if not (t.is_cuda and t.dtype == torch.float16 and t.dim() == 4):
            raise ValueError("q, k, v must be fp16 CUDA tensors of shape [B, H, N, D]")
    if not (q.shape == k.shape == v.shape):
        raise ValueError("q, k, v must have the same shape (self-attention prefill)")
    if q.shape[-1] not in (64, 128):
        raise ValueError("head_dim must be 64 or 128")
    return q.contiguous(), k.contiguous(), v.contiguous()


def naive_attention(q, k, v, causal=False, scale=None):
    """softmax(scale * Q K^T [+ causal mask]) V with the scores in DRAM."""
    q, k, v = _check_prefill(q, k, v)
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    return load_extension().naive_attention(q, k, v, causal, scale)


def flash_attention(q, k, v, causal=False, scale=None, variant="wmma", block_n=None):
    """Tiled attention with online softmax. q, k, v: fp16 [B, H, N, D], D in {64, 128}.

    variant: "simt" (CUDA cores) or "wmma" (tensor cores: the tcgen05 kernel).
    block_n: 32 or 64, accepted for compatibility (see WMMA_BLOCK_N).
    """
    q, k, v = _check_prefill(q, k, v)
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    ext = load_extension()
    if variant == "simt":
        return ext.flash_simt(q, k, v, causal, scale)
    if variant == "wmma":
        bn = WMMA_BLOCK_N[q.shape[-1]] if block_n is None else block_n
        return ext.flash_wmma(q, k, v, causal, scale, bn)
    raise ValueError(f"unknown variant {variant!r}")


@functools.lru_cache(maxsize=None)
def _sm_count(device_index):
    return torch.cuda.get_device_properties(device_index).multi_processor_count


def decode_partition(batch, num_kv_heads, max_context_len, device=None, sm_count=None,
                     num_heads=None, head_dim=128):
    """Tokens per split for paged_decode.

    Same contract as attnkernels/__init__.py:93-101 (a multiple of CHUNK, at
    least one chunk per split, more splits when batch * kv heads is small), with
    the B200 target: about _UNITS_PER_WARP (sequence, kv head, split) units per
    resident decode warp (8 per SM, 16 at head_dim 64), so the persistent kernel
    balances ragged batches, and at most _MAX_SPLITS * G splits per sequence, G =
    num_heads / num_kv_heads (1 when num_heads is not given), which bounds the
    merge. `sm_count` overrides the device query.
    """
    if sm_count is None:
        dev = torch.cuda.current_device() if device is None else device
        sm_count = _sm_count(dev)
    group = max(1, num_heads // num_kv_heads) if num_heads else 1
    return _partition(int(batch), int(num_kv_heads), int(max_context_len), int(sm_count),
                      group, int(head_dim))


@functools.lru_cache(maxsize=4096)
def _partition(batch, num_kv_heads, max_context_len, sm_count, group, head_dim=128):
    seqs = max(1, batch * num_kv_heads)
    want = -(-_UNITS_PER_WARP * _DECODE_WARPS_PER_SM * sm_count // seqs)
    max_chunks = max(1, -(-max_context_len // CHUNK))
    cap = _MAX_SPLITS * group
    splits = max(1, min(want, max_chunks, cap))
    part = -(-max_chunks // splits) * CHUNK
    warps = _decode_warps_per_sm(group, head_dim) * sm_count
    if seqs * -(-max_context_len // part) >= 4 * warps:
        return part
    # Few units for the resident warps: the launch takes about (rounds of units per
    # warp) x (tokens per unit); among partitions of 2^k chunks take the largest of
    # the least such time (fewer parts to merge, whole rounds of warps).
    best_t, best_p = None, part
    p = CHUNK
    while True:
        s = -(-max_context_len // p)
        if s <= cap:
            t = -(-seqs * s // warps) * p
            if best_t is None or t <= best_t:
                best_t, best_p = t, p
        if s <= 1:
            break
        p *= 2
    return best_p


def _check_decode(q, k_cache, v_cache):
    """attnkernels/__init__.py:116-119, plus the 4-D q [B, H, 1, D] of BASELINE config 4."""
    if not (q.dtype == k_cache.dtype == v_cache.dtype == torch.float16):
        raise ValueError("q and caches must be fp16")
    if q.shape[-1] not in (64, 128) or k_cache.shape[-1] != q.shape[-1]:
        raise ValueError("head_dim must be 64 or 128 and match the cache")
    if q.dim() == 4:
        if q.shape[2] != 1:
            raise ValueError("a 4-D decode q must be [B, H, 1, D]")
        return q.reshape(q.shape[0], q.shape[1], q.shape[3])
    if q.dim() != 3:
        raise ValueError("q must be [B, H, D] (or [B, H, 1, D])")
    return q


def _decode_args(q, k_cache, v_cache, block_tables, context_lens, max_context_len, scale,
                 partition_size):
    q3 = _check_decode(q, k_cache, v_cache)
    if not (q.is_cuda and k_cache.is_cuda and v_cache.is_cuda):
        raise ValueError("q and caches must be CUDA tensors")
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    if partition_size is None:
        partition_size = decode_partition(q3.shape[0], k_cache.shape[1], max_context_len,
                                          q.device.index, num_heads=q3.shape[1],
                                          head_dim=q3.shape[2])
    partition_size = -(-int(partition_size) // CHUNK) * CHUNK
    return (q3.contiguous(), k_cache.contiguous(), v_cache.contiguous(),
            block_tables.to(device=q.device, dtype=torch.int32).contiguous(),
            context_lens.to(device=q.device, dtype=torch.int32).contiguous(),
            int(max_context_len), float(scale), partition_size)


def paged_decode(q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                 scale=None, partition_size=None):
    """Decode attention over a paged KV cache.

    q:            [B, H, D] (or [B, H, 1, D]) fp16, one query token per sequence
    k_cache:      [num_blocks, H_kv, block_size, D] fp16 (v_cache the same)
    block_tables: [B, max_blocks_per_seq] int32, physical block ids
    context_lens: [B] int32, tokens of context per sequence (>= 1)
    max_context_len: Python int, max(context_lens) (passed in to avoid a sync)
    partition_size: tokens per split (multiple of 256). None picks one from the
                  batch size; a value >= max_context_len disables split-K.
    Returns fp16 of q's shape.
    """
    args = _decode_args(q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                        scale, partition_size)
    return load_extension().paged_decode(*args).reshape(q.shape)


def paged_decode_partials(q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                          scale=None, partition_size=None, out=None):
    """Softmax state of each (sequence, head) row over this cache's context.

    Returns (o fp32 [B, H, D] normalised, m fp32 [B, H] max score in log2 units
    of scale * q.k, l fp32 [B, H] = sum 2^(s - m)); rows with no context are
    (0, -inf, 0). `out` may supply the three output tensors. Used when a
    sequence's context is split across GPUs (attnkernels.parallel).
    """
    args = _decode_args(q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                        scale, partition_size)
    o, m, l = (None, None, None) if out is None else out
    return load_extension().paged_decode_partials(*args, o=o, m=m, l=l)


def merge_partials(o_parts, m_parts, l_parts, out=None):
    """Merge P partials per row into fp16: o_parts [P, ..., D], m/l_parts [P, ...].

    M = max m_p, w_p = l_p 2^(m_p - M), out = sum w_p o_p / sum w_p (the merge of
    attnkernels/csrc/paged_decode.cu:207-215, across GPUs). Parts may be strided
    views into one gathered buffer (dim 0 stride arbitrary, rows contiguous).
    """
    P = o_parts.shape[0]
    D = o_parts.shape[-1]
    rows = m_parts[0].numel() if P > 0 else o_parts[0].numel() // D
    if out is None:
        out = torch.empty(o_parts.shape[1:], dtype=torch.float16, device=o_parts.device)
    for t in (o_parts, m_parts, l_parts):
        if t.dtype != torch.float32 or not t.is_cuda:
            raise ValueError("partials must be fp32 CUDA tensors")
    o_stride = o_parts.stride(0) if P > 1 else rows * D
    ml_stride = m_parts.stride(0) if P > 1 else rows
    if P > 1 and l_parts.stride(0) != ml_stride:
        raise ValueError("m_parts and l_parts must share their part stride")
    return load_extension().merge_partials(o_parts, m_parts, l_parts, rows, D, o_stride,
                                           ml_stride, P, out)


def release_workspaces():
    """Drop the decode scratch buffers kept per (device, stream) between calls (the
    split-K partials), so the caching allocator can reuse or free their memory.
    Call it when no decode is in flight on those streams."""
    _native._decode_ws.clear()


def device_status(device=None):
    """(code, site) of the kernels' device status word, then clear it (syncs)."""
    return load_extension().device_status(device)


def check_device_status(device=None):
    """Raise RuntimeError if a kernel reported a timed-out wait or a bad block id."""
    code, site = device_status(device)
    if code == _native.DEVICE_WAIT_TIMEOUT:
        raise RuntimeError(f"attention kernel wait timed out (site {site})")
    if code == _native.DEVICE_BAD_BLOCK:
        raise RuntimeError(f"block table holds an id outside the cache (site {site})")
    if code != _native.DEVICE_OK:
        raise RuntimeError(f"attention kernel error code {code} (site {site})")
