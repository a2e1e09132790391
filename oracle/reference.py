"""CPU oracle for the attention hot paths: test infrastructure, not product code.

This module restates, in plain PyTorch fp32, the reference project's own oracle
attnkernels/reference.py (sonhoang/flash-attention-from-scratch). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use it, always as the
checker or as the timed CPU baseline, never inside the CUDA product path.

Parity of this restatement is pinned by tests/golden/*.npz: fixtures produced by
running the reference module itself (tests/golden/make_golden.py), which
tests/test_oracle.py compares against.

Differences from the reference's code are in evaluation order only:
attention_fp32 processes query rows in blocks so that long sequences do not
materialise the full [B, H, N, N] score tensor (each row's softmax is
independent, so the result is the same).
"""
from __future__ import annotations

import math

import torch

_LOG2E = 1.4426950408889634


def attention_fp32(q, k, v, causal=False, scale=None, row_block=1024, q_start=0):
    """softmax(scale * q k^T [+ top-left causal mask]) v in fp32.

    Follows attnkernels/reference.py:9-18: inputs of any float dtype are
    promoted to fp32; the causal mask hides key j > query i (triu(1)).
    q, k, v: [B, H, N, D] (k and v may have another length than q). q may be
    a slice of rows starting at position q_start of the full sequence (the
    causal mask then uses those positions). Returns fp32.
    """
    q, k, v = q.float(), k.float(), v.float()
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    n_q, n_k = q.shape[-2], k.shape[-2]
    out = torch.empty(*q.shape[:-1], v.shape[-1], dtype=torch.float32, device=q.device)
    kt = k.transpose(-1, -2)
    for r0 in range(0, n_q, row_block):
        r1 = min(n_q, r0 + row_block)
        s = (q[..., r0:r1, :] @ kt) * scale
        if causal:
            rows = torch.arange(q_start + r0, q_start + r1, device=q.device)[:, None]
            cols = torch.arange(n_k, device=q.device)[None, :]
            s = s.masked_fill(cols > rows, float("-inf"))
        out[..., r0:r1, :] = torch.softmax(s, dim=-1) @ v
    return out


def make_paged_cache(context_lens, num_kv_heads, head_dim, block_size=16, dtype=torch.float16,
                     device="cpu", extra_blocks=0, generator=None):
    """Random paged K/V caches with scattered physical blocks.

    Follows attnkernels/reference.py:21-45: ceil(ctx / block_size) blocks per
    sequence plus `extra_blocks` unused ones; the pool is handed out in the
    order of one random permutation (drawn from `generator`), so block_tables
    [B, max_blocks] int32 holds a sequence's blocks scattered through the pool;
    unused table slots are 0. K then V are drawn N(0, 1) with the global RNG of
    `device` (as the reference does; `generator` only drives the permutation).
    Returns k_cache, v_cache [num_blocks, num_kv_heads, block_size, head_dim],
    block_tables, context_lens (int32).
    """
    blocks_per_seq = [(c + block_size - 1) // block_size for c in context_lens]
    pool = sum(blocks_per_seq) + extra_blocks
    order = torch.randperm(pool, generator=generator).to(torch.int32)
    tables = torch.zeros(len(context_lens), max(blocks_per_seq), dtype=torch.int32)
    start = 0
    for b, nb in enumerate(blocks_per_seq):
        tables[b, :nb] = order[start:start + nb]
        start += nb
    shape = (pool, num_kv_heads, block_size, head_dim)
    k_cache = torch.randn(shape, device=device, dtype=dtype)
    v_cache = torch.randn(shape, device=device, dtype=dtype)
    lens = torch.tensor(list(context_lens), dtype=torch.int32, device=device)
    return k_cache, v_cache, tables.to(device), lens


def gather_kv(cache, block_tables, n_blocks):
    """Paged [num_blocks, H_kv, bs, D] -> contiguous [B, H_kv, n_blocks * bs, D].

    Follows attnkernels/reference.py:48-53.
    """
    picked = cache.index_select(0, block_tables[:, :n_blocks].reshape(-1).long())
    b = block_tables.shape[0]
    h, bs, d = cache.shape[1], cache.shape[2], cache.shape[3]
    picked = picked.view(b, n_blocks, h, bs, d)
    return picked.transpose(1, 2).reshape(b, h, n_blocks * bs, d)


def _sequence_kv(k_cache, v_cache, block_tables, b, c, group):
    bs = k_cache.shape[2]
    nb = (c + bs - 1) // bs
    k = gather_kv(k_cache, block_tables[b:b + 1], nb)[0, :, :c].float()
    v = gather_kv(v_cache, block_tables[b:b + 1], nb)[0, :, :c].float()
    return k.repeat_interleave(group, dim=0), v.repeat_interleave(group, dim=0)


def paged_decode_fp32(q, k_cache, v_cache, block_tables, context_lens, scale=None):
    """Decode attention per sequence in fp32; q [B, H, D] -> fp32 [B, H, D].

    Follows attnkernels/reference.py:56-70: query head h uses kv head h // G,
    scores over the first context_lens[b] tokens, softmax, weighted sum of V.
    """
    B, H, D = q.shape
    group = H // k_cache.shape[1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    out = torch.empty(B, H, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        c = int(context_lens[b])
        k, v = _sequence_kv(k_cache, v_cache, block_tables, b, c, group)
        s = (k @ q[b].float().unsqueeze(-1)).squeeze(-1) * scale  # [H, c]
        out[b] = (torch.softmax(s, dim=-1).unsqueeze(1) @ v).squeeze(1)
    return out


def paged_decode_torch(q, k_cache, v_cache, block_tables, n_blocks, context_lens=None):
    """Gather-then-SDPA decode baseline of attnkernels/reference.py:73-89.

    The blocks are gathered into a padded contiguous cache; the G query heads of
    a kv head become G query rows; with context_lens, keys past each sequence's
    length are masked.
    """
    B, H, D = q.shape
    hkv = k_cache.shape[1]
    k = gather_kv(k_cache, block_tables, n_blocks)
    v = gather_kv(v_cache, block_tables, n_blocks)
    qg = q.reshape(B, hkv, H // hkv, D)
    mask = None
    if context_lens is not None:
        pos = torch.arange(k.shape[2], device=q.device)
        mask = (pos[None, :] < context_lens.long()[:, None])[:, None, None, :]
    o = torch.nn.functional.scaled_dot_product_attention(qg, k, v, attn_mask=mask)
    return o.reshape(B, H, D)


def paged_decode_partials_fp32(q, k_cache, v_cache, block_tables, context_lens, scale=None):
    """Un-merged softmax state of each (sequence, head) row over the given cache.

    Returns (o [B, H, D] = softmax-weighted V, m [B, H] = max of
    scale * log2(e) * s, l [B, H] = sum of 2^(that - m)); rows with no
    context get (0, -inf, 0). This is the split state of the reference's
    paged_decode_kernel (attnkernels/csrc/paged_decode.cu:182-192), here for a
    whole cache (one GPU's context range).
    """
    B, H, D = q.shape
    group = H // k_cache.shape[1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    o = torch.zeros(B, H, D, dtype=torch.float32)
    m = torch.full((B, H), float("-inf"), dtype=torch.float32)
    l = torch.zeros(B, H, dtype=torch.float32)
    for b in range(B):
        c = int(context_lens[b])
        if c == 0:
            continue
        k, v = _sequence_kv(k_cache, v_cache, block_tables, b, c, group)
        x = (k @ q[b].float().unsqueeze(-1)).squeeze(-1) * (scale * _LOG2E)  # [H, c]
        mb = x.max(dim=-1).values
        p = torch.exp2(x - mb[:, None])
        lb = p.sum(dim=-1)
        o[b] = (p.unsqueeze(1) @ v).squeeze(1) / lb[:, None]
        m[b] = mb
        l[b] = lb
    return o, m, l


def merge_partials_fp32(o, m, l):
    """Merge P partials per row: o [P, ..., D], m and l [P, ...] -> fp32 [..., D].

    M = max_p m_p, w_p = l_p 2^(m_p - M), out = sum_p w_p o_p / sum_p w_p, as in
    the reference's paged_reduce_kernel (attnkernels/csrc/paged_decode.cu:207-215).
    Rows with no mass (all l = 0) are 0.
    """
    big = m.max(dim=0).values
    safe = torch.where(torch.isinf(big), torch.zeros_like(big), big)
    w = l * torch.exp2(m - safe.unsqueeze(0))
    den = w.sum(dim=0)
    num = (w.unsqueeze(-1) * o).sum(dim=0)
    out = num / torch.where(den > 0, den, torch.ones_like(den)).unsqueeze(-1)
    return torch.where((den > 0).unsqueeze(-1), out, torch.zeros_like(out))
