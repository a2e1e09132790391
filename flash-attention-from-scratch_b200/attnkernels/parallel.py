"""Multi-GPU partitioning of the two hot paths (one process per GPU).

The reference is single-GPU; this module is the B200 box layer:

* Prefill shards by head (or by (batch, head) pair): the units are independent,
  so each rank runs flash_attention on its own slice and there is no
  collective. `head_range` / `pair_range` give a rank's contiguous share.

* Long-context decode shards each sequence's context into contiguous,
  block-aligned ranges, one per rank (`context_range`); each rank holds the
  K/V pages of its range. A rank computes the softmax state (o, m, l) of every
  (sequence, head) row over its range with paged_decode_partials, the states
  are all-gathered over NCCL (the only collective: B * H * (D + 2) fp32 per
  rank), and every rank merges them with merge_partials into the fp16 output.
  With exchange="peer" the all-gather and the merge are one kernel instead
  (attn_exchange_merge_partials): each rank pushes its partials into every
  peer's receive area over NVLink (torch symmetric memory gives the peer
  pointers), signals each peer with a flag, waits for the peers' flags and
  merges; no collective launch.

The compute steps are injectable so that the orchestration (packing, the
collective, the merge layout) can be tested on CPU ranks with gloo and the CPU
oracle; the defaults are the CUDA kernels.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous near-equal share [begin, end) of `total` items for `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    return total * rank // world, total * (rank + 1) // world


def head_range(num_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Heads of `rank` when prefill is sharded by head (no collective)."""
    return shard_range(num_heads, world, rank)


def pair_range(batch: int, num_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Flattened (batch, head) pairs [begin, end) of `rank`."""
    return shard_range(batch * num_heads, world, rank)


def context_range(context_len: int, block_size: int, world: int, rank: int) -> tuple[int, int]:
    """Token range [begin, end) of one sequence held by `rank`.

    The sequence's blocks are split into contiguous near-equal runs, so every
    rank owns whole blocks (the last rank's run may end in a partial block).
    """
    blocks = -(-context_len // block_size)
    b0, b1 = shard_range(blocks, world, rank)
    return min(context_len, b0 * block_size), min(context_len, b1 * block_size)


def _gather_flat(buf: torch.Tensor, world: int, group, out=None) -> torch.Tensor:
    if out is None:
        out = torch.empty((world, buf.numel()), dtype=buf.dtype, device=buf.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, buf, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), buf, group=group)
    return out


class _PeerArea:
    """Receive areas of the peer exchange for one (device, rows, head_dim): two
    areas (alternated by call parity) of `world` slots, each slot o [rows][D],
    m [rows], l [rows] fp32 padded to 16 bytes, then the flag words
    [world][ceil(rows / 8)]; one symmetric allocation, rendezvoused over the group
    so that every rank holds every rank's device addresses."""

    def __init__(self, group, device, rows, d, world, rank):
        import torch.distributed._symmetric_memory as symm_mem

        self.rows, self.d, self.world, self.rank = rows, d, world, rank
        self.stride = -(-(rows * (d + 2)) // 4) * 4
        self.area_floats = world * self.stride
        blocks = -(-rows // 8)
        total = 2 * self.area_floats + world * blocks
        group = group if group is not None else dist.group.WORLD
        name = group.group_name
        self.buf = symm_mem.empty(total, dtype=torch.float32, device=device)
        self.buf.zero_()  # the flags start at 0
        torch.cuda.synchronize(device)
        handle = symm_mem.rendezvous(self.buf, name)
        base = [int(x) for x in handle.buffer_ptrs]
        self.handle = handle
        self.slots = [[b + 4 * par * self.area_floats for b in base] for par in (0, 1)]
        self.flags = [b + 4 * 2 * self.area_floats for b in base]
        self.epoch = 0
        dist.barrier(group)  # every rank's flags are zero before anyone signals

    def own_slot(self, par):
        """This rank's slot of its own receive area for call parity `par`."""
        start = par * self.area_floats + self.rank * self.stride
        return self.buf[start:start + self.stride]


class ContextParallelDecode:
    """Decode with each sequence's context split across the ranks of `group`.

    __call__(q, k_cache, v_cache, block_tables, context_lens, max_context_len,
    scale=None, partition_size=None) takes this rank's cache, block tables and
    per-sequence token counts of its range (context_lens may be 0 for some
    sequences) and returns the merged output, fp16 [B, H, D], on every rank.

    partials_fn(q, kc, vc, bt, lens, max_len, scale, partition, out=(o, m, l))
    fills o [B, H, D], m and l [B, H] (fp32); merge_fn(o_parts, m_parts,
    l_parts) merges [P, B, H, D] / [P, B, H] views. Defaults: the CUDA kernels.

    exchange="peer" (the default with the CUDA kernels and one chunk) replaces the
    all-gather and the merge by attn_exchange_merge_partials over peer memory (see
    the module doc); exchange="nccl" keeps the all-gather (and is what custom steps
    or chunks use).

    chunks > 1 (CUDA tensors only) splits the batch: the all-gather of one
    chunk's partials runs on a side stream while the next chunk is decoded, so
    only the last chunk's exchange and the merges are exposed.

    The partials buffer and the gather buffer of each chunk are kept between
    calls (per device and shape), so a decode loop allocates nothing after its
    first step. Reuse is ordered by the streams: a call's partials kernel is
    enqueued on the compute stream after the previous call's merge, which
    itself waited for that call's gather; and a gather waits for the compute
    stream before it overwrites its buffer.
    """

    def __init__(self, group=None, partials_fn=None, merge_fn=None, chunks=1, exchange=None):
        if exchange is None:  # the fused peer kernel unless the steps are customised
            custom = partials_fn is not None or merge_fn is not None or chunks != 1
            exchange = "nccl" if custom else "peer"
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange must be 'nccl' or 'peer', got {exchange!r}")
        if exchange == "peer" and (partials_fn is not None or merge_fn is not None or chunks != 1):
            raise ValueError("exchange='peer' runs the CUDA kernels, in one chunk")
        self.exchange = exchange
        self._areas = {}
        self.group = group
        self.custom_merge = merge_fn is not None
        if partials_fn is None or merge_fn is None:
            from . import merge_partials, paged_decode_partials
            partials_fn = partials_fn or paged_decode_partials
            merge_fn = merge_fn or merge_partials
        self.partials_fn = partials_fn
        self.merge_fn = merge_fn
        self.chunks = max(1, int(chunks))
        self._comm = {}
        self._bufs = {}

    @staticmethod
    def _views(buf, rows_b, heads, d):
        rows = rows_b * heads
        return (buf[..., : rows * d].unflatten(-1, (rows_b, heads, d)),
                buf[..., rows * d: rows * (d + 1)].unflatten(-1, (rows_b, heads)),
                buf[..., rows * (d + 1): rows * (d + 2)].unflatten(-1, (rows_b, heads)))

    def _buffers(self, device, B, H, D, world, chunk, side_stream=None):
        """(partials buffer, gather buffer) of one chunk, kept between calls."""
        key = (str(device), B, H, D, world, chunk)
        bufs = self._bufs.get(key)
        if bufs is None:
            # One fp32 buffer per rank: o [rows, D], m [rows], l [rows], padded to
            # 16 bytes so every part's o rows stay 16-byte aligned after the gather.
            stride = -(-(B * H * (D + 2)) // 4) * 4
            buf = torch.empty(stride, dtype=torch.float32, device=device)
            gathered = torch.empty((world, stride), dtype=torch.float32, device=device)
            if side_stream is not None:
                # Used on the side stream too: the allocator must not hand the
                # memory out again before that stream is done with it.
                buf.record_stream(side_stream)
                gathered.record_stream(side_stream)
            bufs = self._bufs[key] = (buf, gathered)
        return bufs

    def _exchange(self, q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                  scale, partition_size, world, chunk=0, side_stream=None):
        B, H, D = q.shape
        buf, gathered = self._buffers(q.device, B, H, D, world, chunk, side_stream)
        self.partials_fn(q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                         scale, partition_size, out=self._views(buf, B, H, D))
        return buf, gathered

    def __call__(self, q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                 scale=None, partition_size=None):
        world = dist.get_world_size(self.group)
        if q.dim() == 4:
            q = q.reshape(q.shape[0], q.shape[1], q.shape[3])
        B, H, D = q.shape
        if self.exchange == "peer" and q.is_cuda:
            return self._peer_call(q, k_cache, v_cache, block_tables, context_lens,
                                   max_context_len, scale, partition_size, world)
        nchunks = min(self.chunks, B) if q.is_cuda and not self.custom_merge else 1
        if nchunks == 1:
            buf, gathered = self._exchange(q, k_cache, v_cache, block_tables, context_lens,
                                           max_context_len, scale, partition_size, world)
            _gather_flat(buf, world, self.group, out=gathered)
            return self.merge_fn(*self._views(gathered, B, H, D))
        compute = torch.cuda.current_stream(q.device)
        comm = self._comm.get(q.device)
        if comm is None:
            comm = self._comm[q.device] = torch.cuda.Stream(q.device)
        out = torch.empty(B, H, D, dtype=torch.float16, device=q.device)
        pending = []
        for c in range(nchunks):
            b0, b1 = shard_range(B, nchunks, c)
            buf, gathered = self._exchange(q[b0:b1], k_cache, v_cache, block_tables[b0:b1],
                                           context_lens[b0:b1], max_context_len, scale,
                                           partition_size, world, chunk=c, side_stream=comm)
            comm.wait_stream(compute)
            with torch.cuda.stream(comm):
                _gather_flat(buf, world, self.group, out=gathered)
            pending.append((b0, b1, gathered))
        compute.wait_stream(comm)
        for b0, b1, gathered in pending:
            self.merge_fn(*self._views(gathered, b1 - b0, H, D), out=out[b0:b1])
        return out

    def _peer_call(self, q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                   scale, partition_size, world):
        from . import load_extension

        B, H, D = q.shape
        key = (str(q.device), B * H, D, world)
        area = self._areas.get(key)
        if area is None:
            area = self._areas[key] = _PeerArea(self.group, q.device, B * H, D, world,
                                                dist.get_rank(self.group))
        area.epoch += 1
        par = area.epoch & 1
        self.partials_fn(q, k_cache, v_cache, block_tables, context_lens, max_context_len,
                         scale, partition_size, out=self._views(area.own_slot(par), B, H, D))
        out = torch.empty(B, H, D, dtype=torch.float16, device=q.device)
        return load_extension().exchange_merge_partials(
            area.slots[par], area.flags, area.rank, area.epoch, B * H, D, area.stride, out)
