"""Context-parallel paged decode across 2, 4 and 8 GPUs, with the CUDA kernels.

Each rank holds the blocks of its block-aligned slice of every sequence's
context, computes the (o, m, l) partials with attn_paged_decode_partials, the
partials are exchanged (all-gathered over NCCL and merged with
attn_merge_partials, or pushed over NVLink peer memory and merged in one kernel
by attn_exchange_merge_partials) and every rank's result must match single-GPU
paged_decode over the whole context. Also
checks head-sharded prefill: each rank's heads equal the same heads computed on
one GPU. Each world size is skipped on hosts with fewer GPUs.
"""
import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
MAX_ABS = 2e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    for p in (str(ROOT), str(ROOT / "flash-attention-from-scratch_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    import attnkernels as ak
    from attnkernels.parallel import ContextParallelDecode, context_range, head_range
    from oracle.reference import make_paged_cache

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    lines = []
    try:
        # Same cache on every rank (same seeds), so each can check against the full decode.
        torch.manual_seed(7)
        g = torch.Generator().manual_seed(7)
        ctx = [5000, 17, 1024, 300]
        bs = 16
        kc, vc, tables, lens = make_paged_cache(ctx, 4, 128, block_size=bs, device=dev,
                                                generator=g)
        q = torch.randn(len(ctx), 16, 128, generator=torch.Generator(device=dev).manual_seed(8),
                        device=dev).half()
        rows, sub = [], []
        for b, c in enumerate(ctx):
            t0, t1 = context_range(c, bs, world, rank)
            b0, nb = t0 // bs, -(-(t1 - t0) // bs)
            row = torch.zeros(tables.shape[1], dtype=torch.int32, device=dev)
            row[:nb] = tables[b, b0:b0 + nb]
            rows.append(row)
            sub.append(t1 - t0)
        bt_local = torch.stack(rows)
        lens_local = torch.tensor(sub, dtype=torch.int32, device=dev)
        cp = ContextParallelDecode(exchange="nccl")
        out = cp(q, kc, vc, bt_local, lens_local, max(1, max(sub)), partition_size=512)
        full = ak.paged_decode(q, kc, vc, tables, lens, max(ctx), partition_size=512)
        lines.append(f"decode {(out.float() - full.float()).abs().max().item()}")
        # A second step reuses the exchange buffers kept by the first.
        q2 = torch.randn(q.shape, generator=torch.Generator(device=dev).manual_seed(18),
                         device=dev).half()
        out_b = cp(q2, kc, vc, bt_local, lens_local, max(1, max(sub)), partition_size=512)
        full_b = ak.paged_decode(q2, kc, vc, tables, lens, max(ctx), partition_size=512)
        lines.append(f"second {(out_b.float() - full_b.float()).abs().max().item()}")
        # The exchange over peer memory fused with the merge (two calls: both areas).
        cpp = ContextParallelDecode(exchange="peer")
        for tag, qq, ref in (("peer", q, full), ("peer2", q2, full_b)):
            got = cpp(qq, kc, vc, bt_local, lens_local, max(1, max(sub)), partition_size=512)
            lines.append(f"{tag} {(got.float() - ref.float()).abs().max().item()}")
        # The batch in chunks, exchange of one chunk overlapping the next one's decode.
        out2 = ContextParallelDecode(chunks=3)(q, kc, vc, bt_local, lens_local, max(1, max(sub)),
                                               partition_size=512)
        lines.append(f"chunked {(out2.float() - full.float()).abs().max().item()}")
        # Head-sharded prefill: no collective.
        gq = torch.Generator(device=dev).manual_seed(9)
        qp, kp, vp = (torch.randn(2, 8, 700, 128, generator=gq, device=dev).half() for _ in range(3))
        h0, h1 = head_range(8, world, rank)
        mine = ak.flash_attention(qp[:, h0:h1], kp[:, h0:h1], vp[:, h0:h1], causal=True)
        ref = ak.flash_attention(qp, kp, vp, causal=True)[:, h0:h1]
        lines.append(f"prefill {(mine.float() - ref.float()).abs().max().item()}")
        ak.check_device_status(dev)
    except Exception as e:  # noqa: BLE001  reported to the parent
        lines.append(f"error {type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()
    Path(f"{result_path}.{rank}").write_text("\n".join(lines))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_context_parallel_decode(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    res = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, res)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    for r in range(world):
        text = Path(f"{res}.{r}").read_text()
        assert "error" not in text, text
        vals = dict(line.split() for line in text.splitlines())
        assert float(vals["decode"]) < MAX_ABS, (r, text)
        assert float(vals["second"]) < MAX_ABS, (r, text)
        assert float(vals["peer"]) < MAX_ABS, (r, text)
        assert float(vals["peer2"]) < MAX_ABS, (r, text)
        assert float(vals["chunked"]) < MAX_ABS, (r, text)
        assert float(vals["prefill"]) == 0.0, (r, text)
