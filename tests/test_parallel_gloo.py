"""The context-parallel decode orchestration on 2 CPU ranks (gloo).

Each rank holds the blocks of its block-aligned context range, computes the
softmax state of every row with the CPU oracle (injected in place of the CUDA
kernel), the states are all-gathered and merged: the result must equal
single-rank decode over the whole context. A second test makes one rank fail
before the collective and checks that the other rank gets an error, not a hang.
"""
import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    for p in (str(ROOT), str(ROOT / "flash-attention-from-scratch_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _local_slice(k_cache, v_cache, tables, lens, bs, world, rank):
    from attnkernels.parallel import context_range

    local_tabs, local_lens = [], []
    for b, c in enumerate(lens.tolist()):
        t0, t1 = context_range(c, bs, world, rank)
        b0, nb = t0 // bs, -(-(t1 - t0) // bs)
        row = torch.zeros(tables.shape[1], dtype=torch.int32)
        row[:nb] = tables[b, b0:b0 + nb]
        local_tabs.append(row)
        local_lens.append(t1 - t0)
    return torch.stack(local_tabs), torch.tensor(local_lens, dtype=torch.int32)


def _worker(rank, world, port, ctx, fail_rank, result_path):
    _paths()
    from attnkernels.parallel import ContextParallelDecode
    from oracle import reference as ref

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        torch.manual_seed(1)
        g = torch.Generator().manual_seed(1)
        bs, hkv, hq, d = 16, 2, 4, 64
        kc, vc, tables, lens = ref.make_paged_cache(ctx, hkv, d, block_size=bs, device="cpu",
                                                    generator=g)
        q = torch.randn(len(ctx), hq, d).half()
        bt_local, lens_local = _local_slice(kc, vc, tables, lens, bs, world, rank)

        def partials(q, kc, vc, bt, ln, max_len, scale, partition, out):
            o, m, l = ref.paged_decode_partials_fp32(q, kc, vc, bt, ln, scale)
            for dst, src in zip(out, (o, m, l)):
                dst.copy_(src)

        if rank == fail_rank:
            raise SystemExit(3)  # leaves before the collective
        run = ContextParallelDecode(partials_fn=partials, merge_fn=ref.merge_partials_fp32)
        out = run(q, kc, vc, bt_local, lens_local, int(lens_local.max()))
        full = ref.paged_decode_fp32(q, kc, vc, tables, lens)
        err = (out - full).abs().max().item()
        # A second step with another query reuses the kept buffers.
        q2 = torch.randn(len(ctx), hq, d).half()
        out2 = run(q2, kc, vc, bt_local, lens_local, int(lens_local.max()))
        full2 = ref.paged_decode_fp32(q2, kc, vc, tables, lens)
        err = max(err, (out2 - full2).abs().max().item())
        assert len(run._bufs) == 1
        Path(result_path + f".{rank}").write_text(f"ok {err}")
    except RuntimeError as e:  # the collective failed: expected when a peer left
        Path(result_path + f".{rank}").write_text(f"error {type(e).__name__}")
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(world, ctx, fail_rank, tmp_path):
    port = _free_port()
    res = str(tmp_path / "res")
    ctx_mp = mp.get_context("spawn")
    procs = [ctx_mp.Process(target=_worker, args=(r, world, port, ctx, fail_rank, res))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    return {r: Path(res + f".{r}").read_text() if Path(res + f".{r}").exists() else None
            for r in range(world)}, [p.exitcode for p in procs]


@pytest.mark.parametrize("ctx", [[300, 1, 47], [4096, 2000]])
def test_context_parallel_matches_single_rank(ctx, tmp_path):
    results, codes = _run(2, ctx, -1, tmp_path)
    assert codes == [0, 0]
    for r, text in results.items():
        kind, err = text.split()
        assert kind == "ok"
        assert float(err) < 1e-5, (r, err)


def test_rank_failure_is_reported_not_hung(tmp_path):
    results, codes = _run(2, [200, 100], 1, tmp_path)
    assert codes[1] == 3
    assert results[0] is not None and results[0].startswith("error")
