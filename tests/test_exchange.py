"""The peer-memory exchange + merge kernel of context-parallel decode, on one GPU.

attn_exchange_merge_partials pushes this rank's partials to every peer, raises a
flag in each peer's memory and waits for the peers' flags before it merges. On
one GPU the other ranks are emulated without a second kernel: their partials
and flags are written into this rank's receive area before the launch, so the
kernel finds them ready (kernels that wait on each other never run as separate
launches on one GPU). The last test leaves a flag unset: the bounded wait must
give up, report ATTN_DEVICE_WAIT_TIMEOUT at the exchange's site, and leave the
context usable.
"""
import time

import pytest
import torch

import attnkernels as ak
from oracle.reference import merge_partials_fp32

pytestmark = pytest.mark.gpu

ROWS, D = 40, 128
BLOCKS = -(-ROWS // 8)
STRIDE = -(-(ROWS * (D + 2)) // 4) * 4


def fill_slot(slot, o, m, l):
    slot[: ROWS * D].copy_(o.reshape(-1))
    slot[ROWS * D: ROWS * (D + 1)].copy_(m)
    slot[ROWS * (D + 1): ROWS * (D + 2)].copy_(l)


def partial(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    o = torch.randn(ROWS, D, generator=g, device="cuda")
    m = torch.randn(ROWS, generator=g, device="cuda") * 4
    l = torch.rand(ROWS, generator=g, device="cuda") * 50 + 1
    return o, m, l


def run(ext, world, ready_from, epoch=1):
    """Rank 0 of `world`; peers in `ready_from` have their data and flag in place."""
    area = torch.zeros(world * STRIDE, device="cuda")
    peers = [torch.zeros(world * STRIDE, device="cuda") for _ in range(1, world)]
    flags = [torch.zeros(world * BLOCKS, dtype=torch.int32, device="cuda") for _ in range(world)]
    parts = [partial(100 + r) for r in range(world)]
    fill_slot(area[:STRIDE], *parts[0])
    for r in ready_from:
        fill_slot(area[r * STRIDE:(r + 1) * STRIDE], *parts[r])
        flags[0].view(world, BLOCKS)[r].fill_(epoch)
    out = torch.empty(ROWS, D, dtype=torch.float16, device="cuda")
    slots = [area.data_ptr()] + [x.data_ptr() for x in peers]
    ext.exchange_merge_partials(slots, [f.data_ptr() for f in flags], 0, epoch, ROWS, D, STRIDE,
                                out)
    torch.cuda.synchronize()
    return out, parts, peers, flags


def test_single_rank_is_its_own_merge(ext):
    out, parts, _, _ = run(ext, 1, [])
    o, m, l = parts[0]
    want = merge_partials_fp32(o[None].cpu(), m[None].cpu(), l[None].cpu())
    assert (out.float().cpu() - want).abs().max().item() < 2e-3
    ak.check_device_status()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_merge_of_emulated_peers_and_push(ext, world):
    out, parts, peers, flags = run(ext, world, range(1, world), epoch=7)
    o = torch.stack([x[0] for x in parts]).cpu()
    m = torch.stack([x[1] for x in parts]).cpu()
    l = torch.stack([x[2] for x in parts]).cpu()
    want = merge_partials_fp32(o, m, l)
    assert (out.float().cpu() - want).abs().max().item() < 2e-3
    # Rank 0's partials landed in slot 0 of every peer, with flag 7 for every block.
    for q in range(1, world):
        got = peers[q - 1][:STRIDE]
        assert torch.equal(got[: ROWS * D].view(ROWS, D), parts[0][0])
        assert torch.equal(got[ROWS * D: ROWS * (D + 1)], parts[0][1])
        assert (flags[q].view(world, BLOCKS)[0] == 7).all()
    ak.check_device_status()


def test_missing_peer_times_out_without_a_fault(ext):
    ak.check_device_status()
    t0 = time.perf_counter()
    run(ext, 2, [])  # rank 1 never raises its flag
    code, site = ak.device_status()
    assert (code, site) == (1, 401)
    assert time.perf_counter() - t0 < 30
    # The context still works.
    out, _, _, _ = run(ext, 1, [])
    assert torch.isfinite(out).all()
    ak.check_device_status()
