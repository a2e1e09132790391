"""The kernels inside CUDA graphs: a captured paged decode (split-K, so its merge
kernel runs as a programmatic dependent of the decode kernel) and a captured
prefill replay with new inputs copied into the captured buffers, and match the
eager calls bit for bit."""
import pytest
import torch

import attnkernels as ak
from oracle.reference import make_paged_cache

pytestmark = pytest.mark.gpu


def _capture(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # workspaces and schedules set up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


@pytest.mark.parametrize("heads", [(32, 32), (32, 8)])
def test_paged_decode_in_a_graph(heads):
    g = torch.Generator().manual_seed(21)
    ctx = [5000, 700, 33]
    kc, vc, tables, lens = make_paged_cache(ctx, heads[1], 128, device="cuda", generator=g)
    q = torch.randn(len(ctx), heads[0], 128, device="cuda").half()
    fn = lambda: ak.paged_decode(q, kc, vc, tables, lens, 5000, partition_size=256)  # noqa: E731
    graph, out = _capture(fn)
    for seed in (1, 2):
        q.copy_(torch.randn(q.shape, generator=torch.Generator().manual_seed(seed)).half())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, fn())
    ak.check_device_status()


def test_prefill_in_a_graph():
    shape = (2, 4, 1000, 128)
    q, k, v = (torch.randn(shape, device="cuda").half() for _ in range(3))
    fn = lambda: ak.flash_attention(q, k, v, causal=True)  # noqa: E731
    graph, out = _capture(fn)
    for seed in (3, 4):
        gen = torch.Generator().manual_seed(seed)
        for t in (q, k, v):
            t.copy_(torch.randn(shape, generator=gen).half())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, fn())
    ak.check_device_status()
