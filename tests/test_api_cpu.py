"""Host-side logic of the attnkernels package, on CPU: argument checks (the
reference's ValueError conditions), the split-size heuristic and the shard
arithmetic of the multi-GPU layer."""
import pytest
import torch

import attnkernels as ak
from attnkernels import parallel


def test_public_api_matches_reference():
    for name in ["naive_attention", "flash_attention", "paged_decode", "decode_partition",
                 "load_extension"]:
        assert callable(getattr(ak, name))
    assert ak.CHUNK == 256
    assert set(ak.WMMA_BLOCK_N) == {64, 128}


def qkv(d=64, device="cpu", dtype=torch.float16, n=16):
    return tuple(torch.zeros(1, 2, n, d, dtype=dtype, device=device) for _ in range(3))


def test_prefill_rejects_bad_input():
    with pytest.raises(ValueError):
        ak.flash_attention(*qkv())  # CPU tensors: the reference requires CUDA too
    with pytest.raises(ValueError):
        ak.naive_attention(*qkv())
    q = torch.zeros(1, 2, 16, 64, dtype=torch.float32)
    with pytest.raises(ValueError):
        ak.flash_attention(q, q, q)


def test_decode_rejects_bad_input():
    q = torch.zeros(2, 4, 64, dtype=torch.float16)
    kc = torch.zeros(3, 4, 16, 64, dtype=torch.float32)
    with pytest.raises(ValueError):
        ak.paged_decode(q, kc, kc, torch.zeros(2, 1), torch.ones(2), 1)
    kc = torch.zeros(3, 4, 16, 32, dtype=torch.float16)
    with pytest.raises(ValueError):
        ak.paged_decode(q, kc, kc, torch.zeros(2, 1), torch.ones(2), 1)
    kc = torch.zeros(3, 4, 16, 64, dtype=torch.float16)
    with pytest.raises(ValueError):  # CPU tensors
        ak.paged_decode(q, kc, kc, torch.zeros(2, 1), torch.ones(2), 1)


def test_decode_partition_contract():
    for batch, hkv, ctx in [(1, 8, 32768), (64, 32, 8192), (8, 32, 131072), (4, 2, 1),
                            (1, 1, 100), (512, 32, 4096)]:
        p = ak.decode_partition(batch, hkv, ctx, sm_count=148)
        assert p % ak.CHUNK == 0 and p >= ak.CHUNK
        splits = -(-ctx // p)
        assert splits <= max(1, -(-ctx // ak.CHUNK))
    # A small batch is split (at most 32 ways); a big one not at all.
    assert ak.decode_partition(1, 8, 32768, sm_count=148) == 1024
    # Grouped-query layers (G query heads per kv head) allow G times as many splits.
    assert ak.decode_partition(1, 8, 32768, sm_count=148, num_heads=32) == 256
    assert ak.decode_partition(1, 32, 32768, sm_count=148, num_heads=32) == 1024
    assert ak.decode_partition(4096, 32, 4096, sm_count=148) == 4096
    # BASELINE config 4 (64 x 32 heads, ctx up to 8192) lands on its stated 512.
    assert ak.decode_partition(64, 32, 8192, sm_count=148) == 512
    # One rank's share of config 5 at 8 GPUs (8 x 32 heads, 16384 tokens): 512.
    assert ak.decode_partition(8, 32, 16384, sm_count=148) == 512
    # head_dim 64 runs twice the warps per SM: a contract-valid partition either way,
    # and for these shapes no fewer splits than at head_dim 128.
    for batch, hkv, ctx in [(1, 8, 32768), (16, 8, 4096), (64, 8, 8192)]:
        p64 = ak.decode_partition(batch, hkv, ctx, sm_count=148, head_dim=64)
        p128 = ak.decode_partition(batch, hkv, ctx, sm_count=148, head_dim=128)
        assert p64 % ak.CHUNK == 0 and p64 <= p128


def test_shard_range_partitions():
    for total in [0, 1, 7, 32, 131072]:
        for world in [1, 2, 3, 4, 8]:
            spans = [parallel.shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1
    with pytest.raises(ValueError):
        parallel.shard_range(4, 2, 2)


def test_context_range_is_block_aligned():
    for ctx in [1, 15, 16, 17, 1000, 131072]:
        for world in [1, 2, 4, 8]:
            spans = [parallel.context_range(ctx, 16, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == ctx
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(s % 16 == 0 for s, _ in spans)
    assert parallel.context_range(131072, 16, 8, 3) == (3 * 16384, 4 * 16384)


def test_head_and_pair_ranges():
    assert parallel.head_range(32, 8, 7) == (28, 32)
    assert parallel.pair_range(4, 16, 8, 1) == (8, 16)


def test_release_workspaces_empties_the_cache():
    from attnkernels import _native
    ak.release_workspaces()
    assert _native._decode_ws._bufs == {}
