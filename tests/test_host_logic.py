"""CPU tests of the host-side logic: block tables, the LIFO block allocator
(against the reference's golden cache lifecycle), table packing, head
sharding, and the entry points' error conventions without a GPU."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from engine.cache import BlockAllocator, BlockTable, pack_tables
from engine.head_shard import rank_major_to_heads, shard_heads


# reference tests/cache/test_block_table.py:8-29
def test_logical_to_physical():
    t = BlockTable(block_size=4, blocks=[10, 11, 12], length=9)
    assert t.logical_to_physical(0) == (10, 0)
    assert t.logical_to_physical(3) == (10, 3)
    assert t.logical_to_physical(4) == (11, 0)
    assert t.logical_to_physical(8) == (12, 0)


def test_clone_independent():
    t = BlockTable(block_size=2, blocks=[1, 2], length=4)
    c = t.clone()
    c.blocks.append(3)
    c.length = 5
    assert t.blocks == [1, 2] and t.length == 4


def test_truncate_drops_blocks():
    t = BlockTable(block_size=2, blocks=[1, 2, 3], length=6)
    t.truncate(3)
    assert t.length == 3 and t.blocks == [1, 2]
    with pytest.raises(ValueError):
        t.truncate(4)


def test_allocator_replays_reference_lifecycle(golden):
    """Same block ids and free list as the reference cache for the golden script."""
    log = json.loads(bytes(golden["life_log"]).decode())
    al = BlockAllocator(12, 4)
    a, b = al.new_sequence(), al.new_sequence()
    mine = []

    def append(t, n, start):
        al.reserve(t, start + n)
        t.length = max(t.length, start + n)

    append(a, 6, 0)
    mine.append(["append_a6", list(a.blocks), a.length, list(al._free)])
    append(b, 3, 0)
    mine.append(["append_b3", list(b.blocks), b.length, list(al._free)])
    append(a, 3, 6)
    mine.append(["append_a3", list(a.blocks), a.length, list(al._free)])
    f = BlockTable(4, al.fork_blocks(a), a.length)
    mine.append(["fork_a", list(f.blocks), f.length, list(al._free)])
    al.rollback(a, 5)
    mine.append(["rollback_a5", list(a.blocks), a.length, list(al._free)])
    append(a, 4, 5)
    mine.append(["append_a4", list(a.blocks), a.length, list(al._free)])
    al.free_sequence(b)
    mine.append(["free_b", list(b.blocks), b.length, list(al._free)])
    assert mine == [list(x) for x in log]


def test_allocator_out_of_blocks():
    al = BlockAllocator(2, 4)
    t = al.new_sequence()
    al.reserve(t, 8)
    with pytest.raises(RuntimeError, match="out of blocks"):
        al.reserve(t, 9)


def test_pack_tables_cpu():
    tabs = [BlockTable(16, [5, 3], 20), BlockTable(16, [], 0), BlockTable(16, [7, 1, 2], 33)]
    tab, lens = pack_tables(tabs, "cpu")
    assert tab.dtype == torch.int32 and lens.dtype == torch.int32
    assert tab.tolist() == [[5, 3, 0], [0, 0, 0], [7, 1, 2]]
    assert lens.tolist() == [20, 0, 33]


def test_shard_heads():
    shards = [shard_heads(32, 8, 4, r) for r in range(4)]
    assert [s.hq for s in shards] == [8] * 4 and [s.hkv for s in shards] == [2] * 4
    assert [s.q0 for s in shards] == [0, 8, 16, 24] and [s.kv0 for s in shards] == [0, 2, 4, 6]
    # every query head's kv head stays on its rank
    for s in shards:
        for h in range(s.q0, s.q0 + s.hq):
            assert s.kv0 <= h // 4 < s.kv0 + s.hkv
    with pytest.raises(ValueError):
        shard_heads(32, 8, 3, 0)


def test_rank_major_to_heads():
    W, B, M, hl, d = 2, 1, 3, 4, 2
    g = torch.arange(W * B * M * hl * d, dtype=torch.float32).view(W, B, M, hl, d)
    full = rank_major_to_heads(g)
    assert full.shape == (B, M, W * hl, d)
    assert torch.equal(full[:, :, hl:], g[1])


def test_entry_points_refuse_cpu_tensors():
    from kernels.flash_attention import apply_rotary, flash_attention, paged_attention

    q = torch.randn(1, 2, 4, 64)
    with pytest.raises(RuntimeError, match="requires CUDA"):
        flash_attention(q, q, q)
    with pytest.raises(RuntimeError, match="requires CUDA"):
        paged_attention(q, q, q, torch.zeros(1, 1, dtype=torch.int32),
                        torch.zeros(1, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="requires CUDA"):
        apply_rotary(q, q, q)


def test_engine_call_site_conventions():
    from engine.attention import flash_attention

    with pytest.raises(RuntimeError, match="requires CUDA"):
        flash_attention(torch.randn(1, 1, 2, 64), torch.randn(1, 1, 2, 64), torch.randn(1, 1, 2, 64))


def test_rope_tables_match_reference_formula(golden):
    from kernels import build_rope_cache

    for name, (L, d, theta) in (("d16", (64, 16, 10000.0)), ("d64", (520, 64, 500000.0))):
        c, s = build_rope_cache(L, d, theta=theta)
        assert c.dtype == torch.float32 and c.shape == (L, d // 2)
        # same torch arithmetic as the reference: bit-identical tables
        np.testing.assert_array_equal(c.numpy(), golden[f"rope_{name}_cos"])
        np.testing.assert_array_equal(s.numpy(), golden[f"rope_{name}_sin"])


def test_paged_cache_requires_cuda():
    from engine.cache import KVCacheConfig, PagedKVCache

    with pytest.raises(RuntimeError, match="CUDA"):
        PagedKVCache(KVCacheConfig(1, 2, 16, 4, 4, device="cpu"))


class _HostCache:
    """The host-side part of PagedKVCache that begin_step uses (the real cache
    holds its pools on a CUDA device)."""

    def __init__(self, num_blocks, block_size):
        self.alloc = BlockAllocator(num_blocks, block_size)
        self.device = torch.device("cpu")

    def device_tables(self, tables):
        return pack_tables(tables, self.device)


def test_begin_step_reserves_and_packs_once():
    from engine.attention import begin_step

    cache = _HostCache(16, 4)
    a, b, c = (cache.alloc.new_sequence() for _ in range(3))
    cache.alloc.reserve(a, 5)
    a.length = 5
    cache.alloc.reserve(b, 8)
    b.length = 8
    step = begin_step(cache, [a, b, c], 3)
    assert step.starts == [5, 8, 0]
    assert [t.length for t in (a, b, c)] == [8, 11, 3]
    # blocks now cover the new tokens of every sequence
    assert [len(t.blocks) for t in (a, b, c)] == [2, 3, 1]
    assert step.kv_lens.tolist() == [8, 11, 3]
    assert step.start_pos.tolist() == [5, 8, 0]
    assert step.block_tables.dtype == torch.int32
    assert step.block_tables.tolist() == [a.blocks + [0], b.blocks, c.blocks + [0, 0]]
    with pytest.raises(ValueError):
        begin_step(cache, [a], 0)
    with pytest.raises(ValueError):
        begin_step(cache, [], 1)
