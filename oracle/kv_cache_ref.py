"""numpy restatement of the reference paged KV cache (test oracle only).

Follows engine/cache/kv_cache.py:34-194 and engine/cache/block_table.py:6-36:
per-layer pools (num_blocks, block_size, Hkv, D), a LIFO free list
(``_free.pop()`` from list(range(num_blocks)), kv_cache.py:64,76-79), block-walked
append (:102-139), index-select gather trimmed to the sequence length (:141-165),
deep-copy fork (:169-185) and rollback that frees tail blocks (:187-194).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class BlockTableRef:
    block_size: int
    blocks: list[int] = field(default_factory=list)
    length: int = 0

    def num_blocks_needed(self, new_length: int) -> int:
        return (new_length + self.block_size - 1) // self.block_size

    def logical_to_physical(self, pos: int) -> tuple[int, int]:
        return self.blocks[pos // self.block_size], pos % self.block_size

    def clone(self) -> "BlockTableRef":
        return BlockTableRef(self.block_size, list(self.blocks), self.length)

    def truncate(self, new_length: int) -> None:
        assert new_length <= self.length
        self.length = new_length
        del self.blocks[self.num_blocks_needed(new_length):]


class PagedKVCacheRef:
    def __init__(self, num_layers, num_kv_heads, head_dim, num_blocks, block_size,
                 dtype=np.float32):
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.num_blocks = num_blocks
        self.block_size = block_size
        shape = (num_blocks, block_size, num_kv_heads, head_dim)
        self.k = [np.zeros(shape, dtype=dtype) for _ in range(num_layers)]
        self.v = [np.zeros(shape, dtype=dtype) for _ in range(num_layers)]
        self._free = list(range(num_blocks))

    def _alloc_block(self) -> int:
        if not self._free:
            raise RuntimeError("KV cache out of blocks")
        return self._free.pop()

    def _free_block(self, bid: int) -> None:
        self._free.append(bid)

    def new_sequence(self) -> BlockTableRef:
        return BlockTableRef(self.block_size)

    def free_sequence(self, table: BlockTableRef) -> None:
        for b in table.blocks:
            self._free_block(b)
        table.blocks.clear()
        table.length = 0

    def append(self, layer, table, k, v, start=None) -> None:
        L = k.shape[0]
        if start is None:
            start = table.length
        end = start + L
        while len(table.blocks) < table.num_blocks_needed(end):
            table.blocks.append(self._alloc_block())
        pos, src = start, 0
        while src < L:
            bid, off = table.logical_to_physical(pos)
            take = min(self.block_size - off, L - src)
            self.k[layer][bid, off:off + take] = k[src:src + take]
            self.v[layer][bid, off:off + take] = v[src:src + take]
            pos += take
            src += take
        table.length = max(table.length, end)

    def gather(self, layer, table):
        L = table.length
        shape = (L, self.num_kv_heads, self.head_dim)
        if L == 0:
            return np.zeros(shape, self.k[layer].dtype), np.zeros(shape, self.v[layer].dtype)
        idx = np.asarray(table.blocks, dtype=np.int64)
        k = self.k[layer][idx].reshape(-1, self.num_kv_heads, self.head_dim)[:L]
        v = self.v[layer][idx].reshape(-1, self.num_kv_heads, self.head_dim)[:L]
        return k, v

    def fork(self, table):
        new_blocks = [self._alloc_block() for _ in range(len(table.blocks))]
        if new_blocks:
            src = np.asarray(table.blocks)
            dst = np.asarray(new_blocks)
            for layer in range(self.num_layers):
                self.k[layer][dst] = self.k[layer][src]
                self.v[layer][dst] = self.v[layer][src]
        return BlockTableRef(self.block_size, new_blocks, table.length)

    def rollback(self, table, new_length: int) -> None:
        assert new_length <= table.length
        needed = table.num_blocks_needed(new_length)
        for bid in table.blocks[needed:]:
            self._free_block(bid)
        table.blocks[needed:] = []
        table.length = new_length


def gather_tables(pool: np.ndarray, tables: np.ndarray, kv_lens: np.ndarray, out_len: int):
    """Batched gather: out[b, t] = pool[tables[b, t // bs], t % bs] for t < kv_lens[b], else 0."""
    nb, bs, H, D = pool.shape
    B = tables.shape[0]
    out = np.zeros((B, out_len, H, D), dtype=pool.dtype)
    for b in range(B):
        L = int(kv_lens[b])
        if L == 0:
            continue
        nblk = (L + bs - 1) // bs
        rows = pool[tables[b, :nblk]].reshape(-1, H, D)[:L]
        out[b, :L] = rows
    return out
