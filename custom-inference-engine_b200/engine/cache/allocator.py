"""Host-side block bookkeeping of the paged KV cache (no device data).

The free list is LIFO over ``list(range(num_blocks))`` exactly as the
reference's PagedKVCache (engine/cache/kv_cache.py:64, 76-79), so a workload
replayed against both caches gets the same physical block ids — which is what
lets the GPU tests compare against the reference's golden cache lifecycle.
"""

from __future__ import annotations

from engine.cache.block_table import BlockTable


class BlockAllocator:
    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._free: list[int] = list(range(num_blocks))

    @property
    def num_free(self) -> int:
        return len(self._free)

    def alloc(self) -> int:
        if not self._free:
            raise RuntimeError("KV cache out of blocks")
        return self._free.pop()

    def free(self, block_id: int) -> None:
        self._free.append(block_id)

    def new_sequence(self) -> BlockTable:
        return BlockTable(block_size=self.block_size)

    def free_sequence(self, table: BlockTable) -> None:
        for b in table.blocks:
            self.free(b)
        table.blocks.clear()
        table.length = 0

    def reserve(self, table: BlockTable, end: int) -> None:
        """Make sure positions [0, end) have blocks (appending in logical order)."""
        while len(table.blocks) < table.num_blocks_needed(end):
            table.blocks.append(self.alloc())

    def rollback(self, table: BlockTable, new_length: int) -> None:
        """Free the blocks made unnecessary by truncating to new_length (kv_cache.py:187-194)."""
        if new_length > table.length:
            raise ValueError(f"cannot roll back {table.length} tokens to {new_length}")
        needed = table.num_blocks_needed(new_length)
        for bid in table.blocks[needed:]:
            self.free(bid)
        table.blocks[needed:] = []
        table.length = new_length

    def fork_blocks(self, table: BlockTable) -> list[int]:
        """Fresh blocks for a deep copy of ``table`` (data copied by the caller)."""
        return [self.alloc() for _ in range(len(table.blocks))]
