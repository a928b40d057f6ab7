"""Per-sequence logical -> physical block mapping.

Same interface and semantics as the reference's BlockTable
(engine/cache/block_table.py:6-36): ``blocks`` lists physical block ids in
logical order, ``length`` counts written tokens, position p lives in block
``blocks[p // block_size]`` at offset ``p % block_size``.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class BlockTable:
    block_size: int
    blocks: list[int] = field(default_factory=list)
    length: int = 0

    def num_blocks_needed(self, new_length: int) -> int:
        return (new_length + self.block_size - 1) // self.block_size

    def logical_to_physical(self, pos: int) -> tuple[int, int]:
        return self.blocks[pos // self.block_size], pos % self.block_size

    def clone(self) -> "BlockTable":
        return BlockTable(block_size=self.block_size, blocks=list(self.blocks), length=self.length)

    def truncate(self, new_length: int) -> None:
        """Roll back to new_length tokens, releasing no blocks (the caller frees)."""
        if new_length > self.length:
            raise ValueError(f"cannot truncate {self.length} tokens to {new_length}")
        self.length = new_length
        del self.blocks[self.num_blocks_needed(new_length):]
