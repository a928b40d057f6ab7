"""Paged KV cache on the GPU, written and read by the B200 kernels.

Mirrors the reference's PagedKVCache (engine/cache/kv_cache.py:10-210): per
layer K and V pools of shape (num_blocks, block_size, num_kv_heads, head_dim),
a LIFO free list, per-sequence BlockTables, append / gather / fork / rollback /
free with the same semantics. The data path is native:

* ``append`` scatters rows with the ``rope_append`` kernel (optionally rotating
  K at its positions on the way in, as Attention.forward does before appending,
  engine/model/block.py:53-64) instead of ceil(L/bs)+1 slice copies;
* ``gather`` is the bit-exact ``gather_kv`` kernel;
* ``device_tables`` packs several sequences' block lists into the int32
  (B, max_blocks) table + (B,) lengths that ``paged_attention`` reads.

Pools live on a CUDA device; there is no CPU data path.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from engine.cache.allocator import BlockAllocator
from engine.cache.block_table import BlockTable


@dataclass
class KVCacheConfig:
    num_layers: int
    num_kv_heads: int
    head_dim: int
    num_blocks: int
    block_size: int
    dtype: torch.dtype = torch.bfloat16
    device: torch.device | str = "cuda"

    def bytes_required(self) -> int:
        """Total VRAM footprint across all layers and K+V."""
        per_elem = torch.tensor([], dtype=self.dtype).element_size()
        return (2 * self.num_layers * self.num_blocks * self.block_size * self.num_kv_heads *
                self.head_dim * per_elem)


class PagedKVCache:
    def __init__(self, cfg: KVCacheConfig):
        device = torch.device(cfg.device)
        if device.type != "cuda":
            raise RuntimeError("PagedKVCache requires a CUDA device (no CPU data path)")
        if cfg.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"KV cache dtype must be bf16 or fp16, got {cfg.dtype}")
        free, _ = torch.cuda.mem_get_info(device)
        need = cfg.bytes_required()
        if need > free:
            raise RuntimeError(f"PagedKVCache would need {need / 2**30:.2f} GiB but only "
                               f"{free / 2**30:.2f} GiB free on {device}")
        self.cfg = cfg
        shape = (cfg.num_blocks, cfg.block_size, cfg.num_kv_heads, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=cfg.dtype, device=device) for _ in range(cfg.num_layers)]
        self.v = [torch.zeros(shape, dtype=cfg.dtype, device=device) for _ in range(cfg.num_layers)]
        self.alloc = BlockAllocator(cfg.num_blocks, cfg.block_size)

    # --- reference-compatible surface ---
    @property
    def device(self) -> torch.device:
        return self.k[0].device

    @property
    def dtype(self) -> torch.dtype:
        return self.k[0].dtype

    @property
    def _free(self) -> list[int]:
        return self.alloc._free

    def new_sequence(self) -> BlockTable:
        return self.alloc.new_sequence()

    def free_sequence(self, table: BlockTable) -> None:
        self.alloc.free_sequence(table)

    def _validate(self, t: torch.Tensor) -> None:
        if t.device != self.device or t.dtype != self.dtype:
            raise ValueError(f"tensor device/dtype ({t.device}/{t.dtype}) does not match "
                             f"cache ({self.device}/{self.dtype})")

    def _table_tensor(self, table: BlockTable) -> torch.Tensor:
        return torch.tensor([table.blocks or [0]], dtype=torch.int32).to(self.device,
                                                                           non_blocking=True)

    def append(self, layer: int, table: BlockTable, k: torch.Tensor, v: torch.Tensor,
               start: int | None = None, rope: tuple[torch.Tensor, torch.Tensor] | None = None
               ) -> None:
        """Write k, v of shape (L, num_kv_heads, head_dim) at positions start..start+L-1.

        With ``rope`` = (cos, sin) fp32 tables, K rows are rotated at their positions.
        """
        from kernels.flash_attention import rope_append

        L = k.shape[0]
        if v.shape[0] != L:
            raise ValueError("k and v must have the same number of rows")
        self._validate(k)
        self._validate(v)
        if start is None:
            start = table.length
        end = start + L
        self.alloc.reserve(table, end)
        if L > 0:
            rope_append(k.unsqueeze(0), v.unsqueeze(0), self.k[layer], self.v[layer],
                        self._table_tensor(table),
                        torch.tensor([start], dtype=torch.int32).to(self.device, non_blocking=True),
                        rope=rope)
        if end > table.length:
            table.length = end

    def gather(self, layer: int, table: BlockTable) -> tuple[torch.Tensor, torch.Tensor]:
        """Dense (L, Hk, D) copies of the sequence's K and V (bit-exact)."""
        from kernels.flash_attention import gather_kv

        L = table.length
        shape = (L, self.cfg.num_kv_heads, self.cfg.head_dim)
        if L == 0:
            empty = self.k[layer].new_zeros(shape)
            return empty, empty.clone()
        tab = self._table_tensor(table)
        lens = torch.tensor([L], dtype=torch.int32).to(self.device, non_blocking=True)
        k = gather_kv(self.k[layer], tab, lens, out_len=L)[0]
        v = gather_kv(self.v[layer], tab, lens, out_len=L)[0]
        return k, v

    def fork(self, table: BlockTable) -> BlockTable:
        """A new BlockTable whose K/V are a deep copy of ``table``'s (kv_cache.py:169-185)."""
        new_blocks = self.alloc.fork_blocks(table)
        if new_blocks:
            src = torch.tensor(table.blocks, dtype=torch.long, device=self.device)
            dst = torch.tensor(new_blocks, dtype=torch.long, device=self.device)
            for layer in range(self.cfg.num_layers):
                self.k[layer].index_copy_(0, dst, self.k[layer].index_select(0, src))
                self.v[layer].index_copy_(0, dst, self.v[layer].index_select(0, src))
        return BlockTable(block_size=self.cfg.block_size, blocks=new_blocks, length=table.length)

    def rollback(self, table: BlockTable, new_length: int) -> None:
        self.alloc.rollback(table, new_length)

    def stats(self) -> dict:
        total = self.cfg.num_blocks
        free = self.alloc.num_free
        return {"bytes": self.cfg.bytes_required(), "total_blocks": total,
                "allocated_blocks": total - free, "free_blocks": free}

    # --- batched access for the kernels ---
    def device_tables(self, tables: list[BlockTable]) -> tuple[torch.Tensor, torch.Tensor]:
        """int32 (B, max_blocks) block table and int32 (B,) lengths on the cache's device."""
        return pack_tables(tables, self.device)


def pack_tables(tables: list[BlockTable], device) -> tuple[torch.Tensor, torch.Tensor]:
    """Pack per-sequence block lists into the (B, max_blocks) int32 layout the kernels read.

    Unused tail entries are 0 (never read: the kernels stop at each sequence's length).
    """
    width = max([len(t.blocks) for t in tables] + [1])
    rows = [t.blocks + [0] * (width - len(t.blocks)) for t in tables]
    tab = torch.tensor(rows, dtype=torch.int32)
    lens = torch.tensor([t.length for t in tables], dtype=torch.int32)
    if torch.device(device).type == "cuda":
        tab = tab.pin_memory().to(device, non_blocking=True)
        lens = lens.pin_memory().to(device, non_blocking=True)
    return tab, lens
