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
  (B, max_blocks) table + (B,) lengths that ``paged_attention`` reads;
* ``fork`` copies the blocks with the ``copy_blocks`` kernel (one launch per
  pool) instead of an index_select + index_copy_ per layer.

Block tables reach the device through pinned host buffers and non-blocking
copies, and a packed table is reused for as long as the sequence's blocks and
length are unchanged: every layer of one forward step shares the copy the first
layer made, where the reference builds ``torch.tensor(blocks)`` per layer
(engine/cache/kv_cache.py:154). Pools live on a CUDA device; there is no CPU
data path.
"""

from __future__ import annotations

import ctypes
from collections import OrderedDict
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
        # (kind, key) -> device tensor; small LRU of packed tables / positions
        self._packed: OrderedDict = OrderedDict()

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

    _PACK_CACHE = 64

    def _cached(self, key, make):
        hit = self._packed.get(key)
        if hit is not None:
            self._packed.move_to_end(key)
            return hit
        val = make()
        self._packed[key] = val
        if len(self._packed) > self._PACK_CACHE:
            self._packed.popitem(last=False)
        return val

    def _table_tensor(self, table: BlockTable) -> torch.Tensor:
        """int32 (1, n_blocks) device copy of the table's block ids (cached)."""
        blocks = tuple(table.blocks) or (0,)
        return self._cached(("blocks", blocks), lambda: _to_device(
            torch.tensor([blocks], dtype=torch.int32), self.device))

    def _int_tensor(self, value: int) -> torch.Tensor:
        """int32 (1,) device tensor holding ``value`` (cached)."""
        return self._cached(("int", int(value)), lambda: _to_device(
            torch.tensor([int(value)], dtype=torch.int32), self.device))

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
                        self._table_tensor(table), self._int_tensor(start), rope=rope)
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
        lens = self._int_tensor(L)
        k = gather_kv(self.k[layer], tab, lens, out_len=L)[0]
        v = gather_kv(self.v[layer], tab, lens, out_len=L)[0]
        return k, v

    def fork(self, table: BlockTable) -> BlockTable:
        """A new BlockTable whose K/V are a deep copy of ``table``'s (kv_cache.py:169-185).

        The new blocks come from the LIFO free list in logical order, as in the
        reference; the data moves with one ``copy_blocks`` launch per pool, fed by
        block ids copied from pinned memory without a host sync.
        """
        from kernels import _lib
        from kernels.flash_attention import _require, _stream

        new_blocks = self.alloc.fork_blocks(table)
        n = len(new_blocks)
        if n:
            lib = _require()
            ids = _to_device(torch.tensor([table.blocks, new_blocks], dtype=torch.int32),
                             self.device)
            pools = self.k + self.v
            arr = (ctypes.c_void_p * len(pools))(*[p.data_ptr() for p in pools])
            block_bytes = self.k[0][0].numel() * self.k[0].element_size()
            rc = lib.cie_copy_blocks(arr, len(pools), ctypes.c_void_p(ids[0].data_ptr()),
                                     ctypes.c_void_p(ids[1].data_ptr()), n, self.cfg.num_blocks,
                                     block_bytes, _stream(self.k[0]))
            _lib.check(rc, "fork")
        return BlockTable(block_size=self.cfg.block_size, blocks=new_blocks, length=table.length)

    def rollback(self, table: BlockTable, new_length: int) -> None:
        self.alloc.rollback(table, new_length)

    def stats(self, verbose: bool = True) -> dict:
        """Footprint and block usage; printed like the reference's ``stats``
        (engine/cache/kv_cache.py:196-210) and also returned."""
        total = self.cfg.num_blocks
        free = self.alloc.num_free
        out = {"bytes": self.cfg.bytes_required(), "total_blocks": total,
               "allocated_blocks": total - free, "free_blocks": free}
        if verbose:
            print(f"Cache Memory Footprint: {out['bytes']}")
            print(f"Total Blocks: {total}")
            print(f"Allocated Blocks: {total - free}")
            print(f"Freed Blocks: {free}")
        return out

    # --- batched access for the kernels ---
    def device_tables(self, tables: list[BlockTable]) -> tuple[torch.Tensor, torch.Tensor]:
        """int32 (B, max_blocks) block table and int32 (B,) lengths on the cache's device.

        Reused while the tables are unchanged (same blocks and lengths), so the
        layers of one step share a single host-to-device copy."""
        key = ("tables", tuple((t.length, tuple(t.blocks)) for t in tables))
        return self._cached(key, lambda: pack_tables(tables, self.device))


def _to_device(t: torch.Tensor, device) -> torch.Tensor:
    """Copy a small host tensor to ``device`` through pinned memory, without a host sync."""
    if torch.device(device).type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t.to(device)


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
