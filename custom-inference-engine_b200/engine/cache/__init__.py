from engine.cache.allocator import BlockAllocator
from engine.cache.block_table import BlockTable
from engine.cache.kv_cache import KVCacheConfig, PagedKVCache, pack_tables

__all__ = ["PagedKVCache", "KVCacheConfig", "BlockTable", "BlockAllocator", "pack_tables"]
