"""CPU oracle for the attention hot path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's own CPU path:

* ``build_rope_cache`` / ``apply_rotary``   kernels/ref/rope_apply_ref.py:6-53
* ``attention``                             kernels/ref/flash_attention_ref.py:8-56
* ``PagedKVCacheRef`` / ``BlockTableRef``   engine/cache/kv_cache.py:34-194,
                                            engine/cache/block_table.py:6-36
* ``int8_matmul`` / ``dequantize_int8``     kernels/ref/int8_matmul_ref.py:7-47

Parity is pinned: tests/test_oracle_golden.py checks these functions against
golden vectors produced by the reference itself (tests/golden/make_golden.py
imports the reference's kernels.ref and engine.cache and records their
outputs on seeded inputs).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this package, and only as the checker or the timed CPU baseline. The product
(custom-inference-engine_b200/) never imports it and has no CPU fallback.
"""

from oracle.attention_ref import (
    apply_rotary,
    attention,
    bf16_round,
    build_rope_cache,
    decode_case_ref,
    prefill_case_ref,
)
from oracle.int8_ref import dequantize_int8, int8_matmul
from oracle.kv_cache_ref import BlockTableRef, PagedKVCacheRef, gather_tables

__all__ = [
    "apply_rotary",
    "attention",
    "bf16_round",
    "build_rope_cache",
    "prefill_case_ref",
    "decode_case_ref",
    "BlockTableRef",
    "PagedKVCacheRef",
    "gather_tables",
    "dequantize_int8",
    "int8_matmul",
]
