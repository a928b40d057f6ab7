"""Engine-side attention call site.

``flash_attention`` keeps the signature and checks of the reference's call
site (engine/attention.py:6-32) minus its fp16-only rule: bf16 and fp16 both
run on the B200 kernels.

``attention_forward`` is the body of the reference's Attention.forward between
the QKV projections and o_proj (engine/model/block.py:53-71) — rotate q and k,
append K/V to the paged cache, attend over the history — done with fused
kernels: RoPE of K happens inside the paged append, RoPE of q inside the
attention kernel, and the dense history gather is skipped for decode and
speculative verify (the paged kernel reads the block table directly).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from engine.cache.block_table import BlockTable
from engine.cache.kv_cache import PagedKVCache

# Query rows per kv head up to which the paged split-KV kernel serves a call;
# longer query blocks (prefill) go to the tcgen05 prefill kernel.
PAGED_MAX_ROWS = 64


def flash_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    scale: float | None = None,
) -> torch.Tensor:
    """Flash attention on CUDA. Shapes: q (B, H, M, D); k/v (B, Hk, N, D). Supports GQA."""
    if not q.is_cuda:
        raise RuntimeError("flash_attention requires CUDA tensors")
    D = q.shape[-1]
    if D & (D - 1):
        raise ValueError(f"head_dim must be power of 2, got {D}")
    if D < 16:
        raise ValueError(f"head_dim must be >= 16, got {D}")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"flash_attention expects FP16 or BF16 Q/K/V, got {q.dtype}")
    from kernels.flash_attention import flash_attention as _flash_attention

    return _flash_attention(q, k, v, causal=causal, scale=scale)


def attention_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cache: PagedKVCache,
    layer_idx: int,
    table: BlockTable,
    start: int | None = None,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    scale: float | None = None,
) -> torch.Tensor:
    """Causal attention of L new tokens against the sequence's whole history.

    q: (1, Hq, L, d); k, v: (1, Hkv, L, d) — not yet rotated. The new tokens sit
    at positions start..start+L-1 (default: the table's current length). K/V are
    appended to the cache (K rotated with ``rope`` on the way in), then q attends
    bottom-right causally to all table.length keys. Returns (1, Hq, L, d).
    """
    from kernels.flash_attention import flash_attention as _fa
    from kernels.flash_attention import gather_kv, paged_attention

    if q.shape[0] != 1:
        raise ValueError("attention_forward serves one sequence (B == 1), as the reference")
    _, Hq, L, d = q.shape
    Hkv = k.shape[1]
    if start is None:
        start = table.length
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    cache.append(layer_idx, table, k[0].transpose(0, 1), v[0].transpose(0, 1), start=start,
                 rope=rope)
    N = table.length
    if start + L != N:
        raise ValueError(f"new tokens end at {start + L} but the history holds {N}")
    if (Hq // Hkv) * L <= PAGED_MAX_ROWS:
        tab, lens = cache.device_tables([table])
        return paged_attention(q, cache.k[layer_idx], cache.v[layer_idx], tab, lens, True,
                               scale, rope=rope)
    if N == L:
        # whole sequence in this call: attend over the new tokens directly
        return _fa(q, k, v, True, scale, rope=rope, rope_q_pos0=start, rope_k=True)
    hk, hv = cache.gather(layer_idx, table)  # rotated K as stored
    return _fa(q, hk.transpose(0, 1).unsqueeze(0), hv.transpose(0, 1).unsqueeze(0), True, scale,
               rope=rope, rope_q_pos0=start, rope_k=False)


@dataclass
class BatchStep:
    """One forward step of a batch of sequences that each add ``new_tokens`` tokens
    (decode: 1; speculative verify: gamma + 1; a batch of fresh prompts: L).

    Built once per step by :func:`begin_step` and shared by every layer: the new
    tokens' blocks are reserved and all block tables are packed into the device
    layout the kernels read a single time, where the reference packs
    ``torch.tensor(blocks)`` per layer inside ``PagedKVCache.gather``
    (engine/cache/kv_cache.py:141-165) and serves one sequence at a time
    (engine/model/block.py:48).
    """

    tables: list[BlockTable]
    new_tokens: int
    starts: list[int]             # host copy: first new position of each sequence
    block_tables: torch.Tensor    # int32 (B, max_blocks) on the cache's device
    kv_lens: torch.Tensor         # int32 (B,) lengths after the step
    start_pos: torch.Tensor       # int32 (B,) = starts, on the device


def begin_step(cache: PagedKVCache, tables: list[BlockTable], new_tokens: int) -> BatchStep:
    """Reserve ``new_tokens`` positions at the end of every table and pack the tables."""
    if not tables:
        raise ValueError("begin_step needs at least one sequence")
    if new_tokens <= 0:
        raise ValueError(f"new_tokens must be positive, got {new_tokens}")
    starts = [t.length for t in tables]
    for t, s in zip(tables, starts):
        cache.alloc.reserve(t, s + new_tokens)
        t.length = s + new_tokens
    tab, lens = cache.device_tables(tables)
    start_pos = torch.tensor(starts, dtype=torch.int32)
    if torch.device(cache.device).type == "cuda":
        start_pos = start_pos.pin_memory().to(cache.device, non_blocking=True)
    return BatchStep(tables=list(tables), new_tokens=new_tokens, starts=starts,
                     block_tables=tab, kv_lens=lens, start_pos=start_pos)


def attention_forward_batch(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cache: PagedKVCache,
    layer_idx: int,
    step: BatchStep,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    scale: float | None = None,
) -> torch.Tensor:
    """Causal attention of a batch step: q (B, Hq, L, d), k/v (B, Hkv, L, d) not yet
    rotated, L == step.new_tokens, token i of sequence b at position
    step.starts[b] + i. One fused RoPE + paged append writes every sequence's K/V;
    decode / verify blocks (Hq/Hkv * L <= 64 rows per kv head) then take one
    split-KV paged attention launch over the whole batch. Longer blocks go to the
    tcgen05 prefill kernel: in one launch when every history is empty, else per
    sequence over its gathered history. Returns (B, Hq, L, d).
    """
    from kernels.flash_attention import flash_attention as _fa
    from kernels.flash_attention import paged_attention, rope_append

    B, Hq, L, d = q.shape
    Hkv = k.shape[1]
    if B != len(step.tables) or L != step.new_tokens:
        raise ValueError(f"q is ({B} sequences, {L} tokens) but the step holds "
                         f"({len(step.tables)}, {step.new_tokens})")
    if k.shape != (B, Hkv, L, d) or v.shape != k.shape:
        raise ValueError("k and v must be (B, Hkv, L, d) like q")
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    rope_append(k.transpose(1, 2), v.transpose(1, 2), cache.k[layer_idx], cache.v[layer_idx],
                step.block_tables, step.start_pos, rope=rope)
    if (Hq // Hkv) * L <= PAGED_MAX_ROWS:
        return paged_attention(q, cache.k[layer_idx], cache.v[layer_idx], step.block_tables,
                               step.kv_lens, True, scale, rope=rope)
    if all(s == 0 for s in step.starts):
        return _fa(q, k, v, True, scale, rope=rope, rope_q_pos0=0, rope_k=True)
    outs = []
    for b, table in enumerate(step.tables):
        hk, hv = cache.gather(layer_idx, table)
        outs.append(_fa(q[b:b + 1], hk.transpose(0, 1).unsqueeze(0),
                        hv.transpose(0, 1).unsqueeze(0), True, scale, rope=rope,
                        rope_q_pos0=step.starts[b], rope_k=False))
    return torch.cat(outs, 0)
