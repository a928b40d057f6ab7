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

``fused_attention_forward`` is a drop-in for the whole ``Attention.forward``
of the reference's decoder block (engine/model/block.py:39-75): the same
arguments (x, layer_idx, cache, table, positions), the same projections
(the module's own q/k/v/o ``Int8Linear``s) and the same result, with the
attention in between done by ``attention_forward``. ``use_fused_attention``
binds it onto every such module of a model; ``rope_tables`` turns the
engine's ``RotaryEmbedding`` (whose buffers the runtime casts to fp16,
engine/runtime.py:22-37) into the fp32 tables the kernels read.
"""

from __future__ import annotations

import math
import weakref
from dataclasses import dataclass

import torch

from engine.cache.block_table import BlockTable
from engine.cache.kv_cache import PagedKVCache

# Query rows per kv head up to which the paged split-KV kernel serves a call;
# longer query blocks (prefill) go to the tcgen05 prefill kernel.
PAGED_MAX_ROWS = 64


def _paged_long_ok(cache: PagedKVCache, d: int) -> bool:
    """Long query blocks over a history read the pools through the block table on
    the tcgen05 kernel when its 16-token boxes fit the cache geometry."""
    return cache.cfg.block_size % 16 == 0 and d in (64, 128)


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
    if _paged_long_ok(cache, d):
        # chunked prefill: the tcgen05 kernel reads the history through the table
        tab, lens = cache.device_tables([table])
        return paged_attention(q, cache.k[layer_idx], cache.v[layer_idx], tab, lens, True,
                               scale, rope=rope)
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
    tcgen05 prefill kernel in one launch too: over the new tokens when every
    history is empty, else reading each sequence's history through the block
    table (block sizes that are multiples of 16, d 64 / 128; other geometries
    gather each history and launch per sequence). Returns (B, Hq, L, d).
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
    if _paged_long_ok(cache, d):
        return paged_attention(q, cache.k[layer_idx], cache.v[layer_idx], step.block_tables,
                               step.kv_lens, True, scale, rope=rope)
    outs = []
    for b, table in enumerate(step.tables):
        hk, hv = cache.gather(layer_idx, table)
        outs.append(_fa(q[b:b + 1], hk.transpose(0, 1).unsqueeze(0),
                        hv.transpose(0, 1).unsqueeze(0), True, scale, rope=rope,
                        rope_q_pos0=step.starts[b], rope_k=False))
    return torch.cat(outs, 0)


# ------------------------------------------------------------------ drop-in block forward
_ROPE_CACHE: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()


def rope_tables(rope) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 (cos, sin) tables for the fused kernels.

    ``rope`` is either a ``(cos, sin)`` pair or the engine's ``RotaryEmbedding``
    (engine/model/rope.py:9-19, buffers ``cos`` / ``sin`` of shape
    (max_seq_len, head_dim/2)). The engine casts those buffers to the activation
    dtype (engine/runtime.py:22-37); widening fp16 / bf16 back to fp32 is exact,
    so the kernels rotate with the very table values the engine's
    ``apply_rotary_ref`` uses, in fp32 arithmetic. The widened pair is made once
    per module and reused until its buffers change (another cast or ``.to``).
    """
    if isinstance(rope, (tuple, list)):
        cos, sin = rope
        if cos.dtype == torch.float32 and sin.dtype == torch.float32:
            return cos, sin
        return cos.float().contiguous(), sin.float().contiguous()
    cos, sin = rope.cos, rope.sin
    key = (cos.data_ptr(), sin.data_ptr(), cos._version, sin._version, cos.dtype, cos.device)
    hit = _ROPE_CACHE.get(rope)
    if hit is not None and hit[0] == key:
        return hit[1]
    tabs = (cos.float().contiguous(), sin.float().contiguous()) if cos.dtype != torch.float32 \
        else (cos.contiguous(), sin.contiguous())
    _ROPE_CACHE[rope] = (key, tabs)
    return tabs


def _first_position(positions: torch.Tensor | None, table: BlockTable, L: int,
                    layer_idx: int) -> int:
    """First absolute position of the new tokens.

    The reference reads ``positions[0]`` with ``.item()`` in every layer
    (engine/model/block.py:57). TransformerLM hands the same ``positions``
    tensor to all layers of one forward, so the value is read once per forward
    and remembered on that tensor; positions held on the host cost no sync.
    """
    if positions is None:
        # layer 0 appends first; later layers see the grown table
        return table.length if layer_idx == 0 else table.length - L
    hit = getattr(positions, "_cie_first_position", None)
    if hit is not None and hit[0] == positions._version:
        return hit[1]
    start = int(positions.reshape(-1)[0].item())
    positions._cie_first_position = (positions._version, start)
    return start


def fused_attention_forward(attn, x: torch.Tensor, layer_idx: int, cache: PagedKVCache,
                            table: BlockTable, positions: torch.Tensor | None = None
                            ) -> torch.Tensor:
    """Drop-in body of the reference's ``Attention.forward`` (engine/model/block.py:39-75).

    ``attn`` is the engine's attention module (its ``q_proj``, ``k_proj``,
    ``v_proj``, ``o_proj``, ``rope``, ``num_heads``, ``num_kv_heads`` and
    ``head_dim`` are used as they are). x: (1, L, hidden); positions: (L,)
    consecutive absolute positions of the new tokens. The projections run as in
    the reference; RoPE of K is fused into the paged append, RoPE of q into the
    attention kernel, and decode / verify read the paged history directly (no
    gather). Returns o_proj(attention) of shape (1, L, hidden), like the
    reference.
    """
    B, L, _ = x.shape
    if B != 1:
        raise ValueError("batch size must be 1 (engine/model/block.py:48)")
    hq, hkv, d = attn.num_heads, attn.num_kv_heads, attn.head_dim
    q = attn.q_proj(x).view(B, L, hq, d).transpose(1, 2)
    k = attn.k_proj(x).view(B, L, hkv, d).transpose(1, 2)
    v = attn.v_proj(x).view(B, L, hkv, d).transpose(1, 2)
    start = _first_position(positions, table, L, layer_idx)
    out = attention_forward(q, k, v, cache, layer_idx, table, start=start,
                            rope=rope_tables(attn.rope), scale=1.0 / math.sqrt(d))
    out = out.transpose(1, 2).contiguous().view(B, L, hq * d)
    return attn.o_proj(out)


def _is_engine_attention(mod) -> bool:
    return all(hasattr(mod, a) for a in ("q_proj", "k_proj", "v_proj", "o_proj", "rope",
                                         "num_heads", "num_kv_heads", "head_dim"))


def use_fused_attention(model) -> int:
    """Route every engine attention module of ``model`` through
    :func:`fused_attention_forward` (bound per instance; the engine's classes are
    not modified). Returns the number of modules rerouted."""
    n = 0
    for mod in model.modules():
        if _is_engine_attention(mod):
            mod.forward = fused_attention_forward.__get__(mod)
            n += 1
    return n
