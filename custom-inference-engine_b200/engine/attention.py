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
