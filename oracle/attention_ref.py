"""numpy fp32 restatement of the reference attention + RoPE (test oracle only).

Follows, step for step:
  build_rope_cache   kernels/ref/rope_apply_ref.py:6-19
  apply_rotary       kernels/ref/rope_apply_ref.py:22-53
  attention          kernels/ref/flash_attention_ref.py:8-56
All arithmetic is float32 with one rounding per elementwise op, as torch does
on CPU for these expressions.
"""

from __future__ import annotations

import math

import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def build_rope_cache(max_seq_len: int, head_dim: int, theta: float = 10000.0):
    """(cos, sin), each float32 (max_seq_len, head_dim // 2).  rope_apply_ref.py:6-19"""
    assert head_dim % 2 == 0
    exponent = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    # theta ** exponent correctly rounded to fp32 (evaluated in fp64), as torch's
    # fp32 pow returns; then the fp32 reciprocal and fp32 outer product
    powed = np.power(np.float64(theta), exponent.astype(np.float64)).astype(np.float32)
    inv_freq = np.float32(1.0) / powed
    t = np.arange(max_seq_len, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    # cos / sin of the fp32 angles, rounded once to fp32 (within 1 ulp of torch)
    f64 = freqs.astype(np.float64)
    return np.cos(f64).astype(np.float32), np.sin(f64).astype(np.float32)


def apply_rotary(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, positions=None) -> np.ndarray:
    """Half-split rotation of x (B, H, L, D) at ``positions`` (L,) or (B, L).

    rope_apply_ref.py:22-53: out = cat(x1*c - x2*s, x1*s + x2*c).
    """
    B, H, L, D = x.shape
    if positions is None:
        positions = np.arange(L)
    positions = np.asarray(positions)
    if positions.ndim == 1:
        c = cos[positions].reshape(1, 1, L, D // 2)
        s = sin[positions].reshape(1, 1, L, D // 2)
    else:
        c = cos[positions].reshape(B, 1, L, D // 2)
        s = sin[positions].reshape(B, 1, L, D // 2)
    x = x.astype(np.float32, copy=False)
    x1 = x[..., : D // 2]
    x2 = x[..., D // 2:]
    rot1 = x1 * c - x2 * s
    rot2 = x1 * s + x2 * c
    return np.concatenate([rot1, rot2], axis=-1).astype(np.float32)


def attention(q, k, v, mask=None, causal: bool = False, scale: float | None = None) -> np.ndarray:
    """fp32 scaled-dot-product attention, GQA by head broadcast.  flash_attention_ref.py:8-56

    q (B, H, Lq, D), k/v (B, Hk, Lk, D); causal is bottom-right aligned: query i
    sees keys j <= Lk - Lq + i. Fully masked rows give NaN, an empty key axis
    gives zeros, as torch.softmax / matmul do.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    B, H, Lq, D = q.shape
    Hk, Lk = k.shape[1], k.shape[2]
    if Hk != H:
        assert H % Hk == 0
        k = np.repeat(k, H // Hk, axis=1)
        v = np.repeat(v, H // Hk, axis=1)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if Lk == 0:
        return np.zeros((B, H, Lq, D), dtype=np.float32)
    scores = np.matmul(q, np.swapaxes(k, -1, -2)) * np.float32(scale)
    if causal:
        i = np.arange(Lq)[:, None]
        j = np.arange(Lk)[None, :]
        scores = np.where(j > (Lk - Lq + i), np.float32(-np.inf), scores)
    if mask is not None:
        scores = scores + mask
    mx = scores.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp(scores - mx)
        probs = e / e.sum(axis=-1, keepdims=True)
    return np.matmul(probs, v).astype(np.float32)


def prefill_case_ref(q, k, v, cos, sin, causal=True, scale=None, q_pos0=None, rope_k=True):
    """The fused-RoPE prefill contract: rotate q (positions q_pos0 + i, default
    N - M + i) and k (positions 0..N-1) in fp32, then fp32 attention."""
    M, N = q.shape[2], k.shape[2]
    if q_pos0 is None:
        q_pos0 = N - M
    if cos is not None:
        q = apply_rotary(q, cos, sin, np.arange(q_pos0, q_pos0 + M))
        if rope_k:
            k = apply_rotary(k, cos, sin, np.arange(N))
    return attention(q, k, v, causal=causal, scale=scale)


def decode_case_ref(q, k_hist, v_hist, cos, sin, causal=True, scale=None):
    """One sequence of the paged decode / verify contract.

    q (1, Hq, M, D) raw; k_hist/v_hist (1, Hkv, L, D) with K already rotated as
    stored. Query i is rotated at position L - M + i.
    """
    M, L = q.shape[2], k_hist.shape[2]
    if cos is not None:
        q = apply_rotary(q, cos, sin, np.arange(L - M, L))
    return attention(q, k_hist, v_hist, causal=causal, scale=scale)
