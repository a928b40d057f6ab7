"""RoPE cos/sin tables for the fused kernels.

Same table as the reference's ``build_rope_cache`` (kernels/ref/rope_apply_ref.py:6-19):
inv_freq = 1 / theta ** (arange(0, d, 2) / d) in fp32, angles = outer(t, inv_freq),
returned as fp32 (max_seq_len, d/2) cos and sin. The kernels always read fp32
tables, whatever the activation dtype (the reference engine casts these buffers to
the activation dtype at engine/runtime.py:33-37; the fused kernels keep fp32).
"""

from __future__ import annotations

import torch


def build_rope_cache(
    max_seq_len: int,
    head_dim: int,
    theta: float = 10000.0,
    device: torch.device | str = "cpu",
    dtype: torch.dtype = torch.float32,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Return (cos, sin), each (max_seq_len, head_dim // 2), contiguous."""
    if head_dim % 2:
        raise ValueError(f"head_dim must be even for RoPE, got {head_dim}")
    exponent = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
    inv_freq = 1.0 / (theta ** exponent)
    t = torch.arange(max_seq_len, dtype=torch.float32)
    angles = torch.outer(t, inv_freq)
    cos = angles.cos().to(dtype).contiguous()
    sin = angles.sin().to(dtype).contiguous()
    return cos.to(device), sin.to(device)
