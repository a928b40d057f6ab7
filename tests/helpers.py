"""Shared helpers for the parity tests."""

from __future__ import annotations

import numpy as np

# Tolerance of the north-star contract: the kernel against the reference's fp32
# attention + RoPE on the same bf16-rounded inputs.
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def assert_close_attn(out, ref, max_abs: float = MAX_ABS, mean_abs: float = MEAN_ABS, what=""):
    """max |out - ref| <= max_abs and mean |out - ref| <= mean_abs; NaN rows must agree."""
    out = np.asarray(out, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert out.shape == ref.shape, (what, out.shape, ref.shape)
    nan_o, nan_r = np.isnan(out), np.isnan(ref)
    assert np.array_equal(nan_o, nan_r), f"{what}: NaN pattern differs ({nan_o.sum()} vs {nan_r.sum()})"
    ok = ~nan_r
    if not ok.any():
        return
    err = np.abs(out[ok] - ref[ok])
    mx, mean = float(err.max()), float(err.mean())
    assert mx <= max_abs and mean <= mean_abs, f"{what}: max abs {mx:.3e}, mean abs {mean:.3e}"


def to_torch(x: np.ndarray, dtype, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=dtype)


def to_np(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()
