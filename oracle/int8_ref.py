"""Weight-only INT8 GEMM — TEST INFRASTRUCTURE ONLY (numpy restatement).

Follows kernels/ref/int8_matmul_ref.py of the reference:
* ``dequantize_int8``  :7-28  per-channel scales (N,) or per-group (N, K/group)
* ``int8_matmul``      :31-47 y = x @ dequantize(w, scales).T (+ bias), computed
                       in fp32 and returned in x's dtype.
"""

from __future__ import annotations

import numpy as np


def dequantize_int8(w_int8: np.ndarray, scales: np.ndarray, group_size: int | None = None):
    w = w_int8.astype(np.float32)
    s = scales.astype(np.float32)
    if group_size is None or s.ndim == 1:
        return w * s[:, None]
    out, in_ = w.shape
    assert in_ % group_size == 0 and s.shape == (out, in_ // group_size)
    return (w.reshape(out, -1, group_size) * s[:, :, None]).reshape(out, in_)


def int8_matmul(x: np.ndarray, w_int8: np.ndarray, scales: np.ndarray,
                group_size: int | None = None, bias: np.ndarray | None = None) -> np.ndarray:
    w = dequantize_int8(w_int8, scales, group_size)
    y = x.astype(np.float32) @ w.T
    if bias is not None:
        y = y + bias.astype(np.float32)
    return y.astype(x.dtype)
