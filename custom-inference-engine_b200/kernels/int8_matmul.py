"""Weight-only INT8 GEMM on B200 (sm_100a tensor cores).

``int8_matmul`` is the drop-in for the reference's Triton entry
(kernels/int8_matmul.py:76-110): y = x @ (w_int8 * scales[:, None]).T (+ bias),
per-channel fp scales of shape (N,), fp32 accumulation, y in x's dtype, the
same exception types for bad input (:83-86) and the same shape check (:93).
bf16 and fp16 activations are both accepted. The int8 weights are widened to
x's dtype in registers (exact for int8) and either held in tensor memory as the
A operand of tcgen05 MMAs or fed to mma.sync for the smallest batches; the
scale (and bias) are applied once to the fp32 accumulator, and the result is
rounded once to x's dtype, as the reference's fp32 formula
(kernels/ref/int8_matmul_ref.py:31-47) does. The Triton path instead rounds
x @ w * s to x's dtype and then adds the rounded bias (:107-108), so with a
bias the two can differ by one unit in the last place of x's dtype.
"""

from __future__ import annotations

import torch

from kernels import _lib

_DTYPES = {torch.bfloat16: _lib.CIE_DTYPE_BF16, torch.float16: _lib.CIE_DTYPE_FP16}


def int8_matmul(
    x: torch.Tensor,
    w_int8: torch.Tensor,
    scales: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """Per-channel INT8 x FP16/BF16 matmul on CUDA. x: (..., K), w_int8: (N, K)."""
    if not x.is_cuda:
        raise RuntimeError("int8_matmul requires CUDA tensors")
    if scales.ndim != 1:
        raise ValueError("int8_matmul expects per-channel scales with shape (N,)")
    if x.dtype not in _DTYPES:
        raise ValueError(f"int8_matmul expects FP16 or BF16 activations, got {x.dtype}")
    if w_int8.dtype != torch.int8 or w_int8.ndim != 2:
        raise ValueError("int8_matmul expects int8 weights of shape (N, K)")
    lib = _lib.load()

    x_2d = x.reshape(-1, x.shape[-1])
    M, K = x_2d.shape
    N, K2 = w_int8.shape
    assert K == K2
    if scales.shape[0] != N:
        raise ValueError(f"scales has {scales.shape[0]} entries for {N} output channels")
    # The kernels need 16-byte aligned rows; a copy (padded rows when K does not
    # fill 16 bytes) fixes any other layout, including a contiguous view at an
    # unaligned offset, which .contiguous() would hand back unchanged.
    if x_2d.stride(1) != 1 or x_2d.stride(0) % 8 or x_2d.data_ptr() % 16:
        x_2d = x_2d.clone(memory_format=torch.contiguous_format)
        if K % 8:
            x_2d = torch.nn.functional.pad(x_2d, (0, 8 - K % 8))[:, :K]
    if w_int8.stride(1) != 1 or w_int8.stride(0) % 16 or w_int8.data_ptr() % 16:
        w_int8 = w_int8.clone(memory_format=torch.contiguous_format)
        if K % 16:
            w_int8 = torch.nn.functional.pad(w_int8, (0, 16 - K % 16))[:, :K]
    s32 = scales.to(device=x.device, dtype=torch.float32).contiguous()
    b32 = bias.to(device=x.device, dtype=torch.float32).contiguous() if bias is not None else None
    y = torch.empty((M, N), device=x.device, dtype=x.dtype)
    if M > 0:
        ws_n = lib.cie_int8_matmul_workspace(M, N, K)
        ws = torch.empty(ws_n, dtype=torch.uint8, device=x.device) if ws_n else None
        rc = lib.cie_int8_matmul(
            x_2d.data_ptr(), w_int8.data_ptr(), s32.data_ptr(),
            b32.data_ptr() if b32 is not None else None, y.data_ptr(), M, N, K,
            x_2d.stride(0), w_int8.stride(0), y.stride(0), _DTYPES[x.dtype],
            ws.data_ptr() if ws is not None else None, ws_n,
            torch.cuda.current_stream(x.device).cuda_stream)
        _lib.check(rc, "int8_matmul")
    return y.reshape(*x.shape[:-1], N)
