"""Weight-only INT8 GEMM parity: kernels.int8_matmul.int8_matmul (tcgen05 CUDA)
against the pinned oracle (kernels/ref/int8_matmul_ref.py) and against the
reference's own GPU test (tests/kernels/test_triton_kernels.py:26-41).

Outputs are rounded to bf16/fp16 once; both sides accumulate in fp32, so the
tolerance is a few units in the last place of the output type plus fp32
summation-order noise: |y - ref| <= RTOL * |ref| + ATOL_FRAC * rms(ref).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.inputs import INT8_CASES, int8_inputs

pytestmark = pytest.mark.gpu

TOL = {"bf16": (8e-3, 2e-3), "fp16": (2e-3, 5e-4)}


def _check(y, ref, dtype, what):
    rtol, afrac = TOL[dtype]
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    lim = rtol * np.abs(ref) + afrac * np.sqrt(np.mean(ref.astype(np.float64) ** 2))
    assert np.isfinite(y).all(), what
    bad = err > lim
    assert not bad.any(), f"{what}: {bad.sum()} elements out of tolerance, max err {err.max():.3e}"


def _run(cuda, x, w, scales, bias, dtype):
    import torch

    from kernels.int8_matmul import int8_matmul

    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    tx = torch.from_numpy(x).to(cuda, tdt)
    y = int8_matmul(tx, torch.from_numpy(w).to(cuda), torch.from_numpy(scales).to(cuda),
                    None if bias is None else torch.from_numpy(bias).to(cuda))
    return y.float().cpu().numpy(), tx.float().cpu().numpy()


@pytest.mark.parametrize("name", ["decode_bias", "prefill"])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_golden_cases(cuda, golden, name, dtype):
    case = INT8_CASES[name]
    x, w, scales, bias = int8_inputs(case)
    y, xr = _run(cuda, x, w, scales, bias, dtype)
    # the golden vectors are the reference on bf16-rounded x; the fp16 run
    # rounds x differently, so it is checked against the oracle on its own x
    ref = golden[f"int8_{name}"] if dtype == "bf16" else oracle.int8_matmul(xr, w, scales,
                                                                           bias=bias)
    _check(y, ref, dtype, f"{name} {dtype}")


SHAPES = [
    # M, N, K, bias
    (1, 4096, 4096, False),    # decode, one token: mma.sync GEMV, x staged in shared memory
    (7, 6144, 4096, True),     # decode batch (QKV of a Llama-3-8B layer), x staged
    (2, 512, 65536, False),    # x too large to stage: per-chunk x loads
    (8, 768, 4096, True),      # 64 KB of x: per-chunk x loads
    (9, 1000, 1024, True),     # mma.sync GEMV, two token blocks, ragged channel tile
    (32, 256, 64, False),      # tcgen05 GEMV, a single 64-column chunk
    (3, 256, 100, True),       # K not a multiple of 64 at small M: tcgen05 GEMV, split-K
    (20, 1000, 512, True),     # 32-token tcgen05 GEMV tile, ragged channel tile
    (40, 384, 4096, False),    # 64-token tcgen05 GEMV tile
    (24, 20000, 256, True),    # more channel tiles than SMs: two GEMV CTAs per SM, ragged N
    (64, 512, 320, False),     # K not a multiple of 64 (zero-filled tail tile)
    (200, 300, 256, True),     # ragged M and N tiles
    (1024, 1024, 1024, False), # enough tiles for no split
    (130, 96, 16, False),      # K smaller than one tile
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_shapes_vs_oracle(cuda, shape, dtype):
    M, N, K, with_bias = shape
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    scales = rng.uniform(0.5, 2.0, size=N).astype(np.float32) / (127.0 * np.sqrt(K))
    bias = rng.standard_normal(N).astype(np.float32) if with_bias else None
    y, xr = _run(cuda, x, w, scales, bias, dtype)
    _check(y, oracle.int8_matmul(xr, w, scales, bias=bias), dtype, f"{shape} {dtype}")


def test_reference_triton_test(cuda):
    """tests/kernels/test_triton_kernels.py:26-41 of the reference: symmetric
    per-channel quantization of randn weights, fp16 activations and scales."""
    import torch

    from kernels.int8_matmul import int8_matmul

    torch.manual_seed(0)
    M, N, K = 64, 128, 64
    w_fp = torch.randn(N, K)
    scales = (w_fp.abs().amax(dim=1) / 127.0).clamp_min(1e-8)
    w_int8 = (w_fp / scales.unsqueeze(-1)).round().clamp(-128, 127).to(torch.int8)
    x = torch.randn(M, K, dtype=torch.float16, device=cuda)
    scales_cu = scales.to(cuda).to(torch.float16)
    y = int8_matmul(x, w_int8.to(cuda), scales_cu)
    ref = oracle.int8_matmul(x.float().cpu().numpy(), w_int8.numpy(),
                             scales_cu.float().cpu().numpy())
    _check(y.float().cpu().numpy(), ref, "fp16", "reference test")


def test_layouts_and_errors(cuda):
    import torch

    from kernels.int8_matmul import int8_matmul

    rng = np.random.default_rng(3)
    w = torch.from_numpy(rng.integers(-128, 128, size=(256, 128), dtype=np.int8)).to(cuda)
    s = torch.full((256,), 0.01, device=cuda)
    # (B, L, K) input and a strided row view
    x3 = torch.randn(2, 5, 128, device=cuda, dtype=torch.bfloat16)
    y3 = int8_matmul(x3, w, s)
    assert y3.shape == (2, 5, 256) and y3.dtype == torch.bfloat16
    ref = oracle.int8_matmul(x3.float().cpu().numpy().reshape(10, 128), w.cpu().numpy(),
                             s.cpu().numpy()).reshape(2, 5, 256)
    _check(y3.float().cpu().numpy(), ref, "bf16", "3-d input")
    big = torch.randn(10, 192, device=cuda, dtype=torch.bfloat16)
    xs = big[:, 32:160]
    assert not xs.is_contiguous()
    _check(int8_matmul(xs, w, s).float().cpu().numpy(),
           oracle.int8_matmul(xs.float().cpu().numpy(), w.cpu().numpy(), s.cpu().numpy()),
           "bf16", "strided rows")
    # a few strided rows: the GEMV that copies x into shared memory row by row
    xs4 = big[:4, 32:160]
    _check(int8_matmul(xs4, w, s).float().cpu().numpy(),
           oracle.int8_matmul(xs4.float().cpu().numpy(), w.cpu().numpy(), s.cpu().numpy()),
           "bf16", "strided rows, x staged")
    assert int8_matmul(torch.empty(0, 128, device=cuda, dtype=torch.bfloat16), w, s).shape == (0, 256)
    with pytest.raises(RuntimeError):
        int8_matmul(x3.cpu(), w.cpu(), s.cpu())
    with pytest.raises(ValueError):
        int8_matmul(x3, w, s[None])
    with pytest.raises(AssertionError):
        int8_matmul(torch.randn(4, 64, device=cuda, dtype=torch.bfloat16), w, s)


def test_unaligned_contiguous_views(cuda):
    """x and w as contiguous views that start 2 / 1 bytes past a 16-byte boundary
    (e.g. slices of a flat buffer): the wrapper copies them to aligned storage
    instead of handing the C ABI an unaligned pointer."""
    import torch

    from kernels.int8_matmul import int8_matmul

    M, N, K = 5, 256, 128
    rng = np.random.default_rng(77)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.integers(-128, 128, size=(N, K)).astype(np.int8)
    s = (rng.random(N) * 0.01 + 1e-3).astype(np.float32)
    flat_x = torch.zeros(M * K + 1, dtype=torch.bfloat16, device=cuda)
    tx = flat_x[1:].view(M, K)
    tx.copy_(torch.from_numpy(x).to(cuda, torch.bfloat16))
    flat_w = torch.zeros(N * K + 1, dtype=torch.int8, device=cuda)
    tw = flat_w[1:].view(N, K)
    tw.copy_(torch.from_numpy(w).to(cuda))
    assert tx.is_contiguous() and tx.data_ptr() % 16 and tw.data_ptr() % 16
    y = int8_matmul(tx, tw, torch.from_numpy(s).to(cuda)).float().cpu().numpy()
    ref = oracle.int8_matmul(tx.float().cpu().numpy(), w, s)
    _check(y, ref, "bf16", "unaligned views")
