"""cie_paged_attn_noalloc: paged decode / verify for callers that cannot
allocate device memory (hosts that keep all device memory to themselves and
give plugins no allocator, or loops that cannot pay cudaMalloc's device
synchronisation). The entry point keeps its split-KV partials in a fixed array
inside the library instead of a caller workspace.

Checked through the C ABI against the existing entry point (cie_paged_attn
with a torch workspace, via kernels.flash_attention.paged_attention), within
the attention tolerance the other parity tests use, on two calls in a row with
different queries (the shared array keeps the previous call's contents). This
file is collected last so that a stop-at-first-failure run has already run
every other test; it also passes on its own in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from tests.golden.inputs import normal
from tests.helpers import assert_close_attn, to_np, to_torch

pytestmark = pytest.mark.gpu


def _pools(lens, hkv, d, bs, max_blocks, seed):
    nblk = [(L + bs - 1) // bs for L in lens]
    pool = sum(nblk)
    rng = np.random.default_rng(seed)
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.zeros((len(lens), max_blocks), np.int32)  # unused tail entries: block 0
    o = 0
    for i, n in enumerate(nblk):
        tables[i, :n] = perm[o:o + n]
        o += n
    kp = normal(seed + 1, (pool, bs, hkv, d))
    vp = normal(seed + 2, (pool, bs, hkv, d))
    return kp, vp, tables


def _noalloc(lib, q, kp, vp, tables, lens, out, rope, split_tokens=0):
    import torch

    from kernels import _lib

    cos, sin = rope
    B, Hq, M, d = q.shape
    nb, bs, Hkv, _ = kp.shape
    vp_ = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    return lib.cie_paged_attn_noalloc(
        vp_(q), vp_(kp), vp_(vp), vp_(tables), vp_(lens), vp_(out), B, Hq, Hkv, M, d, nb, bs,
        tables.shape[1], _lib.strides3(q.stride()[:3]), _lib.strides3(out.stride()[:3]),
        ctypes.c_float(1.0 / d ** 0.5), 1, _lib.CIE_DTYPE_BF16, vp_(cos), vp_(sin),
        int(cos.shape[0]), int(split_tokens),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("geom", [
    # B, Hq, Hkv, M, d, block size, table width, length range
    (16, 32, 8, 1, 64, 16, 200, (1, 3000)),       # decode, partials fit the default plan
    (64, 32, 8, 1, 128, 16, 4096, (1, 2000)),     # wide tables: partition size is grown to fit
    (8, 32, 8, 5, 128, 16, 400, (5, 6000)),       # speculative verify
], ids=["decode_d64", "wide_table_d128", "verify_d128"])
def test_noalloc_matches_workspace_entry_point(cuda, geom):
    import torch

    from kernels import _lib, build_rope_cache
    from kernels.flash_attention import paged_attention

    lib = _lib.load()
    B, Hq, Hkv, M, d, bs, width, (lo, hi) = geom
    lens = np.random.default_rng(B + d).integers(lo, hi + 1, size=B).tolist()
    kp, vp, tables = _pools(lens, Hkv, d, bs, width, seed=B * 7 + d)
    kpt, vpt = to_torch(kp, torch.bfloat16, cuda), to_torch(vp, torch.bfloat16, cuda)
    tab = torch.from_numpy(tables).to(cuda)
    lt = torch.tensor(lens, dtype=torch.int32, device=cuda)
    rope = build_rope_cache(hi + 8, d, theta=500000.0, device=cuda)
    for call in range(2):  # two calls in a row, different queries
        q = to_torch(normal(1000 * call + B, (B, Hq, M, d)), torch.bfloat16, cuda)
        want = paged_attention(q, kpt, vpt, tab, lt, True, rope=rope)
        got = torch.full_like(want, float("nan"))
        rc = _noalloc(lib, q, kpt, vpt, tab, lt, got, rope)
        assert rc == _lib.CIE_OK, _lib.last_error(lib)
        torch.cuda.synchronize()
        assert_close_attn(to_np(got), to_np(want), what=f"{geom} call {call}")
    assert _lib.device_status(clear=True) == 0


def test_noalloc_rejects_partials_beyond_the_fixed_scratch(cuda):
    import torch

    from kernels import _lib, build_rope_cache

    lib = _lib.load()
    lens = [100] * 64
    kp, vp, tables = _pools(lens, 8, 128, 16, 4096, seed=3)
    kpt, vpt = to_torch(kp, torch.bfloat16, cuda), to_torch(vp, torch.bfloat16, cuda)
    q = to_torch(normal(4, (64, 32, 1, 128)), torch.bfloat16, cuda)
    out = torch.empty_like(q)
    rope = build_rope_cache(128, 128, theta=500000.0, device=cuda)
    # 64-token partitions over a 65536-token table need far more than the array holds
    rc = _noalloc(lib, q, kpt, vpt, torch.from_numpy(tables).to(cuda),
                  torch.tensor(lens, dtype=torch.int32, device=cuda), out, rope, split_tokens=64)
    assert rc == _lib.CIE_ERR_WORKSPACE
    assert "fixed scratch" in _lib.last_error(lib)
