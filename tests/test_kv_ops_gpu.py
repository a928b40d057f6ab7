"""Byte-level parity of the K/V movers: the gather must be bit-exact with the
reference's PagedKVCache.gather, and RoPE / RoPE+append bit-exact with the
oracle's fp32 rotation rounded to bf16."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.inputs import normal
from tests.helpers import to_np, to_torch

pytestmark = pytest.mark.gpu


def test_gather_kv_bit_exact(cuda):
    import torch
    from kernels.flash_attention import gather_kv

    rng = np.random.default_rng(0)
    for bs, lens in ((16, [1, 16, 17, 300, 0]), (8, [5, 64]), (2, [3, 9, 1])):
        nblk = [(L + bs - 1) // bs for L in lens]
        pool_n = sum(nblk) + 2
        perm = rng.permutation(pool_n)
        tables = np.zeros((len(lens), max(max(nblk), 1)), np.int32)
        o = 0
        for i, n in enumerate(nblk):
            tables[i, :n] = perm[o: o + n]
            o += n
        pool = to_torch(normal(bs, (pool_n, bs, 8, 64)), torch.bfloat16, cuda)
        out_len = tables.shape[1] * bs
        out = torch.full((len(lens), out_len, 8, 64), -7.0, dtype=torch.bfloat16, device=cuda)
        gather_kv(pool, torch.from_numpy(tables).cuda(), torch.tensor(lens, dtype=torch.int32).cuda(),
                  out=out)
        ref = oracle.gather_tables(to_np(pool), tables, np.array(lens), out_len)
        got = out.view(torch.int16).cpu().numpy()
        want = to_torch(ref, torch.bfloat16, "cpu").view(torch.int16).numpy()
        for i, L in enumerate(lens):
            assert np.array_equal(got[i, :L], want[i, :L])
            assert (to_np(out[i, L:]) == -7.0).all()  # rows past the length untouched


def test_apply_rotary_bit_exact(cuda):
    import torch
    from kernels import build_rope_cache
    from kernels.flash_attention import apply_rotary

    for d in (16, 64, 128):
        x = normal(d, (2, 3, 37, d))
        cos, sin = build_rope_cache(100, d, theta=500000.0, device=cuda)
        y = apply_rotary(to_torch(x, torch.bfloat16, cuda), cos, sin, pos0=5)
        ref = oracle.bf16_round(oracle.apply_rotary(x, cos.cpu().numpy(), sin.cpu().numpy(),
                                                    np.arange(5, 42)))
        assert np.array_equal(to_np(y), ref), d


def test_rope_append_matches_reference_append(cuda):
    import torch
    from kernels import build_rope_cache
    from kernels.flash_attention import rope_append

    Hkv, d, bs = 2, 64, 16
    cos, sin = build_rope_cache(256, d, theta=500000.0, device=cuda)
    cn, sn = cos.cpu().numpy(), sin.cpu().numpy()
    ref = oracle.PagedKVCacheRef(1, Hkv, d, 32, bs)
    kp = torch.zeros(32, bs, Hkv, d, dtype=torch.bfloat16, device=cuda)
    vp = torch.zeros_like(kp)
    seqs = [ref.new_sequence(), ref.new_sequence()]
    steps = [(0, 20), (1, 3), (0, 1), (1, 30), (0, 5)]
    for i, (si, L) in enumerate(steps):
        t = seqs[si]
        start = t.length
        k_raw = normal(100 + i, (L, Hkv, d))
        v_raw = normal(200 + i, (L, Hkv, d))
        k_rot = oracle.bf16_round(oracle.apply_rotary(k_raw.transpose(1, 0, 2)[None], cn, sn,
                                                      np.arange(start, start + L))[0]
                                  .transpose(1, 0, 2))
        ref.append(0, t, k_rot, v_raw)
        table = torch.tensor([t.blocks], dtype=torch.int32, device=cuda)
        rope_append(to_torch(k_raw[None], torch.bfloat16, cuda),
                    to_torch(v_raw[None], torch.bfloat16, cuda), kp, vp, table,
                    torch.tensor([start], dtype=torch.int32, device=cuda), rope=(cos, sin))
    for t in seqs:
        gk, gv = ref.gather(0, t)
        idx = torch.tensor(t.blocks, device=cuda)
        k = kp[idx].reshape(-1, Hkv, d)[: t.length]
        v = vp[idx].reshape(-1, Hkv, d)[: t.length]
        assert np.array_equal(to_np(k), gk)
        assert np.array_equal(to_np(v), gv)
