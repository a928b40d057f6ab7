"""Paged decode / speculative-verify parity: kernels.paged_attention vs the
reference's PagedKVCache.gather + fp32 flash_attention_ref (golden vectors and
the pinned oracle)."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.inputs import DECODE_CASES, decode_inputs, normal
from tests.helpers import assert_close_attn, to_np, to_torch

pytestmark = pytest.mark.gpu


def build_paged(kv_lens, Hkv, d, bs, seed, cos=None, sin=None, extra_blocks=3, perm_seed=None):
    """Random raw K/V per sequence, K rotated at positions 0..L-1 and rounded to
    bf16 as stored, scattered into a pool through seeded random block tables."""
    nblk = [(L + bs - 1) // bs for L in kv_lens]
    pool_blocks = sum(nblk) + extra_blocks
    rng = np.random.default_rng(perm_seed if perm_seed is not None else seed)
    perm = rng.permutation(pool_blocks)
    kp = np.zeros((pool_blocks, bs, Hkv, d), np.float32)
    vp = np.zeros_like(kp)
    maxb = max(max(nblk), 1)
    tables = np.full((len(kv_lens), maxb), 0, np.int32)
    ks, vs = [], []
    off = 0
    for i, L in enumerate(kv_lens):
        k = normal(seed * 1000 + 2 * i, (L, Hkv, d))
        v = normal(seed * 1000 + 2 * i + 1, (L, Hkv, d))
        if cos is not None and L > 0:
            k = oracle.bf16_round(
                oracle.apply_rotary(k.transpose(1, 0, 2)[None], cos, sin, np.arange(L))[0]
                .transpose(1, 0, 2))
        blocks = perm[off: off + nblk[i]]
        off += nblk[i]
        tables[i, : nblk[i]] = blocks
        for t in range(L):
            kp[blocks[t // bs], t % bs] = k[t]
            vp[blocks[t // bs], t % bs] = v[t]
        ks.append(k)
        vs.append(v)
    return kp, vp, tables, ks, vs


def ref_paged(q, ks, vs, kv_lens, cos, sin, causal=True):
    outs = []
    for i, L in enumerate(kv_lens):
        outs.append(oracle.decode_case_ref(q[i: i + 1], ks[i].transpose(1, 0, 2)[None],
                                           vs[i].transpose(1, 0, 2)[None], cos, sin,
                                           causal=causal))
    return np.concatenate(outs)


@pytest.mark.parametrize("name", sorted(DECODE_CASES))
def test_golden_decode_verify(cuda, golden, name):
    """Same sequences, same reference block ids, same attention as the reference
    engine's decode (M=1) / verify (M=5) step."""
    import torch
    from kernels import build_rope_cache
    from kernels.flash_attention import paged_attention

    case = DECODE_CASES[name]
    qs, ks_raw, vs = decode_inputs(case)
    bs, Hkv, d, M = case["block_size"], case["Hkv"], case["d"], case["M"]
    tables = golden[f"decode_{name}_tables"]
    nb = int(tables.max()) + 5
    c, s = oracle.build_rope_cache(max(case["kv_lens"]) + 8, d, case["theta"])
    kp = np.zeros((nb, bs, Hkv, d), np.float32)
    vp = np.zeros_like(kp)
    for i, L in enumerate(case["kv_lens"]):
        krot = oracle.apply_rotary(ks_raw[i].transpose(1, 0, 2)[None], c, s, np.arange(L))[0]
        krot = krot.transpose(1, 0, 2)
        for t in range(L):
            kp[tables[i, t // bs], t % bs] = krot[t]
            vp[tables[i, t // bs], t % bs] = vs[i][t]
    dev_tables = torch.from_numpy(np.where(tables < 0, 0, tables)).int().to(cuda)
    kv_lens = torch.tensor(case["kv_lens"], dtype=torch.int32, device=cuda)
    q = to_torch(np.concatenate(qs), torch.bfloat16, cuda)
    rope = build_rope_cache(max(case["kv_lens"]) + 8, d, theta=case["theta"], device=cuda)
    out = paged_attention(q, to_torch(kp, torch.bfloat16, cuda), to_torch(vp, torch.bfloat16, cuda),
                          dev_tables, kv_lens, True, rope=rope)
    assert_close_attn(to_np(out), golden[f"decode_{name}_out"], what=name)


PAGED_CASES = [
    # B, Hq, Hkv, M, d, bs, kv_lens
    (4, 32, 8, 1, 64, 16, [1, 15, 16, 17]),
    (6, 32, 8, 1, 64, 16, [300, 1000, 257, 4000, 64, 2049]),
    (3, 32, 8, 5, 128, 16, [5, 1100, 3000]),
    (5, 8, 8, 1, 128, 16, [33, 700, 2, 129, 1500]),
    (3, 4, 1, 7, 64, 8, [7, 100, 513]),         # G*M = 28 rows, block size 8
    (2, 16, 2, 5, 64, 32, [900, 37]),           # G*M = 40 rows -> 4 m-tiles
    (2, 8, 1, 9, 128, 16, [400, 1000]),          # G*M = 72 rows -> 3 row groups
    (3, 2, 2, 1, 16, 4, [3, 50, 9]),            # reference tiny-model geometry
    (2, 4, 2, 3, 16, 8, [200, 70]),             # d=16 over several partitions
    (1, 8, 1, 5, 16, 16, [300]),                # d=16, G*M = 40 rows: 64-row groups
    (2, 4, 2, 3, 32, 16, [100, 3]),
    (2, 4, 2, 1, 256, 16, [100, 500]),
]


@pytest.mark.parametrize("case", PAGED_CASES, ids=lambda c: f"B{c[0]}H{c[1]}-{c[2]}M{c[3]}d{c[4]}bs{c[5]}")
@pytest.mark.parametrize("split", [0, 64])
def test_random_vs_oracle(cuda, case, split):
    import torch
    from kernels import build_rope_cache
    from kernels.flash_attention import paged_attention

    B, Hq, Hkv, M, d, bs, lens = case
    seed = (B * 131 + Hq * 17 + M * 7 + d + bs) % 9973
    c, s = oracle.build_rope_cache(max(lens) + 4, d, 500000.0)
    kp, vp, tables, ks, vs = build_paged(lens, Hkv, d, bs, seed, c, s)
    q = normal(seed + 99, (B, Hq, M, d))
    rope = build_rope_cache(max(lens) + 4, d, theta=500000.0, device=cuda)
    out = paged_attention(to_torch(q, torch.bfloat16, cuda), to_torch(kp, torch.bfloat16, cuda),
                          to_torch(vp, torch.bfloat16, cuda), torch.from_numpy(tables).to(cuda),
                          torch.tensor(lens, dtype=torch.int32, device=cuda), True, rope=rope,
                          split_tokens=split)
    assert_close_attn(to_np(out), ref_paged(q, ks, vs, lens, c, s), what=str(case))


def test_splits_agree_and_fp16(cuda):
    import torch
    from kernels.flash_attention import paged_attention

    lens = [2000, 513, 4096, 1]
    kp, vp, tables, ks, vs = build_paged(lens, 8, 64, 16, 77)
    q = normal(78, (4, 32, 1, 64))
    args = [torch.from_numpy(tables).cuda(), torch.tensor(lens, dtype=torch.int32).cuda()]
    outs = []
    for split in (0, 16, 64, 512, 4096):
        outs.append(to_np(paged_attention(to_torch(q, torch.float16, cuda),
                                          to_torch(kp, torch.float16, cuda),
                                          to_torch(vp, torch.float16, cuda), *args, True,
                                          split_tokens=split)))
    ref = ref_paged(q, ks, vs, lens, None, None)
    for o in outs:
        assert_close_attn(o, ref, what="fp16 split")


def test_non_causal_and_strided_q(cuda):
    import torch
    from kernels.flash_attention import paged_attention

    lens = [50, 300]
    kp, vp, tables, ks, vs = build_paged(lens, 2, 64, 16, 5)
    q = normal(6, (2, 5, 8, 64))  # (B, M, Hq, d) buffer, viewed as (B, Hq, M, d)
    tq = to_torch(q, torch.bfloat16, cuda).transpose(1, 2)
    out = paged_attention(tq, to_torch(kp, torch.bfloat16, cuda), to_torch(vp, torch.bfloat16, cuda),
                          torch.from_numpy(tables).cuda(), torch.tensor(lens, dtype=torch.int32).cuda(),
                          causal=False)
    ref = ref_paged(q.transpose(0, 2, 1, 3), ks, vs, lens, None, None, causal=False)
    assert_close_attn(to_np(out), ref, what="non-causal strided")


def test_bad_block_id_sets_status_without_fault(cuda):
    """A table entry outside the pool is refused by the kernel's own bounds check:
    it raises a status bit, reads nothing, and the context stays usable."""
    import torch
    from kernels import _lib
    from kernels.flash_attention import paged_attention

    _lib.device_status(clear=True)
    lens = [40]
    kp, vp, tables, ks, vs = build_paged(lens, 2, 64, 16, 9)
    tables[0, 1] = kp.shape[0] + 1000
    q = to_torch(normal(10, (1, 4, 1, 64)), torch.bfloat16, cuda)
    out = paged_attention(q, to_torch(kp, torch.bfloat16, cuda), to_torch(vp, torch.bfloat16, cuda),
                          torch.from_numpy(tables).cuda(), torch.tensor(lens, dtype=torch.int32).cuda())
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) & _lib.CIE_DEV_BAD_BLOCK_ID
    assert torch.isfinite(out).all()
    assert _lib.device_status(clear=True) == 0


def test_config3_full_size_sampled(cuda):
    """B=64 decode, ctx ~ U[256, 8192], block size 16, random tables;
    checked on sampled sequences against the oracle."""
    import torch
    from kernels import build_rope_cache
    from kernels.flash_attention import paged_attention

    rng = np.random.default_rng(0)
    ctx = rng.integers(256, 8193, size=64)
    lens = (ctx + 1).tolist()
    c, s = oracle.build_rope_cache(max(lens) + 1, 64, 500000.0)
    kp, vp, tables, ks, vs = build_paged(lens, 8, 64, 16, 123, c, s, extra_blocks=0, perm_seed=0)
    q = normal(124, (64, 32, 1, 64))
    rope = build_rope_cache(max(lens) + 1, 64, theta=500000.0, device=cuda)
    out = to_np(paged_attention(to_torch(q, torch.bfloat16, cuda), to_torch(kp, torch.bfloat16, cuda),
                                to_torch(vp, torch.bfloat16, cuda), torch.from_numpy(tables).cuda(),
                                torch.tensor(lens, dtype=torch.int32).cuda(), True, rope=rope))
    pick = [0, 1, int(np.argmax(lens)), int(np.argmin(lens)), 63]
    ref = ref_paged(q[pick], [ks[i] for i in pick], [vs[i] for i in pick], [lens[i] for i in pick],
                    c, s)
    assert_close_attn(out[pick], ref, what="cfg3 sampled")


def _device_pool(lens, Hkv, d, bs, seed, device):
    """Seeded random bf16 pools built on the device (the full-size configs are too
    large to assemble on the host) and seeded random-permutation block tables."""
    import torch

    nblk = [(L + bs - 1) // bs for L in lens]
    pool = int(sum(nblk))
    rng = np.random.default_rng(seed)
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.zeros((len(lens), max(nblk)), np.int32)
    off = 0
    for i, n in enumerate(nblk):
        tables[i, :n] = perm[off: off + n]
        off += n
    g = torch.Generator(device=device).manual_seed(seed)
    kp = torch.randn(pool, bs, Hkv, d, device=device, generator=g).to(torch.bfloat16)
    vp = torch.randn(pool, bs, Hkv, d, device=device, generator=g).to(torch.bfloat16)
    return kp, vp, tables


def _history(pool, tables, i, L):
    """Sequence i's (L, Hkv, d) history read from the pool with torch indexing (fp32, host)."""
    import torch

    bs = pool.shape[1]
    blocks = torch.from_numpy(tables[i, : (L + bs - 1) // bs].astype(np.int64)).to(pool.device)
    return pool.index_select(0, blocks).reshape(-1, *pool.shape[2:])[:L].float().cpu().numpy()


def _check_sampled(out, q, kp, vp, tables, lens, pick, c, s, what):
    for i in pick:
        k, v = _history(kp, tables, i, lens[i]), _history(vp, tables, i, lens[i])
        ref = oracle.decode_case_ref(q[i: i + 1], k.transpose(1, 0, 2)[None],
                                     v.transpose(1, 0, 2)[None], c, s, causal=True)
        assert_close_attn(out[i: i + 1], ref, what=f"{what} seq {i} (len {lens[i]})")


@pytest.mark.parametrize("hkv,split", [(8, 0), (1, 0), (1, 512)],
                         ids=["all_heads", "one_kv_head_slice", "one_kv_head_split512"])
def test_config5_full_size_sampled(cuda, hkv, split):
    """speculative verify, B=32, M=5, ctx ~ U[1024, 32768], d=128, block
    size 16, random-permutation tables, at full size; checked on sampled sequences
    (shortest, longest and three more) against the oracle. ``one_kv_head_slice`` is
    what one rank of eight holds (Hq=4, Hkv=1), with the automatic partition size;
    with 512-token partitions every sequence (sequence 0 is given the longest
    context the config allows, 32768: 65 partitions) has more partitions than the
    merge kernel's shared-memory path takes (32), so they are merged by its
    fallback path on full-length data."""
    import torch
    from kernels import _lib, build_rope_cache
    from kernels.flash_attention import paged_attention

    _lib.device_status(clear=True)
    rng = np.random.default_rng(4)
    ctx = rng.integers(1024, 32769, size=32)
    ctx[0] = 32768
    M, d, G = 5, 128, 4
    lens = (ctx + M).tolist()
    kp, vp, tables = _device_pool(lens, hkv, d, 16, 41 + hkv, cuda)
    q = normal(400 + hkv, (32, G * hkv, M, d))
    c, s = oracle.build_rope_cache(max(lens) + 1, d, 500000.0)
    rope = build_rope_cache(max(lens) + 1, d, theta=500000.0, device=cuda)
    out = to_np(paged_attention(to_torch(q, torch.bfloat16, cuda), kp, vp,
                                torch.from_numpy(tables).to(cuda),
                                torch.tensor(lens, dtype=torch.int32, device=cuda), True,
                                rope=rope, split_tokens=split))
    assert _lib.device_status(clear=True) == 0
    assert np.isfinite(out).all()
    pick = sorted({0, 31, int(np.argmax(lens)), int(np.argmin(lens)), 17})
    _check_sampled(out, q, kp, vp, tables, lens, pick, c, s, f"cfg5 Hkv={hkv}")


PAGED_PREFILL_CASES = [
    # B, Hq, Hkv, M, d, bs, kv_lens (history incl. the M new tokens)
    (3, 8, 2, 100, 64, 16, [100, 137, 1100]),
    (2, 8, 2, 300, 128, 16, [300, 2000]),
    (3, 16, 2, 77, 128, 32, [77, 500, 1029]),
    (1, 32, 8, 513, 64, 16, [4000]),
    (2, 4, 1, 129, 128, 64, [129, 1000]),
]


@pytest.mark.parametrize("case", PAGED_PREFILL_CASES,
                         ids=lambda c: f"B{c[0]}H{c[1]}-{c[2]}M{c[3]}d{c[4]}bs{c[5]}")
@pytest.mark.parametrize("dt", ["bf16", "fp16"])
def test_paged_prefill_vs_oracle(cuda, case, dt):
    """Chunked prefill of a batch: M new tokens per sequence (G*M > 64 rows per kv
    head) against ragged paged histories, on the tcgen05 kernel reading the pools
    through the block table; q rotated at positions kv_len - M + i."""
    import torch
    from kernels import build_rope_cache
    from kernels.flash_attention import paged_attention

    B, Hq, Hkv, M, d, bs, lens = case
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    seed = (B * 31 + Hq * 7 + M + d + bs) % 9973
    c, s = oracle.build_rope_cache(max(lens) + 4, d, 500000.0)
    kp, vp, tables, ks, vs = build_paged(lens, Hkv, d, bs, seed, c, s)
    q = normal(seed + 7, (B, Hq, M, d))
    rope = build_rope_cache(max(lens) + 4, d, theta=500000.0, device=cuda)
    out = paged_attention(to_torch(q, tdt, cuda), to_torch(kp, tdt, cuda), to_torch(vp, tdt, cuda),
                          torch.from_numpy(tables).to(cuda),
                          torch.tensor(lens, dtype=torch.int32, device=cuda), True, rope=rope)
    assert_close_attn(to_np(out), ref_paged(q, ks, vs, lens, c, s), what=str(case))


def test_paged_prefill_bad_block_id_sets_status(cuda):
    """A refused block id in the tcgen05 paged path: status bit, zeros fetched,
    finite output, and the context stays usable."""
    import torch
    from kernels import _lib
    from kernels.flash_attention import paged_attention

    _lib.device_status(clear=True)
    lens = [400]
    kp, vp, tables, ks, vs = build_paged(lens, 2, 64, 16, 19)
    tables[0, 3] = kp.shape[0] + 7
    q = to_torch(normal(20, (1, 8, 200, 64)), torch.bfloat16, cuda)
    out = paged_attention(q, to_torch(kp, torch.bfloat16, cuda), to_torch(vp, torch.bfloat16, cuda),
                          torch.from_numpy(tables).cuda(), torch.tensor(lens, dtype=torch.int32).cuda())
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) & _lib.CIE_DEV_BAD_BLOCK_ID
    assert torch.isfinite(out).all()
    assert _lib.device_status(clear=True) == 0
