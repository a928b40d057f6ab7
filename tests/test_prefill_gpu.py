"""Prefill parity: kernels.flash_attention (tcgen05 / mma.sync CUDA) vs the
reference's fp32 attention + RoPE (golden vectors and the pinned oracle), in
the style of the reference's tests/kernels/test_triton_kernels.py:11-22."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.inputs import ATTN_CASES, CFG1, attn_inputs, cfg1_inputs, normal
from tests.helpers import assert_close_attn, to_np, to_torch

pytestmark = pytest.mark.gpu


def _tables(torch, L, d, theta, device):
    from kernels import build_rope_cache

    return build_rope_cache(L, d, theta=theta, device=device)


@pytest.mark.parametrize("name", sorted(ATTN_CASES))
def test_golden_cases(cuda, golden, name):
    import torch
    from kernels.flash_attention import flash_attention

    case = ATTN_CASES[name]
    q, k, v, mask = attn_inputs(case)
    D = q.shape[-1]
    tq, tk, tv = (to_torch(a, torch.bfloat16, cuda) for a in (q, k, v))
    if D < 16:
        with pytest.raises(ValueError):
            flash_attention(tq, tk, tv, causal=case["causal"])
        return
    if mask is not None:
        pytest.skip("additive masks are an oracle-only feature of the reference")
    rope = None
    if case.get("rope"):
        rope = _tables(torch, max(q.shape[2], k.shape[2]) + 8, D, case["theta"], cuda)
    out = flash_attention(tq, tk, tv, case["causal"], case.get("scale"), rope=rope)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == tq.shape
    assert_close_attn(to_np(out), golden[f"attn_{name}"], what=name)


def test_config1_llama32_1b_prefill(cuda, golden):
    """B=1, Hq=32, Hkv=8, S=512, d=64, RoPE theta 5e5, causal."""
    import torch
    from kernels.flash_attention import flash_attention

    q, k, v = cfg1_inputs()
    rope = _tables(torch, CFG1["S"], CFG1["d"], CFG1["theta"], cuda)
    out = flash_attention(*(to_torch(a, torch.bfloat16, cuda) for a in (q, k, v)), True, 1 / 8,
                          rope=rope)
    o = to_np(out)
    assert_close_attn(o[:, :, CFG1["sample_rows"]], golden["cfg1_rows"], what="cfg1 rows")
    assert abs(o.astype(np.float64).sum() - golden["cfg1_sum"][0]) < 5.0


CASES = [
    # B, Hq, Hkv, M, N, D, causal
    (1, 4, 1, 128, 128, 64, True),
    (2, 8, 2, 256, 256, 64, True),
    (1, 4, 4, 200, 200, 128, True),
    (2, 4, 2, 130, 333, 128, True),    # chunked prefill: N > M, ragged tiles
    (1, 8, 2, 300, 300, 64, False),
    (1, 2, 1, 1000, 1000, 128, True),
    (1, 4, 1, 64, 64, 64, True),       # G*M = 256 rows -> tcgen05 with a partial tile
    (1, 8, 8, 5, 900, 128, True),      # short query block -> split-KV mma path
    (2, 4, 2, 33, 77, 32, True),       # d=32 -> mma path
    (1, 2, 2, 40, 40, 16, False),      # d=16 (the reference's tiny-model head dim)
    (1, 2, 1, 20, 50, 256, True),      # d=256 -> mma path
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c)))
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_random_vs_oracle(cuda, case, dtype):
    import torch
    from kernels.flash_attention import flash_attention

    B, H, Hk, M, N, D, causal = case
    seed = hash(case) % 10000
    q = normal(seed + 1, (B, H, M, D))
    k = normal(seed + 2, (B, Hk, N, D))
    v = normal(seed + 3, (B, Hk, N, D))
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    c, s = oracle.build_rope_cache(N + 4, D, 500000.0)
    rope = _tables(torch, N + 4, D, 500000.0, cuda)
    out = flash_attention(*(to_torch(a, tdt, cuda) for a in (q, k, v)), causal, rope=rope)
    ref = oracle.prefill_case_ref(q, k, v, c, s, causal=causal)
    assert_close_attn(to_np(out), ref, what=f"{case} {dtype}")


@pytest.mark.parametrize("D", [64, 128])
def test_running_max_jumps(cuda, D):
    """Keys whose scores jump far above everything before them in later key tiles:
    exercises the lazy rescale of O and the recomputation of a speculatively
    exponentiated half row (a jump of ~2^10 and one of ~2^40 in the log2 domain)."""
    import torch
    from kernels.flash_attention import flash_attention

    B, H, Hk, L = 1, 4, 2, 1000
    rng = np.random.default_rng(D)
    u = rng.standard_normal(D).astype(np.float32)
    u /= np.linalg.norm(u)
    q = normal(11, (B, H, L, D)) + 2.0 * u
    k = normal(12, (B, Hk, L, D))
    v = normal(13, (B, Hk, L, D))
    spike = 1.1 * np.sqrt(D) * 8.0
    k[:, :, 517, :] = spike * u          # key tile 4 (of 128 keys)
    k[:, :, 900, :] = 4.0 * spike * u    # key tile 7
    k[:, :, 901:, :] *= 0.5
    t = [to_torch(a, torch.bfloat16, cuda) for a in (q, k, v)]
    out = flash_attention(*t, causal=True)
    ref = oracle.attention(*(oracle.bf16_round(a) for a in (q, k, v)), causal=True)
    assert np.isfinite(to_np(out)).all()
    assert_close_attn(to_np(out), ref, what=f"max jumps d={D}")


def test_no_rope_and_q_positions(cuda):
    import torch
    from kernels.flash_attention import flash_attention

    B, H, Hk, M, N, D = 1, 4, 2, 150, 150, 128
    q, k, v = normal(1, (B, H, M, D)), normal(2, (B, Hk, N, D)), normal(3, (B, Hk, N, D))
    t = [to_torch(a, torch.bfloat16, cuda) for a in (q, k, v)]
    out = flash_attention(*t, causal=True)
    assert_close_attn(to_np(out), oracle.attention(q, k, v, causal=True), what="no rope")
    # K already rotated (read from the cache): rotate only q, at explicit positions
    c, s = oracle.build_rope_cache(400, D, 500000.0)
    k_rot = oracle.bf16_round(oracle.apply_rotary(k, c, s, np.arange(N)))
    rope = _tables(torch, 400, D, 500000.0, cuda)
    out = flash_attention(t[0], to_torch(k_rot, torch.bfloat16, cuda), t[2], True, rope=rope,
                          rope_q_pos0=0, rope_k=False)
    ref = oracle.attention(oracle.apply_rotary(q, c, s, np.arange(M)), k_rot, v, causal=True)
    assert_close_attn(to_np(out), ref, what="rope_k=False")


def test_strided_views_like_the_engine(cuda):
    """q/k/v as the engine builds them: (B, L, H, D) buffers viewed as (B, H, L, D)."""
    import torch
    from kernels.flash_attention import flash_attention

    B, H, Hk, L, D = 2, 8, 2, 260, 64
    q, k, v = normal(5, (B, L, H, D)), normal(6, (B, L, Hk, D)), normal(7, (B, L, Hk, D))
    tq, tk, tv = (to_torch(a, torch.bfloat16, cuda).transpose(1, 2) for a in (q, k, v))
    assert not tq.is_contiguous()
    out = flash_attention(tq, tk, tv, True)
    ref = oracle.attention(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3),
                           v.transpose(0, 2, 1, 3), causal=True)
    assert_close_attn(to_np(out), ref, what="strided")


def test_unaligned_contiguous_view(cuda):
    """A contiguous q that starts 2 bytes past a 16-byte boundary (a slice of a flat
    buffer) is copied to aligned storage by the wrapper, not refused by the C ABI."""
    import torch
    from kernels.flash_attention import flash_attention

    B, H, Hk, L, D = 1, 8, 2, 300, 64
    q, k, v = normal(15, (B, H, L, D)), normal(16, (B, Hk, L, D)), normal(17, (B, Hk, L, D))
    flat = torch.zeros(q.size + 1, dtype=torch.bfloat16, device=cuda)
    tq = flat[1:].view(B, H, L, D)
    tq.copy_(to_torch(q, torch.bfloat16, cuda))
    assert tq.is_contiguous() and tq.data_ptr() % 16
    out = flash_attention(tq, to_torch(k, torch.bfloat16, cuda), to_torch(v, torch.bfloat16, cuda),
                          True)
    assert_close_attn(to_np(out), oracle.attention(q, k, v, causal=True), what="unaligned q")


def test_edge_cases(cuda):
    import torch
    from kernels.flash_attention import flash_attention

    # empty key axis -> zeros (reference fp32 attention), fully masked rows -> NaN
    q = torch.randn(1, 4, 130, 64, device=cuda, dtype=torch.bfloat16)
    kv = torch.randn(1, 2, 0, 64, device=cuda, dtype=torch.bfloat16)
    out = flash_attention(q, kv, kv, causal=False)
    assert torch.count_nonzero(out).item() == 0
    k = torch.randn(1, 2, 100, 64, device=cuda, dtype=torch.bfloat16)
    out = flash_attention(q, k, k, causal=True)  # M > N: first 30 rows see no key
    o = to_np(out)
    assert np.isnan(o[:, :, :30]).all() and not np.isnan(o[:, :, 30:]).any()
    # empty query axis
    out = flash_attention(q[:, :, :0], k, k, causal=True)
    assert out.shape == (1, 4, 0, 64)


def test_error_conventions(cuda):
    import torch
    from kernels.flash_attention import flash_attention

    q = torch.randn(1, 2, 8, 64)
    with pytest.raises(RuntimeError, match="requires CUDA"):
        flash_attention(q, q, q)
    qc = torch.randn(1, 2, 8, 48, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        flash_attention(qc, qc, qc)
    qf = torch.randn(1, 2, 8, 64, device=cuda, dtype=torch.float32)
    with pytest.raises(ValueError):
        flash_attention(qf, qf, qf)


@pytest.mark.parametrize("cfg", ["cfg2", "cfg4"])
def test_full_size_configs_sampled_rows(cuda, cfg):
    """configs[1] / configs[3] at full size; every sampled query row is checked
    against an fp32 torch reference of that row (size-independent property)."""
    import torch
    from kernels.flash_attention import flash_attention

    B, H, Hk, S, D = (8, 32, 8, 2048, 64) if cfg == "cfg2" else (4, 32, 8, 8192, 128)
    g = torch.Generator(device=cuda).manual_seed(0)
    q = torch.randn(B, H, S, D, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hk, S, D, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hk, S, D, device=cuda, generator=g).to(torch.bfloat16)
    from kernels import build_rope_cache

    cos, sin = build_rope_cache(S, D, theta=500000.0, device=cuda)
    out = flash_attention(q, k, v, True, 1 / D ** 0.5, rope=(cos, sin))
    torch.cuda.synchronize()
    assert not torch.isnan(out).any()

    def rot(x, pos):
        x = x.float()
        c, s = cos[pos], sin[pos]
        x1, x2 = x[..., : D // 2], x[..., D // 2:]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], -1)

    kr = rot(k, torch.arange(S, device=cuda))
    rows = torch.tensor([0, 1, 127, 128, 1000, S // 2 + 3, S - 129, S - 1], device=cuda)
    errs = []
    for b in range(0, B, max(1, B // 2)):
        for h in range(0, H, 7):
            qr = rot(q[b, h, rows], rows)
            sc = (qr @ kr[b, h // (H // Hk)].T) / D ** 0.5
            sc = sc.masked_fill(torch.arange(S, device=cuda)[None, :] > rows[:, None], float("-inf"))
            ref = torch.softmax(sc, -1) @ v[b, h // (H // Hk)].float()
            errs.append((out[b, h, rows].float() - ref).abs())
    err = torch.cat([e.flatten() for e in errs])
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, (err.max().item(), err.mean().item())


@pytest.mark.parametrize("n_copies", [1, 7])
def test_output_copies_inside_the_kernel(cuda, n_copies):
    """cie_prefill_attn_peers on one GPU: the 'peer' outputs are other buffers of
    the same device, so the copy warp's path (its counters, the copy loop, the final
    fence) runs without a second GPU. Short units (S = 512) and seven copies make
    the copy warp fall several units behind the softmax warpgroups, the case its
    counters exist for. Every copy must equal the local output bit for bit, and the
    local output must match the oracle."""
    import torch
    from kernels import _lib, build_rope_cache
    from kernels.flash_attention import flash_attention

    _lib.device_status(clear=True)
    # 512 one-pair units over at most 148 CTAs: each CTA walks several of them
    B, H, Hk, S, D = 8, 64, 16, 512, 128
    q, k, v = normal(31, (B, H, S, D)), normal(32, (B, Hk, S, D)), normal(33, (B, Hk, S, D))
    tq, tk, tv = (to_torch(a, torch.bfloat16, cuda) for a in (q, k, v))
    rope = build_rope_cache(S, D, theta=500000.0, device=cuda)
    # a (B, S, H, D) output layout, as an engine keeps it, viewed as (B, H, S, D)
    out = torch.full((B, S, H, D), float("nan"), dtype=torch.bfloat16, device=cuda)
    copies = [torch.full_like(out, float("nan")) for _ in range(n_copies)]
    view = out.transpose(1, 2)
    res = flash_attention(tq, tk, tv, True, rope=rope, out=view,
                          out_peers=[c.data_ptr() for c in copies])
    torch.cuda.synchronize()
    assert res.data_ptr() == view.data_ptr()
    assert _lib.device_status(clear=True) == 0
    for i, c in enumerate(copies):
        assert torch.equal(c, out), f"copy {i} differs from the local output"
    c_, s_ = oracle.build_rope_cache(S, D, 500000.0)
    assert_close_attn(to_np(view), oracle.prefill_case_ref(q, k, v, c_, s_, causal=True),
                      what="local output")
