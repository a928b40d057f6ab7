"""Pin the CPU oracle to the reference: every golden vector produced by the
reference's own kernels.ref / engine.cache code (tests/golden/make_golden.py)
must be reproduced by oracle/ on the same seeded inputs."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

import oracle
from tests.golden.inputs import (
    INT8_CASES,
    int8_inputs,
    ATTN_CASES,
    CFG1,
    DECODE_CASES,
    ROPE_TABLE_CASES,
    ROTARY_CASES,
    attn_inputs,
    cfg1_inputs,
    decode_inputs,
    rotary_inputs,
)


@pytest.mark.parametrize("name", sorted(ROPE_TABLE_CASES))
def test_rope_tables_match_reference(golden, name):
    L, d, theta = ROPE_TABLE_CASES[name]
    c, s = oracle.build_rope_cache(L, d, theta)
    # identical angles; cos/sin within one fp32 ulp of torch's
    np.testing.assert_allclose(c, golden[f"rope_{name}_cos"], rtol=0, atol=1.2e-7)
    np.testing.assert_allclose(s, golden[f"rope_{name}_sin"], rtol=0, atol=1.2e-7)


@pytest.mark.parametrize("name", sorted(ROTARY_CASES))
def test_apply_rotary_matches_reference(golden, name):
    case = ROTARY_CASES[name]
    x, pos = rotary_inputs(case)
    c, s = oracle.build_rope_cache(case["max_pos"], case["shape"][-1], case["theta"])
    y = oracle.apply_rotary(x, c, s, pos)
    np.testing.assert_allclose(y, golden[f"rotary_{name}"], rtol=0, atol=1e-5)


def test_rotary_identity_at_zero_and_norm_preserving():
    # the reference's own properties (tests/kernels/test_rope_ref.py:9-27)
    c, s = oracle.build_rope_cache(32, 16)
    x = np.random.default_rng(0).standard_normal((2, 4, 5, 16)).astype(np.float32)
    y0 = oracle.apply_rotary(x[:, :, :1], c, s, np.array([0]))
    np.testing.assert_allclose(y0, x[:, :, :1], atol=1e-6)
    y = oracle.apply_rotary(x, c, s)
    np.testing.assert_allclose(x[..., :8] ** 2 + x[..., 8:] ** 2,
                               y[..., :8] ** 2 + y[..., 8:] ** 2, atol=1e-5)


@pytest.mark.parametrize("name", sorted(ATTN_CASES))
def test_attention_matches_reference(golden, name):
    case = ATTN_CASES[name]
    q, k, v, mask = attn_inputs(case)
    if case.get("rope"):
        L = max(q.shape[2], k.shape[2]) + 8
        c, s = oracle.build_rope_cache(L, q.shape[-1], case["theta"])
        M, N = q.shape[2], k.shape[2]
        q = oracle.apply_rotary(q, c, s, np.arange(N - M, N))
        k = oracle.apply_rotary(k, c, s, np.arange(N))
    o = oracle.attention(q, k, v, mask=mask, causal=case["causal"], scale=case.get("scale"))
    ref = golden[f"attn_{name}"]
    assert o.shape == ref.shape
    np.testing.assert_array_equal(np.isnan(o), np.isnan(ref))
    ok = ~np.isnan(ref)
    np.testing.assert_allclose(o[ok], ref[ok], rtol=0, atol=2e-5)


def test_attention_matches_manual_softmax():
    # reference tests/kernels/test_flash_attention_ref.py:11-20
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((2, 4, 8, 16)).astype(np.float32) for _ in range(3))
    out = oracle.attention(q, k, v)
    sc = q @ k.transpose(0, 1, 3, 2) / math.sqrt(16)
    e = np.exp(sc - sc.max(-1, keepdims=True))
    np.testing.assert_allclose(out, (e / e.sum(-1, keepdims=True)) @ v, atol=1e-5)


def test_config1_matches_reference(golden):
    q, k, v = cfg1_inputs()
    c, s = oracle.build_rope_cache(CFG1["S"], CFG1["d"], CFG1["theta"])
    o = oracle.prefill_case_ref(q, k, v, c, s, causal=True, scale=1 / 8)
    np.testing.assert_allclose(o[:, :, CFG1["sample_rows"]], golden["cfg1_rows"], atol=2e-5)
    tot = o.astype(np.float64).sum()
    assert abs(tot - golden["cfg1_sum"][0]) < 1e-2
    assert abs(np.abs(o.astype(np.float64)).sum() - golden["cfg1_sum"][1]) < 1e-1


@pytest.mark.parametrize("name", sorted(DECODE_CASES))
def test_paged_decode_matches_reference(golden, name):
    case = DECODE_CASES[name]
    qs, ks, vs = decode_inputs(case)
    bs, Hkv, d = case["block_size"], case["Hkv"], case["d"]
    nblocks = sum((L + bs - 1) // bs for L in case["kv_lens"]) + 4
    cache = oracle.PagedKVCacheRef(1, Hkv, d, nblocks, bs)
    c, s = oracle.build_rope_cache(max(case["kv_lens"]) + 8, d, case["theta"])
    outs = []
    for i, L in enumerate(case["kv_lens"]):
        t = cache.new_sequence()
        krot = oracle.apply_rotary(ks[i].transpose(1, 0, 2)[None], c, s, np.arange(L))[0]
        cache.append(0, t, krot.transpose(1, 0, 2), vs[i])
        gk, gv = cache.gather(0, t)
        # block ids follow the reference's LIFO allocator exactly
        ref_tab = golden[f"decode_{name}_tables"][i]
        assert t.blocks == [int(x) for x in ref_tab if x >= 0]
        # K was rotated with tables that agree with torch's to one fp32 ulp; the
        # gather itself is bit-exact (test_cache_lifecycle_matches_reference)
        np.testing.assert_allclose(gk, golden[f"decode_{name}_gk{i}"], rtol=0, atol=2e-6)
        outs.append(oracle.decode_case_ref(qs[i], gk.transpose(1, 0, 2)[None],
                                           gv.transpose(1, 0, 2)[None], c, s))
    np.testing.assert_allclose(np.concatenate(outs), golden[f"decode_{name}_out"], atol=2e-5)


def test_cache_lifecycle_matches_reference(golden):
    log = json.loads(bytes(golden["life_log"]).decode())
    cache = oracle.PagedKVCacheRef(2, 2, 16, 12, 4)
    rng = np.random.default_rng(1234)
    a, b = cache.new_sequence(), cache.new_sequence()

    def rows(n):
        return rng.standard_normal((n, 2, 16)).astype(np.float32)

    mine = []
    for layer in range(2):
        cache.append(layer, a, rows(6), rows(6), start=0)
    mine.append(("append_a6", list(a.blocks), a.length, list(cache._free)))
    for layer in range(2):
        cache.append(layer, b, rows(3), rows(3), start=0)
    mine.append(("append_b3", list(b.blocks), b.length, list(cache._free)))
    for layer in range(2):
        cache.append(layer, a, rows(3), rows(3), start=6)
    mine.append(("append_a3", list(a.blocks), a.length, list(cache._free)))
    f = cache.fork(a)
    mine.append(("fork_a", list(f.blocks), f.length, list(cache._free)))
    cache.rollback(a, 5)
    mine.append(("rollback_a5", list(a.blocks), a.length, list(cache._free)))
    for layer in range(2):
        cache.append(layer, a, rows(4), rows(4), start=5)
    mine.append(("append_a4", list(a.blocks), a.length, list(cache._free)))
    cache.free_sequence(b)
    mine.append(("free_b", list(b.blocks), b.length, list(cache._free)))
    assert [list(x) for x in mine] == [list(x) for x in log]
    for layer in range(2):
        ak, av = cache.gather(layer, a)
        fk, _ = cache.gather(layer, f)
        np.testing.assert_array_equal(ak, golden[f"life_a_k{layer}"])
        np.testing.assert_array_equal(av, golden[f"life_a_v{layer}"])
        np.testing.assert_array_equal(fk, golden[f"life_f_k{layer}"])


def test_gather_tables_matches_cache_gather():
    rng = np.random.default_rng(3)
    cache = oracle.PagedKVCacheRef(1, 2, 16, 40, 4)
    tabs, lens = [], []
    for L in (1, 4, 9, 30):
        t = cache.new_sequence()
        cache.append(0, t, rng.standard_normal((L, 2, 16)).astype(np.float32),
                     rng.standard_normal((L, 2, 16)).astype(np.float32))
        tabs.append(t)
        lens.append(L)
    maxb = max(len(t.blocks) for t in tabs)
    table = np.array([t.blocks + [0] * (maxb - len(t.blocks)) for t in tabs], dtype=np.int32)
    out = oracle.gather_tables(cache.k[0], table, np.array(lens), 32)
    for i, t in enumerate(tabs):
        np.testing.assert_array_equal(out[i, :lens[i]], cache.gather(0, t)[0])


# reference kernels/ref/int8_matmul_ref.py:31-47 (and tests/quant's dequantize round trip)
@pytest.mark.parametrize("name", sorted(INT8_CASES))
def test_int8_matmul_matches_reference(golden, name):
    case = INT8_CASES[name]
    x, w, scales, bias = int8_inputs(case)
    y = oracle.int8_matmul(x, w, scales, group_size=case["group"] or None, bias=bias)
    np.testing.assert_allclose(y, golden[f"int8_{name}"], rtol=1e-5, atol=1e-5)


def test_dequantize_per_group_equals_per_channel_when_uniform():
    rng = np.random.default_rng(7)
    w = rng.integers(-128, 128, size=(8, 64), dtype=np.int8)
    s = rng.uniform(0.01, 0.1, size=8).astype(np.float32)
    per_group = np.repeat(s[:, None], 4, axis=1)
    np.testing.assert_array_equal(oracle.dequantize_int8(w, s),
                                  oracle.dequantize_int8(w, per_group, group_size=16))
