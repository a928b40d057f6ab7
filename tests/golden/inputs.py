"""Seeded inputs shared by the golden generator and the tests.

Everything is drawn from numpy's PCG64 (``np.random.default_rng(seed)``), whose
stream is fixed by specification, and rounded to bfloat16 (kept as float32), so
the tests regenerate exactly the inputs the goldens were computed from.
"""

from __future__ import annotations

import numpy as np


def bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def normal(seed: int, shape) -> np.ndarray:
    return bf16(np.random.default_rng(seed).standard_normal(shape, dtype=np.float32))


ROPE_TABLE_CASES = {
    "d16": (64, 16, 10000.0),
    "d64": (520, 64, 500000.0),
    "d128": (64, 128, 500000.0),
}

ROTARY_CASES = {
    "pos1d": {"shape": (2, 3, 5, 16), "max_pos": 32, "theta": 10000.0, "seed": 11,
              "positions": [0, 1, 7, 30, 4]},
    "pos2d": {"shape": (2, 2, 4, 64), "max_pos": 600, "theta": 500000.0, "seed": 12,
              "positions": [[0, 5, 511, 599], [3, 3, 100, 200]]},
}


def rotary_inputs(case):
    x = normal(case["seed"], case["shape"])
    pos = np.asarray(case["positions"], dtype=np.int64)
    return x, pos


# (B, H, Hk, Lq, Lk, D)
ATTN_CASES = {
    "ref_small": {"shape": (1, 2, 2, 4, 4, 8), "causal": False, "seed": 21},
    "ref_b2": {"shape": (2, 4, 4, 8, 16, 16), "causal": False, "seed": 22},
    "causal_sq": {"shape": (1, 1, 1, 4, 4, 8), "causal": True, "seed": 23},
    "gqa": {"shape": (1, 4, 2, 3, 3, 8), "causal": False, "seed": 24},
    "causal_br_gqa": {"shape": (1, 8, 2, 5, 37, 16), "causal": True, "seed": 25},
    "causal_m_gt_n": {"shape": (1, 2, 1, 6, 3, 16), "causal": True, "seed": 26},
    "empty_keys": {"shape": (1, 2, 2, 3, 0, 16), "causal": False, "seed": 27},
    "masked": {"shape": (1, 2, 2, 4, 6, 16), "causal": False, "seed": 28, "mask": True},
    "scaled": {"shape": (1, 2, 1, 7, 9, 32), "causal": True, "seed": 29, "scale": 0.3},
    "rope_d64": {"shape": (1, 4, 2, 140, 140, 64), "causal": True, "seed": 30, "rope": True,
                 "theta": 500000.0},
    "rope_d128_chunk": {"shape": (1, 4, 1, 130, 200, 128), "causal": True, "seed": 31,
                        "rope": True, "theta": 500000.0},
}


def attn_inputs(case):
    B, H, Hk, Lq, Lk, D = case["shape"]
    s = case["seed"]
    q = normal(s * 10 + 1, (B, H, Lq, D))
    k = normal(s * 10 + 2, (B, Hk, Lk, D))
    v = normal(s * 10 + 3, (B, Hk, Lk, D))
    mask = None
    if case.get("mask"):
        mask = (np.random.default_rng(s * 10 + 4).standard_normal((1, 1, Lq, Lk)) *
                2.0).astype(np.float32)
    return q, k, v, mask


CFG1 = {"B": 1, "Hq": 32, "Hkv": 8, "S": 512, "d": 64, "theta": 500000.0, "seed": 5,
        "sample_rows": list(range(0, 512, 32)) + [1, 2, 511]}


def cfg1_inputs():
    c = CFG1
    q = normal(c["seed"] * 10 + 1, (c["B"], c["Hq"], c["S"], c["d"]))
    k = normal(c["seed"] * 10 + 2, (c["B"], c["Hkv"], c["S"], c["d"]))
    v = normal(c["seed"] * 10 + 3, (c["B"], c["Hkv"], c["S"], c["d"]))
    return q, k, v


# paged decode / verify: per sequence q (1, Hq, M, d), raw K/V rows (L, Hkv, d)
DECODE_CASES = {
    "decode_d64": {"Hq": 8, "Hkv": 2, "d": 64, "M": 1, "block_size": 16,
                   "kv_lens": [5, 17, 33, 130], "theta": 500000.0, "seed": 41},
    "verify_d128": {"Hq": 8, "Hkv": 2, "d": 128, "M": 5, "block_size": 16,
                    "kv_lens": [5, 16, 21, 77], "theta": 500000.0, "seed": 42},
    "decode_bs8_d16": {"Hq": 2, "Hkv": 2, "d": 16, "M": 1, "block_size": 8,
                       "kv_lens": [1, 8, 9, 23], "theta": 10000.0, "seed": 43},
}


def decode_inputs(case):
    qs, ks, vs = [], [], []
    for i, L in enumerate(case["kv_lens"]):
        s = case["seed"] * 100 + i * 3
        qs.append(normal(s + 1, (1, case["Hq"], case["M"], case["d"])))
        ks.append(normal(s + 2, (L, case["Hkv"], case["d"])))
        vs.append(normal(s + 3, (L, case["Hkv"], case["d"])))
    return qs, ks, vs


# weight-only INT8 GEMM (kernels/ref/int8_matmul_ref.py); "group" > 0 uses the
# reference function's per-group scale layout (oracle only: the GPU entry, like
# the reference's Triton entry, takes per-channel scales)
INT8_CASES = {
    "decode_bias": dict(seed=101, M=3, N=96, K=160, bias=True, group=0),
    "prefill": dict(seed=102, M=130, N=200, K=256, bias=False, group=0),
    "per_group": dict(seed=103, M=5, N=64, K=128, bias=False, group=32),
}


def int8_inputs(case):
    rng = np.random.default_rng(case["seed"])
    M, N, K = case["M"], case["N"], case["K"]
    x = bf16(rng.standard_normal((M, K)).astype(np.float32))
    w = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    if case["group"]:
        scales = rng.uniform(0.001, 0.02, size=(N, K // case["group"])).astype(np.float32)
    else:
        scales = rng.uniform(0.001, 0.02, size=(N,)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32) if case["bias"] else None
    return x, w, scales, bias
