"""Generate the golden vectors that pin the oracle to the reference.

Run in a container that has the reference source tree (it is read, never
modified, and never needed at test time):

    python tests/golden/make_golden.py --reference /path/to/Custom-Inference-Engine

It imports the reference's own CPU code —
  kernels.ref.build_rope_cache / apply_rotary_ref   (kernels/ref/rope_apply_ref.py)
  kernels.ref.flash_attention_ref                   (kernels/ref/flash_attention_ref.py)
  engine.cache.PagedKVCache / BlockTable            (engine/cache/*.py)
  kernels.ref.int8_matmul_ref.int8_matmul_ref       (kernels/ref/int8_matmul_ref.py)
— runs them on seeded inputs (numpy PCG64, so the inputs can be regenerated
bit-identically anywhere) and writes the results to tests/golden/*.npz.
Inputs are rounded to bfloat16 first, as the GPU path stores them.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))  # repo root, for tests.golden.inputs
from tests.golden.inputs import (  # noqa: E402
    ATTN_CASES,
    CFG1,
    DECODE_CASES,
    INT8_CASES,
    ROPE_TABLE_CASES,
    ROTARY_CASES,
    attn_inputs,
    cfg1_inputs,
    decode_inputs,
    int8_inputs,
    rotary_inputs,
)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference source tree")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from engine.cache.kv_cache import KVCacheConfig, PagedKVCache
    from kernels.ref import apply_rotary_ref, build_rope_cache, flash_attention_ref

    torch.set_num_threads(1)
    out: dict[str, np.ndarray] = {}

    # 1) RoPE tables
    for name, (L, d, theta) in ROPE_TABLE_CASES.items():
        c, s = build_rope_cache(L, d, theta=theta)
        out[f"rope_{name}_cos"] = c.numpy()
        out[f"rope_{name}_sin"] = s.numpy()

    # 2) apply_rotary_ref
    for name, case in ROTARY_CASES.items():
        x, pos = rotary_inputs(case)
        c, s = build_rope_cache(case["max_pos"], case["shape"][-1], theta=case["theta"])
        y = apply_rotary_ref(torch.from_numpy(x), c, s, positions=torch.from_numpy(pos))
        out[f"rotary_{name}"] = y.numpy()

    # 3) flash_attention_ref (+ RoPE on q/k where the case asks for it)
    for name, case in ATTN_CASES.items():
        q, k, v, mask = attn_inputs(case)
        qt, kt, vt = (torch.from_numpy(a) for a in (q, k, v))
        if case.get("rope"):
            L = max(q.shape[2], k.shape[2]) + 8
            c, s = build_rope_cache(L, q.shape[-1], theta=case["theta"])
            M, N = q.shape[2], k.shape[2]
            qt = apply_rotary_ref(qt, c, s, positions=torch.arange(N - M, N))
            kt = apply_rotary_ref(kt, c, s, positions=torch.arange(N))
        mt = torch.from_numpy(mask) if mask is not None else None
        o = flash_attention_ref(qt, kt, vt, mask=mt, causal=case["causal"], scale=case.get("scale"))
        out[f"attn_{name}"] = o.numpy()

    # 4) config 1 (Llama-3.2-1B prefill, CPU path): sampled rows of the output
    q, k, v = cfg1_inputs()
    c, s = build_rope_cache(CFG1["S"], CFG1["d"], theta=CFG1["theta"])
    pos = torch.arange(CFG1["S"])
    qr = apply_rotary_ref(torch.from_numpy(q), c, s, positions=pos)
    kr = apply_rotary_ref(torch.from_numpy(k), c, s, positions=pos)
    o = flash_attention_ref(qr, kr, torch.from_numpy(v), causal=True, scale=1.0 / 8.0)
    out["cfg1_rows"] = o[:, :, CFG1["sample_rows"], :].numpy()
    out["cfg1_sum"] = np.array([o.double().sum().item(), o.double().abs().sum().item()])

    # 5) paged decode / verify through the reference cache + attention
    for name, case in DECODE_CASES.items():
        qs, ks, vs = decode_inputs(case)
        bs, Hkv, d = case["block_size"], case["Hkv"], case["d"]
        nblocks = sum((L + bs - 1) // bs for L in case["kv_lens"]) + 4
        cache = PagedKVCache(KVCacheConfig(num_layers=1, num_kv_heads=Hkv, head_dim=d,
                                           num_blocks=nblocks, block_size=bs,
                                           dtype=torch.float32, device="cpu"))
        c, s = build_rope_cache(max(case["kv_lens"]) + 8, d, theta=case["theta"])
        outs, tables = [], []
        for i, L in enumerate(case["kv_lens"]):
            t = cache.new_sequence()
            kt = torch.from_numpy(ks[i])  # (L, Hkv, d), raw
            krot = apply_rotary_ref(kt.permute(1, 0, 2).unsqueeze(0), c, s,
                                    positions=torch.arange(L))[0].permute(1, 0, 2)
            cache.append(0, t, krot.contiguous(), torch.from_numpy(vs[i]))
            gk, gv = cache.gather(0, t)
            M = case["M"]
            qr = apply_rotary_ref(torch.from_numpy(qs[i]), c, s, positions=torch.arange(L - M, L))
            o = flash_attention_ref(qr, gk.permute(1, 0, 2).unsqueeze(0),
                                    gv.permute(1, 0, 2).unsqueeze(0), causal=True)
            outs.append(o.numpy())
            tables.append(list(t.blocks))
            out[f"decode_{name}_gk{i}"] = gk.numpy()
        out[f"decode_{name}_out"] = np.concatenate(outs, axis=0)
        out[f"decode_{name}_tables"] = np.array(
            [tb + [-1] * (max(map(len, tables)) - len(tb)) for tb in tables], dtype=np.int32)

    # 6) a scripted cache lifecycle (append / decode / fork / rollback / free)
    cache = PagedKVCache(KVCacheConfig(num_layers=2, num_kv_heads=2, head_dim=16, num_blocks=12,
                                       block_size=4, dtype=torch.float32, device="cpu"))
    rng = np.random.default_rng(1234)
    log = []
    a = cache.new_sequence()
    b = cache.new_sequence()

    def rows(n):
        return torch.from_numpy(rng.standard_normal((n, 2, 16)).astype(np.float32))

    for layer in range(2):
        cache.append(layer, a, rows(6), rows(6), start=0)
    log.append(("append_a6", list(a.blocks), a.length, list(cache._free)))
    for layer in range(2):
        cache.append(layer, b, rows(3), rows(3), start=0)
    log.append(("append_b3", list(b.blocks), b.length, list(cache._free)))
    for layer in range(2):
        cache.append(layer, a, rows(3), rows(3), start=6)
    log.append(("append_a3", list(a.blocks), a.length, list(cache._free)))
    f = cache.fork(a)
    log.append(("fork_a", list(f.blocks), f.length, list(cache._free)))
    cache.rollback(a, 5)
    log.append(("rollback_a5", list(a.blocks), a.length, list(cache._free)))
    for layer in range(2):
        cache.append(layer, a, rows(4), rows(4), start=5)
    log.append(("append_a4", list(a.blocks), a.length, list(cache._free)))
    cache.free_sequence(b)
    log.append(("free_b", list(b.blocks), b.length, list(cache._free)))
    for layer in range(2):
        ga_k, ga_v = cache.gather(layer, a)
        gf_k, gf_v = cache.gather(layer, f)
        out[f"life_a_k{layer}"] = ga_k.numpy()
        out[f"life_a_v{layer}"] = ga_v.numpy()
        out[f"life_f_k{layer}"] = gf_k.numpy()
    out["life_log"] = np.frombuffer(json.dumps(log).encode(), dtype=np.uint8)

    # 6) int8_matmul_ref (weight-only INT8 GEMM)
    from kernels.ref.int8_matmul_ref import int8_matmul_ref

    for name, case in INT8_CASES.items():
        x, w, scales, bias = int8_inputs(case)
        y = int8_matmul_ref(torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(scales),
                            group_size=case["group"] or None,
                            bias=torch.from_numpy(bias) if bias is not None else None)
        out[f"int8_{name}"] = y.numpy()

    np.savez_compressed(HERE / "golden.npz", **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {HERE / 'golden.npz'}: {len(out)} arrays, {total / 1e6:.2f} MB raw")


if __name__ == "__main__":
    main()
