"""World-size-2 gloo test of the multi-GPU layer on CPU: each rank computes its
kv-head group (with the oracle standing in for the kernel), one all-gather
reassembles the output, and the result equals the unsharded attention.
Also checks that a rank that fails before the collective surfaces as an error
on the other rank (short process-group timeout), not a hang."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, k, v, ret):
    import sys

    from tests.conftest import PKG, REPO  # noqa: F401  (sets sys.path)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        from engine.head_shard import gather_output, local_heads, rank_major_to_heads, shard_heads

        sh = shard_heads(q.shape[1], k.shape[1], world, rank)
        ql = local_heads(q, sh, kv=False).numpy()
        kl = local_heads(k, sh, kv=True).numpy()
        vl = local_heads(v, sh, kv=True).numpy()
        out = torch.from_numpy(oracle.attention(ql, kl, vl, causal=True))  # (B, hq, M, d)
        gathered = gather_output(out.transpose(1, 2).contiguous())          # (W, B, M, hq, d)
        full = rank_major_to_heads(gathered)                                 # (B, M, Hq, d)
        if rank == 0:
            ret.put(full.numpy())
    finally:
        dist.destroy_process_group()


def test_kv_head_sharding_reassembles_output():
    world = 2
    rng = np.random.default_rng(0)
    B, Hq, Hkv, M, d = 2, 8, 4, 9, 16
    q = torch.from_numpy(rng.standard_normal((B, Hq, M, d), dtype=np.float32))
    k = torch.from_numpy(rng.standard_normal((B, Hkv, M, d), dtype=np.float32))
    v = torch.from_numpy(rng.standard_normal((B, Hkv, M, d), dtype=np.float32))
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, k, v, ret)) for r in range(world)]
    for p in procs:
        p.start()
    full = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    import oracle

    ref = oracle.attention(q.numpy(), k.numpy(), v.numpy(), causal=True).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(full, ref, atol=1e-6)


def _failing_worker(rank, world, port, ret):
    from datetime import timedelta

    from tests.conftest import PKG  # noqa: F401

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # dies between steps, before the collective
    from engine.head_shard import gather_output

    try:
        gather_output(torch.zeros(1, 2, 2, 4))
        ret.put("completed")
    except Exception as e:  # the surviving rank learns of it as an error
        ret.put(f"error: {type(e).__name__}")


def test_dead_rank_surfaces_as_error_not_hang():
    world = 2
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, ret)) for r in range(world)]
    for p in procs:
        p.start()
    msg = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error"), msg
