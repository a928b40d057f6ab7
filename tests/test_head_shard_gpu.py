"""Multi-GPU: kv-head-group sharding gives the one-GPU result, bit for bit.

Two ranks (one process per GPU) each hold half of the kv-head groups of a
causal RoPE prefill and of a paged decode batch (pools split by head, identical
block tables), run the single-GPU kernels on their slice and reassemble the
output, two ways: an NCCL all-gather (rank-major -> global head order), and the
fused path, where the prefill kernel stores each output tile into every rank's
full output over NVLink (symmetric memory) and a peer barrier closes the step.
Every head runs the same kernel on the same inputs as on one GPU, so the
reassembled output must equal the one-GPU output exactly. Skipped with fewer
than two GPUs.
"""

from __future__ import annotations

import os
import socket

import pytest

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errq):
    import sys
    from datetime import timedelta
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (str(repo), str(repo / "custom-inference-engine_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    try:
        import torch
        import torch.distributed as dist

        from engine.head_shard import gather_output, local_heads, shard_heads
        from kernels import build_rope_cache
        from kernels.flash_attention import flash_attention, paged_attention

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        g = torch.Generator(device=dev).manual_seed(5)
        # prefill: B=2, Hq=8, Hkv=2, S=640, d=128, RoPE on q and k
        B, Hq, Hkv, S, d = 2, 8, 2, 640, 128
        q = torch.randn(B, Hq, S, d, device=dev, generator=g).bfloat16()
        k = torch.randn(B, Hkv, S, d, device=dev, generator=g).bfloat16()
        v = torch.randn(B, Hkv, S, d, device=dev, generator=g).bfloat16()
        rope = build_rope_cache(4096, d, theta=500000.0, device=dev)
        sh = shard_heads(Hq, Hkv, world, rank)
        o = flash_attention(local_heads(q, sh, False), local_heads(k, sh, True),
                            local_heads(v, sh, True), True, rope=rope)
        got = gather_output(o)                              # (W, B, hq, S, d)
        got = got.permute(1, 0, 2, 3, 4).reshape(B, Hq, S, d)
        want = flash_attention(q, k, v, True, rope=rope)
        assert torch.equal(got, want), "sharded prefill differs from one GPU"

        # paged decode / verify: B=3, M=5, Hq=8, Hkv=2, d=128, block size 16
        lens = [37, 1500, 3001]
        M, bs = 5, 16
        nblk = [(L + bs - 1) // bs for L in lens]
        perm = torch.randperm(sum(nblk), generator=torch.Generator().manual_seed(3))
        tables = torch.zeros(3, max(nblk), dtype=torch.int32)
        off = 0
        for i, n in enumerate(nblk):
            tables[i, :n] = perm[off: off + n]
            off += n
        tables = tables.to(dev)
        kv_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
        kp = torch.randn(sum(nblk), bs, Hkv, d, device=dev, generator=g).bfloat16()
        vp = torch.randn(sum(nblk), bs, Hkv, d, device=dev, generator=g).bfloat16()
        qd = torch.randn(3, Hq, M, d, device=dev, generator=g).bfloat16()
        od = paged_attention(local_heads(qd, sh, False),
                             local_heads(kp, sh, True, head_dim=2).contiguous(),
                             local_heads(vp, sh, True, head_dim=2).contiguous(),
                             tables, kv_lens, True, rope=rope)
        gotd = gather_output(od).permute(1, 0, 2, 3, 4).reshape(3, Hq, M, d)
        wantd = paged_attention(qd, kp, vp, tables, kv_lens, True, rope=rope)
        assert torch.equal(gotd, wantd), "sharded paged attention differs from one GPU"

        # the fused path: output tiles stored into every rank's full output by the
        # kernel itself (symmetric memory), closed by the peer barrier; three steps
        # so that both alternating buffers are used and one is reused
        from engine.head_shard import PeerOutput

        po = PeerOutput((B, Hq, S, d), torch.bfloat16, dev)
        for step in range(3):
            full = po.attention(local_heads(q, sh, False), local_heads(k, sh, True),
                                local_heads(v, sh, True), sh, True, rope=rope)
            torch.cuda.synchronize()
            assert torch.equal(full, want), f"fused peer gather differs from one GPU (step {step})"
        from kernels import _lib

        assert _lib.device_status(clear=True) == 0
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, which fails the test
        import traceback

        errq.put(f"rank {rank}: {e!r}\n{traceback.format_exc()}")
        raise


def test_two_gpu_sharding_matches_one_gpu():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, errq)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "a rank did not finish in time"
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
