"""KV-head-group sharding of the attention hot path across GPUs.

Attention needs no communication between kv-head groups: with G = Hq / Hkv,
query heads [g*G, (g+1)*G) only read kv head g. Rank r of W owns kv heads
[r*Hkv/W, (r+1)*Hkv/W) and the matching query heads, computes its slice of the
output with the single-GPU kernels, and the output is reassembled on every
rank in one of two ways:

* ``PeerOutput``: the prefill kernel itself writes each finished output tile
  into every rank's copy of the full output (peer stores over NVLink, in
  symmetric memory), overlapping the transfer with the attention math, and a
  stream-ordered peer barrier closes the step; the result is the full output in
  global head order on every rank, with no collective launch;
* ``gather_output``: one NCCL all-gather of the rank-major [W, B, M, Hq/W, d]
  output (``rank_major_to_heads`` permutes it to global head order; an o_proj
  can consume the rank-major layout directly by permuting its input rows once).

The reference is single-GPU; this module is the multi-GPU layer of the B200
build.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    hq: int      # query heads on this rank
    hkv: int     # kv heads on this rank
    q0: int      # first global query head
    kv0: int     # first global kv head


def shard_heads(num_heads: int, num_kv_heads: int, world: int, rank: int) -> HeadShard:
    """Split kv-head groups evenly; every rank keeps whole GQA groups."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if num_heads % num_kv_heads:
        raise ValueError(f"num_heads {num_heads} not a multiple of num_kv_heads {num_kv_heads}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads cannot be split over {world} ranks")
    g = num_heads // num_kv_heads
    hkv = num_kv_heads // world
    return HeadShard(rank, world, hkv * g, hkv, rank * hkv * g, rank * hkv)


def local_heads(x: torch.Tensor, shard: HeadShard, kv: bool, head_dim: int = 1) -> torch.Tensor:
    """This rank's slice of a (B, H, L, d) (head_dim=1) or (B, L, H, d) (head_dim=2) tensor."""
    start, n = (shard.kv0, shard.hkv) if kv else (shard.q0, shard.hq)
    return x.narrow(head_dim, start, n)


def gather_output(local_out: torch.Tensor, group=None, async_op: bool = False):
    """All-gather each rank's (B, M, Hq/W, d) output into (W, B, M, Hq/W, d).

    Uses one ``all_gather_into_tensor`` (NCCL on GPUs, gloo on CPU).
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    # rank-major concatenation along dim 0 (the layout every backend accepts)
    flat = torch.empty((world * local_out.shape[0], *local_out.shape[1:]), dtype=local_out.dtype,
                       device=local_out.device)
    out = flat.view(world, *local_out.shape)
    if world == 1:
        out[0].copy_(local_out)
        return (out, None) if async_op else out
    work = dist.all_gather_into_tensor(flat, local_out.contiguous(), group=group,
                                       async_op=async_op)
    return (out, work) if async_op else out


def rank_major_to_heads(gathered: torch.Tensor) -> torch.Tensor:
    """(W, B, M, Hq/W, d) -> (B, M, Hq, d) in global head order (a copy)."""
    W, B, M, hl, d = gathered.shape
    return gathered.permute(1, 2, 0, 3, 4).reshape(B, M, W * hl, d)


class PeerOutput:
    """The full attention output held in symmetric memory on every rank.

    Each rank runs the fused prefill (``kernels.flash_attention.flash_attention``
    with ``out_peers``) on its kv-head group: the kernel writes every output tile
    to this rank's slice of the full output and copies it, while it computes, to
    the same slice of every other rank's copy; ``cie_peer_barrier`` then closes
    the step. Two output buffers alternate between calls, so a rank that runs
    ahead (by at most one step: the barrier) never writes into a buffer another
    rank is still reading.
    """

    def __init__(self, shape, dtype, device, group=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = torch.device(device)
        self.bufs, self.hdls = [], []
        for _ in range(2):
            t = symm_mem.empty(*shape, dtype=dtype, device=self.device)
            self.bufs.append(t)
            self.hdls.append(symm_mem.rendezvous(t, self.group))
        self.flags = symm_mem.empty(self.world, dtype=torch.int32, device=self.device)
        self.flags.zero_()
        self.fhdl = symm_mem.rendezvous(self.flags, self.group)
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        self.flag_ptrs = [int(p) for p in self.fhdl.buffer_ptrs]
        self.epoch = 0

    def next_buffer(self):
        """The output buffer of the next step (alternating)."""
        return self.bufs[self.epoch % 2], self.hdls[self.epoch % 2]

    def peers_of(self, view, hdl) -> list[int]:
        """Addresses of ``view`` (a slice of a buffer) in the other ranks' buffers."""
        base = self.bufs[self.epoch % 2]
        off = view.data_ptr() - base.data_ptr()
        return [int(hdl.buffer_ptrs[r]) + off for r in range(self.world) if r != self.rank]

    def attention(self, q, k, v, shard: "HeadShard", causal=True, scale=None, *, rope=None,
                  rope_q_pos0=None, rope_k=True, head_dim: int = 1, on_kernel_done=None):
        """This rank's heads of the prefill, written into every rank's full output.
        Returns the full output (global head order along ``head_dim``) of this step.
        ``on_kernel_done`` (e.g. a CUDA event's ``record``) is called between the
        kernel and the barrier."""
        from kernels.flash_attention import flash_attention, peer_barrier

        full, hdl = self.next_buffer()
        view = full.narrow(head_dim, shard.q0, shard.hq)
        if head_dim != 1:
            view = view.transpose(1, head_dim)
        flash_attention(q, k, v, causal, scale, rope=rope, rope_q_pos0=rope_q_pos0, rope_k=rope_k,
                        out=view, out_peers=self.peers_of(view, hdl))
        if on_kernel_done is not None:
            on_kernel_done()
        self.epoch += 1
        peer_barrier(self.flag_ptrs, self.rank, self.epoch, self.device)
        return full
