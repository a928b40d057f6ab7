"""KV-head-group sharding of the attention hot path across GPUs.

Attention needs no communication between kv-head groups: with G = Hq / Hkv,
query heads [g*G, (g+1)*G) only read kv head g. Rank r of W owns kv heads
[r*Hkv/W, (r+1)*Hkv/W) and the matching query heads, computes its slice of the
output with the single-GPU kernels, and one all-gather (NCCL over NVLink /
NVSwitch) reassembles the output, rank-major: [W, B, M, Hq/W, d], which is the
head order of the unsharded [B, M, Hq, d] output after a rank-to-head permute
(an o_proj can consume the rank-major layout directly by permuting its input
rows once). The reference is single-GPU; this module is the multi-GPU layer of
the B200 build.
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
