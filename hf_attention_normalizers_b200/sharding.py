"""Head-group sharding of attention across the GPUs of one node.

(batch, KV-head group) units are independent: a KV head and its
Hq/Hkv query heads need nothing from any other group, and every normalizer's
row reduction (softmax1 denominator, sparsemax/entmax15 threshold) stays
inside one query head.  So a job splits the KV heads into contiguous blocks,
one per rank, runs the single-GPU kernels on its block, and gathers the
per-head results along the head dimension -- the only collective.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    kv_lo: int
    kv_hi: int
    q_lo: int
    q_hi: int


def kv_group_shard(heads_q: int, heads_kv: int, world: int, rank: int) -> HeadShard:
    """Contiguous block of KV heads (and their query heads) owned by `rank`."""
    if heads_q % heads_kv:
        raise ValueError("Query heads must be divisible by KV heads.")
    if heads_kv % world:
        raise ValueError(f"{heads_kv} KV heads cannot be split evenly over {world} ranks")
    per = heads_kv // world
    g = heads_q // heads_kv
    return HeadShard(rank * per, (rank + 1) * per, rank * per * g, (rank + 1) * per * g)


def gather_heads(x: torch.Tensor, head_dim_index: int = 1, group=None) -> torch.Tensor:
    """All-gather per-rank head blocks into the full tensor (heads concatenated
    in rank order along `head_dim_index`)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if world == 1:
        return x
    x = x.movedim(head_dim_index, 0).contiguous()
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)
    return out.movedim(0, head_dim_index)
