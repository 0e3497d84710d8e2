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


def gather_stacked(x: torch.Tensor, group=None, async_op: bool = False):
    """All-gather a contiguous per-rank block ``x`` into a new [world, *x.shape]
    tensor (rank r's block at index r) without repacking it.  Returns
    (gathered, work); work is None unless async_op."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    x = x.contiguous()
    out = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    work = dist.all_gather_into_tensor(out, x, group=group, async_op=async_op)
    return out, work


def gather_heads_into(full: torch.Tensor, group=None, async_op: bool = False):
    """In-place all-gather of a head-major buffer ``full`` [world, ...] whose
    slice ``full[rank]`` this rank has already written (for example through a
    [B, H_rank, S, D] view with strides into it): no packing copy, the
    collective reads the slice where the kernels wrote it."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    return dist.all_gather_into_tensor(full, full[rank], group=group, async_op=async_op)


# ---------------------------------------------------------------------------
# Batch sharding for paged decode: sequences are independent, so the batch is
# split across ranks, balanced by key count (greedy longest-processing-time
# list scheduling on the context lengths).  Each rank keeps only its
# sequences' pages in a compact local pool with a renumbered block table; the
# outputs are all-gathered back into batch order.
# ---------------------------------------------------------------------------
def lpt_partition(costs, world: int) -> list[list[int]]:
    """Items in decreasing cost (ties: lower index first), each to the rank
    with the least load so far (ties: lower rank).  Returns the item indices of
    every rank in increasing order.  Deterministic."""
    if world < 1:
        raise ValueError("world must be positive")
    costs = [float(c) for c in costs]
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0.0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda x: (load[x], x))
        parts[r].append(i)
        load[r] += costs[i]
    return [sorted(p) for p in parts]


@dataclass(frozen=True)
class PagedShard:
    rows: tuple              # global batch indices of this rank's sequences, increasing
    key_cache: torch.Tensor  # [local_pages * page_size, Hkv, D]
    value_cache: torch.Tensor
    block_table: torch.Tensor  # int32 [len(rows), max_blocks], local page ids
    seq_lens: torch.Tensor     # int32 [len(rows)]


def shard_paged_batch(key_cache, value_cache, block_table, seq_lens, page_size: int, rows) -> PagedShard:
    """The pages of sequences ``rows`` copied into a compact local pool (in
    order of first use) with the block table renumbered to it."""
    rows = tuple(int(r) for r in rows)
    lens = seq_lens.to("cpu", torch.int64)[list(rows)]
    table = block_table.to("cpu", torch.int64)[list(rows)]
    npages = [(int(n) + page_size - 1) // page_size for n in lens]
    width = max(npages, default=0) or 1
    local = torch.zeros(len(rows), width, dtype=torch.int32)
    phys = []
    for i, n in enumerate(npages):
        local[i, :n] = torch.arange(len(phys), len(phys) + n, dtype=torch.int32)
        phys.extend(int(x) for x in table[i, :n])
    dev = key_cache.device
    tok = (torch.tensor(phys, dtype=torch.int64)[:, None] * page_size
           + torch.arange(page_size, dtype=torch.int64)[None]).reshape(-1).to(dev)
    return PagedShard(rows, key_cache.index_select(0, tok), value_cache.index_select(0, tok),
                      local.to(block_table.device), lens.to(torch.int32).to(seq_lens.device))


def batch_gather_order(parts: list[list[int]]):
    """(slots per rank, index of every global row in the padded gather buffer)."""
    nmax = max(len(p) for p in parts)
    pos = [r * nmax + j for r in range(len(parts)) for j in range(len(parts[r]))]
    glob = [i for p in parts for i in p]
    order = torch.empty(len(glob), dtype=torch.int64)
    order[torch.tensor(glob, dtype=torch.int64)] = torch.tensor(pos, dtype=torch.int64)
    return nmax, order


def gather_batch(x: torch.Tensor, parts: list[list[int]], group=None, order=None) -> torch.Tensor:
    """All-gather per-rank batch slices (``x`` holds this rank's rows, in the
    order of ``parts[rank]``) back into global batch order.  Slices are padded
    to the largest part so that one all_gather_into_tensor moves them.
    ``order`` may hold a precomputed ``batch_gather_order(parts)``."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    nmax, idx = order if order is not None else batch_gather_order(parts)
    send = x.new_zeros((nmax,) + tuple(x.shape[1:]))
    send[: len(parts[rank])] = x
    buf = x.new_empty((world * nmax,) + tuple(x.shape[1:]))
    dist.all_gather_into_tensor(buf, send, group=group)
    return buf.index_select(0, idx.to(buf.device))
