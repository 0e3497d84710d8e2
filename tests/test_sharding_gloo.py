"""Multi-rank host logic on CPU (gloo, world size 2): each rank computes the
oracle attention of its KV-head block and the head all-gather reassembles the
single-process result exactly."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hf_attention_normalizers_b200.sharding import gather_heads, kv_group_shard


def test_kv_group_shard_partitions_heads():
    shards = [kv_group_shard(32, 8, 4, r) for r in range(4)]
    assert [(s.kv_lo, s.kv_hi, s.q_lo, s.q_hi) for s in shards] == [
        (0, 2, 0, 8), (2, 4, 8, 16), (4, 6, 16, 24), (6, 8, 24, 32)]
    with pytest.raises(ValueError, match="cannot be split evenly"):
        kv_group_shard(32, 8, 3, 0)


def _worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle

    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 8, 24, 16, generator=g, dtype=torch.float64)
    k = torch.randn(2, 4, 24, 16, generator=g, dtype=torch.float64)
    v = torch.randn(2, 4, 24, 16, generator=g, dtype=torch.float64)
    do = torch.randn(2, 8, 24, 16, generator=g, dtype=torch.float64)
    sh = kv_group_shard(8, 4, world, rank)
    outs = []
    for name in ("softmax1", "sparsemax", "entmax15"):
        o, dq, dk, dv = oracle.attention_backward(
            q[:, sh.q_lo:sh.q_hi].numpy(), k[:, sh.kv_lo:sh.kv_hi].numpy(), v[:, sh.kv_lo:sh.kv_hi].numpy(),
            do[:, sh.q_lo:sh.q_hi].numpy(), name, causal=True)
        outs.append([gather_heads(torch.from_numpy(x), 1) for x in (o, dq, dk, dv)])
    if rank == 0:
        full = []
        for name in ("softmax1", "sparsemax", "entmax15"):
            full.append(oracle.attention_backward(q.numpy(), k.numpy(), v.numpy(), do.numpy(), name, causal=True))
        ok = all(np.array_equal(a.numpy(), b) for got, ref in zip(outs, full) for a, b in zip(got, ref))
        with open(result_path, "w") as f:
            f.write("ok" if ok else "mismatch")
    dist.destroy_process_group()


def test_two_rank_gloo_gather_matches_single_process(tmp_path):
    path = str(tmp_path / "result")
    port = 29500 + os.getpid() % 1000
    mp.spawn(_worker, args=(2, port, path), nprocs=2, join=True)
    assert open(path).read() == "ok"
