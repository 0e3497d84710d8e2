"""Benchmark of the fused normalizer-attention engine on B200.

Workload: Qwen3-8B-shaped causal prefill, bf16,
B=4, S=8192, 32 query heads / 8 KV heads (GQA 4:1), D=128, q/k/v ~ N(0,1)
with softmax scale 1/sqrt(D) (seeded synthetic data).  One step = forward +
backward of sparsemax attention and of entmax15 attention on the same inputs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N>1) the 8 KV-head groups are sharded across ranks (strong
scaling: the total problem is fixed); after each step the outputs and
gradients are gathered with NCCL all-gather.  Rank 0 prints one JSON line.

``--impl reference`` times the reference's own CPU algorithm (its eager torch
path restated under oracle/torch_eager.py -- the reference package itself
cannot be imported where the benchmarks run -- all host threads) on a bounded
sample of the same workload and prints the same metric.

Metric: algorithmic attention TFLOP/s of fwd+bwd (FlashAttention convention:
fwd = 4 B Hq D sum_rows(visible keys), bwd = 2.5 x fwd; threshold-solve
recomputation is not counted).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, S, HQ, HKV, D = 4, 8192, 32, 8, 128
NORMS = ("sparsemax", "entmax15")
METRIC = "attn fwd+bwd TFLOP/s (sparsemax+entmax15, Qwen3-8B causal prefill)"


def causal_flops(b, hq, s, d):
    return 4.0 * b * hq * d * s * (s + 1) / 2


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return m["bf16_tflops"], m["bf16_tflops_sustained"], m["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        self.t0 = self.t1 = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a moment to start: wait for its first sample so
            # that the timed region is covered from its first step
            deadline = time.time() + 5.0
            while not self.lines and time.time() < deadline:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def start(self):
        self.t0 = time.time()

    def stop(self):
        self.t1 = time.time()
        time.sleep(0.15)  # the sample that covers the end of the region

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        lines = self.lines
        if self.t0 is not None and self.t1 is not None:
            window = [x for x in lines if self.t0 <= x[0] <= self.t1 + 0.11]
            lines = window or lines
        for _, line in lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        busy = [x for x in sm if smax and x > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- ours
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from hf_attention_normalizers_b200 import _native as N
    from hf_attention_normalizers_b200 import kernels, ops
    from hf_attention_normalizers_b200.sharding import gather_heads, kv_group_shard

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    shard = kv_group_shard(HQ, HKV, world, rank)
    hkv = shard.kv_hi - shard.kv_lo
    hq = shard.q_hi - shard.q_lo
    scale = D ** -0.5
    gen = torch.Generator(device="cpu").manual_seed(1000 + rank)
    host = {
        "q": torch.randn(B, hq, S, D, generator=gen).to(torch.bfloat16),
        "k": torch.randn(B, hkv, S, D, generator=gen).to(torch.bfloat16),
        "v": torch.randn(B, hkv, S, D, generator=gen).to(torch.bfloat16),
        "do": torch.randn(B, hq, S, D, generator=gen).to(torch.bfloat16),
    }
    t = {k: v.to(dev) for k, v in host.items()}
    flops_rank = causal_flops(B, hq, S, D)

    # Multi-GPU: every output and gradient is written by the kernels straight
    # into this rank's block of a rank-major gather buffer [world, B, H_rank,
    # S, D] (no packing copy) and all-gathered in place on NCCL's stream while
    # the next kernels run.  Two buffer sets (by step parity): a set is
    # rewritten only after the gathers that read it two steps earlier are done.
    corr = torch.empty((hq, B * S), dtype=torch.float32, device=dev)
    stats = {n: torch.empty((2, hq, B * S), dtype=torch.float32, device=dev) for n in NORMS}
    masks = {n: torch.empty((ops.mask_words(N.NORMALIZER_IDS[n], hq, B, S, S),), dtype=torch.int32, device=dev)
             for n in NORMS}
    wmeans = {n: ops.new_wmean(t["q"], N.NORMALIZER_IDS[n]) for n in NORMS}
    supports = {n: ops.new_dense_support(t["q"], t["k"], N.NORMALIZER_IDS[n]) for n in NORMS}
    if world > 1:
        from hf_attention_normalizers_b200.sharding import gather_heads_into

        def gbuf(h):
            return torch.empty((world, B, h, S, D), dtype=torch.bfloat16, device=dev)

        sets = [{n: {"o": gbuf(hq), "dq": gbuf(hq), "dk": gbuf(hkv), "dv": gbuf(hkv)} for n in NORMS}
                for _ in range(2)]
        pending = [[], []]
    state = {"i": 0}

    def step():
        if world == 1:
            for name in NORMS:
                nid = N.NORMALIZER_IDS[name]
                o, st, mk, wm, sup = ops.attn_fwd(t["q"], t["k"], t["v"], nid, scale, True, -1, False)
                ops.attn_bwd(t["do"], t["q"], t["k"], t["v"], o, st, mk, nid, scale, True, -1, wmean=wm,
                             support=sup)
            return
        par = state["i"] % 2
        state["i"] += 1
        for w in pending[par]:
            w.wait()  # the compute stream waits for the gathers of step i - 2
        pending[par] = []
        for name in NORMS:
            nid = N.NORMALIZER_IDS[name]
            bf = sets[par][name]
            o = bf["o"][rank]
            ops.attn_fwd_into(t["q"], t["k"], t["v"], o, stats[name], nid, scale, True, mask=masks[name],
                              wmean=wmeans[name], support=supports[name])
            pending[par].append(gather_heads_into(bf["o"], async_op=True))
            ops.attn_bwd_into(t["do"], t["q"], t["k"], t["v"], o, stats[name], corr, bf["dq"][rank],
                              bf["dk"][rank], bf["dv"][rank], nid, scale, True, mask=masks[name],
                              wmean=wmeans[name], support=supports[name])
            for x in ("dq", "dk", "dv"):
                pending[par].append(gather_heads_into(bf[x], async_op=True))

    def drain():
        if world > 1:
            for par in range(2):
                for w in pending[par]:
                    w.wait()
                pending[par] = []

    def gather(*tensors):
        if world == 1:
            return []
        from hf_attention_normalizers_b200.sharding import gather_stacked

        return [gather_stacked(x, async_op=True)[1] for x in tensors]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    drain()
    barrier()
    sampler = ClockSampler(local_rank)
    with sampler:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        sampler.start()
        e0.record()
        for _ in range(args.steps):
            step()
        drain()  # the last gathers belong to the timed region
        e1.record()
        barrier()
        sampler.stop()
    if args.profile_case:
        return None
    ms = e0.elapsed_time(e1) / args.steps
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    total_flops = 3.5 * flops_rank * world * len(NORMS)
    value = total_flops / (ms * 1e-3) / 1e12

    # Per-phase device times (forward / backward of each normalizer) and the
    # dominant launch (the backward of entmax15) for the roofline.
    phases = {}
    for name in NORMS:
        nid = N.NORMALIZER_IDS[name]
        o, st, mk, wm, sup = ops.attn_fwd(t["q"], t["k"], t["v"], nid, scale, True, -1, False)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        reps = 3
        for _trial in range(2):  # the first trial settles the allocator (timed: the second)
            torch.cuda.synchronize()
            ev[0].record()
            for _ in range(reps):
                ops.attn_fwd(t["q"], t["k"], t["v"], nid, scale, True, -1, False)
            ev[1].record()
            for _ in range(reps):
                ops.attn_bwd(t["do"], t["q"], t["k"], t["v"], o, st, mk, nid, scale, True, -1, wmean=wm,
                             support=sup)
            ev[2].record()
            torch.cuda.synchronize()
        fwd = ev[0].elapsed_time(ev[1]) / reps
        bwd = ev[1].elapsed_time(ev[2]) / reps
        phases[name] = {"fwd_ms": round(fwd, 3), "bwd_ms": round(bwd, 3),
                        "fwd_tflops": round(flops_rank / fwd / 1e9, 1),
                        "fwd_bwd_tflops": round(3.5 * flops_rank / (fwd + bwd) / 1e9, 1),
                        # share of the visible (64-row block, key tile) pairs whose
                        # probabilities are all zero: the backward skips them
                        "skipped_tile_frac": round(ops.tile_mask_skipped_fraction(mk, hq, B, S, S), 4)}

    # End to end through the public API: pinned host inputs copied in every
    # step, autograd forward + backward, loss read back to the host.  The
    # copy of step i + 1 runs on a copy stream into the other of two device
    # buffers while step i computes (double-buffered input prefetch).
    pinned = {k: v.pin_memory() for k, v in host.items()}
    fns = {"sparsemax": kernels.hopper_sparsemax_attention, "entmax15": kernels.hopper_entmax15_attention}
    bufs = [{k: torch.empty(v.shape, dtype=v.dtype, device=dev) for k, v in host.items()} for _ in range(2)]
    copy_s = torch.cuda.Stream(dev)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(i):
        b = i % 2
        with torch.cuda.stream(copy_s):
            copy_s.wait_event(free[b])  # the buffer's previous step has finished with it
            for k in host:
                bufs[b][k].copy_(pinned[k], non_blocking=True)
            ready[b].record(copy_s)

    def e2e_steps(n):
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            b = i % 2
            torch.cuda.current_stream().wait_event(ready[b])
            q = bufs[b]["q"].detach().requires_grad_(True)
            k = bufs[b]["k"].detach().requires_grad_(True)
            v = bufs[b]["v"].detach().requires_grad_(True)
            do = bufs[b]["do"]
            loss = 0.0
            works = []
            for name in NORMS:
                o = fns[name](q, k, v, is_causal=True)
                o.backward(do)
                # as in step(): outputs and gradients all-gathered (rank-major, no repacking)
                works += gather(o.detach(), q.grad, k.grad, v.grad)
                loss = loss + torch.sum(o * do, dtype=torch.float32)
                q.grad = k.grad = v.grad = None
            for w in works:
                w.wait()
            free[b].record()
            float(loss.item())

    e2e_steps(2)
    barrier()
    t0 = time.perf_counter()
    e2e_steps_n = max(2, args.steps)  # the first step's copy is not overlapped
    e2e_steps(e2e_steps_n)
    barrier()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps_n
    e2e_t = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_t.item())
    h2d = sum(x.numel() * x.element_size() for x in host.values())

    burst, sustained, hbm, peak_kind = peaks()
    # Dominant single launch: the entmax15 forward (tc_fwd_kernel).  Its DRAM
    # traffic comes from one ncu capture of `bench.py --shape 1,8192,32,8
    # --profile-case` (Q+K+V+O = 168 MB, larger than L2): dram__bytes_read.sum
    # + dram__bytes_write.sum = 101.5 + 35.7 MB on that case, one quarter of
    # the config's (batch) units, so x4.  Reads are Q+K+V once; part of O is
    # still in L2 when the launch ends.
    dom = phases["entmax15"]
    achieved = flops_rank / dom["fwd_ms"] / 1e9
    traffic = 137.2e6 * 4 if (B, S, HQ, HKV) == (4, 8192, 32, 8) and world == 1 else None
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: q,k,v,dO ~ N(0,1) bf16, seeded; random, no dataset",
        "config": {"workload": "Qwen3-8B causal prefill fwd+bwd (BASELINE configs[1])", "batch": B,
                   "seq_len": S, "heads_q": HQ, "heads_kv": HKV, "head_dim": D, "normalizers": list(NORMS),
                   "parallelism": f"kv-head groups sharded over {world} GPU(s)",
                   "l2": "inputs (~670 MB) exceed L2; no flush"},
        "phases": phases,
        "roofline": {"kernel": "tc_fwd_kernel<128,bf16,entmax15> (entmax15 forward, one launch)",
                     "bound": "tensor", "achieved": round(achieved, 1), "peak": sustained, "unit": "TFLOP/s",
                     "frac": round(achieved / sustained, 3), "peak_kind": f"{peak_kind} bf16 sustained",
                     "traffic": traffic,
                     "traffic_unit": "DRAM bytes per launch (ncu, B=1 case larger than L2, x4 batches)",
                     "algorithmic_bytes": 2 * (B * HQ + B * HKV) * S * D * 2},
        "e2e": {"value": round(total_flops / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "path": "kernels.hopper_{sparsemax,entmax15}_attention + autograd, pinned host inputs copied every step (copy stream, double-buffered prefetch of the next step)"},
        # per step: entmax15 forward, tile dQ, tile dK/dV; sparsemax forward,
        # the five support-list kernels and the two tile kernels (which read
        # the overflow flag and return at once)
        "gpu_launches": args.steps * (3 + 8),
        "clocks": sampler.summary(),
    }
    extra = {}
    if args.decode:
        if world > 1:
            del sets
        extra["paged_decode"] = bench_decode(dev, hbm, world=world, rank=rank)
        extra["varlen"] = bench_varlen(dev, world=world, rank=rank)
        if world == 1:
            extra["prescaled_worst_case"] = bench_prescaled(t, flops_rank)
        del t
        for bufs_ in (bufs,):
            bufs_.clear()
        torch.cuda.empty_cache()
        try:
            extra["model_step"] = bench_model(dev, world=world, rank=rank)
        except Exception as exc:  # the prefill/decode line above stands on its own
            extra["model_step"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    if rank != 0:
        return None
    line.update(extra)
    if args.cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_seconds)
    return line


def _max_over_ranks(ms, dev, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return ms
    x = torch.tensor([ms], device=dev)
    dist.all_reduce(x, op=dist.ReduceOp.MAX)
    return float(x.item())


def bench_decode(dev, hbm_peak, bsz=256, norms=("softmax1", "sparsemax", "entmax15"), world=1, rank=0):
    """paged decode, batch 256, contexts U[1024, 32768]
    (seed 0), 32-token pages in a randomly permuted pool (seed 1), 32 query /
    8 KV heads, D=128, bf16, one query token per sequence.  Reported as
    algorithmic GB/s: every valid page's K and V bytes plus q, o and the block
    table, divided by the device time of one call.

    With N ranks the batch is sharded by greedy LPT on context length; each
    rank holds only its sequences' pages (its own pool and block table) and
    the outputs are all-gathered back into batch order (2 MB) inside the timed
    call.  Whole-job GB/s = all sequences' bytes / the slowest rank's time."""
    import torch

    from hf_attention_normalizers_b200 import _native as N
    from hf_attention_normalizers_b200 import ops
    from hf_attention_normalizers_b200.sharding import batch_gather_order, gather_batch, lpt_partition

    page, hq, hkv, d = 32, 32, 8, 128
    lens_all = torch.randint(1024, 32769, (bsz,), generator=torch.Generator().manual_seed(0))
    parts = lpt_partition(lens_all.tolist(), world)
    mine = parts[rank]
    lens = lens_all[mine]
    npages = [(int(x) + page - 1) // page for x in lens]
    pool = sum(npages)
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(1 + rank)).int()
    table = torch.zeros(len(mine), 1024, dtype=torch.int32)
    off = 0
    for i, n in enumerate(npages):
        table[i, :n] = perm[off:off + n]
        off += n
    gen = torch.Generator(device=dev).manual_seed(2 + rank)
    kc = torch.randn(pool * page, hkv, d, device=dev, generator=gen, dtype=torch.bfloat16)
    vc = torch.randn(pool * page, hkv, d, device=dev, generator=gen, dtype=torch.bfloat16)
    qg = torch.Generator(device=dev).manual_seed(3)
    q_all = torch.randn(bsz, hq, 1, d, device=dev, generator=qg, dtype=torch.bfloat16)
    q = q_all[torch.tensor(mine, device=dev)].contiguous()
    table_d, lens_d = table.to(dev), lens.int().to(dev)
    max_len = int(lens.max())
    pool_all = sum((int(x) + page - 1) // page for x in lens_all)
    kv_bytes = pool_all * page * hkv * d * 2 * 2
    alg = kv_bytes + 2 * q_all.numel() * 2 + bsz * 1024 * 4 + bsz * 4
    order = batch_gather_order(parts) if world > 1 else None
    out = {"config": "BASELINE configs[3]" if bsz == 256 else f"configs[3] shape, batch {bsz}",
           "kv_gb": round(kv_bytes / 1e9, 3)}
    if world > 1:
        out["sharding"] = (f"batch by greedy LPT on context length over {world} ranks; per-rank pool and "
                           "block table; outputs all-gathered (inside the timed call)")
        out["rank0_kv_gb"] = round(pool * page * hkv * d * 4 / 1e9, 3)
    for name in norms:
        nid = N.NORMALIZER_IDS[name]

        def f():
            o, _ = ops.paged_fwd(q, kc, vc, table_d, lens_d, page, max_len, nid, d ** -0.5, True)
            if world > 1:
                gather_batch(o, parts, order=order)

        for _ in range(3):
            f()
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        e0.record()
        for _ in range(reps):
            f()
        e1.record()
        torch.cuda.synchronize()
        ms = _max_over_ranks(e0.elapsed_time(e1) / reps, dev, world)
        gbs = alg / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 3), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm_peak / world, 3)}
        if name != "softmax1":
            # DRAM bytes of a sparse call: K once, the score rows, and V only for
            # support keys -- 0.59 of the algorithmic bytes in an ncu capture of
            # the same shape with 16 sequences (dram__bytes_read + write)
            dram = 0.59 * alg
            out[name]["dram_GB/s"] = round(dram / (ms * 1e-3) / 1e9, 1)
            out[name]["dram_frac"] = round(dram / (ms * 1e-3) / 1e9 / hbm_peak / world, 3)
    out["note"] = ("sparsemax/entmax15 read V only for keys in the support, so their algorithmic GB/s "
                   "can exceed the DRAM bandwidth; dram_GB/s / dram_frac count the bytes that reach DRAM "
                   "(ncu ratio 0.59 of the algorithmic bytes); fractions are per GPU")
    return out


def bench_varlen(dev, norms=("softmax1", "entmax15"), world=1, rank=0):
    """64 packed sequences with lengths U[128, 4096]
    (seed 0), cu_seqlens_k = cu_seqlens_q, 16 query / 8 KV heads, D=128, bf16
    N(0,1) (seeded, generated on the device), causal; forward and backward
    device times per normalizer through the varlen ops, in algorithmic TFLOP/s
    (fwd = 4 Hq D sum L(L+1)/2).  With N ranks the KV-head groups are sharded
    and o, dq, dk, dv are all-gathered (rank-major, inside the timed region);
    the figures are whole-job, over the slowest rank's time."""
    import torch

    from hf_attention_normalizers_b200 import _native as N
    from hf_attention_normalizers_b200 import ops
    from hf_attention_normalizers_b200.sharding import gather_stacked, kv_group_shard

    HQv, HKVv, d = 16, 8, 128
    sh = kv_group_shard(HQv, HKVv, world, rank)
    hq, hkv = sh.q_hi - sh.q_lo, sh.kv_hi - sh.kv_lo
    lens = torch.randint(128, 4097, (64,), generator=torch.Generator().manual_seed(0))
    cu = torch.zeros(65, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0).int()
    tot, mx = int(cu[-1]), int(lens.max())
    gen = torch.Generator(device=dev).manual_seed(10 + rank)
    q = torch.randn(tot, hq, d, device=dev, generator=gen, dtype=torch.bfloat16)
    k = torch.randn(tot, hkv, d, device=dev, generator=gen, dtype=torch.bfloat16)
    v = torch.randn(tot, hkv, d, device=dev, generator=gen, dtype=torch.bfloat16)
    do = torch.randn(tot, hq, d, device=dev, generator=gen, dtype=torch.bfloat16)
    cu_d = cu.to(dev)
    flops = 4.0 * HQv * d * float(sum(int(x) * (int(x) + 1) / 2 for x in lens))
    out = {"config": "BASELINE configs[2]", "tokens": tot, "fwd_flop": flops}
    if world > 1:
        out["sharding"] = f"KV-head groups over {world} ranks; o, dq, dk, dv all-gathered"

    def gathers(*xs):
        if world == 1:
            return []
        return [gather_stacked(x, async_op=True)[1] for x in xs]

    for name in norms:
        nid = N.NORMALIZER_IDS[name]
        fwd = lambda: ops.varlen_fwd(q, k, v, cu_d, cu_d, mx, mx, nid, d ** -0.5, True)
        o, st, mk, wm, sup = fwd()
        bwd = lambda: ops.varlen_bwd(do, q, k, v, o, st, mk, cu_d, cu_d, mx, mx, nid, d ** -0.5, True, wm, sup)
        bwd()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        reps = 5
        ev[0].record()
        for _ in range(reps):
            fwd()
        ev[1].record()
        for _ in range(reps):
            bwd()
        ev[2].record()
        works = []
        for _ in range(reps):  # the sharded step: forward, backward and the gathers
            o2 = fwd()[0]
            works += gathers(o2)
            works += gathers(*bwd())
        for w in works:
            w.wait()
        ev[3].record()
        torch.cuda.synchronize()
        f_ms = _max_over_ranks(ev[0].elapsed_time(ev[1]) / reps, dev, world)
        b_ms = _max_over_ranks(ev[1].elapsed_time(ev[2]) / reps, dev, world)
        s_ms = _max_over_ranks(ev[2].elapsed_time(ev[3]) / reps, dev, world)
        out[name] = {"fwd_ms": round(f_ms, 3), "bwd_ms": round(b_ms, 3),
                     "fwd_tflops": round(flops / f_ms / 1e9, 1),
                     "fwd_bwd_tflops": round(3.5 * flops / (f_ms + b_ms) / 1e9, 1)}
        if world > 1:
            out[name]["step_ms_with_gathers"] = round(s_ms, 3)
            out[name]["step_tflops_with_gathers"] = round(3.5 * flops / s_ms / 1e9, 1)
    return out


def bench_prescaled(t, flops, norms=NORMS):
    """The no-skip worst case of the prefill config: q and k additionally
    scaled by D^-1/4 each, so the scores are ~N(0, 1/128) and the supports are
    wide (hundreds of keys for sparsemax, nearly dense for entmax15)."""
    import torch

    from hf_attention_normalizers_b200 import _native as N
    from hf_attention_normalizers_b200 import ops

    qs, ks = t["q"] * D ** -0.25, t["k"] * D ** -0.25
    out = {}
    for name in norms:
        nid = N.NORMALIZER_IDS[name]
        o, st, mk, wm, sup = ops.attn_fwd(qs, ks, t["v"], nid, D ** -0.5, True, -1, False)
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        ops.attn_fwd(qs, ks, t["v"], nid, D ** -0.5, True, -1, False)
        ev[1].record()
        ops.attn_bwd(t["do"], qs, ks, t["v"], o, st, mk, nid, D ** -0.5, True, -1, wmean=wm, support=sup)
        ev[2].record()
        torch.cuda.synchronize()
        f_ms, b_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
        out[name] = {"fwd_ms": round(f_ms, 3), "bwd_ms": round(b_ms, 3),
                     "fwd_bwd_tflops": round(3.5 * flops / (f_ms + b_ms) / 1e9, 1),
                     "skipped_tile_frac": round(ops.tile_mask_skipped_fraction(mk, qs.shape[1], qs.shape[0],
                                                                               qs.shape[2], ks.shape[2]), 4)}
    return out


def bench_model(dev, steps=3, warmup=2, world=1, rank=0):
    """BASELINE configs[4], one data-parallel replica: Qwen3-1.7B-shaped
    model (28 layers, hidden 2048, 16 query / 8 KV heads, D=128), random init
    (seed 0), bf16, one sequence of 4096 random tokens; a training step =
    forward + LM loss + backward + AdamW step.  Reports tokens/s per
    normalizer routed through set_softmax_attention_backend(..., "sdpa"),
    HF's own SDPA softmax as the reference point, the number of fused
    attention calls per step, and the attention share (the fused kernels
    timed alone at the model's shapes x 28 layers / step time).  With N ranks
    the model is data-parallel (DistributedDataParallel, NCCL all-reduce of the
    gradients overlapped with the backward), one 4096-token sequence per rank;
    tokens/s is whole-job over the slowest rank's step time."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from hf_attention_normalizers_b200 import _native as N
    from hf_attention_normalizers_b200 import backends, ops

    cfg = Qwen3Config(hidden_size=2048, num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                      head_dim=128, intermediate_size=6144, vocab_size=151936, rope_theta=1e6,
                      max_position_embeddings=8192)
    torch.manual_seed(0)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        model = Qwen3ForCausalLM(cfg)
    torch.set_default_dtype(prev)
    model.train()
    seq = 4096
    ids = torch.randint(0, cfg.vocab_size, (1, seq), generator=torch.Generator().manual_seed(rank)).to(dev)
    net = model
    if world > 1:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[dev.index], gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-5, foreach=True)
    calls = {"n": 0, "skipped": []}
    real_fwd = ops.attn_fwd

    def counting_fwd(*a, **k):
        calls["n"] += 1
        out_ = real_fwd(*a, **k)
        if len(calls["skipped"]) < 28:  # the support masks of one step's layers (the model's activations)
            q_, k_ = a[0], a[1]
            calls["skipped"].append((out_[2], q_.shape[1], q_.shape[0], q_.shape[2], k_.shape[2]))
        return out_

    def step():
        loss = net(input_ids=ids, labels=ids).loss
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)

    out = {"config": "BASELINE configs[4]" + (f", data-parallel over {world} GPUs (DDP)" if world > 1
                                                else " (one replica)"),
           "tokens_per_step": seq * world}
    ops.attn_fwd = counting_fwd
    try:
        for norm in ("hf_sdpa_softmax", "softmax1", "sparsemax", "entmax15"):
            if norm == "hf_sdpa_softmax":
                model.config._attn_implementation = "sdpa"
            else:
                backends.set_softmax_attention_backend(model, "sdpa", norm)
            for _ in range(warmup):
                step()
            torch.cuda.synchronize()
            calls["n"] = 0
            calls["skipped"] = []
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                step()
            e1.record()
            torch.cuda.synchronize()
            ms = _max_over_ranks(e0.elapsed_time(e1) / steps, dev, world)
            res = {"ms_per_step": round(ms, 2), "tokens_per_s": round(world * seq / ms * 1e3, 1),
                   "fused_attention_calls_per_step": calls["n"] // steps}
            if norm in ("sparsemax", "entmax15") and calls["skipped"]:
                fr = [ops.tile_mask_skipped_fraction(*x) for x in calls["skipped"]]
                res["skipped_tile_frac_mean_over_layers"] = round(sum(fr) / len(fr), 4)
            if norm != "hf_sdpa_softmax":
                nid = N.NORMALIZER_IDS[norm]
                q = torch.randn(1, 16, seq, 128, device=dev, dtype=torch.bfloat16)
                k = torch.randn(1, 8, seq, 128, device=dev, dtype=torch.bfloat16)
                v = torch.randn(1, 8, seq, 128, device=dev, dtype=torch.bfloat16)
                o, st, mk, wm, sup = real_fwd(q, k, v, nid, 128 ** -0.5, True, -1, False)
                ops.attn_bwd(q, q, k, v, o, st, mk, nid, 128 ** -0.5, True, -1, wmean=wm, support=sup)
                torch.cuda.synchronize()
                a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record()
                for _ in range(28):
                    o, st, mk, wm, sup = real_fwd(q, k, v, nid, 128 ** -0.5, True, -1, False)
                    ops.attn_bwd(q, q, k, v, o, st, mk, nid, 128 ** -0.5, True, -1, wmean=wm, support=sup)
                a1.record()
                torch.cuda.synchronize()
                res["attention_ms"] = round(a0.elapsed_time(a1), 2)
                res["attention_share"] = round(a0.elapsed_time(a1) / ms, 3)
            out[norm] = res
    finally:
        ops.attn_fwd = real_fwd
    return out


# --------------------------------------------------------------------------- CPU
REF_ROWS = 512  # query rows of the CPU sample (reference arm step and cpu_baseline)


def cpu_sample(threads: int, rows: int):
    """One bounded sample of the workload through the reference's eager path
    restated in torch (``oracle/torch_eager.py``: the same sort / cumsum
    thresholds, closed-form backwards and matmuls), on the host cores.

    The last `rows` query rows of one (batch, KV group) slice -- 4 query heads
    against all S keys under the causal mask, forward + backward of both
    normalizers, float32.  Returns (seconds, algorithmic FLOPs of the sample).
    """
    import torch

    from oracle import torch_eager

    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(0)
    g = HQ // HKV
    q = torch.randn(1, g, rows, D, generator=gen)
    k = torch.randn(1, 1, S, D, generator=gen)
    v = torch.randn(1, 1, S, D, generator=gen)
    do = torch.randn(1, g, rows, D, generator=gen)
    t0 = time.perf_counter()
    for name in NORMS:
        torch_eager.attention_backward(q, k, v, do, name, scale=D ** -0.5, causal=True)
    sec = time.perf_counter() - t0
    visible = sum(S - rows + i + 1 for i in range(rows))
    flops = 3.5 * 4.0 * g * D * visible * len(NORMS)
    return sec, flops


def cpu_baseline(budget_s: float = 20.0):
    """The reference arm's sample (REF_ROWS query rows), 1 warm-up and the
    median of up to 5 runs within the time budget, plus config 1 whole."""
    threads = os.cpu_count() or 1
    rows = REF_ROWS
    cpu_sample(threads, rows)
    secs, flops, t_end = [], 0.0, time.perf_counter() + budget_s
    while len(secs) < 5 and (not secs or time.perf_counter() < t_end):
        sec_, flops = cpu_sample(threads, rows)
        secs.append(sec_)
    sec = statistics.median(secs)
    return {"value": round(flops / sec / 1e12, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"last {rows} query rows x 4 heads of one (batch, KV group) slice, all {S} keys, "
                      f"fwd+bwd sparsemax+entmax15, float32, the reference's eager path restated in torch "
                      f"(oracle/torch_eager.py, {threads} threads); median of {len(secs)}, {sec:.2f} s each",
            "config1": cpu_config1(threads)}


def cpu_config1(threads: int):
    """BASELINE configs[0] as a whole problem on the host cores: fp32 q,k,v
    [2, 8, 512, 128] (the reference's seed), causal, fwd + bwd of every
    normalizer through the torch restatement of the reference's eager path
    (1 warm-up, median of 5)."""
    import torch

    from oracle import torch_eager

    torch.set_num_threads(threads)
    torch.manual_seed(0)
    q, k, v, g = (torch.randn(2, 8, 512, 128) for _ in range(4))
    flops = 3.5 * causal_flops(2, 8, 512, 128)
    out = {"workload": "BASELINE configs[0] (B=2 H=8 S=512 D=128 fp32, causal, fwd+bwd)", "cores": threads,
           "path": "oracle/torch_eager.py (the reference's eager torch ops)"}
    for name in ("softmax1", "sparsemax", "entmax15"):
        times = []
        for rep in range(6):
            t0 = time.perf_counter()
            torch_eager.attention_backward(q, k, v, g, name, scale=128 ** -0.5, causal=True)
            if rep:
                times.append(time.perf_counter() - t0)
        sec = statistics.median(times)
        out[name] = {"ms": round(sec * 1e3, 1), "GFLOP/s": round(flops / sec / 1e9, 2)}
    return out


def run_reference(args, rank):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    for _ in range(args.warmup if args.warmup < 2 else 1):
        cpu_sample(threads, 16)
    secs, flops = [], 0.0
    for _ in range(args.steps):
        s_, f_ = cpu_sample(threads, REF_ROWS)
        secs.append(s_)
        flops = f_
    sec = statistics.median(secs)
    value = flops / sec / 1e12
    return {
        "metric": METRIC, "impl": "reference", "value": round(value, 6), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1), seeded",
        "config": {"workload": "Qwen3-8B causal prefill fwd+bwd (BASELINE configs[1])", "batch": B,
                   "seq_len": S, "heads_q": HQ, "heads_kv": HKV, "head_dim": D, "normalizers": list(NORMS)},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"each step: last {REF_ROWS} query rows x 4 heads of one (batch, KV group) "
                                   f"slice, all {S} keys, fwd+bwd sparsemax+entmax15, float32, the reference's "
                                   f"eager path restated in torch (oracle/torch_eager.py, {threads} threads)"},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-decode", dest="decode", action="store_false",
                    help="skip the paged-decode measurement (BASELINE configs[3])")
    ap.add_argument("--decode-only", type=int, default=0, metavar="BATCH",
                    help="only run the paged-decode measurement with this many sequences (profiling)")
    ap.add_argument("--decode-norms", default="softmax1,sparsemax,entmax15")
    ap.add_argument("--shape", default=None,
                    help="B,S,HQ,HKV override for small profiling cases (default: the BASELINE config)")
    ap.add_argument("--model-step", action="store_true",
                    help="only run the Qwen3-1.7B training-step measurement (BASELINE configs[4])")
    ap.add_argument("--nccl-ctas", type=int, default=0,
                    help="cap on the CTAs of NCCL's collectives (0: NCCL's choice)")
    ap.add_argument("--nccl-priority", type=int, default=1,
                    help="1 (default): NCCL's collectives on a high-priority stream; 0: normal priority")
    ap.add_argument("--profile-case", action="store_true",
                    help="run warmup+steps of the step only (no e2e, no phases): for ncu captures")
    args = ap.parse_args()
    if args.shape:
        global B, S, HQ, HKV
        B, S, HQ, HKV = (int(x) for x in args.shape.split(","))

    if args.model_step:
        import torch

        print(json.dumps(bench_model(torch.device("cuda", 0))), flush=True)
        return
    if args.decode_only:
        import torch

        print(json.dumps(bench_decode(torch.device("cuda", 0), peaks()[2], args.decode_only,
                                      tuple(args.decode_norms.split(",")))), flush=True)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank)
    else:
        if world > 1:
            import torch
            import torch.distributed as dist

            # NCCL's communicator lines (rank count, transports) go to the log
            # ahead of the JSON line, which is printed last
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
            torch.cuda.set_device(local_rank)
            # The all-gathers run beside the attention kernels, which fill
            # every SM with one CTA: each CTA NCCL holds is an SM the kernels
            # lose while the gathers run.  --nccl-ctas caps that count; at 8
            # GPUs a cap of 8 made the gathers the bottleneck (7.1 ms per step
            # against 4.2 with NCCL's own choice), so the default is no cap.
            # A high-priority NCCL stream gets the gathers' CTAs onto SMs as
            # soon as attention CTAs retire, so they finish and hand the SMs
            # back sooner (8 GPUs: 3.7 ms per step against 4.2).
            opts = dist.ProcessGroupNCCL.Options()
            if args.nccl_ctas > 0:
                opts.config.max_ctas = args.nccl_ctas
                opts.config.nvls_ctas = args.nccl_ctas
            opts.is_high_priority_stream = args.nccl_priority
            dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank), pg_options=opts)
        args.cpu_baseline = args.cpu_baseline and rank == 0 and world == 1 and not args.shape
        args.decode = args.decode and not args.shape
        line = run_ours(args, rank, world, local_rank)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1 and args.impl != "reference":
        # Every rank is past the last collective.  The process group is not
        # destroyed: NCCL would print its teardown lines after the JSON line
        # (the exit frees the communicator), and the JSON line stays last on
        # stdout.
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


if __name__ == "__main__":
    main()
