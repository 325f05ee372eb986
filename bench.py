#!/usr/bin/env python
"""bench.py -- KV append + paged GQA decode attention on B200.

Default workload (per GPU): 64 sequences with contexts
~U[1024, 32768], 6 full-attention layers (one page pool each), nH=8, KVH=2,
dh=256, 16-token pages scattered by a seeded permutation over a pool of
1.25x the pages.  One step = for every layer, append one K/V row per
sequence and run paged decode attention for every sequence.

  value   appended+attended tokens/s of the whole job (sequences x GPUs per
          step time), inputs resident in HBM, timed with CUDA events, max
          over ranks;
  e2e     the same through the public C-ABI call with pinned HOST q/k/v
          copied in and outputs copied out inside the timed region;
  roofline  the attend kernel: algorithmic bytes / CUDA-event time per
          launch vs the measured HBM copy bandwidth;
  cpu_baseline  the oracle's restatement of hostFlashDecode on a bounded
          sample of the same workload, one host thread.

`--impl reference` times the reference's CPU path (the oracle port: the
reference is Swift over Apple frameworks and cannot be built here) with all
host threads, in complete steps of rank 0's shard (at N=1 the whole job);
when the host lacks memory or the W + K steps would overrun a fixed budget,
a step covers fewer layers and the time is scaled, as the line states.

Multi-GPU (torchrun): weak scaling -- every rank runs its own 64 sequences
with its own pools; no collective on the hot path.  The e2e step adds the
NCCL gather of the outputs into job order and rank 0's copy to the host.
"""
from __future__ import annotations

import argparse
import csv
import dataclasses
import datetime
import io
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from gadeon_b200.workload import (CONFIGS, append_bytes, contexts, decode_bytes, pool_pages,  # noqa: E402
                                  weak_job_contexts, weak_rank_contexts)

METRIC = "KV append+attend tok/s (paged GQA decode, config 2)"
UNIT = "tok/s"
REF_BUDGET_S = 150.0  # --impl reference: host seconds for its W + K steps


# DRAM bytes (read + write) per algorithmic byte of the config-2 attend
# launch, from `ncu --set full` of one launch of the same per-layer workload
# (64 sequences, 1 layer): 2.2913 GB read + 4.6 MB written / 2.2899 GB
# algorithmic.
NCU_C2_TRAFFIC_PER_ALGO_BYTE = (2.291264e9 + 4.597504e6) / 2289898428.0
# The same for the config-3 verify launch (32 of the 128 sequences, one
# launch): 1.0811 GB read + 6.9 MB written / 1.0876 GB algorithmic.
NCU_C3_TRAFFIC_PER_ALGO_BYTE = (1.0811e9 + 6.90688e6) / 1087551873.375
# DRAM bytes per sequence of one config-4 chunk launch, from `ncu --set full`
# of the 2-sequence case (245.2 MB read + 103.4 MB written): every sequence
# streams its own K/V, so a full launch moves about 32 x this.
NCU_C4_DRAM_PER_SEQ = (245.167104e6 + 103.359744e6) / 2
# The same for the fused fp16 GDN rollback launch of config 6 (full-size
# workload, launches 6-8): 2.5335 GB measured / 2.6911 GB algorithmic; the
# shortfall is written state still dirty in L2 when the launch ends.
NCU_C6_TRAFFIC_PER_ALGO_BYTE = (845496320 + 843880448 + 844162560) / (895729664 + 897515520 + 897826816)


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20,
                    help="steps per timed block (config 2's contexts grow by one per step, so long runs "
                         "drift from the configured distribution)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=20251201)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--repeats", type=int, default=10,
                    help="timed blocks of --steps steps each; the line reports the median block")
    ap.add_argument("--c5-parts", type=int, default=8,
                    help="--config 5: partition the job into this many shards (8: the per-GPU shard of the "
                         "8-way partition; = --gpus: the whole job over the GPUs)")
    ap.add_argument("--no-subconfigs", action="store_true",
                    help="config 2 alone: skip the configs 3/4 records (1 GPU) and config 5 (4 and 8 GPUs)")
    # profiling knobs: shrink the workload (ncu captures of one launch);
    # a line measured with them is not the config-2 number
    ap.add_argument("--seqs", type=int, default=None, help="sequences per GPU (default: config 2's 64)")
    ap.add_argument("--layers", type=int, default=None, help="layers (default: config 2's 6)")
    ap.add_argument("--gdn-f32", action="store_true",
                    help="configs 6/7: GDN state and conv tail in fp32 (default fp16, the reference's storage)")
    ap.add_argument("--producer", action="store_true",
                    help="config 2 through gkv_attn_step: raw fp32 q|gate, k, v projections, RMSNorm + RoPE "
                         "+ output gate fused into the decode step (Qwen3.5 attention layer)")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5, 6, 7],
                    help="BASELINE config: 2 decode (default, the headline), 3 MTP verify+rollback, "
                         "4 prefill chunk, 5 long-context sharded decode; 6 = the GDN state rollback "
                         "that runs beside config 3's truncate; 7 = a whole MTP cycle (drafts on the drafter "
                         "pool, verify, truncate, GDN rollback, drafter rewind)")
    return ap.parse_args(argv)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak(sustained: bool):
    """Dense bf16 tensor peak (TFLOP/s): burst for a kernel timed alone,
    sustained for one timed inside a long step."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops_sustained" if sustained else "bf16_tflops"]), "measured"
    except Exception:
        return (1400.0 if sustained else 1590.0), "fallback"


def gpu_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    return int(vis.split(",")[local]) if vis else local


def bind_near_gpu(local: int):
    """Pin this process's host threads to the CPU cores NVML lists as nearest
    to its GPU (matched by PCI bus id), so the page-locked buffers it
    allocates sit in that socket's memory and the kernels' in-place host
    reads stay local.  Changes only this process's CPU affinity; a no-op
    where NVML is missing.  Returns the number of cores kept, or None."""
    try:
        import pynvml
        import torch
        pr = torch.cuda.get_device_properties(local)
        bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        n = os.cpu_count() or 1
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (n + 63) // 64)
        cpus = {w * 64 + b for w, m in enumerate(words) for b in range(64) if (int(m) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 50 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r for r in csv.reader(io.StringIO(self.file.read())) if len(r) >= 9]
        os.unlink(self.file.name)
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_sample(seed: int, n_seqs: int, steps: int, threads: int, cfg, ctx_all):
    """Time the oracle (hostFlashDecode restatement) on a bounded sample:
    n_seqs sequences drawn from the job's contexts, one layer, `steps`
    decode steps of append-one + attend.  Returns (seconds per sequence-
    layer-step normalised to the job's mean context, sample description)."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    pick = rng.choice(len(ctx_all), size=min(n_seqs, len(ctx_all)), replace=False)
    ctx = [int(ctx_all[i]) for i in pick]
    kvh, dh, G, P = cfg.kv_heads, cfg.head_dim, cfg.group, cfg.page_tokens
    pool = O.OraclePool(kvh, dh, P, pool_pages(ctx, P, steps + 4), seed)
    ids = []
    for c in ctx:
        s = pool.seq_create()
        K = rng.standard_normal((kvh, c, dh), dtype=np.float32).astype(np.float16).view(np.uint16)
        V = rng.standard_normal((kvh, c, dh), dtype=np.float32).astype(np.float16).view(np.uint16)
        pool.seed(s, K, V, c)
        ids.append(s)
    scale = dh ** -0.5
    times = []
    for step in range(steps + 1):
        k = rng.standard_normal((len(ids), kvh, dh), dtype=np.float32).astype(np.float16).view(np.uint16)
        q = rng.standard_normal((len(ids), 1, kvh * G, dh), dtype=np.float32).astype(np.float16).view(np.uint16)
        t0 = time.perf_counter()
        pool.append(ids, [1] * len(ids), k, k)
        pool.attend_causal(ids, 1, q, G, scale, n_threads=threads)
        dt = time.perf_counter() - t0
        if step > 0:  # step 0 builds the fp32 mirror (floats32's first call)
            times.append(dt)
    sample_tokens = sum(ctx) + len(ctx) * (steps / 2 + 1)
    per_token_key = statistics.mean(times) / sample_tokens  # seconds per attended key
    desc = (f"{len(ctx)} of the job's sequences (ctx sum {sum(ctx)}), 1 layer, {steps} decode steps "
            f"after a mirror-building step; time scaled by attended keys to the full step")
    return per_token_key, desc, sum(times)


def host_mem_available() -> int:
    """Bytes this process may still allocate on the host: MemAvailable,
    capped by the cgroup's limit when one is set."""
    avail = 8 << 30
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    avail = int(line.split()[1]) * 1024
    except OSError:
        pass
    try:
        with open("/sys/fs/cgroup/memory.max") as f:
            lim = f.read().strip()
        with open("/sys/fs/cgroup/memory.current") as f:
            cur = int(f.read())
        if lim != "max":
            avail = min(avail, int(lim) - cur)
    except (OSError, ValueError):
        pass
    return avail


def config2_dict(S: int, L: int, world: int, ctx, cfg) -> dict:
    """The `config` object of a config-2 line (both arms print the same)."""
    return {
        "workload": (f"config2 decode step: {S} seqs/GPU x {L} layers, append 1 + paged GQA decode attend"
                     + ("" if (S, L) == (cfg.seqs, cfg.layers) else " (REDUCED profiling case)")),
        "seqs_per_gpu": S, "layers": L, "n_heads": cfg.n_heads, "kv_heads": cfg.kv_heads,
        "head_dim": cfg.head_dim, "page_tokens": cfg.page_tokens,
        "ctx": ("U[1024,32768]: %d x %d job sequences token-balanced over the GPUs" % (S, world)
                if world > 1 else "U[1024,32768]"), "ctx_mean": float(np.mean(ctx)),
        "l2": "inputs larger than L2 (%.1f GB of K/V per GPU)"
              % (float(np.sum(ctx)) * L * cfg.kv_heads * cfg.head_dim * 4 / 1e9),
        "parallelism": f"dp{world} (sequences sharded, no hot-path collective)",
    }


def run_reference(args, rank, world):
    """--impl reference: the oracle port of the reference's CPU path
    (PagePool.append, then hostFlashDecode with its fp32 mirror, per
    sequence; PagedAttention.swift:85-94, :46-77, :317-366) on all host
    threads, sequences spread over them.  Each timed step is a complete
    config-2 step of rank 0's shard -- append one row to every sequence and
    attend, layer after layer -- timed with the host clock.  At N=1 the
    shard is the whole job, so the line is measured as is; at N>1 one host
    runs the whole job, so its rate is the shard step's time scaled by the
    job's attended keys over the shard's.  When the host cannot hold every
    layer's pool and mirror, the step runs as many layers as fit and the
    time is scaled by the layer count (stated in the line)."""
    if rank != 0:
        return
    from oracle import oracle as O
    cfg = CONFIGS[2]
    S, L, KVH, dh, P, G, nH = cfg.seqs, cfg.layers, cfg.kv_heads, cfg.head_dim, cfg.page_tokens, cfg.group, cfg.n_heads
    S, L = args.seqs or S, args.layers or L
    W, K = args.warmup, args.steps
    ctx = weak_rank_contexts(2, args.seed, S, world, 0)
    job = weak_job_contexts(2, args.seed, S, world)
    threads = os.cpu_count() or 1
    grow = W + K + 4
    n_pages = pool_pages(ctx, P, grow)
    # pages (fp16 K and V) + the fp32 mirror, whose capacity doubles from 64 rows
    mirror_rows = sum(64 << max(0, math.ceil(math.log2((int(c) + grow) / 64))) for c in ctx)
    per_layer = n_pages * KVH * P * dh * 2 * 2 + mirror_rows * KVH * dh * 4 * 2
    avail = host_mem_available()
    L_mem = max(1, min(L, int(0.7 * avail // per_layer)))
    rng = np.random.default_rng(args.seed + 7)
    span = int(ctx.max()) + 4096
    block = rng.standard_normal((2, KVH, span, dh), dtype=np.float32).astype(np.float16).view(np.uint16)
    t_setup = time.perf_counter()
    pools, ids = [], []
    for layer in range(L_mem):
        pool = O.OraclePool(KVH, dh, P, n_pages, args.seed * 31 + layer)
        lids = []
        for c in ctx:
            c, off = int(c), int(rng.integers(0, 4096))
            s = pool.seq_create()
            assert pool.seed(s, np.ascontiguousarray(block[0, :, off:off + c]),
                             np.ascontiguousarray(block[1, :, off:off + c]), c) == 0
            lids.append(s)
        pools.append(pool)
        ids.append(lids)
    # per-step rows and queries, drawn before the clock starts
    rows = [rng.standard_normal((2, S, KVH, dh), dtype=np.float32).astype(np.float16).view(np.uint16)
            for _ in range(4)]
    qs = [rng.standard_normal((S, 1, nH, dh), dtype=np.float32).astype(np.float16).view(np.uint16)
          for _ in range(4)]
    scale = dh ** -0.5

    def step(i, layers):
        kv, q = rows[i % 4], qs[i % 4]
        for layer in range(layers):
            assert pools[layer].append(ids[layer], [1] * S, kv[0], kv[1]) == 0
            pools[layer].attend_causal(ids[layer], 1, q, G, scale, n_threads=threads)

    step(0, L_mem)  # builds every sequence's fp32 mirror (floats32's first call)
    t0 = time.perf_counter()
    step(1, L_mem)
    per_layer_s = (time.perf_counter() - t0) / L_mem
    setup_s = time.perf_counter() - t_setup
    # as many layers per step as keep the W + K steps within the budget
    L_run = max(1, min(L_mem, int(REF_BUDGET_S // ((W + K) * per_layer_s))))
    for i in range(W):
        step(2 + i, L_run)
    t0 = time.perf_counter()
    for i in range(K):
        step(2 + W + i, L_run)
    step_s = (time.perf_counter() - t0) / K
    key_scale = float(job.sum()) / float(ctx.sum())
    job_step_s = step_s * (L / L_run) * key_scale
    value = len(job) / job_step_s
    measured = (f"rank 0's shard: {S} sequences x {L_run} of {L} layers, complete steps (append 1 row to every "
                f"sequence, then hostFlashDecode of every sequence) on {threads} threads, {K} timed steps after "
                f"{W} warm-up steps; setup {setup_s:.0f} s (pools, the fp32 mirror, one probe step)")
    scaled = []
    if L_run < L:
        scaled.append(f"x{L / L_run:g} for the layers left out (%s)" %
                      ("host memory" if L_run == L_mem else f"the {REF_BUDGET_S:.0f} s budget for {W + K} steps"))
    if world > 1:
        scaled.append(f"x{key_scale:.3f} (the job's attended keys over the shard's): one host runs the whole job")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": step_s * 1e3, "job_ms_per_step": job_step_s * 1e3,
        "timing": "host clock around the K timed steps; ms_per_step is one timed step of the run, "
                  "job_ms_per_step the job's step it stands for",
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (fp16 storage, fp32 mirror)", "data": "synthetic (seeded N(0,1) fp16)",
        "impl": "reference",
        "config": config2_dict(S, L, world, ctx, cfg),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": measured + ("; scaled " + ", ".join(scaled) if scaled else
                                               "; the whole job, no scaling")},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "host_mem_gb": {"available": avail / 1e9, "per_layer": per_layer / 1e9},
    }
    print(json.dumps(line), flush=True)


def mean_decode_bytes(ctx, cfg, first: int, count: int, out_bytes: int = 4) -> float:
    """Mean algorithmic bytes of `count` consecutive decode launches whose
    contexts (after the append) are ctx + first + j, j = 0..count-1."""
    c = np.asarray(ctx, dtype=np.int64)[None, :] + first + np.arange(count, dtype=np.int64)[:, None]
    kv_row = cfg.kv_heads * cfg.head_dim * 2
    per = (c * kv_row * 2 + cfg.n_q * cfg.n_heads * cfg.head_dim * (2 + out_bytes)
           + 4 * ((c + cfg.page_tokens - 1) // cfg.page_tokens))
    return float(per.sum(axis=1).mean())


def subconfigs(args, rank, world, local):
    """The records beside config 2 in the default line: configs 3 and 4 on
    one GPU (their full per-GPU workloads), and config 5's whole job strong-
    scaled over 4 or 8 GPUs (every rank checks its memory first; all ranks
    skip together when one lacks room)."""
    import torch
    import torch.distributed as dist
    out = {}
    R = max(1, args.repeats)

    def guarded(fn):
        # a failing record is reported in the line instead of losing the
        # config-2 measurement before it
        try:
            return fn()
        except Exception as e:  # noqa: BLE001
            torch.cuda.empty_cache()
            return {"error": f"{type(e).__name__}: {e}"[:400]}

    if world == 1:
        out["3"] = guarded(lambda: measure_config3(args, rank, world, local, max(args.warmup, 3),
                                                   max(args.steps, 20), R))
        out["4"] = guarded(lambda: measure_config4(args, rank, world, local, max(args.warmup, 3), 3, 1))
    elif world in (4, 8):
        from gadeon_b200.workload import lpt_partition
        cfg = CONFIGS[5]
        job = contexts(5, args.seed, cfg.seqs)
        mine = job[lpt_partition(job, world)[rank]]
        need = pool_pages(mine, cfg.page_tokens, 128, 1.02) * cfg.kv_heads * cfg.page_tokens * cfg.head_dim * 4
        need = need * cfg.layers + (4 << 30)
        free = torch.cuda.mem_get_info(local)[0]
        room = torch.tensor([free - need], device=torch.device("cuda", local), dtype=torch.float64)
        dist.all_reduce(room, op=dist.ReduceOp.MIN)
        if room.item() < 0:
            out["5"] = {"skipped": "a GPU lacks room for its share of the job (%.1f GB short)"
                                   % (-room.item() / 1e9)}
        else:
            out["5"] = guarded(lambda: measure_config5(args, rank, world, local, max(args.warmup, 3),
                                                       min(args.steps, 20), 3, world))
    return out


def run_ours(args, rank, world, local):
    import torch
    import torch.distributed as dist

    from gadeon_b200 import BlockPool
    from gadeon_b200.shard import gather_outputs
    from gadeon_b200.workload import capped_partition

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    host_cores = bind_near_gpu(local)
    cfg = CONFIGS[2]
    L, S, KVH, dh, P, G, nH = cfg.layers, cfg.seqs, cfg.kv_heads, cfg.head_dim, cfg.page_tokens, cfg.group, cfg.n_heads
    L = args.layers or L
    S = args.seqs or S
    W, K, R = args.warmup, args.steps, max(1, args.repeats)
    ctx = weak_rank_contexts(2, args.seed, S, world, rank)
    # the N-GPU job: S * world sequences; rank r holds shard r of the count-
    # capped token-balanced partition, rows of its outputs in shard order
    job_ctx = weak_job_contexts(2, args.seed, S, world)
    shards = capped_partition(job_ctx, world, S) if world > 1 else [list(range(S))]
    # every timed block is rewound to the contexts after the warm-up
    steps_total = W + K + 4
    max_pps = int(math.ceil((int(ctx.max()) + steps_total) / P)) + 2
    n_pages = pool_pages(ctx, P, steps_total)

    # ---- pools, seeded contexts (device RNG, seeded per rank and layer)
    pools, ids = [], []
    scratch = torch.empty(KVH * int(ctx.max()) * dh * 2, dtype=torch.float16, device=dev)
    gen = torch.Generator(device=dev)
    for layer in range(L):
        pool = BlockPool(KVH, dh, P, n_pages, S + 1, max_pps, seed=(args.seed * 1_000_003 + rank * 4099 + layer),
                         device=local)
        gen.manual_seed(args.seed * 7919 + rank * 131 + layer)
        lids = []
        for c in ctx:
            c = int(c)
            s = pool.seq_create()
            buf = scratch[: 2 * KVH * c * dh]
            torch.randn(buf.shape, generator=gen, device=dev, dtype=torch.float16, out=buf)
            kv = buf.view(2, KVH, c, dh)
            pool.seed(s, kv[0], kv[1], c)
            lids.append(s)
        pools.append(pool)
        ids.append(lids)
    del scratch
    # per-step inputs for warm-up + timed steps (every timed block reuses steps W..W+K-1)
    NS = W + K
    q_all = torch.randn((NS, L, S, 1, nH, dh), generator=gen, device=dev, dtype=torch.float16)
    k_all = torch.randn((NS, L, S, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    v_all = torch.randn((NS, L, S, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    outs = [torch.empty((S, 1, nH, dh), dtype=torch.float32, device=dev) for _ in range(L)]
    torch.cuda.synchronize()

    def step(i, ti):
        # one public call per layer: append the step's K/V row of every
        # sequence and attend (the append rides inside the attend kernel).
        # No event between the launches: each launch's start-up overlaps the
        # previous one's tail, and the per-launch time is the step's / L.
        for layer in range(L):
            pools[layer].append_attend(ids[layer], 1, G, k_all[i, layer], v_all[i, layer], q_all[i, layer],
                                       out=outs[layer])

    def rewind():
        # every timed block starts from the same contexts (those after the
        # warm-up): drop the rows the block appended (host bookkeeping,
        # outside the timed blocks)
        for layer in range(L):
            pools[layer].truncate(ids[layer], base_len)

    base_len = [int(c) + W for c in ctx]

    def job_outputs():
        # every layer's outputs of the step, gathered over the GPUs into job
        # order (one NCCL all-gather, one index_select)
        local_out = torch.stack([o.reshape(S, -1) for o in outs], dim=1).reshape(S, -1)
        return gather_outputs(local_out, shards, rank)

    # ---- the same step end to end through the public call with host buffers
    legs = [step]
    e2e = None
    if not args.no_e2e:
        qh = q_all[W:].cpu().pin_memory()
        kh = k_all[W:].cpu().pin_memory()
        vh = v_all[W:].cpu().pin_memory()
        qp, kp, vp = q_all[W:].cpu(), k_all[W:].cpu(), v_all[W:].cpu()  # plain (pageable) host arrays
        n_job = S * world
        if world == 1:
            oh = torch.empty((K, L, S, 1, nH, dh), dtype=torch.float32).pin_memory()
            op = torch.empty((K, L, S, 1, nH, dh), dtype=torch.float32)
        else:  # rank 0 receives the job's outputs
            oh = torch.empty((K, n_job, L * nH * dh), dtype=torch.float32).pin_memory()
            op = torch.empty((K, n_job, L * nH * dh), dtype=torch.float32)
        qd, kd, vd = torch.empty_like(q_all[0, 0]), torch.empty_like(k_all[0, 0]), torch.empty_like(v_all[0, 0])
        copy_stream = torch.cuda.Stream(device=dev)

        def job_to_host(dst, job, ti):
            # N GPUs, rank 0: the step's gathered outputs to page-locked host
            # memory on a copy stream, so the copy engine moves them while the
            # next step's launches run; a block's last step makes the launch
            # stream wait for it, so each timed block ends with all its copies
            main = torch.cuda.current_stream()
            copy_stream.wait_stream(main)
            with torch.cuda.stream(copy_stream):
                dst.copy_(job, non_blocking=True)
            job.record_stream(copy_stream)
            if ti == K - 1:
                main.wait_stream(copy_stream)

        def zero_copy(i, ti):
            # the public call given page-locked host q/k/v (read in place by
            # the kernel over the host link); one GPU: out written in place to
            # host memory; N GPUs: out on the device, gathered in job order,
            # rank 0 copies the job's outputs to host memory
            for layer in range(L):
                pools[layer].append_attend(ids[layer], 1, G, kh[ti, layer], vh[ti, layer], qh[ti, layer],
                                           out=oh[ti, layer] if world == 1 else outs[layer])
            if world > 1:
                job = job_outputs()
                if rank == 0:
                    job_to_host(oh[ti], job, ti)

        # staged copies: device buffers for two steps (by step parity).  The
        # next step's q/k/v move on one copy stream while this step runs, each
        # layer's output moves back on another while the next layer runs, and
        # the launch stream waits on events once per step (so the launches of
        # a step stay chained back to back).
        h2d_stream, d2h_stream = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        qd_s = [[torch.empty_like(qd) for _ in range(L)] for _ in range(2)]
        kd_s = [[torch.empty_like(kd) for _ in range(L)] for _ in range(2)]
        vd_s = [[torch.empty_like(vd) for _ in range(L)] for _ in range(2)]
        od_s = [[torch.empty_like(outs[0]) for _ in range(L)] for _ in range(2)]
        in_ready, in_free, out_free = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
        for ev_ in in_free + out_free:
            ev_.record()

        def stage_step_in(ti):
            sb = ti % 2
            h2d_stream.wait_event(in_free[sb])  # the step two back has read these buffers
            with torch.cuda.stream(h2d_stream):
                for layer in range(L):
                    qd_s[sb][layer].copy_(qh[ti, layer], non_blocking=True)
                    kd_s[sb][layer].copy_(kh[ti, layer], non_blocking=True)
                    vd_s[sb][layer].copy_(vh[ti, layer], non_blocking=True)
                in_ready[sb].record(h2d_stream)

        def staged(i, ti):
            # the call on device buffers that copy engines fill from and drain
            # to page-locked host memory; N GPUs: the gathered job's outputs
            # go to the host instead of each layer's
            main = torch.cuda.current_stream()
            sb = ti % 2
            if ti == 0:
                stage_step_in(0)  # a block's first step: nothing prefetched it
            if ti + 1 < K:
                stage_step_in(ti + 1)
            main.wait_event(in_ready[sb])
            if world == 1:
                main.wait_event(out_free[sb])  # the outputs of the step two back are out
            for layer in range(L):
                pools[layer].append_attend(ids[layer], 1, G, kd_s[sb][layer], vd_s[sb][layer], qd_s[sb][layer],
                                           out=od_s[sb][layer] if world == 1 else outs[layer])
                if world == 1:
                    d2h_stream.wait_stream(main)
                    with torch.cuda.stream(d2h_stream):
                        oh[ti, layer].copy_(od_s[sb][layer], non_blocking=True)
            in_free[sb].record(main)
            if world > 1:
                job = job_outputs()
                if rank == 0:
                    job_to_host(oh[ti], job, ti)
            else:
                out_free[sb].record(d2h_stream)
                if ti == K - 1:
                    main.wait_stream(d2h_stream)  # the block ends with its last copy

        def pageable(i, ti):
            # plain host arrays through the public call: the library stages
            # them through its page-locked bounce buffer (the call returns with
            # out in place)
            for layer in range(L):
                pools[layer].append_attend(ids[layer], 1, G, kp[ti, layer], vp[ti, layer], qp[ti, layer],
                                           out=op[ti, layer] if world == 1 else outs[layer])
            if world > 1:
                job = job_outputs()
                if rank == 0:
                    op[ti].copy_(job)

        legs += [zero_copy, staged, pageable]

    times, clk = interleaved_blocks(torch, dist, world, W, K, legs, local, R, rewind)
    # one GPU: every block ran the same K steps from the same contexts, so
    # the host buffers the last e2e blocks wrote must equal, bit for bit, the
    # outputs of the same steps run on device buffers
    e2e_check = None
    if not args.no_e2e and world == 1:
        ref = torch.empty((K, L, S, 1, nH, dh), dtype=torch.float32, device=dev)
        for ti in range(K):
            step(W + ti, ti)
            for layer in range(L):
                ref[ti, layer].copy_(outs[layer])
        rewind()
        ref_h = ref.cpu()
        e2e_check = {"what": "outputs of the last staged-copy and pageable blocks vs the same steps on device "
                             "buffers, bit for bit",
                     "staged_equal": bool(torch.equal(oh.view(torch.int32), ref_h.view(torch.int32))),
                     "pageable_equal": bool(torch.equal(op.view(torch.int32), ref_h.view(torch.int32)))}
        del ref, ref_h
    blocks = times[0]
    ms = statistics.median(blocks)
    attend_avg_ms = ms / L  # back-to-back launches: gaps between them included
    # algorithmic bytes of each timed attend launch (contexts after its append;
    # every block runs the same K steps from the same contexts)
    bytes_per_launch = mean_decode_bytes(ctx, cfg, W + 1, K) + append_bytes(S, cfg)
    hbm_peak, peak_kind = peaks()
    achieved = bytes_per_launch / (attend_avg_ms * 1e-3) / 1e9
    job_bytes = bytes_per_launch * L
    if world > 1:
        t = torch.tensor([job_bytes], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        job_bytes = float(t.item())
    if not args.no_e2e:
        e2e_ms, e2e_copy_ms, e2e_page_ms = (statistics.median(b) for b in times[1:])
        h2d = L * (qd.numel() + kd.numel() + vd.numel()) * 2 * world
        d2h = (L * outs[0].numel() * 4) * world
        e2e = [e2e_ms, h2d, d2h, e2e_copy_ms, e2e_page_ms, times[1], times[2], times[3]]

    # ---- the output gather on its own (N GPUs), after the timed region
    gather_ms = None
    if world > 1:
        for _ in range(3):
            job_outputs()
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(K):
            job_outputs()
        g1.record()
        torch.cuda.synchronize()
        gather_ms = g0.elapsed_time(g1) / K

    # ---- max over ranks
    vals = torch.tensor([ms, e2e[0] if e2e else 0.0, gather_ms or 0.0, attend_avg_ms, e2e[3] if e2e else 0.0,
                         e2e[4] if e2e else 0.0], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms_max, gather_max, attend_max, e2e_copy_max, e2e_page_max = vals.tolist()
    for p in pools:
        st = p.device_status()
        assert st == 0, f"device status {st}"
    del pools, q_all, k_all, v_all, outs
    torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        per_key, desc, cpu_s = cpu_sample(args.seed + 7, 32, 15, 1, cfg, ctx)  # ~10 s of one core
        job_keys = float(ctx.sum()) * L
        cpu_step = per_key * job_keys
        cpu = {"value": S / cpu_step, "unit": UNIT, "cores": 1, "kind": "port",
               "sample": desc + f" ({cpu_s:.1f} s of CPU time)"}

    sub = None
    if not args.no_subconfigs and (args.seqs, args.layers) == (None, None):
        sub = subconfigs(args, rank, world, local)

    if rank != 0:
        return
    tokens = S * world
    line = {
        "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "repeats": R, "ms_per_step": ms, "block_ms_per_step": blocks,
        "timing": (f"{R} rounds; each times one block of exactly {K} steps of the device-resident step and then "
                   f"of each e2e variant, between barrier + synchronize brackets with CUDA events (max over ranks), "
                   f"and after every block drops the block's appended rows (gkv_truncate, outside the timed "
                   f"blocks), so every block starts from the contexts after the warm-up; ms_per_step is the "
                   f"median block's"),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 accumulate, fp16 K/V/Q storage", "data": "synthetic (seeded N(0,1) fp16)",
        "config": config2_dict(S, L, world, ctx, cfg),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_kind": peak_kind,
                     "traffic": NCU_C2_TRAFFIC_PER_ALGO_BYTE * bytes_per_launch,
                     "traffic_source": "ncu dram__bytes_read+write of one launch of the same per-layer workload "
                                       "(bench.py --seqs 64 --layers 1), scaled by algorithmic bytes",
                     "kernel": "attend_kernel<256,TMA,fused append>", "bytes_per_launch": bytes_per_launch,
                     "launch_ms": attend_avg_ms, "launch_ms_max_rank": attend_max,
                     "launch_timing": "CUDA-event step time / layers (launches back to back, gaps included)"},
        "job_gb_per_step": job_bytes / 1e9, "job_gbs": job_bytes / (ms * 1e-3) / 1e9,
        "job_gbs_per_gpu": job_bytes / (ms * 1e-3) / 1e9 / world,
        "cpu_baseline": cpu,
        "e2e": ({"value": tokens / (min(e2e_ms_max, e2e_copy_max) * 1e-3), "unit": UNIT,
                 "h2d_bytes_per_step": e2e[1], "d2h_bytes_per_step": e2e[2],
                 "ms_per_step": min(e2e_ms_max, e2e_copy_max),
                 "transfer": ("the faster of two ways through gkv_append_attend with page-locked host buffers: "
                              + (("the kernel reading q/k/v in place" + (" and writing out in place to host memory"
                                                                         if world == 1 else ""))
                                 if e2e_ms_max <= e2e_copy_max else
                                 ("cudaMemcpyAsync of q/k/v to the device" + (" and of the outputs back" if world == 1
                                                                              else "")
                                  + ", on copy streams overlapping the launches"))
                              + ("" if world == 1 else
                                 "; every step's outputs gathered over NCCL into job order (shard.gather_outputs) "
                                 "and copied by rank 0 to page-locked host memory on a copy stream that overlaps "
                                 "the next step's launches; each timed block ends after its last copy")),
                 "block_ms_per_step": e2e[5] if e2e_ms_max <= e2e_copy_max else e2e[6],
                 "in_place_value": tokens / (e2e_ms_max * 1e-3),
                 "staged_copy_value": tokens / (e2e_copy_max * 1e-3),
                 "staged_copy_note": "same step with cudaMemcpyAsync of q/k/v to device buffers (the next step's "
                                     "during this one) and of each layer's output back (during the next layer), "
                                     "on two copy streams; the launch stream waits on them once per step",
                 "pageable_value": tokens / (e2e_page_max * 1e-3),
                 "check": e2e_check,
                 "pageable_note": "same step given plain (pageable) host arrays, which the library copies "
                                  "through a pool-owned page-locked bounce buffer read and written in place"}
                if e2e else None),
        "gpu_launches": K * L * R,
        "gpu_launches_note": "attend launches in the timed blocks of the device-resident step; each e2e "
                             "variant launches as many in its own blocks",
        "clocks": clk,
        "host_cores_near_gpu": host_cores,
    }
    if gather_ms is not None:
        line["gather_ms_per_step"] = gather_max
        line["gather_note"] = ("all layers' outputs of a step gathered into job order (NCCL all-gather + "
                               "reorder), timed on its own after the timed region; inside every e2e step")
    if sub:
        line["configs"] = sub
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- configs 3-5

def make_pools(torch, cfg, ctx, L, rank, seed, growth, local, factor=1.25, distinct=True):
    """One BlockPool per layer (its own seeded page permutation); sequence i
    seeded with ctx[i] rows of N(0,1) fp16 from torch's seeded device RNG.
    distinct=False fills every sequence by appends of one 4,096-row block
    drawn per layer (it stays in L2, so filling costs only the page writes;
    values do not change the memory traffic of the timed steps)."""
    from gadeon_b200 import BlockPool
    KVH, dh, P = cfg.kv_heads, cfg.head_dim, cfg.page_tokens
    dev = torch.device("cuda", local)
    cmax = int(max(ctx))
    max_pps = int(math.ceil((cmax + growth) / P)) + 2
    n_pages = pool_pages(ctx, P, growth, factor)
    block = 4096
    scratch = torch.empty(2 * KVH * (cmax if distinct else block) * dh, dtype=torch.float16, device=dev)
    gen = torch.Generator(device=dev)
    pools, ids = [], []
    for layer in range(L):
        pool = BlockPool(KVH, dh, P, n_pages, len(ctx) + 1, max_pps,
                         seed=(seed * 1_000_003 + rank * 4099 + layer), device=local)
        gen.manual_seed(seed * 7919 + rank * 131 + layer)
        if not distinct:
            torch.randn(scratch.shape, generator=gen, device=dev, dtype=torch.float16, out=scratch)
            rows = scratch.view(2, block, KVH, dh)  # token-major K and V rows
        lids = []
        for c in ctx:
            c = int(c)
            sid = pool.seq_create()
            if distinct:
                buf = scratch[: 2 * KVH * c * dh]
                torch.randn(buf.shape, generator=gen, device=dev, dtype=torch.float16, out=buf)
                kv = buf.view(2, KVH, c, dh)
                pool.seed(sid, kv[0], kv[1], c)
            else:
                for t0 in range(0, c, block):
                    n = min(block, c - t0)
                    pool.append([sid], [n], rows[0, :n], rows[1, :n])
            lids.append(sid)
        pools.append(pool)
        ids.append(lids)
    del scratch
    torch.cuda.synchronize()
    return pools, ids, gen


def timed_loop(torch, dist, world, W, K, step, local, repeats=1):
    """W untimed steps, then `repeats` blocks of exactly K steps, each block
    between barrier + synchronize brackets and timed with CUDA events on the
    launching stream; clocks sampled meanwhile.  step(i, ti) runs step i
    (ti = its index in the timed block, None while warming up); every block
    runs steps W..W+K-1.  Returns (the median block's ms per step, each
    block max over ranks; the blocks' ms per step; clocks)."""
    for i in range(W):
        step(i, None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(gpu_index(local))
    clocks.start()
    time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    blocks = []
    for _ in range(repeats):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start.record()
        for i in range(K):
            step(W + i, i)
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        blocks.append(start.elapsed_time(end) / K)
    clk = clocks.stop()
    t = torch.tensor(blocks, device=torch.device("cuda", local), dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    blocks = t.tolist()
    return statistics.median(blocks), blocks, clk


def interleaved_blocks(torch, dist, world, W, K, legs, local, repeats, rewind):
    """Times several variants of one step under the same conditions: W
    untimed steps of legs[0]; one untimed step of every other leg (its first
    call's set-up), each followed by rewind(); then `repeats` rounds, each
    timing one block of exactly K steps of every leg in turn, between
    barrier + synchronize brackets with CUDA events on the launching stream,
    and calling rewind() after every block so that every block starts from
    the same state.  Clocks are sampled over the rounds.  Returns (per leg,
    the blocks' ms per step, each the max over ranks; clocks)."""
    for i in range(W):
        legs[0](i, None)
    torch.cuda.synchronize()
    for leg in legs[1:]:
        leg(W, 0)
        torch.cuda.synchronize()
        rewind()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(gpu_index(local))
    clocks.start()
    time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = [[] for _ in legs]
    for _ in range(repeats):
        for li, leg in enumerate(legs):
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            start.record()
            for i in range(K):
                leg(W + i, i)
            end.record()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            times[li].append(start.elapsed_time(end) / K)
            rewind()
    clk = clocks.stop()
    t = torch.tensor(times, device=torch.device("cuda", local), dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist(), clk


def max_over_ranks(torch, dist, world, local, x):
    t = torch.tensor([x], device=torch.device("cuda", local), dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure_config3(args, rank, world, local, W, K, repeats):
    """Config 3: MTP verify + rollback.  128 sequences at context 8192 (per
    GPU), nH=16, KVH=4, dh=256, P=16, one layer.  A step appends 4 draft
    rows per sequence, attends them causally (16 query rows per kv head),
    then truncates to len + accepted, accepted ~ U{0..4} from a seeded RNG.
    Returns this config's record (rank 0's view; timings max over ranks)."""
    import torch
    import torch.distributed as dist
    cfg = CONFIGS[3]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    S, L = args.seqs or cfg.seqs, cfg.layers
    KVH, dh, G, nH, nq = cfg.kv_heads, cfg.head_dim, cfg.group, cfg.n_heads, cfg.n_q
    ctx = contexts(3, args.seed + 1000 * rank, S)
    pools, ids, gen = make_pools(torch, cfg, ctx, L, rank, args.seed, (W + K * repeats) * nq + 8, local)
    rng = np.random.default_rng(args.seed + 17 * rank)
    acc = rng.integers(0, nq + 1, size=(W + K, S))
    q = torch.randn((S, nq, nH, dh), generator=gen, device=dev, dtype=torch.float16)
    kk = torch.randn((S * nq, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    vv = torch.randn((S * nq, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    out = torch.empty((S, nq, nH, dh), dtype=torch.float32, device=dev)
    lens = ctx.copy()
    # per timed block: the contexts each launch attends over, and an event
    # pair around each launch
    lens_at = [[] for _ in range(repeats)]
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K * L)]
          for _ in range(repeats)]
    timed = 0

    def step(i, ti):
        # one public call per layer appends the drafts and verifies them (the
        # append rides in the attend launch); the event bracket times it
        nonlocal lens, timed
        blk = timed // K
        for layer in range(L):
            if ti is not None:
                ev[blk][ti * L + layer][0].record()
            pools[layer].append_attend(ids[layer], nq, G, kk, vv, q, out=out)
            if ti is not None:
                ev[blk][ti * L + layer][1].record()
        if ti is not None:
            lens_at[blk].append(lens + nq)
            timed += 1
        lens = lens + acc[i]
        for layer in range(L):
            pools[layer].truncate(ids[layer], lens)

    ms, blocks, clk = timed_loop(torch, dist, world, W, K, step, local, repeats)
    # each block's mean launch time (max over ranks) and algorithmic bytes;
    # the roofline is the median block's
    blk_ms = torch.tensor([statistics.mean(a.elapsed_time(b) for a, b in e) for e in ev],
                          device=torch.device("cuda", local), dtype=torch.float64)
    if world > 1:
        dist.all_reduce(blk_ms, op=dist.ReduceOp.MAX)
    blk_bytes = [statistics.mean(decode_bytes(la, cfg) for la in b) + append_bytes(S * nq, cfg) for b in lens_at]
    blk_gbs = [by / (t * 1e-3) / 1e9 for by, t in zip(blk_bytes, blk_ms.tolist())]
    mid = sorted(range(repeats), key=lambda r: blk_gbs[r])[repeats // 2]
    launch_ms, bpl = blk_ms.tolist()[mid], blk_bytes[mid]
    hbm, kind = peaks()
    for p in pools:
        assert p.device_status() == 0
    del pools
    torch.cuda.empty_cache()
    achieved = bpl / (launch_ms * 1e-3) / 1e9
    return {
        "metric": "MTP verify+rollback: draft tokens verified/s (config 3)",
        "value": S * nq * world / (ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "repeats": repeats, "ms_per_step": ms, "block_ms_per_step": blocks, "higher_is_better": True,
        "scaling": "weak", "dtype": "f32 accumulate, fp16 K/V/Q storage", "data": "synthetic (seeded N(0,1) fp16)",
        "config": {"workload": f"config3: {S} seqs/GPU at ctx 8192, {L} layer, 4 drafts appended + causal "
                               "attend in one gkv_append_attend (16 rows/kv head, split-K mma.sync kernel, "
                               "append fused), truncate to len+U{0..4}",
                   "kv_heads": KVH, "n_heads": nH, "head_dim": dh, "page_tokens": cfg.page_tokens,
                   "l2": "inputs larger than L2 (%.1f GB of K/V per GPU)" % (float(ctx.sum()) * KVH * dh * 4 / 1e9)},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "traffic": NCU_C3_TRAFFIC_PER_ALGO_BYTE * bpl,
                     "traffic_source": "ncu dram__bytes_read+write of one verify launch over 32 of the sequences, "
                                       "scaled by algorithmic bytes",
                     "kernel": "attend_kernel<256,TMA,fused append> (n_q=4)",
                     "bytes_per_launch": bpl, "launch_ms": launch_ms,
                     "block_gbs": blk_gbs,
                     "launch_timing": "CUDA events around each launch; the block with the median GB/s"},
        "accepted_draft_tok_per_s": float(acc[W:].sum() * world / (K * ms * 1e-3)),
        "gpu_launches": K * L * repeats, "clocks": clk}


def run_config3(args, rank, world, local):
    rec = measure_config3(args, rank, world, local, max(args.warmup, 3), max(args.steps, 64), args.repeats)
    if rank == 0:
        rec.update({"vs_baseline": None, "cpu_baseline": None, "e2e": None})
        print(json.dumps(rec), flush=True)


def chunk_flops(ctx_before, n_q, cfg):
    """QK^T + P.V flops of one chunk launch: row s of a sequence sees
    ctx_before + s + 1 keys, for every query head."""
    f = 0.0
    for c in ctx_before:
        keys = n_q * (int(c) + 1) + n_q * (n_q - 1) / 2
        f += cfg.n_heads * keys * cfg.head_dim * 4
    return f


def measure_config4(args, rank, world, local, W, K, repeats, seqs=None):
    """Config 4: prefill-chunk ingest.  32 sequences (per GPU) with a seeded
    16384-token context each ingest a 4096-token chunk per layer (append +
    causal chunk attention on the tcgen05 kernel), 8 layers, nH=16, KVH=4,
    dh=256, P=16; the chunk is truncated away after each step so every step
    has the same shape.  Returns this config's record."""
    import torch
    import torch.distributed as dist
    cfg = CONFIGS[4]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    S, L = seqs or cfg.seqs, cfg.layers
    KVH, dh, G, nH, nq = cfg.kv_heads, cfg.head_dim, cfg.group, cfg.n_heads, cfg.n_q
    ctx = contexts(4, args.seed + 1000 * rank, S)
    pools, ids, gen = make_pools(torch, cfg, ctx, L, rank, args.seed, nq + 16, local, distinct=False)
    q = torch.randn((S, nq, nH, dh), generator=gen, device=dev, dtype=torch.float16)
    kk = torch.randn((S * nq, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    vv = torch.randn((S * nq, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    out = torch.empty((S, nq, nH, dh), dtype=torch.float32, device=dev)
    rows = [nq] * S
    # events around each chunk launch of the last timed block, per variant
    ev = {pf: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K * L)]
          for pf in (False, True)}

    def make_step(pf):
        # pf: GKV_ATTEND_P_F16 (softmax weights rounded once to fp16)
        def step(i, ti):
            for layer in range(L):
                pools[layer].append(ids[layer], rows, kk, vv)
                if ti is not None:
                    ev[pf][ti * L + layer][0].record()
                pools[layer].attend(ids[layer], nq, G, q, out=out, p_f16=pf)
                if ti is not None:
                    ev[pf][ti * L + layer][1].record()
                pools[layer].truncate(ids[layer], ctx)
        return step

    # the default and the P_F16 variant in alternating blocks (the same clock
    # conditions); every step truncates its chunk away, so nothing to rewind
    times, clk = interleaved_blocks(torch, dist, world, W, K, [make_step(False), make_step(True)], local,
                                    repeats, lambda: None)
    blocks, blocks16 = times
    ms, ms16 = statistics.median(blocks), statistics.median(blocks16)
    launch_ms, launch16 = (max_over_ranks(torch, dist, world, local,
                                          statistics.mean(a.elapsed_time(b) for a, b in ev[pf]))
                           for pf in (False, True))
    fl = chunk_flops(ctx, nq, cfg)
    peak, kind = tensor_peak(sustained=True)
    for p in pools:
        assert p.device_status() == 0
    del pools
    torch.cuda.empty_cache()
    achieved = fl / (launch_ms * 1e-3) / 1e12
    achieved16 = fl / (launch16 * 1e-3) / 1e12
    return {
        "metric": "prefill chunk ingest tok/s (config 4)", "value": S * nq * world / (ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": K, "warmup": W, "repeats": repeats, "ms_per_step": ms, "block_ms_per_step": blocks,
        "higher_is_better": True, "scaling": "weak",
        "dtype": "fp16 x fp16 -> fp32 (tcgen05 kind::f16; P.V as P_hi.V + P_lo.V)",
        "data": "synthetic (seeded N(0,1) fp16)",
        "config": {"workload": f"config4: {S} seqs/GPU x {L} layers, 16384-token context + 4096-token chunk "
                               "(append + causal chunk attention)", "kv_heads": KVH, "n_heads": nH,
                   "head_dim": dh, "page_tokens": cfg.page_tokens, "l2": "inputs larger than L2"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_kind": kind + " sustained bf16 (fp16 runs at the same rate)",
                     "traffic": NCU_C4_DRAM_PER_SEQ * S,
                     "traffic_source": "ncu dram__bytes_read+write of one launch of the 2-sequence case, scaled by "
                                       "sequences",
                     "kernel": "chunk_kernel<256,pair>", "flops_per_launch": fl,
                     "flops_note": "algorithmic Q.K^T + P.V flops; the tensor cores also run the P_lo.V "
                                   "correction (1.5x these flops)",
                     "issued_tflops": 1.5 * achieved, "launch_ms": launch_ms,
                     "launch_timing": "CUDA events around each chunk launch (the last timed block)"},
        "p_f16": {"what": "the same steps with GKV_ATTEND_P_F16: the softmax weights rounded once to fp16 and "
                          "one P.V per key tile, the arithmetic of the reference's Metal attn_batch_mm; each "
                          "output element within 2^-10 x sum_i w_i |V_i| of the exact result instead of the "
                          "element-wise tolerance of the default; timed in blocks alternating with the default's",
                  "value": S * nq * world / (ms16 * 1e-3), "ms_per_step": ms16, "block_ms_per_step": blocks16,
                  "launch_ms": launch16, "achieved_tflops": achieved16, "frac": achieved16 / peak},
        "gpu_launches": K * L * 2 * repeats, "clocks": clk}


def run_config4(args, rank, world, local):
    rec = measure_config4(args, rank, world, local, max(args.warmup, 3), min(args.steps, 5), 1, args.seqs)
    if rank == 0:
        rec.update({"vs_baseline": None, "cpu_baseline": None, "e2e": None})
        print(json.dumps(rec), flush=True)


def measure_config5(args, rank, world, local, W, K, repeats, parts):
    """Config 5: long-context sharded decode.  The job is 512 sequences with
    contexts log-uniform in [4096, 131072] (8 layers, nH=16, KVH=4, dh=256,
    P=16, ~0.6 TB of KV).  Sequences are token-balanced over `parts` shards
    (greedy LPT) and rank r runs shard r % parts: parts = world is the whole
    job strong-scaled over the GPUs; parts = 8 at fewer GPUs is the per-GPU
    shard of the 8-way partition (weak scaling).  One step = per layer
    append 1 + decode attend; no collective on the hot path.  After the
    timed region the outputs are gathered in job order (NCCL all-gather)
    and that gather is timed on its own.  Returns this config's record."""
    import torch
    import torch.distributed as dist
    from gadeon_b200.shard import gather_outputs
    from gadeon_b200.workload import lpt_partition
    cfg = CONFIGS[5]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = args.layers or cfg.layers
    KVH, dh, G, nH = cfg.kv_heads, cfg.head_dim, cfg.group, cfg.n_heads
    job = contexts(5, args.seed, cfg.seqs)
    shards = lpt_partition(job, parts)
    if args.seqs:  # a reduced case: the first --seqs sequences of every shard
        shards = [sh[: args.seqs] for sh in shards]
    mine = shards[rank % parts]
    ctx = job[mine]
    loads = [int(job[s_].sum()) for s_ in shards]  # tokens per shard
    if args.seqs:  # the reduced job's sequences renumbered 0..n-1 for the gather
        kept = {j: n for n, j in enumerate(sorted(i for sh in shards for i in sh))}
        shards = [[kept[i] for i in sh] for sh in shards]
    pools, ids, gen = make_pools(torch, cfg, ctx, L, rank, args.seed, W + K * repeats + 4, local, factor=1.02,
                                 distinct=False)
    S = len(ctx)
    q = torch.randn((S, 1, nH, dh), generator=gen, device=dev, dtype=torch.float16)
    kk = torch.randn((S, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    vv = torch.randn((S, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    outs = [torch.empty((S, 1, nH, dh), dtype=torch.float32, device=dev) for _ in range(L)]

    def step(i, ti):
        # one public call per layer: the append rides inside the attend kernel
        for layer in range(L):
            pools[layer].append_attend(ids[layer], 1, G, kk, vv, q, out=outs[layer])

    ms, blocks, clk = timed_loop(torch, dist, world, W, K, step, local, repeats)
    launch_ms = ms / L  # back-to-back launches: gaps between them included
    bpl = statistics.mean(decode_bytes(ctx + W + i + 1, cfg) for i in range(K)) + append_bytes(S, cfg)
    hbm, kind = peaks()
    gather_ms = None
    full_job = parts == world  # every rank holds one shard of the job (reduced by --seqs if given)
    if world > 1 and full_job:
        # every layer's outputs of the step, gathered into job order
        local_out = torch.stack([o.reshape(S, -1) for o in outs], dim=1).reshape(S, -1)
        gather_outputs(local_out, shards, rank)
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(10):
            gather_outputs(local_out, shards, rank)
        g1.record()
        torch.cuda.synchronize()
        gather_ms = max_over_ranks(torch, dist, world, local, g0.elapsed_time(g1) / 10)
    tok_sum = max_over_ranks(torch, dist, world, local, float(ctx.sum()))
    job_bytes = bpl * L
    if world > 1:
        t = torch.tensor([job_bytes], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        job_bytes = float(t.item())
    for p in pools:
        assert p.device_status() == 0
    del pools
    torch.cuda.empty_cache()
    achieved = bpl / (launch_ms * 1e-3) / 1e9
    n_job = sum(len(s_) for s_ in shards) if full_job else S * world
    return {
        "metric": "long-context sharded decode tok/s (config 5)", "value": n_job / (ms * 1e-3),
        "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "repeats": repeats, "ms_per_step": ms,
        "block_ms_per_step": blocks, "higher_is_better": True,
        "scaling": (("strong (the whole 512-sequence job)" if not args.seqs else
                     f"strong (REDUCED: {args.seqs} seqs of every shard)") if full_job
                    else "weak (8-way shard per GPU)"),
        "dtype": "f32 accumulate, fp16 K/V/Q storage", "data": "synthetic (seeded N(0,1) fp16)",
        "config": {"workload": f"config5: shard {rank % parts} of a {parts}-way LPT partition of 512 seqs "
                               f"(ctx log-U[4096,131072]); {S} seqs/GPU x {L} layers",
                   "kv_gb_per_gpu": float(ctx.sum()) * L * KVH * dh * 4 / 1e9,
                   "shard_tokens_max_over_mean": max(loads) / (sum(loads) / len(loads)),
                   "max_rank_shard_tokens": tok_sum, "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "traffic": None, "kernel": "attend_kernel<256,TMA,fused append>",
                     "bytes_per_launch": bpl, "launch_ms": launch_ms,
                     "launch_timing": "CUDA-event step time / layers (launches back to back, gaps included)"},
        "job_gb_per_step": job_bytes / 1e9, "job_gbs": job_bytes / (ms * 1e-3) / 1e9,
        "job_gbs_per_gpu": job_bytes / (ms * 1e-3) / 1e9 / world,
        "gather_ms_per_step": gather_ms,
        "gather_note": ("all layers' outputs gathered into job order (shard.gather_outputs: NCCL "
                        "all_gather_into_tensor + reorder), timed after the timed region") if gather_ms else None,
        "gpu_launches": K * L * repeats, "clocks": clk}


def run_config5(args, rank, world, local):
    rec = measure_config5(args, rank, world, local, max(args.warmup, 3), min(args.steps, 50), args.repeats,
                          args.c5_parts)
    if rank == 0:
        rec.update({"vs_baseline": None, "cpu_baseline": None, "e2e": None})
        print(json.dumps(rec), flush=True)


def run_config2_producer(args, rank, world, local):
    """Config 2 geometry through gkv_attn_step: per layer, one call takes
    each sequence's raw fp32 q|gate [nH, 2*dh], k and v [KVH, dh]
    projections, RMSNorm's q and k, applies the partial NEOX rope (64 of 256
    dims, base 1e7, per-position tables), appends, attends and gates the
    output.  Same contexts, pools and timing as the default line."""
    import torch
    import torch.distributed as dist
    import gadeon_b200 as gk
    cfg = CONFIGS[2]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L, S = args.layers or cfg.layers, args.seqs or cfg.seqs
    KVH, dh, G, nH = cfg.kv_heads, cfg.head_dim, cfg.group, cfg.n_heads
    n_rot, base = 64, 1e7
    W, K = max(args.warmup, 3), args.steps
    ctx = weak_rank_contexts(2, args.seed, S, world, rank)
    pools, ids, gen = make_pools(torch, cfg, ctx, L, rank, args.seed, W + K + 2, local)
    NS = W + K
    qg = torch.randn((L, S, nH, 2 * dh), generator=gen, device=dev)
    kr = torch.randn((L, S, KVH, dh), generator=gen, device=dev)
    vr = torch.randn((L, S, KVH, dh), generator=gen, device=dev)
    q_norm = 1 + 0.1 * torch.randn((L, dh), generator=gen, device=dev)
    k_norm = 1 + 0.1 * torch.randn((L, dh), generator=gen, device=dev)
    # rope tables of every step's positions (host helper), resident on the device
    cos_np = np.empty((NS, S, n_rot // 2), dtype=np.float32)
    sin_np = np.empty_like(cos_np)
    for i in range(NS):
        cos_np[i], sin_np[i] = gk.rope_table(n_rot, base, ctx + i)
    cos_t, sin_t = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    outs = [torch.empty((S, nH, dh), dtype=torch.float32, device=dev) for _ in range(L)]
    def step(i, ti):
        for layer in range(L):
            pools[layer].attn_step(ids[layer], G, qg[layer], kr[layer], vr[layer], q_norm[layer], k_norm[layer],
                                   cos_t[i], sin_t[i], eps=1e-6, out=outs[layer])

    ms, _, clk = timed_loop(torch, dist, world, W, K, step, local)
    launch_ms = ms / L  # back-to-back launches: gaps between them included
    # algorithmic bytes: the decode bytes (K/V once, q as fp16, fp32 out,
    # table) with the fp16 q replaced by the fp32 q|gate row, plus the raw
    # k/v read, the fp16 rows written, the rope rows and norm weights
    prod_bytes = S * (nH * (2 * dh * 4 - dh * 2) + KVH * dh * (4 * 2 + 2 * 2) + n_rot * 4) + 2 * dh * 4
    bpl = statistics.mean(decode_bytes(ctx + W + i + 1, cfg) for i in range(K)) + prod_bytes
    hbm, kind = peaks()
    for p_ in pools:
        assert p_.device_status() == 0
    if rank != 0:
        return
    achieved = bpl / (launch_ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "KV append+attend tok/s through gkv_attn_step (config 2, producer fused)",
        "value": S * world / (ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 projections in, fp16 K/V/Q storage, f32 accumulate",
        "data": "synthetic (seeded N(0,1): fp16 contexts, fp32 projections)",
        "config": {"workload": f"config2 + producer: {S} seqs/GPU x {L} layers, ctx ~U[1024,32768], "
                               f"q/k RMSNorm, rope {n_rot}/{dh} base {base:g}, sigmoid output gate",
                   "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "traffic": None, "kernel": "attend_kernel<256,TMA,fused append,producer>",
                     "bytes_per_launch": bpl, "launch_ms": launch_ms,
                     "launch_timing": "CUDA-event step time / layers (launches back to back, gaps included)"},
        "cpu_baseline": None, "e2e": None, "gpu_launches": K * L, "clocks": clk}), flush=True)


def run_config6(args, rank, world, local):
    """GDN rollback beside config 3: per step, every one of 128 sequences
    (per GPU) rolls back the recurrent state and conv tail of its 3 GDN
    layers to an accepted length m ~ U{1..5} (seeded).  One state launch and
    one conv launch cover all (sequence, layer) items; the state and conv
    tail stored in fp16 as the reference stores them (fp32 with --gdn-f32),
    inputs far larger than L2."""
    import torch
    import torch.distributed as dist
    import gadeon_b200 as gk
    from gadeon_b200.workload import GDN, rollback_bytes
    g = GDN
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n = (args.seqs or g.seqs) * (args.layers or g.layers)
    H, D, Cw, CD, T = g.value_heads, g.head_dim, g.chunk, g.conv_dim, g.taps
    W, K = max(args.warmup, 3), max(args.steps, 50)
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + 31 * rank)
    sdt = torch.float32 if args.gdn_f32 else torch.float16
    sb = 4 if args.gdn_f32 else 2
    s0 = (torch.randn((n, H, D, D), generator=gen, device=dev) * 0.1).to(sdt)
    out = torch.empty_like(s0)
    kk = torch.randn((n, H, Cw, D), generator=gen, device=dev) / math.sqrt(D)
    delta = torch.randn((n, H, Cw, D), generator=gen, device=dev) * 0.5
    gcum = torch.cumsum(-torch.rand((n, H, Cw), generator=gen, device=dev) * 0.7, dim=-1)
    proj = torch.randn((n, Cw, CD), generator=gen, device=dev)
    pre = torch.randn((n, CD, T), generator=gen, device=dev).to(sdt)
    conv = torch.empty_like(pre)
    rng = np.random.default_rng(args.seed + 17 * rank)
    ms_acc = rng.integers(1, Cw + 1, size=(W + K, n)).astype(np.int32)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]

    def step(i, ti):
        # the state and conv tail of every item in one launch
        # (gkv_gdn_rollback_f16, or gkv_gdn_rollback with --gdn-f32)
        if ti is not None:
            ev[ti][0].record()
        gk.gdn_rollback(ms_acc[i], s0, delta, kk, gcum, proj, pre, out=out, conv_out=conv)
        if ti is not None:
            ev[ti][1].record()

    ms, _, clk = timed_loop(torch, dist, world, W, K, step, local)
    launch_ms = max_over_ranks(torch, dist, world, local, statistics.mean(a.elapsed_time(b) for a, b in ev))
    step_bytes = statistics.mean(sum(rollback_bytes(ms_acc[W + i], g, sb)) for i in range(K))
    bpl = step_bytes  # one launch per step
    hbm, kind = peaks()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        ns = 8
        a = [x[:ns].cpu().numpy() for x in (s0, delta, kk, gcum)]
        mm = ms_acc[0, :ns]
        orc = O.mtp_rollback if args.gdn_f32 else O.mtp_rollback_f16
        orc(mm, *a)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0:
            orc(mm, *a)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        cpu = {"value": ns / g.layers / dt, "unit": "seq/s", "cores": 1, "kind": "port",
               "sample": f"{ns} (sequence, layer) state rollbacks of the same shapes, oracle restatement of "
                         f"MtpRollback.stateAfter, one thread, {reps} repetitions"}
    if rank != 0:
        return
    achieved = bpl / (launch_ms * 1e-3) / 1e9
    seqs = n // (args.layers or g.layers)
    print(json.dumps({
        "metric": "GDN MTP rollback: sequences rolled back/s (all GDN layers of one attention block)",
        "value": seqs * world / (ms * 1e-3), "unit": "seq/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 compute, " + ("f32 state" if args.gdn_f32 else "fp16 state and conv tail (reference storage)"),
        "data": "synthetic (seeded torch.randn state, keys, deltas; gates = negative cumsums)",
        "config": {"workload": f"config6: {seqs} seqs/GPU x {n // seqs} GDN layers; value heads {H}, "
                               f"DK=DV={D}, C={Cw}, conv {CD}x{T} taps; m ~ U{{1..{Cw}}}",
                   "step_bytes": step_bytes, "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "traffic": None if args.gdn_f32 else NCU_C6_TRAFFIC_PER_ALGO_BYTE * bpl,
                     "kernel": "gdn_rollback_%s_kernel (state + conv tail)" % ("f32" if args.gdn_f32 else "f16"),
                     "bytes_per_launch": bpl, "launch_ms": launch_ms},
        "step_gbs": step_bytes / (ms * 1e-3) / 1e9,
        "cpu_baseline": cpu, "e2e": None, "gpu_launches": K, "clocks": clk}), flush=True)


def run_config7(args, rank, world, local):
    """A whole MTP speculative cycle's cache work (Engine.decodeSpecStep,
    LLM/src/CoreML/Engine.swift:2742-2812) on config 3's geometry: 128
    sequences (per GPU) at context 8192, nH=16, KVH=4, dh=256, P=16; one
    full-attention layer, its 3 GDN layers, and the MTP drafter's own pool
    (same geometry, the committed history).  Per cycle: 3 draft steps on the
    drafter pool (append 1 + decode, each depending on the last), the verify
    of 4 rows on the main pool (append + causal attend), accepted length
    m ~ U{1..4} (seeded), main truncate to p0 + m, GDN state + conv-tail
    rollback, drafter rewind to its base + m rows re-appended."""
    import torch
    import torch.distributed as dist
    import gadeon_b200 as gk
    from gadeon_b200.workload import GDN, rollback_bytes
    cfg, g = CONFIGS[3], GDN
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    S = args.seqs or cfg.seqs
    KVH, dh, G, nH, nq = cfg.kv_heads, cfg.head_dim, cfg.group, cfg.n_heads, cfg.n_q
    n_draft = nq - 1
    cfg1 = dataclasses.replace(cfg, n_q=1)  # a drafter step: one query row per sequence
    W, K = max(args.warmup, 3), min(max(args.steps, 20), 200)
    ctx = contexts(3, args.seed + 1000 * rank, S)
    growth = (W + K) * (nq + n_draft) + 8
    (main,), (mids,), gen = make_pools(torch, cfg, ctx, 1, rank, args.seed, growth, local)
    (drafter,), (dids,), _ = make_pools(torch, cfg, ctx, 1, rank, args.seed + 1, growth, local)
    q1 = torch.randn((S, 1, nH, dh), generator=gen, device=dev, dtype=torch.float16)
    k1 = torch.randn((S, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    q4 = torch.randn((S, nq, nH, dh), generator=gen, device=dev, dtype=torch.float16)
    k4 = torch.randn((S * nq, KVH, dh), generator=gen, device=dev, dtype=torch.float16)
    out1 = torch.empty((S, 1, nH, dh), dtype=torch.float32, device=dev)
    out4 = torch.empty((S, nq, nH, dh), dtype=torch.float32, device=dev)
    n_items = S * g.layers
    H, D, Cw = g.value_heads, g.head_dim, nq
    # GDN state and conv tail in fp16, as the reference stores them (fp32 with --gdn-f32)
    sdt = torch.float32 if args.gdn_f32 else torch.float16
    s0 = (torch.randn((n_items, H, D, D), generator=gen, device=dev) * 0.1).to(sdt)
    s_out = torch.empty_like(s0)
    gk_ = torch.randn((n_items, H, Cw, D), generator=gen, device=dev) / math.sqrt(D)
    gd = torch.randn((n_items, H, Cw, D), generator=gen, device=dev) * 0.5
    gc = torch.cumsum(-torch.rand((n_items, H, Cw), generator=gen, device=dev) * 0.7, dim=-1)
    proj = torch.randn((n_items, Cw, g.conv_dim), generator=gen, device=dev)
    pre = torch.randn((n_items, g.conv_dim, g.taps), generator=gen, device=dev).to(sdt)
    conv = torch.empty_like(pre)
    rng = np.random.default_rng(args.seed + 17 * rank)
    acc = rng.integers(1, nq + 1, size=(W + K, S))  # m = accepted drafts + 1
    lens = ctx.copy()
    dlens = ctx.copy()
    att_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K * nq)]
    att_bytes = []

    def step(i, ti):
        nonlocal lens, dlens
        base = dlens.copy()
        for d in range(n_draft):  # each draft depends on the previous one
            if ti is not None:
                att_ev[ti * nq + d][0].record()
                att_bytes.append(decode_bytes(base + d + 1, cfg1) + append_bytes(S, cfg))
            drafter.append_attend(dids, 1, G, k1, k1, q1, out=out1)
            if ti is not None:
                att_ev[ti * nq + d][1].record()
        if ti is not None:
            att_ev[ti * nq + n_draft][0].record()
            att_bytes.append(decode_bytes(lens + nq, cfg))
        main.append_attend(mids, nq, G, k4, k4, q4, out=out4)
        if ti is not None:
            att_ev[ti * nq + n_draft][1].record()
        m = acc[i]
        lens = lens + m
        main.truncate(mids, lens)
        mm = np.repeat(m, g.layers).astype(np.int32)
        gk.gdn_rollback(mm, s0, gd, gk_, gc, proj, pre, out=s_out, conv_out=conv)  # state + conv tail, one launch
        drafter.rewind_append(dids, base, m, k4[: int(m.sum())], k4[: int(m.sum())])
        dlens = base + m

    ms, _, clk = timed_loop(torch, dist, world, W, K, step, local)
    att_ms = sum(a.elapsed_time(b) for a, b in att_ev)
    committed = float(acc[W:].sum())
    hbm, kind = peaks()
    achieved = max_over_ranks(torch, dist, world, local, sum(att_bytes) / (att_ms * 1e-3) / 1e9)
    for p_ in (main, drafter):
        assert p_.device_status() == 0
    if rank != 0:
        return
    rb = statistics.mean(sum(rollback_bytes(np.repeat(acc[W + i], g.layers), g, 4 if args.gdn_f32 else 2))
                         for i in range(K))
    cycle_bytes = sum(att_bytes) / K + append_bytes(S * nq, cfg) + append_bytes(int(acc[W:].sum() / K), cfg) + rb
    print(json.dumps({
        "metric": "MTP cycle: committed tokens/s (drafts + verify + rollback + drafter rewind, config 3 geometry)",
        "value": committed * world / (K * ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 accumulate, fp16 K/V/Q storage, " + ("f32 GDN state" if args.gdn_f32 else "fp16 GDN state"),
        "data": "synthetic (seeded)",
        "config": {"workload": f"config7: {S} seqs/GPU at ctx 8192, 1 attention layer + its drafter pool + "
                               f"{g.layers} GDN layers; {n_draft} drafts, verify {nq} rows, m ~ U{{1..{nq}}}",
                   "mean_committed_per_seq_cycle": committed / (K * S), "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "traffic": None,
                     "kernel": "attend_kernel<256,TMA> (3 drafter decodes + 1 verify per cycle, fused appends)",
                     "bytes_per_cycle": sum(att_bytes) / K, "attend_ms_per_cycle": att_ms / K},
        "cycle_gbs": cycle_bytes / (ms * 1e-3) / 1e9,
        "cpu_baseline": None, "e2e": None, "gpu_launches": K * (n_draft + 1 + 1 + 1), "clocks": clk}), flush=True)


def _json_only_stdout():
    """Keep the process's stdout for the JSON line alone: Python's sys.stdout
    moves to a duplicate of the original descriptor, and descriptor 1 itself
    is pointed at stderr, so whatever a native library prints there (NCCL's
    version banner at communicator set-up) lands on stderr."""
    sys.stdout.flush()
    fd = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = os.fdopen(fd, "w", buffering=1)


def main():
    args = parse_args()
    _json_only_stdout()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.config != 2:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "reference arm is measured on config 2"}))
            return
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        runner = {2: run_ours, 3: run_config3, 4: run_config4, 5: run_config5, 6: run_config6,
                  7: run_config7}[args.config]
        if args.config == 2 and args.producer:
            runner = run_config2_producer
        runner(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
