"""Synthetic workloads of the five BASELINE configurations and the
token-balanced sharding of sequences across GPUs.

Contexts and page permutations are drawn from documented seeds; K/V/Q values
are N(0,1) cast to fp16.  Each GPU owns a private pool per layer, seeded
per (GPU, layer), and no data crosses GPUs on the hot path.
"""
from __future__ import annotations

import dataclasses
import math
from typing import List, Sequence

import numpy as np


@dataclasses.dataclass(frozen=True)
class Config:
    name: str
    seqs: int          # sequences in the whole job (per GPU for weak-scaled configs)
    layers: int
    n_heads: int
    kv_heads: int
    head_dim: int
    page_tokens: int
    n_q: int           # query rows per sequence per step (1 = decode, 4 = MTP verify)
    description: str

    @property
    def group(self) -> int:
        return self.n_heads // self.kv_heads


CONFIGS = {
    1: Config("config1", 1, 1, 8, 2, 256, 16, 1,
              "single layer, B=1, 512-token prefill append then decode (ctx 513..640)"),
    2: Config("config2", 64, 6, 8, 2, 256, 16, 1,
              "batched decode, ctx ~U[1024,32768], 6 layers, nH=8, KVH=2, dh=256, P=16"),
    3: Config("config3", 128, 1, 16, 4, 256, 16, 4,
              "MTP verify: 4 drafts appended + causal attend, truncate to len+U{0..4}, ctx 8192"),
    4: Config("config4", 32, 8, 16, 4, 256, 16, 4096,
              "prefill chunk: 4096 new tokens over 16384 prior, 8 layers"),
    5: Config("config5", 512, 8, 16, 4, 256, 16, 1,
              "long-context sharded decode, ctx log-U[4096,131072], 8 layers, 512 seqs / job"),
}


@dataclasses.dataclass(frozen=True)
class GdnConfig:
    """GDN rollback beside config 3's truncate: every sequence of the MTP
    verify batch rolls back the recurrent state and conv tail of the GDN
    layers that share its full-attention layer (3 GDN : 1 attention in the
    hybrid).  Head geometry of the Qwen3.5 GDN layers: 16 key heads and 32
    value heads of dim 128, conv kernel 4 (3 carried taps) over q|k|v
    channels; verify width C = 1 + 4 drafts."""
    seqs: int = 128
    layers: int = 3
    value_heads: int = 32
    key_heads: int = 16
    head_dim: int = 128
    chunk: int = 5
    taps: int = 3

    @property
    def conv_dim(self) -> int:
        return (2 * self.key_heads + self.value_heads) * self.head_dim


GDN = GdnConfig()


def rollback_bytes(m: Sequence[int], g: GdnConfig, state_bytes: int = 4) -> tuple:
    """Algorithmic HBM bytes of one rollback call pair over items with
    accepted lengths m: (state kernel, conv kernel).  The state (elements of
    state_bytes: 4 fp32, 2 fp16) is read and written once; only the m
    accepted rows of k and delta (fp32) and the gate row are read; the conv
    tail (state_bytes per element) is written once and each tap read once --
    from the fp32 projection rows or the carried tail."""
    H, D = g.value_heads, g.head_dim
    state = sum(H * (2 * D * D * state_bytes + (int(x) * 2 * D + g.chunk) * 4) for x in m)
    conv = 0
    for x in m:
        from_proj = min(int(x), g.taps)  # taps at positions m - taps + t >= 0
        conv += g.conv_dim * (g.taps * state_bytes + from_proj * 4 + (g.taps - from_proj) * state_bytes)
    return state, conv


def contexts(cfg_id: int, seed: int, n: int) -> np.ndarray:
    """Context lengths of config cfg_id drawn from `seed`."""
    rng = np.random.default_rng(seed)
    if cfg_id == 1:
        return np.full(n, 512, dtype=np.int64)
    if cfg_id == 2:
        return rng.integers(1024, 32768, size=n, endpoint=True).astype(np.int64)
    if cfg_id == 3:
        return np.full(n, 8192, dtype=np.int64)
    if cfg_id == 4:
        return np.full(n, 16384, dtype=np.int64)
    if cfg_id == 5:
        return np.exp(rng.uniform(math.log(4096), math.log(131072), size=n)).astype(np.int64)
    raise ValueError(cfg_id)


def lpt_partition(tokens: Sequence[int], parts: int) -> List[List[int]]:
    """Greedy longest-processing-time partition: sequences by context
    descending, each to the currently least-loaded part (ties -> lowest
    index).  Returns the sequence indices of every part, ascending."""
    order = sorted(range(len(tokens)), key=lambda i: (-int(tokens[i]), i))
    load = [0] * parts
    out: List[List[int]] = [[] for _ in range(parts)]
    for i in order:
        p = min(range(parts), key=lambda r: (load[r], r))
        out[p].append(i)
        load[p] += int(tokens[i])
    return [sorted(o) for o in out]


def capped_partition(tokens: Sequence[int], parts: int, per_part: int) -> List[List[int]]:
    """Token-balanced partition with exactly per_part sequences per part
    (len(tokens) == parts * per_part): sequences by context descending, each
    to the least-loaded part that still has room (ties -> lowest index).
    Returns the sequence indices of every part, ascending."""
    if len(tokens) != parts * per_part:
        raise ValueError(f"{len(tokens)} sequences do not fill {parts} parts of {per_part}")
    order = sorted(range(len(tokens)), key=lambda i: (-int(tokens[i]), i))
    load = [0] * parts
    out: List[List[int]] = [[] for _ in range(parts)]
    for i in order:
        p = min((r for r in range(parts) if len(out[r]) < per_part), key=lambda r: (load[r], r))
        out[p].append(i)
        load[p] += int(tokens[i])
    return [sorted(o) for o in out]


def weak_job_contexts(cfg_id: int, seed: int, per_gpu: int, world: int) -> np.ndarray:
    """Contexts of a weak-scaled job on `world` GPUs: per_gpu * world
    sequences drawn from `seed`, in job order (world = 1: the one-GPU job)."""
    return contexts(cfg_id, seed, per_gpu * world)


def weak_rank_contexts(cfg_id: int, seed: int, per_gpu: int, world: int, rank: int) -> np.ndarray:
    """This rank's sequences of the weak-scaled job: the job's contexts
    token-balanced over the GPUs with per_gpu sequences each (the path
    shards by sequence; every GPU streams the same number of K/V bytes)."""
    job = weak_job_contexts(cfg_id, seed, per_gpu, world)
    if world == 1:
        return job
    return job[capped_partition(job, world, per_gpu)[rank]]


def pool_pages(ctx: Sequence[int], page_tokens: int, growth_tokens: int, factor: float = 1.25) -> int:
    """Physical pages for a layer pool: `factor` x the pages the contexts
    occupy, plus room for `growth_tokens` more per sequence."""
    need = sum((int(c) + page_tokens - 1) // page_tokens for c in ctx)
    grow = len(ctx) * ((growth_tokens + page_tokens - 1) // page_tokens + 1)
    return int(math.ceil(need * factor)) + grow


def decode_bytes(ctx_after: Sequence[int], cfg: Config, out_bytes: int = 4) -> int:
    """Algorithmic HBM bytes of one attend launch (one layer) over sequences
    whose contexts (after the append) are ctx_after: each K and V byte read
    once, q read, out written, block-table entries read."""
    kv_row = cfg.kv_heads * cfg.head_dim * 2
    total = 0
    for c in ctx_after:
        c = int(c)
        total += c * kv_row * 2
        total += cfg.n_q * cfg.n_heads * cfg.head_dim * (2 + out_bytes)
        total += 4 * ((c + cfg.page_tokens - 1) // cfg.page_tokens)
    return total


def append_bytes(n_rows: int, cfg: Config) -> int:
    """Bytes one append moves: rows read + written, K and V."""
    return n_rows * cfg.kv_heads * cfg.head_dim * 2 * 2 * 2
