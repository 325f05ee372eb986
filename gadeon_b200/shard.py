"""Sequence sharding across the GPUs of one node, and the output gather.

The paged-KV path shards by sequence: every GPU owns private page pools (one
per layer) for the sequences assigned to it, and the hot path has no
cross-GPU traffic.  The only collective is the gather of attention outputs
after a step, which goes over NCCL (NVLink) on GPUs and gloo in the CPU
tests.  The reference runs on one device and has no counterpart
(leok7v/gadeon has no multi-device code).
"""
from __future__ import annotations

from typing import List, Sequence

import numpy as np

from .workload import lpt_partition


def assign(tokens: Sequence[int], world: int) -> List[List[int]]:
    """Token-balanced assignment of job sequences to `world` ranks (greedy
    LPT: contexts descending, each to the least-loaded rank)."""
    return lpt_partition(tokens, world)


def imbalance(tokens: Sequence[int], shards: List[List[int]]) -> float:
    """max / mean tokens per rank (1.0 = perfectly balanced)."""
    loads = [sum(int(tokens[i]) for i in s) for s in shards]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean else 1.0


# Device index of each job sequence's row in the gathered buffer, per
# (partition, padded shard size, device): built and validated once.
_ORDER_CACHE: dict = {}


def _job_order(shards: List[List[int]], n_max: int, device):
    import torch

    key = (tuple(tuple(int(i) for i in s) for s in shards), n_max, str(device))
    idx = _ORDER_CACHE.get(key)
    if idx is None:
        # the shards must partition 0..n_job-1 (checked here, before an index
        # ever reaches a device kernel)
        n_all = sum(len(s) for s in shards)
        if sorted(i for s in key[0] for i in s) != list(range(n_all)):
            raise ValueError("shards do not partition the job's sequence indices 0..n-1")
        src = np.empty(n_all, dtype=np.int64)
        for r, s in enumerate(key[0]):
            src[np.asarray(s, dtype=np.int64)] = r * n_max + np.arange(len(s), dtype=np.int64)
        idx = torch.as_tensor(src, device=device)
        _ORDER_CACHE[key] = idx
    return idx


def gather_outputs(local, shards: List[List[int]], rank: int, group=None):
    """All-gather every rank's per-sequence outputs (rows in the order of
    its shard) and return them in job order: a tensor [n_job, *row_shape].

    Ranks hold different numbers of sequences, so each pads to the largest
    shard before one all_gather_into_tensor (NCCL) / all_gather (gloo); one
    index_select then puts the rows in job order, with an index built once
    per partition (no host-device transfer on later calls)."""
    import torch
    import torch.distributed as dist

    world = len(shards)
    n_max = max(len(s) for s in shards)
    row_shape = tuple(local.shape[1:])
    if local.shape[0] != len(shards[rank]):
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows for a shard of {len(shards[rank])}")
    order = _job_order(shards, n_max, local.device)
    if local.shape[0] == n_max and local.is_contiguous():
        padded = local
    else:
        padded = torch.zeros((n_max,) + row_shape, dtype=local.dtype, device=local.device)
        padded[: local.shape[0]] = local
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * n_max,) + row_shape, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, padded, group=group)
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
        out = torch.cat(parts, 0)
    return out.index_select(0, order)
