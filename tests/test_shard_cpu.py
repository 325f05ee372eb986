"""Multi-process host logic of the sequence-sharded path on CPU (gloo,
world size 2): token-balanced assignment, the padded output gather back to
job order, and failure detection when a rank dies before the collective
(the failure is made on the host; no GPU is involved)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from gadeon_b200.shard import assign, imbalance
from gadeon_b200.workload import contexts


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_assign_is_a_token_balanced_partition():
    tokens = contexts(5, 123, 512)
    for world in (1, 2, 4, 8):
        shards = assign(tokens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(512))
        assert imbalance(tokens, shards) < 1.01
    # LPT places the longest context first, on rank 0
    shards = assign([5, 9, 1, 7], 2)
    assert 1 in shards[0] and shards == [[1, 2], [0, 3]]


def test_weak_scaled_job_is_count_capped_and_token_balanced():
    """Config 2 at N GPUs: 64*N job sequences, exactly 64 per rank, token
    loads within 0.1% of each other; N=1 is the one-GPU job unchanged."""
    from gadeon_b200.workload import capped_partition, weak_job_contexts, weak_rank_contexts
    assert np.array_equal(weak_rank_contexts(2, 7, 64, 1, 0), contexts(2, 7, 64))
    for world in (2, 4, 8):
        job = weak_job_contexts(2, 7, 64, world)
        parts = capped_partition(job, world, 64)
        assert sorted(i for p in parts for i in p) == list(range(64 * world))
        assert all(len(p) == 64 for p in parts)
        assert imbalance(job, parts) < 1.001
        for r in range(world):
            assert np.array_equal(weak_rank_contexts(2, 7, 64, world, r), job[parts[r]])
    with pytest.raises(ValueError):
        capped_partition([1, 2, 3], 2, 2)
    # the cap binds: plain LPT would put all three short sequences beside each
    # other; with two per part the last one joins the long sequence
    assert capped_partition([100, 1, 1, 1], 2, 2) == [[0, 3], [1, 2]]


def _worker(rank, world, port, fail_rank, q):
    import torch
    import torch.distributed as dist

    from gadeon_b200.shard import gather_outputs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    tokens = [100, 900, 50, 400, 300, 700, 20]
    shards = assign(tokens, world)
    # each sequence's "attention output" row encodes its job index
    local = torch.tensor([[float(i), float(i) * 2] for i in shards[rank]], dtype=torch.float32)
    try:
        if rank == fail_rank:
            raise RuntimeError("rank failed before the gather")
        job = gather_outputs(local, shards, rank)
        # again with other rows on the same partition (the cached index), and
        # on an equal-size partition (no padding copy)
        job2 = gather_outputs(local * 10, shards, rank)
        equal = [[0, 2, 5, 6], [1, 3, 4, 7]][:world] if world == 2 else None
        job3 = (gather_outputs(torch.tensor([[float(i)] for i in equal[rank]]), equal, rank).numpy().tolist()
                if equal else None)
        q.put((rank, "ok", (job.numpy().tolist(), job2.numpy().tolist(), job3)))
    except Exception as e:  # the surviving rank must see an error, not hang
        q.put((rank, "error", type(e).__name__))
    finally:
        if rank == fail_rank:
            q.close()
            q.join_thread()  # deliver the report before the hard exit
            os._exit(0)  # leave without the collective
        dist.destroy_process_group()


def _run(world, fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=120)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_gather_outputs_job_order_gloo():
    res = _run(2, fail_rank=-1)
    want = [[float(i), float(i) * 2] for i in range(7)]
    for rank in range(2):
        status, (job, job2, job3) = res[rank]
        assert status == "ok"
        assert job == want
        assert job2 == [[10 * a, 10 * b] for a, b in want]
        assert job3 == [[float(i)] for i in range(8)]


def test_dead_rank_is_detected_by_the_collective():
    res = _run(2, fail_rank=1)
    assert res[1][0] == "error"
    assert res[0][0] == "error", res  # the gather fails instead of hanging


def test_partition_properties():
    """For random context lists: every sequence lands in exactly one part;
    the capped partition gives every part exactly per_part sequences; the
    LPT partition keeps the heaviest part within the list-scheduling bound
    (mean load + the largest context)."""
    hypothesis = pytest.importorskip("hypothesis")
    from hypothesis import given, settings, strategies as st
    from gadeon_b200.workload import capped_partition, lpt_partition

    @settings(max_examples=200, deadline=None)
    @given(parts=st.integers(1, 8), per=st.integers(1, 12), data=st.data())
    def check(parts, per, data):
        tokens = data.draw(st.lists(st.integers(0, 131072), min_size=parts * per, max_size=parts * per))
        for split in (capped_partition(tokens, parts, per), lpt_partition(tokens, parts)):
            assert sorted(i for p in split for i in p) == list(range(len(tokens)))
            assert len(split) == parts and all(p == sorted(p) for p in split)
        assert all(len(p) == per for p in capped_partition(tokens, parts, per))
        loads = [sum(tokens[i] for i in p) for p in lpt_partition(tokens, parts)]
        assert max(loads) <= sum(tokens) / parts + max(tokens) + 1e-9

    check()


def test_gather_outputs_refuses_shards_that_do_not_partition_the_job():
    """Row indices that fall outside 0..n-1 (or repeat) are refused on the
    host, before any collective or index kernel runs."""
    import pytest
    import torch
    from gadeon_b200.shard import gather_outputs
    local = torch.zeros((2, 3))
    for shards in ([[0, 5], [1, 2]], [[0, 1], [1, 2]], [[0, 2], [2]]):
        with pytest.raises(ValueError, match="partition"):
            gather_outputs(local, shards, 0)
    with pytest.raises(ValueError, match="rows"):  # the rank's rows do not match its shard
        gather_outputs(torch.zeros((3, 3)), [[0, 1], [2, 3]], 0)
