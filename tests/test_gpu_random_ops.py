"""Seeded random mixes of pool operations, GPU vs oracle, checked after every step.

The fixed scenarios of test_gpu_parity.py pin each operation on its own; here
the operations interleave the way an engine drives them: new sequences,
batched appends (chunks and single rows), the fused decode step, MTP verify
rows, prefill chunks on the tensor-core kernel, truncates (the rollback of
Engine.decodeSpecStep), clones (PagePool.clone: shared pages, copy-on-write
tails), releases and drafter rewinds -- including appends that exhaust the
pool, which must fail on both sides and change nothing.  After every step
the block tables, free list, lengths and reference counts must be bit-exact
with the oracle's restatement of PagePool (LLM/src/CoreML/PagedAttention.swift
:21-287 plus the explicit free-list policy), page bytes every few steps, and
every attention output within the BASELINE tolerance of the oracle's
hostFlashDecode / causal verify restatement.
"""
import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair, dev_f16

pytestmark = pytest.mark.gpu

OPS = ["new", "append", "decode", "verify", "chunk", "truncate", "clone", "release", "rewind", "fverify"]
WEIGHTS = np.array([1.0, 3.0, 4.0, 1.5, 0.5, 2.0, 1.0, 0.7, 1.0, 1.5])


@pytest.mark.parametrize("seed,P,dh,num_pages,grow,kvh,G", [
    (11, 8, 128, 260, 3, 2, 2), (12, 16, 256, 200, 3, 2, 2), (13, 16, 128, 120, 3, 2, 2),
    (14, 16, 128, 48, 10, 2, 2),
    (1010, 32, 128, 152, 2, 2, 2),  # two sequences sharing a partial tail page append in one batch
    (15, 16, 256, 220, 3, 4, 4),    # config 3's heads: verify rows fill the 16-row tile
])
def test_random_operation_mix(cuda, oracle, seed, P, dh, num_pages, grow, kvh, G):
    """grow: an append adds up to grow * P rows per sequence (10: the pool
    runs out now and then, and both sides must refuse the same appends)."""
    from gadeon_b200 import GKV_ERR_NO_PAGES, GkvError
    torch = cuda
    rng = np.random.default_rng(seed)
    # block-table rows longer than the pool, so running out of pages is the only refusal
    pr = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=num_pages, max_seqs=16, max_pps=2 * num_pages, seed=seed)
    live = []
    counts = {op: 0 for op in OPS}
    refused = 0

    def subset(k_max):
        k = int(rng.integers(1, min(k_max, len(live)) + 1))
        return [int(x) for x in rng.choice(live, size=k, replace=False)]

    def append_both(ids, n_new):
        """Append on both sides; a pool that cannot place it refuses on both."""
        nonlocal refused
        k, v = pr.rows(int(sum(n_new)))
        try:
            pr.gpu.append(ids, n_new, dev_f16(torch, k), dev_f16(torch, v))
        except GkvError as e:
            assert e.code == GKV_ERR_NO_PAGES, e
            assert pr.orc.append(ids, n_new, k, v) != 0, "oracle placed an append the GPU refused"
            refused += 1
            return False
        assert pr.orc.append(ids, n_new, k, v) == 0, "GPU placed an append the oracle refused"
        return True

    for step in range(140):
        op = OPS[int(rng.choice(len(OPS), p=WEIGHTS / WEIGHTS.sum()))]
        if op != "new" and not live:
            op = "new"
        if op == "new":
            if len(live) >= 10:
                continue
            live.append(pr.new_seq())
        elif op == "append":
            ids = subset(4)
            n_new = [int(x) for x in rng.integers(0, grow * P, size=len(ids))]
            append_both(ids, n_new)
        elif op == "decode":
            # the fused single-token step (unfused when a tail page is shared)
            ids = subset(6)
            k, v = pr.rows(len(ids))
            q = oracle.normal_f16(seed, 1000 + step, (len(ids), 1, kvh * G, dh))
            try:
                got = pr.gpu.append_attend(ids, 1, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
            except GkvError as e:
                assert e.code == GKV_ERR_NO_PAGES, e
                assert pr.orc.append(ids, [1] * len(ids), k, v) != 0
                refused += 1
                continue
            assert pr.orc.append(ids, [1] * len(ids), k, v) == 0
            want = pr.orc.attend_causal(ids, 1, q, G, dh ** -0.5, n_threads=8)
            assert_attn_close(got.cpu().numpy(), want, f"step {step} decode")
        elif op == "fverify":
            # drafts appended and verified in one call (fused into the attend
            # launch unless a tail page is shared)
            ids = subset(4)
            n_q = int(rng.integers(2, 9))
            k, v = pr.rows(len(ids) * n_q)
            q = oracle.normal_f16(seed, 5000 + step, (len(ids), n_q, kvh * G, dh))
            try:
                got = pr.gpu.append_attend(ids, n_q, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
            except GkvError as e:
                assert e.code == GKV_ERR_NO_PAGES, e
                assert pr.orc.append(ids, [n_q] * len(ids), k, v) != 0
                refused += 1
                continue
            assert pr.orc.append(ids, [n_q] * len(ids), k, v) == 0
            want = pr.orc.attend_causal(ids, n_q, q, G, dh ** -0.5, n_threads=8)
            assert_attn_close(got.cpu().numpy(), want, f"step {step} fused verify n_q={n_q}")
        elif op in ("verify", "chunk"):
            n_q = int(rng.integers(2, 9)) if op == "verify" else int(rng.integers(9, 48))
            ids = [s for s in live if pr.gpu.length(s) >= n_q]
            if not ids:
                continue
            ids = [int(x) for x in rng.choice(ids, size=min(3, len(ids)), replace=False)]
            got, want = pr.attend(ids, n_q, G)  # n_q*G > 16 runs the tcgen05 chunk kernel
            assert_attn_close(got, want, f"step {step} {op} n_q={n_q}")
        elif op == "truncate":
            ids = subset(4)
            new_len = [int(rng.integers(0, pr.gpu.length(s) + 1)) for s in ids]
            pr.truncate(ids, new_len)
        elif op == "clone":
            if len(live) >= 10:
                continue
            src = int(rng.choice(live))
            try:
                c = pr.gpu.clone(src)
            except GkvError as e:  # no free page for the tail copy: refused on both sides
                assert e.code == GKV_ERR_NO_PAGES, e
                assert pr.orc.clone(src) < 0, "oracle cloned where the GPU refused"
                refused += 1
                continue
            assert pr.orc.clone(src) == c
            pr.seqs.append(c)
            live.append(c)
        elif op == "release":
            s = int(rng.choice(live))
            pr.gpu.seq_release(s)
            assert pr.orc.seq_release(s) == 0
            live.remove(s)
            pr.seqs.remove(s)
        elif op == "rewind":
            # drafter upkeep: back to a base length, then m committed rows
            # (only when the free list surely holds the rows: an append
            # needs at most a copied tail page plus one page per P rows)
            ids = subset(3)
            base = [int(rng.integers(0, pr.gpu.length(s) + 1)) for s in ids]
            n_new = [int(x) for x in rng.integers(0, 6, size=len(ids))]
            if pr.gpu.free_page_count() < sum(n // P + 2 for n in n_new):
                continue
            k, v = pr.rows(int(sum(n_new)))
            pr.gpu.rewind_append(ids, base, n_new, dev_f16(torch, k), dev_f16(torch, v))
            assert pr.orc.truncate(ids, base) == 0
            assert pr.orc.append(ids, n_new, k, v) == 0
        counts[op] += 1
        pr.check_state(pages=(step % 10 == 9))
    pr.check_state(pages=True)
    # the mix exercised the operations that move pages
    assert counts["decode"] > 10 and counts["truncate"] > 5 and counts["clone"] > 0, (counts, refused)
    if grow >= 10:
        assert refused > 0, "the small pool never ran out"


def test_random_large_batches(cuda, oracle):
    """Batches of 129-300 sequences -- past the 128 whose descriptors ride in
    the kernel parameter block, so every call uploads its descriptor through
    the pool's staging ring -- in a seeded mix of fused decode, fused verify,
    appends, truncates and clones; state bit-exact, outputs in tolerance."""
    torch = cuda
    seed, P, dh, G, kvh = 5001, 16, 128, 2, 2
    rng = np.random.default_rng(seed)
    pr = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=9000, max_seqs=400, max_pps=2000, seed=seed)
    live = [pr.new_seq() for _ in range(300)]
    pr.append(live, [int(x) for x in rng.integers(1, 200, size=len(live))])
    for step in range(20):
        op = rng.choice(["decode", "fverify", "append", "truncate", "clone"], p=[0.35, 0.25, 0.15, 0.15, 0.10])
        ids = [int(x) for x in rng.choice(live, size=int(rng.integers(129, len(live) + 1)), replace=False)]
        if op in ("decode", "fverify"):
            n_q = 1 if op == "decode" else int(rng.integers(2, 5))
            k, v = pr.rows(len(ids) * n_q)
            q = oracle.normal_f16(seed, step, (len(ids), n_q, kvh * G, dh))
            got = pr.gpu.append_attend(ids, n_q, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
            assert pr.orc.append(ids, [n_q] * len(ids), k, v) == 0
            want = pr.orc.attend_causal(ids, n_q, q, G, dh ** -0.5, n_threads=8)
            assert_attn_close(got.cpu().numpy(), want, f"step {step} {op}")
        elif op == "append":
            pr.append(ids, [int(x) for x in rng.integers(0, 3 * P, size=len(ids))])
        elif op == "truncate":
            pr.truncate(ids, [int(rng.integers(1, pr.gpu.length(s) + 1)) for s in ids])
        elif op == "clone":
            for s in ids[:5]:
                c = pr.gpu.clone(s)
                assert pr.orc.clone(s) == c
                pr.seqs.append(c)
                live.append(c)
        pr.check_state(pages=(step % 10 == 9))
    pr.check_state(pages=True)
