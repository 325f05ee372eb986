"""Launch chaining and descriptor placement of the attend kernel, vs the oracle.

A call with up to 128 sequences carries its work descriptor in the kernel's
parameter block and is launched with programmatic stream serialization, so
its CTAs may start while the previous kernel of the stream drains; a larger
call uploads the descriptor to a device slot first.  These tests queue many
dependent launches with no host synchronisation between them (each step's
block table and page writes are read by the next step's launch) and cross the
128-sequence boundary, then compare every output with the oracle's
hostFlashDecode restatement (LLM/src/CoreML/PagedAttention.swift:317-366) and
the cache state bit for bit.
"""
import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair, dev_f16

pytestmark = pytest.mark.gpu


def test_back_to_back_fused_steps_two_pools(cuda, oracle):
    """16 decode steps on two pools (layers), all queued before any result is
    read: fresh pages appear mid-chain (contexts sit just below page
    boundaries), so a launch reads table entries the previous launch on the
    same pool wrote."""
    torch = cuda
    G, dh, P = 4, 256, 16
    pairs = [Pair(cuda, oracle, kvh=2, dh=dh, P=P, num_pages=900, seed=41 + i) for i in range(2)]
    ctx = [1, P - 2, 2 * P - 1, 100, 1000, 3 * P]
    ids = []
    for pr in pairs:
        ids.append([pr.new_seq() for _ in ctx])
        pr.append(ids[-1], ctx)
    torch.cuda.synchronize()
    steps = 16
    rows, qs, outs = [], [], []
    for step in range(steps):
        for li, pr in enumerate(pairs):
            k, v = pr.rows(len(ctx))
            q = oracle.normal_f16(23 + li, step, (len(ctx), 1, 2 * G, dh))
            out = torch.empty((len(ctx), 1, 2 * G, dh), dtype=torch.float32, device="cuda")
            pr.gpu.append_attend(ids[li], 1, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q), out=out)
            rows.append((k, v))
            qs.append(q)
            outs.append(out)
    torch.cuda.synchronize()
    for step in range(steps):
        for li, pr in enumerate(pairs):
            i = step * len(pairs) + li
            k, v = rows[i]
            assert pr.orc.append(ids[li], [1] * len(ctx), k, v) == 0
            want = pr.orc.attend_causal(ids[li], 1, qs[i], G, dh ** -0.5)
            assert_attn_close(outs[i].cpu().numpy(), want, f"step {step} pool {li}")
    for pr in pairs:
        pr.check_state()


@pytest.mark.parametrize("n_seqs", [128, 129, 200])
def test_descriptor_inline_and_uploaded(cuda, oracle, n_seqs):
    """Around the 128-sequence inline limit: plain decode attend, fused
    decode append + attend and fused MTP verify (4 drafts x G=4 rows) all
    match."""
    torch = cuda
    G, dh, P, kvh = 4, 128, 16, 2
    pr = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=n_seqs * 8, max_seqs=n_seqs, seed=5)
    rng = np.random.default_rng(n_seqs)
    ctx = [int(c) for c in rng.integers(1, 70, size=n_seqs)]
    ids = [pr.new_seq() for _ in range(n_seqs)]
    pr.append(ids, ctx)
    got, want = pr.attend(ids, 1, G)
    assert_attn_close(got, want, f"attend n={n_seqs}")
    k, v = pr.rows(n_seqs)
    q = oracle.normal_f16(31, n_seqs, (n_seqs, 1, kvh * G, dh))
    got = pr.gpu.append_attend(ids, 1, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
    assert pr.orc.append(ids, [1] * n_seqs, k, v) == 0
    want = pr.orc.attend_causal(ids, 1, q, G, dh ** -0.5)
    assert_attn_close(got.cpu().numpy(), want, f"fused n={n_seqs}")
    # verify rows appended in the same call (fused: the two-page tails travel
    # inline up to 128 sequences, uploaded beyond)
    k, v = pr.rows(n_seqs * 4)
    q = oracle.normal_f16(32, n_seqs, (n_seqs, 4, kvh * G, dh))
    got = pr.gpu.append_attend(ids, 4, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
    assert pr.orc.append(ids, [4] * n_seqs, k, v) == 0
    want = pr.orc.attend_causal(ids, 4, q, G, dh ** -0.5)
    assert_attn_close(got.cpu().numpy(), want, f"fused verify n={n_seqs}")
    pr.check_state()


@pytest.mark.parametrize("P,dh,n_q,G", [(8, 256, 4, 4), (8, 128, 8, 2), (16, 256, 4, 4), (16, 128, 16, 1),
                                        (64, 256, 3, 4), (128, 128, 5, 2)])
def test_fused_verify_append(cuda, oracle, P, dh, n_q, G):
    """gkv_append_attend with n_q > 1 on the split-K kernel writes the n_q
    draft rows inside the attend launch: rows straddling a page boundary, a
    fresh page starting among them, pages larger than the key tile, and a
    cloned (shared) tail that takes the two-kernel path.  Tables, free list
    and page bytes bit-exact; outputs within tolerance of the causal verify
    restatement (Engine.swift:2620-2646)."""
    torch = cuda
    pr = Pair(cuda, oracle, kvh=2, dh=dh, P=P, num_pages=900, seed=61)
    ctx = [1, P - 2, P - 1, P, 2 * P + 1, 300]
    ids = [pr.new_seq() for _ in ctx]
    pr.append(ids, ctx)
    for step in range(6):
        if step == 2:  # share a partial tail: this step appends through the unfused path
            c = pr.gpu.clone(ids[4])
            assert pr.orc.clone(ids[4]) == c
            pr.seqs.append(c)
            ids.append(c)
        k, v = pr.rows(len(ids) * n_q)
        q = oracle.normal_f16(71, step, (len(ids), n_q, 2 * G, dh))
        got = pr.gpu.append_attend(ids, n_q, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
        assert pr.orc.append(ids, [n_q] * len(ids), k, v) == 0
        want = pr.orc.attend_causal(ids, n_q, q, G, dh ** -0.5)
        assert_attn_close(got.cpu().numpy(), want, f"fused verify step {step}")
        pr.check_state()
        # the rejected drafts go (Engine.decodeSpecStep's truncate)
        keep = [pr.gpu.length(s) - (step + s) % (n_q + 1) for s in ids]
        pr.truncate(ids, keep)
        pr.check_state(pages=False)
