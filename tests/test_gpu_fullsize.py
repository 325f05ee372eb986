"""Parity at the BASELINE configurations' real sizes, against the oracle.

The other parity tests use small shapes; here each kernel runs on its
configuration's real geometry and context lengths (drawn by the bench's own
workload generators), with the element-wise tolerance of conftest.py:

* config 2 -- all 64 sequences, contexts ~U[1024, 32768], nH 8 / KVH 2 /
  dh 256, P 16, a pool of 1.25x the pages with a seeded permutation; 8 fused
  decode steps (append inside the attend launch), every output row checked;
* config 3 -- 128 sequences at 8,192, nH 16 / KVH 4; 16 MTP cycles of 4
  drafts appended and attended causally in one launch, then truncated to
  the pre-draft length + U{0..4}; every output row checked, block tables and
  free list bit-exact after every cycle;
* config 4 -- 2 sequences, each a seeded 16,384-token context plus one
  4,096-row chunk (the tensor-core chunk kernel); 512 rows of every head
  checked (the first 64, the last 64 and 384 spread between); the same rows
  again with GKV_ATTEND_P_F16, within that option's error bound;
* config 5 -- 16 sequences of the long-context job, contexts log-uniform in
  [4096, 131072] (the longest of the job included), 4 fused decode steps.

After every step the sequences' lengths, block tables, the free list and
the tail pages' bytes (rows past the end included) are bit-exact; at the end
every sequence's whole content is compared (compact)."""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair, dev_f16

pytestmark = pytest.mark.gpu

THREADS = max(1, min(16, os.cpu_count() or 1))
BENCH_SEED = 20251201  # bench.py's default --seed


def seed_contexts(pr, lens, seed):
    """One new sequence per length in both pools, filled with seeded N(0,1)
    fp16 rows [KVH, n, dh] (drawn on THREADS host threads)."""
    def gen(i):
        n = int(lens[i])
        return (pr.O.normal_f16(seed, 2 * i, (pr.kvh, n, pr.dh)),
                pr.O.normal_f16(seed, 2 * i + 1, (pr.kvh, n, pr.dh)))

    ids = []
    with ThreadPoolExecutor(THREADS) as ex:
        for i, (K, V) in enumerate(ex.map(gen, range(len(lens)))):
            s = pr.new_seq()
            pr.gpu.seed(s, dev_f16(pr.torch, K), dev_f16(pr.torch, V), int(lens[i]))
            assert pr.orc.seed(s, K, V, int(lens[i])) == 0
            ids.append(s)
    return ids


def check_state(pr, ids, what):
    """Lengths, block tables, free list and every sequence's tail page (the
    page an append writes, rows past the end included) bit-exact."""
    assert np.array_equal(pr.gpu.export_free_list(), pr.orc.free_list()), f"{what}: free list"
    for s in ids:
        assert pr.gpu.length(s) == pr.orc.length(s), f"{what}: length of {s}"
        t = pr.gpu.export_table(s)
        assert np.array_equal(t, pr.orc.pages(s)), f"{what}: table of {s}"
        if len(t):
            gk, gv = pr.gpu.export_page(int(t[-1]))
            ok, ov = pr.orc.page_bytes(int(t[-1]))
            assert np.array_equal(gk, ok) and np.array_equal(gv, ov), f"{what}: tail page of {s}"
    assert pr.gpu.device_status() == 0, what


def check_contents(pr, ids, what):
    """Every sequence's rows, compacted, bit-exact."""
    for s in ids:
        K, V = pr.gpu.compact(s)
        oK, oV = pr.orc.compact(s)
        assert np.array_equal(K.cpu().numpy().view(np.uint16), oK), f"{what}: K of {s}"
        assert np.array_equal(V.cpu().numpy().view(np.uint16), oV), f"{what}: V of {s}"


def new_pair(cuda, oracle, cfg_id, lens, growth, seed):
    from gadeon_b200 import workload as W
    cfg = W.CONFIGS[cfg_id]
    P = cfg.page_tokens
    return Pair(cuda, oracle, kvh=cfg.kv_heads, dh=cfg.head_dim, P=P,
                num_pages=W.pool_pages(lens, P, growth), max_seqs=len(lens),
                max_pps=(int(max(lens)) + growth + P - 1) // P + 1, seed=seed), cfg


def test_config2_full_size_decode(cuda, oracle):
    from gadeon_b200 import workload as W
    steps = 8
    lens = W.contexts(2, BENCH_SEED, 64)
    pr, cfg = new_pair(cuda, oracle, 2, lens, steps, seed=2002)
    ids = seed_contexts(pr, lens, 2202)
    check_state(pr, ids, "config 2 seeded")
    G, scale = cfg.group, cfg.head_dim ** -0.5
    for step in range(steps):
        k, v = pr.rows(len(ids))
        q = oracle.normal_f16(2302, step, (len(ids), 1, cfg.n_heads, cfg.head_dim))
        got = pr.gpu.append_attend(ids, 1, G, dev_f16(cuda, k), dev_f16(cuda, v), dev_f16(cuda, q)).cpu().numpy()
        assert pr.orc.append(ids, [1] * len(ids), k, v) == 0
        want = pr.orc.attend_causal(ids, 1, q, G, scale, n_threads=THREADS)
        assert_attn_close(got, want, f"config 2 step {step}")
        check_state(pr, ids, f"config 2 step {step}")
    check_contents(pr, ids, "config 2")


def test_config3_full_size_verify_rollback(cuda, oracle):
    from gadeon_b200 import workload as W
    cycles, S = 16, 4
    lens = W.contexts(3, BENCH_SEED, 128)
    pr, cfg = new_pair(cuda, oracle, 3, lens, cycles * S + S, seed=3003)
    ids = seed_contexts(pr, lens, 3203)
    G, scale = cfg.group, cfg.head_dim ** -0.5
    rng = np.random.default_rng(3303)
    for c in range(cycles):
        before = np.array([pr.orc.length(s) for s in ids], dtype=np.int64)
        k, v = pr.rows(len(ids) * S)
        q = oracle.normal_f16(3403, c, (len(ids), S, cfg.n_heads, cfg.head_dim))
        got = pr.gpu.append_attend(ids, S, G, dev_f16(cuda, k), dev_f16(cuda, v), dev_f16(cuda, q)).cpu().numpy()
        assert pr.orc.append(ids, [S] * len(ids), k, v) == 0
        want = pr.orc.attend_causal(ids, S, q, G, scale, n_threads=THREADS)
        assert_attn_close(got, want, f"config 3 cycle {c}")
        pr.truncate(ids, before + rng.integers(0, S, size=len(ids), endpoint=True))
        check_state(pr, ids, f"config 3 cycle {c}")
    check_contents(pr, ids, "config 3")


def test_config4_full_size_chunk(cuda, oracle):
    from gadeon_b200 import workload as W
    n_seqs, n_q = 2, W.CONFIGS[4].n_q
    lens = W.contexts(4, BENCH_SEED, n_seqs)
    pr, cfg = new_pair(cuda, oracle, 4, lens, n_q, seed=4004)
    ids = seed_contexts(pr, lens, 4204)
    G, scale = cfg.group, cfg.head_dim ** -0.5
    k, v = pr.rows(n_seqs * n_q)
    q = oracle.normal_f16(4304, 0, (n_seqs, n_q, cfg.n_heads, cfg.head_dim))
    got = pr.gpu.append_attend(ids, n_q, G, dev_f16(cuda, k), dev_f16(cuda, v), dev_f16(cuda, q)).cpu().numpy()
    assert pr.orc.append(ids, [n_q] * n_seqs, k, v) == 0
    rows = np.unique(np.concatenate([np.arange(64), np.arange(n_q - 64, n_q),
                                     np.linspace(64, n_q - 65, 384).astype(np.int64)]))
    assert len(rows) == 512
    want = pr.orc.attend_rows(ids, n_q, rows, q[:, rows], G, scale, n_threads=THREADS)
    assert_attn_close(got[:, rows], want, f"config 4: {len(rows)} rows x {cfg.n_heads} heads")
    check_state(pr, ids, "config 4")
    check_contents(pr, ids, "config 4")


def test_config5_full_size_long_context_decode(cuda, oracle):
    from gadeon_b200 import workload as W
    steps = 4
    job = W.contexts(5, BENCH_SEED, 512)
    top = int(np.argmax(job))
    pick = np.sort(np.concatenate([[top], [i for i in range(0, 512, 34) if i != top][:15]]))
    lens = job[pick]
    assert len(lens) == 16 and lens.max() > 120000
    pr, cfg = new_pair(cuda, oracle, 5, lens, steps, seed=5005)
    ids = seed_contexts(pr, lens, 5205)
    G, scale = cfg.group, cfg.head_dim ** -0.5
    for step in range(steps):
        k, v = pr.rows(len(ids))
        q = oracle.normal_f16(5305, step, (len(ids), 1, cfg.n_heads, cfg.head_dim))
        got = pr.gpu.append_attend(ids, 1, G, dev_f16(cuda, k), dev_f16(cuda, v), dev_f16(cuda, q)).cpu().numpy()
        assert pr.orc.append(ids, [1] * len(ids), k, v) == 0
        want = pr.orc.attend_causal(ids, 1, q, G, scale, n_threads=THREADS)
        assert_attn_close(got, want, f"config 5 step {step}")
        check_state(pr, ids, f"config 5 step {step}")
    check_contents(pr, ids, "config 5")


def test_config4_full_size_chunk_p_f16(cuda, oracle):
    """The opt-in GKV_ATTEND_P_F16 at config 4's size: 2 sequences of 16,384
    seeded rows plus a 4,096-row chunk; the same 512 rows of every head as
    the default's test, each element within 2^-10 x sum_i w_i |V_i| + 1e-5
    of the oracle (the bound computed on a twin oracle pool holding |V|)."""
    from gadeon_b200 import BlockPool
    from gadeon_b200 import workload as W
    cfg = W.CONFIGS[4]
    n_seqs, n_q = 2, cfg.n_q
    kvh, dh, P, G = cfg.kv_heads, cfg.head_dim, cfg.page_tokens, cfg.group
    lens = [int(c) + n_q for c in W.contexts(4, BENCH_SEED, n_seqs)]
    pages = sum((n + P - 1) // P for n in lens) + 16
    gpu = BlockPool(kvh, dh, P, pages, n_seqs + 1, pages, seed=4404)
    orc = oracle.OraclePool(kvh, dh, P, pages, 4404)
    absorc = oracle.OraclePool(kvh, dh, P, pages, 4404)

    def gen(i):
        return (oracle.normal_f16(4504, 2 * i, (kvh, lens[i], dh)),
                oracle.normal_f16(4504, 2 * i + 1, (kvh, lens[i], dh)))

    ids = []
    with ThreadPoolExecutor(THREADS) as ex:
        for i, (K, V) in enumerate(ex.map(gen, range(n_seqs))):
            s = gpu.seq_create()
            assert orc.seq_create() == s and absorc.seq_create() == s
            gpu.seed(s, dev_f16(cuda, K), dev_f16(cuda, V), lens[i])
            assert orc.seed(s, K, V, lens[i]) == 0
            assert absorc.seed(s, K, V & np.uint16(0x7FFF), lens[i]) == 0
            ids.append(s)
    scale = dh ** -0.5
    q = oracle.normal_f16(4604, 0, (n_seqs, n_q, cfg.n_heads, dh))
    got = gpu.attend(ids, n_q, G, dev_f16(cuda, q), scale=scale, p_f16=True).cpu().numpy()
    rows = np.unique(np.concatenate([np.arange(64), np.arange(n_q - 64, n_q),
                                     np.linspace(64, n_q - 65, 384).astype(np.int64)]))
    want = orc.attend_rows(ids, n_q, rows, q[:, rows], G, scale, n_threads=THREADS)
    bound = absorc.attend_rows(ids, n_q, rows, q[:, rows], G, scale, n_threads=THREADS)
    err = np.abs(got[:, rows] - want)
    lim = 2.0 ** -10 * bound + 1e-5
    assert np.all(err <= lim), f"max |d| {err.max():.3g}, max |d| / B {np.max(err / np.maximum(bound, 1e-30)):.3g}"
    assert gpu.device_status() == 0
