"""Property tests of the oracle's page bookkeeping (CPU, hypothesis).

The oracle is the checker every GPU parity test trusts, and its block pool
is an explicit model the reference does not have (PagePool owns ARC pages,
LLM/src/CoreML/PagedAttention.swift:21-287).  Under random sequences of
append / truncate / clone / release the model must keep its own invariants:

* every physical page is either on the free list or referenced, never both;
* a page's reference count equals the number of block-table entries naming it;
* a sequence holds exactly ceil(length / P) pages;
* a clone's contents are its source's at clone time, whatever is appended to
  or truncated from either afterwards (copy-on-write, :199-210);
* a refused append changes nothing.
"""
import numpy as np
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402

OPS = st.lists(
    st.tuples(st.sampled_from(["new", "append", "truncate", "clone", "release"]),
              st.integers(0, 10 ** 6), st.integers(0, 10 ** 6)),
    min_size=1, max_size=40)


def check_invariants(pool, seqs, P, num_pages):
    free = [int(x) for x in pool.free_list()]
    assert len(free) == len(set(free))
    refs = np.zeros(num_pages, dtype=np.int64)
    for s in seqs:
        pages = [int(x) for x in pool.pages(s)]
        assert len(pages) == -(-pool.length(s) // P)
        for pid in pages:
            refs[pid] += 1
    for pid in range(num_pages):
        assert pool.page_ref(pid) == refs[pid], pid
        assert (refs[pid] == 0) == (pid in set(free)), pid


@settings(max_examples=150, deadline=None)
@given(ops=OPS, P=st.sampled_from([1, 2, 4, 8]), seed=st.integers(0, 2 ** 32 - 1))
def test_pool_invariants_under_random_operations(oracle, ops, P, seed):
    kvh, dh, num_pages = 1, 8, 24
    pool = oracle.OraclePool(kvh, dh, P, num_pages, seed)
    seqs, snapshots, stream = [], {}, 0
    for op, a, b in ops:
        if op == "new" or not seqs:
            seqs.append(pool.seq_create())
            continue
        s = seqs[a % len(seqs)]
        if op == "append":
            n = b % (3 * P + 1)
            k = oracle.normal_f16(seed % 1000, stream, (n, kvh, dh))
            stream += 1
            before = (pool.free_list().copy(), [pool.pages(x).copy() for x in seqs], [pool.length(x) for x in seqs])
            rc = pool.append([s], [n], k, k)
            if rc != 0:  # refused: nothing changed
                assert np.array_equal(before[0], pool.free_list())
                assert all(np.array_equal(p, pool.pages(x)) for p, x in zip(before[1], seqs))
                assert before[2] == [pool.length(x) for x in seqs]
        elif op == "truncate":
            to = b % (pool.length(s) + 1)
            assert pool.truncate([s], [to]) == 0
            if s in snapshots:  # rows past `to` may be rewritten from now on
                snapshots[s] = (snapshots[s][0], min(snapshots[s][1], to))
        elif op == "clone":
            c = pool.clone(s)
            if c >= 0:
                seqs.append(c)
                snapshots[c] = (pool.compact(s), pool.length(s))
        elif op == "release":
            assert pool.seq_release(s) == 0
            seqs.remove(s)
            snapshots.pop(s, None)
        check_invariants(pool, seqs, P, num_pages)
    # copy-on-write: every clone still holds its source's rows at clone time,
    # up to the shortest length it has been truncated to since
    for c, ((K, V), n) in snapshots.items():
        if c in seqs:
            K2, V2 = pool.compact(c)
            assert np.array_equal(K2[:, :n], K[:, :n]) and np.array_equal(V2[:, :n], V[:, :n])
