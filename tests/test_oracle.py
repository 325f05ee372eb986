"""CPU tests of the oracle (no GPU): known-answer cases for the restated
reference semantics, so the checker itself is trusted before it judges the
CUDA path.

The reference commits no golden vectors for this path and cannot run here
(Swift + Accelerate + CoreML), so the oracle is pinned by analytic cases
derived from the reference's own definitions:
  * PagePool.append / truncate / clone / compact / fromCompact
    (LLM/src/CoreML/PagedAttention.swift:85-276),
  * hostFlashDecode (PagedAttention.swift:317-366),
  * the causal verify route (LLM/src/CoreML/Engine.swift:2620-2646).
"""
import numpy as np
import pytest


def f32(O, a):
    return O.f16_bits_to_f32(a)


def np_flash(K, V, q, scale):
    """float64 softmax attention over fp16-rounded K [n, dh], V [n, dh]."""
    s = (K.astype(np.float64) @ q.astype(np.float64)) * scale
    e = np.exp(s - s.max())
    return (e @ V.astype(np.float64)) / e.sum()


def test_fp16_conversion_exhaustive(oracle):
    L = oracle.lib()
    bits = np.arange(0, 65536, 3, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    ours = np.array([L.orc_f16_to_f32(int(b)) for b in bits], dtype=np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(ours[~nan], ref[~nan])
    x = np.random.default_rng(0).standard_normal(20000).astype(np.float32) * np.float32(500)
    x = np.concatenate([x, np.float32([6.1e-5, 5.96e-8, 2.98e-8, 2.9802322e-8, 65504, 65519.99, -0.0, 1e-9])])
    ours = np.array([L.orc_f32_to_f16(float(v)) for v in x], dtype=np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(ours, x.astype(np.float16).view(np.uint16))


def test_normal_generator_stats(oracle):
    a = f32(oracle, oracle.normal_f16(123, 0, (200000,)))
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1) < 0.01
    b = oracle.normal_f16(123, 0, (16,))
    assert np.array_equal(b, oracle.normal_f16(123, 0, (16,)))
    assert not np.array_equal(b, oracle.normal_f16(123, 1, (16,)))


def test_permutation(oracle):
    p = oracle.permutation(5, 1000)
    assert sorted(p.tolist()) == list(range(1000))
    assert not np.array_equal(p, np.arange(1000))
    assert np.array_equal(p, oracle.permutation(5, 1000))
    # known answer for the spec (splitmix64 Fisher-Yates, identity start)
    assert oracle.permutation(42, 10).tolist() == [0, 9, 5, 8, 6, 4, 7, 2, 1, 3]


def test_append_pages_zeroed_and_layout(oracle):
    """append: fresh zeroed page at len % P == 0, row h at (h*P + slot)*dh."""
    O = oracle
    pool = O.OraclePool(kv_heads=2, head_dim=8, page_tokens=4, num_pages=8, seed=1)
    s = pool.seq_create()
    k = np.arange(5 * 2 * 8, dtype=np.uint16).reshape(5, 2, 8) + 1
    v = k + 1000
    assert pool.append([s], [5], k, v) == 0
    perm = O.permutation(1, 8)
    assert pool.pages(s).tolist() == perm[:2].tolist()
    assert pool.free_list().tolist() == perm[2:].tolist()
    K0, V0 = pool.page_bytes(int(perm[0]))
    for t in range(4):
        for h in range(2):
            assert np.array_equal(K0[h, t], k[t, h]) and np.array_equal(V0[h, t], v[t, h])
    K1, _ = pool.page_bytes(int(perm[1]))
    assert np.array_equal(K1[:, 0], k[4])
    assert (K1[:, 1:] == 0).all()  # zeroPage


def test_truncate_pops_last_first_keeps_stale(oracle):
    O = oracle
    pool = O.OraclePool(2, 8, 4, 16, seed=9)
    s = pool.seq_create()
    k = O.normal_f16(1, 1, (14, 2, 8))
    assert pool.append([s], [14], k, k) == 0
    pages = pool.pages(s).tolist()  # 4 pages
    assert pool.truncate([s], [5]) == 0
    assert pool.length(s) == 5
    assert pool.pages(s).tolist() == pages[:2]
    # freed last-first: pages[3] pushed, then pages[2] -> head is pages[2]
    assert pool.free_list()[:2].tolist() == [pages[2], pages[3]]
    # stale rows of the kept tail survive (slot 1.. of page 1)
    K1, _ = pool.page_bytes(pages[1])
    assert np.array_equal(K1[:, 1], k[5])
    # the next append reuses the most recently freed page and zeroes it
    assert pool.append([s], [4], k[:4], k[:4]) == 0
    assert pool.pages(s).tolist() == pages[:2] + [pages[2]]
    K2, _ = pool.page_bytes(pages[2])
    assert np.array_equal(K2[:, 0], k[3]) and (K2[:, 1:] == 0).all()
    assert pool.truncate([s], [10]) != 0  # beyond length


def test_batch_allocation_order(oracle):
    """Pops follow batch order, ascending slots within a sequence."""
    O = oracle
    pool = O.OraclePool(1, 8, 4, 32, seed=3)
    a, b = pool.seq_create(), pool.seq_create()
    k = O.normal_f16(2, 2, (13, 1, 8))
    assert pool.append([b, a], [9, 4], k, k) == 0
    perm = O.permutation(3, 32).tolist()
    assert pool.pages(b).tolist() == perm[0:3]
    assert pool.pages(a).tolist() == perm[3:4]
    Ka, _ = pool.page_bytes(perm[3])
    assert np.array_equal(Ka[0], k[9:13, 0])


def test_clone_shares_full_pages_copies_tail(oracle):
    O = oracle
    pool = O.OraclePool(1, 8, 4, 16, seed=4)
    s = pool.seq_create()
    k = O.normal_f16(3, 3, (6, 1, 8))
    pool.append([s], [6], k, k)
    c = pool.clone(s)
    ps, pc = pool.pages(s), pool.pages(c)
    assert ps[0] == pc[0] and ps[1] != pc[1]
    assert pool.page_ref(int(ps[0])) == 2 and pool.page_ref(int(pc[1])) == 1
    assert np.array_equal(pool.page_bytes(int(ps[1]))[0], pool.page_bytes(int(pc[1]))[0])
    # full-page boundary: nothing copied
    pool.append([s], [2], k[:2], k[:2])
    c2 = pool.clone(s)
    assert pool.pages(c2).tolist() == pool.pages(s).tolist()


def test_compact_roundtrip(oracle):
    O = oracle
    pool = O.OraclePool(3, 16, 8, 16, seed=5)
    K = O.normal_f16(1, 2, (3, 21, 16))
    V = O.normal_f16(1, 3, (3, 21, 16))
    t = pool.from_compact(K, V, 21)
    assert t >= 0 and pool.length(t) == 21 and len(pool.pages(t)) == 3
    K2, V2 = pool.compact(t)
    assert np.array_equal(K2, K) and np.array_equal(V2, V)


def test_flash_decode_matches_float64(oracle):
    O = oracle
    kvh, G, dh, P, n = 2, 4, 64, 4, 37
    pool = O.OraclePool(kvh, dh, P, 64, seed=6)
    s = pool.seq_create()
    k = O.normal_f16(9, 1, (n, kvh, dh))
    v = O.normal_f16(9, 2, (n, kvh, dh))
    pool.append([s], [n], k, v)
    q = O.normal_f16(9, 3, (kvh, G, dh))
    got = pool.flash_decode(s, q, G, dh ** -0.5).reshape(kvh, G, dh)
    kf, vf, qf = f32(O, k), f32(O, v), f32(O, q)
    for h in range(kvh):
        for g in range(G):
            want = np_flash(kf[:, h], vf[:, h], qf[h, g], dh ** -0.5)
            np.testing.assert_allclose(got[h, g], want, atol=2e-6, rtol=1e-5)


def test_flash_decode_known_answers(oracle):
    """Equal keys -> uniform softmax -> mean of V; a dominant key -> its V."""
    O = oracle
    dh = 16
    pool = O.OraclePool(1, dh, 4, 8, seed=1)
    s = pool.seq_create()
    one = np.float16(1.0).view(np.uint16)
    k = np.full((6, 1, dh), one, dtype=np.uint16)
    v = np.zeros((6, 1, dh), dtype=np.uint16)
    for t in range(6):
        v[t, 0, :] = np.float16(t).view(np.uint16)
    pool.append([s], [6], k, v)
    q = np.full((1, 1, dh), np.float16(0.5).view(np.uint16), dtype=np.uint16)
    out = pool.flash_decode(s, q, 1, 0.25)
    np.testing.assert_allclose(out, np.full(dh, 2.5, dtype=np.float32), rtol=1e-6)
    # dominant key: K_5 = 8, others 1 -> weight e^(scale*(8-1)*sum q) ~ 1
    k[5, 0, :] = np.float16(8.0).view(np.uint16)
    p2 = O.OraclePool(1, dh, 4, 8, seed=1)
    s2 = p2.seq_create()
    p2.append([s2], [6], k, v)
    out = p2.flash_decode(s2, q, 1, 1.0)
    np.testing.assert_allclose(out, np.full(dh, 5.0, dtype=np.float32), rtol=1e-6)


def test_causal_rows_match_per_token_route(oracle):
    """attend_causal row r == hostFlashDecode after appending rows 0..r
    (Engine.verifyAttn's append-then-attend loop)."""
    O = oracle
    kvh, G, dh, P = 2, 2, 32, 4
    pool = O.OraclePool(kvh, dh, P, 64, seed=8)
    ref = O.OraclePool(kvh, dh, P, 64, seed=8)
    s, r = pool.seq_create(), ref.seq_create()
    k = O.normal_f16(4, 1, (13, kvh, dh))
    v = O.normal_f16(4, 2, (13, kvh, dh))
    pool.append([s], [13], k, v)
    ref.append([r], [9], k[:9], v[:9])
    q = O.normal_f16(4, 3, (1, 4, kvh * G, dh))
    got = pool.attend_causal([s], 4, q, G, dh ** -0.5, n_threads=3)
    for row in range(4):
        ref.append([r], [1], k[9 + row:10 + row], v[9 + row:10 + row])
        want = ref.flash_decode(r, q[0, row].reshape(kvh, G, dh), G, dh ** -0.5)
        np.testing.assert_array_equal(got[0, row].reshape(-1), want)


def test_release_returns_pages(oracle):
    O = oracle
    pool = O.OraclePool(1, 8, 4, 8, seed=2)
    s = pool.seq_create()
    k = O.normal_f16(1, 1, (9, 1, 8))
    pool.append([s], [9], k, k)
    assert len(pool.free_list()) == 5
    assert pool.seq_release(s) == 0
    assert len(pool.free_list()) == 8
    assert pool.seq_create() == s
    assert pool.append([s], [40], np.zeros((40, 1, 8), np.uint16), np.zeros((40, 1, 8), np.uint16)) == O.ORC_ERR_NO_PAGES
    assert len(pool.free_list()) == 8  # failed append mutates nothing


def test_tile_at_windows(oracle):
    """tileAt (PagedAttention.swift:151-161): rows [0, count) are positions
    start.. of compact(), rows past count are zero (zeroPage), for windows
    inside one page, spanning pages, and empty; the reference's carry loop
    (:466-481) covers the sequence tile by tile."""
    kvh, dh, P = 2, 16, 8
    pool = oracle.OraclePool(kvh, dh, P, 32, 3)
    s = pool.seq_create()
    n = 45
    K = oracle.normal_f16(1, 0, (kvh, n, dh))
    V = oracle.normal_f16(1, 1, (kvh, n, dh))
    assert pool.seed(s, K, V, n) == 0
    for start, count, tile_p in [(0, 8, 8), (8, 8, 8), (40, 5, 8), (3, 10, 16), (13, 0, 4), (44, 1, 32)]:
        tk, tv = pool.tile_at(s, start, count, tile_p)
        assert np.array_equal(tk[:, :count], K[:, start:start + count])
        assert np.array_equal(tv[:, :count], V[:, start:start + count])
        assert not tk[:, count:].any() and not tv[:, count:].any()
    tile_p = 16
    got = np.concatenate([pool.tile_at(s, st, min(tile_p, n - st), tile_p)[0] for st in range(0, n, tile_p)], axis=1)
    assert np.array_equal(got[:, :n], K) and not got[:, n:].any()
    for start, count, tile_p in [(40, 6, 8), (-1, 1, 4), (0, 5, 4), (0, 1, 0)]:
        with pytest.raises(ValueError):
            pool.tile_at(s, start, count, tile_p)
