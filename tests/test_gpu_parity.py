"""GPU vs oracle parity through the C ABI (libgadeonkv.so).

Cache state (block tables, free list, reference counts, page bytes) must be
bit-exact after every append / truncate / clone; attention outputs must be
within max-abs 2e-3 and relative 1e-2 of the oracle's restatement of
hostFlashDecode (LLM/src/CoreML/PagedAttention.swift:317-366) and of the
causal verify loop (LLM/src/CoreML/Engine.swift:2620-2646).

The fixture ideas follow the reference's own tests: tiny pages (P=4/8) to
force multi-page gathers (MetalSelfTest.swift:132-147), T=40 / nH=2 / nKV=1 /
hd 256 and 512 (GemmaMetalKernelTests.swift:205-271), a mark mid-page
followed by replay (MetalSelfTest.swift:150-168), and an anti-vacuity check.
"""
import numpy as np
import pytest

from conftest import assert_attn_close

pytestmark = pytest.mark.gpu


def dev_f16(torch, a):
    """uint16 fp16 bit patterns (numpy) -> torch.float16 CUDA tensor."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.float16)


class Pair:
    """A GPU BlockPool and an oracle pool driven with identical calls."""

    def __init__(self, torch, O, kvh, dh, P, num_pages, max_seqs=64, max_pps=None, seed=1234):
        from gadeon_b200 import BlockPool
        self.torch, self.O = torch, O
        self.kvh, self.dh, self.P = kvh, dh, P
        max_pps = max_pps or num_pages
        self.gpu = BlockPool(kvh, dh, P, num_pages, max_seqs, max_pps, seed=seed)
        self.orc = O.OraclePool(kvh, dh, P, num_pages, seed)
        self.seqs = []
        self.stream = 0

    def new_seq(self):
        a = self.gpu.seq_create()
        b = self.orc.seq_create()
        assert a == b
        self.seqs.append(a)
        return a

    def rows(self, n, stream=None):
        s = self.stream if stream is None else stream
        self.stream += 1
        return self.O.normal_f16(99, s, (n, self.kvh, self.dh)), self.O.normal_f16(98, s, (n, self.kvh, self.dh))

    def append(self, ids, n_new):
        n = int(np.sum(n_new))
        k, v = self.rows(n)
        self.gpu.append(ids, n_new, dev_f16(self.torch, k), dev_f16(self.torch, v))
        assert self.orc.append(ids, n_new, k, v) == 0

    def seed(self, sid, count):
        K = self.O.normal_f16(7, self.stream, (self.kvh, count, self.dh))
        V = self.O.normal_f16(8, self.stream, (self.kvh, count, self.dh))
        self.stream += 1
        self.gpu.seed(sid, dev_f16(self.torch, K), dev_f16(self.torch, V), count)
        assert self.orc.seed(sid, K, V, count) == 0

    def truncate(self, ids, new_len):
        self.gpu.truncate(ids, new_len)
        assert self.orc.truncate(ids, new_len) == 0

    def check_state(self, pages=True):
        assert np.array_equal(self.gpu.export_free_list(), self.orc.free_list())
        for s in self.seqs:
            assert self.gpu.length(s) == self.orc.length(s)
            t = self.gpu.export_table(s)
            assert np.array_equal(t, self.orc.pages(s)), f"table of seq {s}"
            if pages:
                for pid in t:
                    gk, gv = self.gpu.export_page(int(pid))
                    ok, ov = self.orc.page_bytes(int(pid))
                    assert np.array_equal(gk, ok) and np.array_equal(gv, ov), f"page {pid}"
                    assert self.gpu.page_refcount(int(pid)) == self.orc.page_ref(int(pid))
        assert self.gpu.device_status() == 0

    def attend(self, ids, n_q, G, scale=None):
        scale = self.dh ** -0.5 if scale is None else scale
        q = self.O.normal_f16(55, self.stream, (len(ids), n_q, self.kvh * G, self.dh))
        self.stream += 1
        got = self.gpu.attend(ids, n_q, G, dev_f16(self.torch, q), scale=scale).cpu().numpy()
        want = self.orc.attend_causal(ids, n_q, q, G, scale, n_threads=8)
        return got, want


@pytest.mark.parametrize("P", [4, 8, 16, 32])
@pytest.mark.parametrize("dh", [256, 512])
def test_decode_small_pages(cuda, oracle, P, dh):
    """GemmaMetalKernelTests shape: T=40, nH=2, nKV=1, hd 256/512."""
    pr = Pair(cuda, oracle, kvh=1, dh=dh, P=P, num_pages=64)
    s = pr.new_seq()
    pr.append([s], [40])
    pr.check_state()
    got, want = pr.attend([s], 1, 2)
    assert_attn_close(got, want, f"P={P} dh={dh}")


@pytest.mark.parametrize("dh", [64, 128, 256, 512])
@pytest.mark.parametrize("G", [1, 4, 6, 8])
def test_decode_geometries(cuda, oracle, dh, G):
    pr = Pair(cuda, oracle, kvh=2, dh=dh, P=16, num_pages=400)
    ids = [pr.new_seq() for _ in range(5)]
    pr.append(ids, [1, 17, 64, 300, 1000])
    got, want = pr.attend(ids, 1, G)
    assert_attn_close(got, want, f"dh={dh} G={G}")


def test_config1_prefill_then_decode(cuda, oracle):
    """Config 1: B=1, nH=8, KVH=2, dh=256, P=16: a 512-token prefill append,
    then 128 decode steps of append-one + attend-all.  State is bit-exact
    after every step; outputs within tolerance at every step."""
    pr = Pair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=64, seed=20240611)
    s = pr.new_seq()
    pr.append([s], [512])
    pr.check_state()
    torch = cuda
    for step in range(128):
        k, v = pr.rows(1)
        q = oracle.normal_f16(5, step, (1, 1, 8, 256))
        got = pr.gpu.append_attend([s], 1, 4, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
        assert pr.orc.append([s], [1], k, v) == 0
        want = pr.orc.attend_causal([s], 1, q, 4, 256 ** -0.5)
        assert_attn_close(got.cpu().numpy(), want, f"decode step {step}")
        pr.check_state(pages=(step % 16 == 15))
    assert pr.gpu.length(s) == 640


@pytest.mark.parametrize("P,dh", [(8, 256), (16, 256), (16, 128), (64, 256), (128, 128)])
def test_fused_decode_append(cuda, oracle, P, dh):
    """gkv_append_attend with n_q = 1 writes the new rows inside the attend
    kernel: page contents, tables and free list stay bit-exact step after
    step, across fresh pages and pages larger than the key tile; a shared
    (cloned) tail page falls back to the two-kernel path."""
    torch = cuda
    G = 4
    pr = Pair(cuda, oracle, kvh=2, dh=dh, P=P, num_pages=600, seed=31)
    ids = [pr.new_seq() for _ in range(5)]
    pr.append(ids, [1, P - 1, P, 3 * P + 2, 700])
    for step in range(2 * P + 3):
        if step == 5:  # share a partial tail: the next append copies it first
            c = pr.gpu.clone(ids[3])
            assert pr.orc.clone(ids[3]) == c
            pr.seqs.append(c)
            ids.append(c)
        k, v = pr.rows(len(ids))
        q = oracle.normal_f16(17, step, (len(ids), 1, 2 * G, dh))
        got = pr.gpu.append_attend(ids, 1, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
        assert pr.orc.append(ids, [1] * len(ids), k, v) == 0
        want = pr.orc.attend_causal(ids, 1, q, G, dh ** -0.5)
        assert_attn_close(got.cpu().numpy(), want, f"fused step {step}")
        pr.check_state(pages=(step % 4 == 0 or step > 2 * P))


def test_batched_ragged_decode(cuda, oracle):
    """Config-2 shape (nH=8, KVH=2, dh=256, P=16) with ragged contexts that
    split across many CTAs (the partial-merge path) and tiny ones."""
    pr = Pair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=3000, seed=7)
    ctx = [1, 2, 15, 16, 17, 63, 64, 65, 1024, 4097, 9000, 20000]
    ids = [pr.new_seq() for _ in ctx]
    pr.append(ids, ctx)
    for step in range(3):
        pr.append(ids, [1] * len(ids))
        got, want = pr.attend(ids, 1, 4)
        assert_attn_close(got, want, f"ragged step {step}")
    pr.check_state(pages=False)


@pytest.mark.parametrize("P", [8, 16])
def test_mtp_verify_and_rollback(cuda, oracle, P):
    """Config 3 shape (16 q heads, 4 KV heads, dh=256) scaled down: each step
    appends 4 draft rows, attends them causally (16 query rows per kv head),
    truncates to len + accepted (accepted ~ U{0..4}); the free list and block
    tables stay bit-exact after every rollback."""
    rng = np.random.default_rng(3)
    pr = Pair(cuda, oracle, kvh=4, dh=256, P=P, num_pages=2000, seed=11)
    ids = [pr.new_seq() for _ in range(8)]
    pr.append(ids, list(rng.integers(100, 400, size=8)))
    for step in range(24):
        lens = [pr.gpu.length(s) for s in ids]
        pr.append(ids, [4] * len(ids))
        got, want = pr.attend(ids, 4, 4)
        assert_attn_close(got, want, f"verify step {step}")
        acc = rng.integers(0, 5, size=len(ids))
        pr.truncate(ids, [l + int(a) for l, a in zip(lens, acc)])
        pr.check_state(pages=(step % 8 == 7))


def test_seed_compact_roundtrip(cuda, oracle):
    pr = Pair(cuda, oracle, kvh=4, dh=128, P=16, num_pages=200)
    s = pr.new_seq()
    pr.seed(s, 100)
    pr.check_state()
    K, V = pr.gpu.compact(s)
    oK, oV = pr.orc.compact(s)
    assert np.array_equal(K.cpu().view(cuda.int16).numpy().view(np.uint16), oK)
    assert np.array_equal(V.cpu().view(cuda.int16).numpy().view(np.uint16), oV)
    t = pr.gpu.from_compact(K, V, 100)
    assert pr.orc.from_compact(oK, oV, 100) == t
    pr.seqs.append(t)
    pr.check_state()
    got, want = pr.attend([s, t], 1, 4)
    assert_attn_close(got, want, "seed/fromCompact")
    q1 = oracle.normal_f16(4, 4, (1, 1, 16, 128))
    same = pr.gpu.attend([s, t], 1, 4, dev_f16(cuda, np.concatenate([q1, q1]))).cpu().numpy()
    assert np.array_equal(same[0], same[1])  # identical pages, identical bits


def test_clone_mark_midpage_replay(cuda, oracle):
    """MetalSelfTest.checkMetalBookmark: mark mid-page (clone), decode a path,
    restore (clone the mark again), replay the same feed: identical outputs,
    and the mark's pages stay untouched (copy-on-write)."""
    torch = cuda
    pr = Pair(cuda, oracle, kvh=2, dh=256, P=4, num_pages=100)
    s = pr.new_seq()
    pr.append([s], [6])  # len 6: mid-page for P=4
    mark = pr.gpu.clone(s)
    assert pr.orc.clone(s) == mark
    pr.seqs.append(mark)
    pr.check_state()

    def path(seq, stream0):
        outs = []
        for i in range(5):
            k, v = pr.rows(1, stream=stream0 + i)
            q = oracle.normal_f16(77, stream0 + i, (1, 1, 4, 256))
            out = pr.gpu.append_attend([seq], 1, 2, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
            assert pr.orc.append([seq], [1], k, v) == 0
            want = pr.orc.attend_causal([seq], 1, q, 2, 256 ** -0.5)
            assert_attn_close(out.cpu().numpy(), want, "bookmark path")
            outs.append(out.cpu().numpy())
        return np.stack(outs)

    a = path(s, 1000)
    pr.gpu.seq_release(s)
    assert pr.orc.seq_release(s) == 0
    pr.seqs.remove(s)
    r = pr.gpu.clone(mark)  # restore(b): clone again so the mark stays reusable
    assert pr.orc.clone(mark) == r
    pr.seqs.append(r)
    b = path(r, 1000)
    assert np.array_equal(a, b)
    pr.check_state()


def test_cow_after_truncate_into_shared_page(cuda, oracle):
    """Truncating a clone into a shared full page and appending copies the
    page first, so the sequence it shares with is untouched."""
    pr = Pair(cuda, oracle, kvh=1, dh=64, P=8, num_pages=40)
    s = pr.new_seq()
    pr.append([s], [20])
    c = pr.gpu.clone(s)
    assert pr.orc.clone(s) == c
    pr.seqs.append(c)
    pr.truncate([c], [5])
    pr.append([c], [6])
    pr.check_state()
    got, want = pr.attend([s, c], 1, 1)
    assert_attn_close(got, want, "cow")


def test_pool_exhaustion_leaves_state(cuda, oracle):
    from gadeon_b200 import GKV_ERR_NO_PAGES, GkvError
    pr = Pair(cuda, oracle, kvh=2, dh=128, P=16, num_pages=10)
    a, b = pr.new_seq(), pr.new_seq()
    pr.append([a], [100])  # 7 pages
    k, v = pr.rows(80)
    with pytest.raises(GkvError) as ei:
        pr.gpu.append([a, b], [40, 40], dev_f16(cuda, k), dev_f16(cuda, v))
    assert ei.value.code == GKV_ERR_NO_PAGES
    assert pr.orc.append([a, b], [40, 40], k, v) == oracle.ORC_ERR_NO_PAGES
    pr.check_state()


def test_bad_arguments(cuda, oracle):
    from gadeon_b200 import GKV_ERR_BAD_SEQ, GKV_ERR_INVALID, GKV_ERR_UNSUPPORTED, GkvError
    pr = Pair(cuda, oracle, kvh=2, dh=128, P=16, num_pages=10)
    s = pr.new_seq()
    pr.append([s], [3])
    q = dev_f16(cuda, oracle.normal_f16(1, 1, (1, 4, 8, 128)))
    for call, code in [
        (lambda: pr.gpu.truncate([s], [4]), GKV_ERR_BAD_SEQ),
        (lambda: pr.gpu.truncate([99], [0]), GKV_ERR_BAD_SEQ),
        (lambda: pr.gpu.attend([s], 4, 4, q), GKV_ERR_BAD_SEQ),       # len 3 < n_q 4
        (lambda: pr.gpu.attend([s, s], 1, 4, q), GKV_ERR_INVALID),     # duplicate id
        (lambda: pr.gpu.attend([s], 1, 4, q, scale=0.0), GKV_ERR_INVALID),
    ]:
        with pytest.raises(GkvError) as ei:
            call()
        assert ei.value.code == code
    pr.check_state()
    # more than 16 rows per kv head needs the chunk kernel, which needs P >= 8
    small = Pair(cuda, oracle, kvh=2, dh=128, P=4, num_pages=10)
    t = small.new_seq()
    small.append([t], [5])
    q5 = dev_f16(cuda, oracle.normal_f16(1, 2, (1, 5, 8, 128)))
    with pytest.raises(GkvError) as ei:
        small.gpu.attend([t], 5, 4, q5)
    assert ei.value.code == GKV_ERR_UNSUPPORTED


def test_anti_vacuity_table_matters(cuda, oracle):
    """The output must depend on which pages the table points at: two
    sequences with different data give different outputs, and each matches
    the oracle (a kernel that ignored the table could not pass both)."""
    pr = Pair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=100)
    a, b = pr.new_seq(), pr.new_seq()
    pr.append([a, b], [200, 200])
    torch = cuda
    q1 = oracle.normal_f16(3, 3, (1, 1, 8, 256))
    qq = np.concatenate([q1, q1])
    got = pr.gpu.attend([a, b], 1, 4, dev_f16(torch, qq)).cpu().numpy()
    want = pr.orc.attend_causal([a, b], 1, qq, 4, 256 ** -0.5)
    assert_attn_close(got, want, "anti-vacuity")
    assert np.abs(got[0] - got[1]).max() > 1e-2


def test_pagepool_view_and_host_flash_decode(cuda, oracle):
    """The per-sequence PagePool view (PagedAttention.swift:21-287) and
    host_flash_decode (:317-366) driven like the Swift: an empty pool decodes
    to zeros (:323), then seed / append / clone / truncate, each followed by
    a decode against the oracle's hostFlashDecode restatement."""
    from gadeon_b200 import PagePool, host_flash_decode
    torch = cuda
    kvh, dh, P, G = 2, 256, 8, 4
    pr = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=64, seed=77)

    def decode(pool, oseq, stream):
        q = oracle.normal_f16(55, stream, (kvh, G, dh))
        got = host_flash_decode(dev_f16(torch, q), pool, G).cpu().numpy()
        want = pr.orc.flash_decode(oseq, q, G, dh ** -0.5).reshape(-1)
        assert_attn_close(got, want, f"host_flash_decode at length {pool.length}")

    a = PagePool(pr.gpu)
    assert a.seq_id == pr.orc.seq_create()
    assert (a.P, a.kv_heads, a.dh) == (P, kvh, dh)
    zero = host_flash_decode(dev_f16(torch, oracle.normal_f16(55, 0, (kvh, G, dh))), a, G)
    assert zero.shape == (kvh * G * dh,) and not bool(zero.any())
    K = oracle.normal_f16(3, 1, (kvh, 13, dh))
    V = oracle.normal_f16(3, 2, (kvh, 13, dh))
    a.seed(dev_f16(torch, K), dev_f16(torch, V), 13)
    assert pr.orc.seed(a.seq_id, K, V, 13) == 0
    decode(a, a.seq_id, 1)
    for t in range(5):  # 13 -> 18: across the page boundary at 16
        k, v = pr.rows(1)
        a.append(dev_f16(torch, k[0]), dev_f16(torch, v[0]))
        assert pr.orc.append([a.seq_id], [1], k, v) == 0
        decode(a, a.seq_id, 2 + t)
    assert a.length == 18 and a.page_count == 3
    b = a.clone()
    assert b.seq_id == pr.orc.clone(a.seq_id)
    a.truncate(9)
    pr.orc.truncate([a.seq_id], [9])
    pr.seqs += [a.seq_id, b.seq_id]
    pr.check_state()
    decode(a, a.seq_id, 10)
    decode(b, b.seq_id, 11)
    K2, V2 = b.compact()
    c = PagePool.from_compact(pr.gpu, K2, V2, b.length)
    oK, oV = pr.orc.compact(b.seq_id)
    assert c.seq_id == pr.orc.from_compact(oK, oV, b.length)
    pr.seqs.append(c.seq_id)
    pr.check_state()
    decode(c, c.seq_id, 12)


@pytest.mark.parametrize("tile_p", [4, 16, 32, 512])
def test_tile_at_carry_windows(cuda, oracle, tile_p):
    """tileAt (PagedAttention.swift:151-161) through gkv_tile_at, bit for bit
    against the oracle, over the windows pagedFlashCarry asks for
    (start = i*tile_p, count = min(tile_p, length - start), :466-481): tiles
    inside one page (4, 16) and spanning pages (32, 512), zero rows past the
    sequence; the pool is left as it was; bad windows are refused."""
    from gadeon_b200 import GKV_ERR_BAD_SEQ, GKV_ERR_INVALID, GkvError, PagePool
    pr = Pair(cuda, oracle, kvh=2, dh=128, P=16, num_pages=64, seed=21)
    s = pr.new_seq()
    pr.seed(s, 77)
    pr.append([s], [6])  # 83 positions over 6 pages, the last one partial
    n = pr.gpu.length(s)
    for start in range(0, n, tile_p):
        count = min(tile_p, n - start)
        gk_, gv = pr.gpu.tile_at(s, start, count, tile_p)
        ok, ov = pr.orc.tile_at(s, start, count, tile_p)
        as_u16 = lambda t: t.cpu().view(cuda.int16).numpy().view(np.uint16)
        assert np.array_equal(as_u16(gk_), ok) and np.array_equal(as_u16(gv), ov), (start, count)
    view = PagePool(pr.gpu, s)
    k2, _ = view.tile_at(5, 3, 8)
    assert np.array_equal(k2.cpu().view(cuda.int16).numpy().view(np.uint16), pr.orc.tile_at(s, 5, 3, 8)[0])
    # kPage / vPage (:80-81): the pages as stored, stale or zero rows included; floats32 (:46-62)
    for i, pid in enumerate(pr.orc.pages(s)):
        ok, ov = pr.orc.page_bytes(int(pid))
        assert np.array_equal(view.k_page(i), ok) and np.array_equal(view.v_page(i), ov)
    fk, fv = view.floats32()
    ck, cv = pr.orc.compact(s)
    assert np.array_equal(fk, oracle.f16_bits_to_f32(ck).reshape(2, -1))
    assert np.array_equal(fv, oracle.f16_bits_to_f32(cv).reshape(2, -1))
    for start, count, tp, code in [(n - 2, 3, 8, GKV_ERR_BAD_SEQ), (-1, 1, 8, GKV_ERR_BAD_SEQ),
                                   (0, 9, 8, GKV_ERR_INVALID), (0, 0, 0, GKV_ERR_INVALID)]:
        with pytest.raises(GkvError) as e:
            pr.gpu.tile_at(s, start, count, tp)
        assert e.value.code == code, (start, count, tp)
    cuda.cuda.synchronize()
    pr.check_state()


def test_snapshot_restore_twice(cuda, oracle):
    """MetalKVPool.snapshot / restore (MetalKVPool.swift:102-120) through the
    PagePool view: restore makes the live sequence a copy of the snapshot
    with its own tail, so appends after a restore leave the snapshot intact
    and it restores again to the same state; cache state bit-exact with the
    oracle doing clone + release, attention within tolerance."""
    from gadeon_b200 import PagePool
    pr = Pair(cuda, oracle, kvh=2, dh=128, P=16, num_pages=64, seed=33)
    s = pr.new_seq()
    pr.seed(s, 37)  # partial tail page
    live = PagePool(pr.gpu, s)
    snap = live.snapshot()
    assert snap.seq_id == pr.orc.clone(s)
    pr.seqs.append(snap.seq_id)
    for extra in (20, 5):
        pr.append([live.seq_id], [extra])
        pr.check_state()
        old = live.seq_id
        live.restore(snap)
        nid = pr.orc.clone(snap.seq_id)
        assert pr.orc.seq_release(old) == 0
        assert live.seq_id == nid
        pr.seqs = [x for x in pr.seqs if x != old] + [nid]
        assert live.length == 37
        pr.check_state()
        got, want = pr.attend([live.seq_id, snap.seq_id], 1, 4)
        assert_attn_close(got, want, f"after restore (+{extra})")
        q1 = oracle.normal_f16(6, extra, (1, 1, 8, 128))
        same = pr.gpu.attend([live.seq_id, snap.seq_id], 1, 4, dev_f16(cuda, np.concatenate([q1, q1])))
        same = same.cpu().numpy()
        assert np.array_equal(same[0], same[1])  # equal rows in the pages, equal bits out


@pytest.mark.parametrize("lens", [(11, 9), (4, 30)])
def test_shared_tail_copy_and_in_place_write_in_one_batch(cuda, oracle, lens):
    """Two sequences share one partially filled tail page and both append in
    the same batch: the first takes a copy-on-write copy of the whole page
    (PagePool.clone's duplicate, PagedAttention.swift:199-210), the last then
    owns the page and writes it in place.  The copy must hold the page as it
    was before that write, as the reference's sequential order gives it --
    (11, 9): the writer's slot is a valid row of the copier; (4, 30): only a
    stale row.  24 such pairs in one batch; state bit-exact, attention within
    tolerance."""
    P, G = 32, 2
    pr = Pair(cuda, oracle, kvh=2, dh=128, P=P, num_pages=400, max_seqs=96, seed=44)
    ids, new_len = [], []
    for _ in range(24):
        a = pr.new_seq()
        pr.seed(a, 40)  # a full first page and a partial second one
        b = pr.gpu.clone(a)
        assert pr.orc.clone(a) == b
        pr.seqs.append(b)
        ids += [a, b]
        new_len += list(lens)
    pr.truncate(ids, new_len)  # both back into the shared first page
    pr.check_state()
    for s in ids:
        assert pr.gpu.page_refcount(int(pr.gpu.export_table(s)[0])) == 2
    k, v = pr.rows(len(ids))
    q = oracle.normal_f16(45, lens[0], (len(ids), 1, 2 * G, 128))
    got = pr.gpu.append_attend(ids, 1, G, dev_f16(cuda, k), dev_f16(cuda, v), dev_f16(cuda, q)).cpu().numpy()
    assert pr.orc.append(ids, [1] * len(ids), k, v) == 0
    want = pr.orc.attend_causal(ids, 1, q, G, 128 ** -0.5)
    pr.check_state()
    assert_attn_close(got, want, f"shared tail {lens}")
    # fresh shared pairs, then a plain batched append of 3 rows each (with
    # lens (4, 30) the writer also crosses into a new page)
    batch, batch_len = [], []
    for _ in range(12):
        a = pr.new_seq()
        pr.seed(a, 40)
        b = pr.gpu.clone(a)
        assert pr.orc.clone(a) == b
        pr.seqs.append(b)
        batch += [a, b]
        batch_len += list(lens)
    pr.truncate(batch, batch_len)
    pr.append(batch, [3] * len(batch))
    pr.check_state()
    got, want = pr.attend(batch, 3, G)
    assert_attn_close(got, want, f"shared tail {lens}, 3-row append")
