"""gkv_attend_noalloc: attention over caller-owned device memory that
allocates nothing.

It serves callers that may not call cudaMalloc while serving -- an engine
that reserves one device arena at start-up, or a language binding with its
own allocator -- so they keep K/V pages and block tables in their own
buffers.  Its scratch is a static device array inside the library, and its
device errors (a block-table entry outside the caller's pages) are read
back with gkv_noalloc_status.

The tests own all device memory themselves (torch tensors standing in for
the caller's arena), call the entry point through the C ABI, and check the
results against the CPU oracle loaded with the same K/V rows, and against
gkv_attend on a library pool holding them, within the parity tolerance of
the other tests.  This file is collected last, so a failure here comes
after every other test ran.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_attn_close

pytestmark = pytest.mark.gpu

DEV_ERR_BAD_PAGE = 2


def _noalloc(lib, torch, k_pages, v_pages, table, lens, n_q, G, q, out, scale):
    num_pages, kvh, P, dh = k_pages.shape
    L = np.ascontiguousarray(lens, dtype=np.int32)
    return lib.gkv_attend_noalloc(
        k_pages.data_ptr(), v_pages.data_ptr(), num_pages, kvh, dh, P,
        table.data_ptr(), table.shape[1], len(L), L.ctypes.data_as(C.POINTER(C.c_int32)),
        n_q, G, q.data_ptr(), out.data_ptr(), scale, torch.cuda.current_stream().cuda_stream)


def _status(lib, torch):
    st = C.c_int32(-1)
    rc = lib.gkv_noalloc_status(torch.cuda.current_stream().cuda_stream, C.byref(st))
    assert rc == 0, lib.gkv_last_error().decode()
    return st.value


class CallerArena:
    """The caller's own device buffers: K/V pages [num_pages, kvh, P, dh]
    fp16 and a block table whose rows point at pages drawn from a seeded
    permutation; the same rows (head-major [kvh, n, dh] per sequence) are
    kept on the host for the oracle."""

    def __init__(self, torch, O, kvh, dh, P, lens, stride, seed):
        self.kvh, self.dh, self.P, self.lens = kvh, dh, P, list(lens)
        npg = [(n + P - 1) // P for n in lens]
        self.num_pages = sum(npg) + 7
        perm = O.permutation(seed, self.num_pages)
        k_pages = np.zeros((self.num_pages, kvh, P, dh), dtype=np.uint16)
        v_pages = np.zeros_like(k_pages)
        self.table_h = np.full((len(lens), stride), -1, dtype=np.int32)
        self.K, self.V = [], []
        used = 0
        for i, n in enumerate(lens):
            K = O.normal_f16(seed, 1000 + 2 * i, (kvh, n, dh))
            V = O.normal_f16(seed, 1001 + 2 * i, (kvh, n, dh))
            self.K.append(K)
            self.V.append(V)
            pids = perm[used:used + npg[i]]
            used += npg[i]
            self.table_h[i, :npg[i]] = pids
            for src, dst in ((K, k_pages), (V, v_pages)):
                pad = np.zeros((kvh, npg[i] * P, dh), dtype=np.uint16)
                pad[:, :n] = src
                dst[pids] = pad.reshape(kvh, npg[i], P, dh).transpose(1, 0, 2, 3)
        dev = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.float16)
        self.k_pages, self.v_pages = dev(k_pages), dev(v_pages)
        self.table = torch.from_numpy(self.table_h).cuda()

    def oracle(self, O):
        orc = O.OraclePool(self.kvh, self.dh, self.P, self.num_pages + 8, seed=1)
        ids = []
        for K, V, n in zip(self.K, self.V, self.lens):
            s = orc.seq_create()
            assert orc.seed(s, K, V, n) == 0
            ids.append(s)
        return orc, ids

    def pool(self, torch):
        from gadeon_b200 import BlockPool
        pool = BlockPool(self.kvh, self.dh, self.P, self.num_pages + 8, len(self.lens) + 1,
                         self.table_h.shape[1], seed=3)
        ids = []
        for K, V, n in zip(self.K, self.V, self.lens):
            s = pool.seq_create()
            dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.float16)
            pool.seed(s, dev(K), dev(V), n)
            ids.append(s)
        return pool, ids


def test_noalloc_matches_oracle_and_pool_attend_two_calls(cuda, oracle):
    """Two calls in a row -- a decode, then an MTP-verify-shaped call of 4
    rows -- each checked against the oracle and against gkv_attend."""
    torch = cuda
    from gadeon_b200 import kv
    lib = kv.load_library()
    kvh, dh, P, G = 2, 256, 16, 4
    nH = kvh * G
    arena = CallerArena(torch, oracle, kvh, dh, P, [37, 1024, 3001, 16, 2500, 4, 700], 256, seed=11)
    orc, orc_ids = arena.oracle(oracle)
    pool, pool_ids = arena.pool(torch)
    n = len(arena.lens)
    _status(lib, torch)  # start from a clear status word
    for call, n_q in enumerate([1, 4]):
        q_h = oracle.normal_f16(12, call, (n, n_q, nH, dh))
        q = torch.from_numpy(q_h.view(np.int16)).cuda().view(torch.float16)
        out = torch.full((n, n_q, nH, dh), float("nan"), device="cuda", dtype=torch.float32)
        rc = _noalloc(lib, torch, arena.k_pages, arena.v_pages, arena.table, arena.lens, n_q, G, q, out,
                      dh ** -0.5)
        assert rc == 0, lib.gkv_last_error().decode()
        got = out.cpu().numpy()
        want = orc.attend_causal(orc_ids, n_q, q_h, G, dh ** -0.5, n_threads=8)
        assert_attn_close(got, want, f"no-alloc call {call} vs oracle")
        same = pool.attend(pool_ids, n_q, G, q, scale=dh ** -0.5).cpu().numpy()
        assert_attn_close(got, same, f"no-alloc call {call} vs gkv_attend")
    assert _status(lib, torch) == 0


def test_noalloc_batch_of_many_launches(cuda, oracle):
    """300 sequences: more than one launch's inline descriptor holds, so the
    batch runs as several launches sharing the array; every row checked."""
    torch = cuda
    from gadeon_b200 import kv
    lib = kv.load_library()
    kvh, dh, P, G = 4, 128, 16, 4
    nH = kvh * G
    lens = np.random.default_rng(3).integers(1, 600, 300).tolist()
    arena = CallerArena(torch, oracle, kvh, dh, P, lens, 40, seed=21)
    orc, orc_ids = arena.oracle(oracle)
    q_h = oracle.normal_f16(22, 0, (len(lens), 1, nH, dh))
    q = torch.from_numpy(q_h.view(np.int16)).cuda().view(torch.float16)
    for call in range(2):
        out = torch.full((len(lens), 1, nH, dh), float("nan"), device="cuda", dtype=torch.float32)
        rc = _noalloc(lib, torch, arena.k_pages, arena.v_pages, arena.table, lens, 1, G, q, out, dh ** -0.5)
        assert rc == 0, lib.gkv_last_error().decode()
        want = orc.attend_causal(orc_ids, 1, q_h, G, dh ** -0.5, n_threads=8)
        assert_attn_close(out.cpu().numpy(), want, f"300-sequence call {call}")


def test_noalloc_reports_a_bad_page_id(cuda, oracle):
    """A block-table entry outside the caller's pages is read as page 0 and
    reported by gkv_noalloc_status (then cleared); the other sequences'
    results are unaffected and nothing faults."""
    torch = cuda
    from gadeon_b200 import kv
    lib = kv.load_library()
    kvh, dh, P, G = 2, 256, 16, 4
    nH = kvh * G
    arena = CallerArena(torch, oracle, kvh, dh, P, [300, 500, 129], 64, seed=31)
    orc, orc_ids = arena.oracle(oracle)
    _status(lib, torch)
    bad = arena.table.clone()
    bad[1, 3] = arena.num_pages  # one past the last page
    q_h = oracle.normal_f16(32, 0, (3, 1, nH, dh))
    q = torch.from_numpy(q_h.view(np.int16)).cuda().view(torch.float16)
    out = torch.zeros((3, 1, nH, dh), device="cuda", dtype=torch.float32)
    rc = _noalloc(lib, torch, arena.k_pages, arena.v_pages, bad, arena.lens, 1, G, q, out, dh ** -0.5)
    assert rc == 0, lib.gkv_last_error().decode()
    assert _status(lib, torch) == DEV_ERR_BAD_PAGE
    assert _status(lib, torch) == 0  # read and cleared
    want = orc.attend_causal(orc_ids, 1, q_h, G, dh ** -0.5)
    got = out.cpu().numpy()
    assert_attn_close(got[[0, 2]], want[[0, 2]], "sequences with good tables")
    # the next call with a good table leaves the word clear
    rc = _noalloc(lib, torch, arena.k_pages, arena.v_pages, arena.table, arena.lens, 1, G, q, out, dh ** -0.5)
    assert rc == 0 and _status(lib, torch) == 0
    assert_attn_close(out.cpu().numpy(), want, "after the bad call")


def test_noalloc_leaves_free_device_memory_unchanged(cuda, oracle):
    """After a first call (which loads the kernel), further calls leave the
    device's free memory exactly as it was: the library allocates nothing."""
    torch = cuda
    from gadeon_b200 import kv
    lib = kv.load_library()
    kvh, dh, P, G = 2, 256, 16, 4
    arena = CallerArena(torch, oracle, kvh, dh, P, [100, 2000, 5000, 40] * 40, 320, seed=41)
    n = len(arena.lens)
    q = torch.zeros((n, 4, kvh * G, dh), device="cuda", dtype=torch.float16).normal_()
    out = torch.empty((n, 4, kvh * G, dh), device="cuda", dtype=torch.float32)
    for n_q in (1, 4):  # load every kernel the calls below use
        assert _noalloc(lib, torch, arena.k_pages, arena.v_pages, arena.table, arena.lens, n_q, G, q, out,
                        dh ** -0.5) == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for i in range(6):
        assert _noalloc(lib, torch, arena.k_pages, arena.v_pages, arena.table, arena.lens, 1 + 3 * (i % 2), G, q,
                        out, dh ** -0.5) == 0
    assert _status(lib, torch) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_sizes_beyond_its_limits(cuda):
    torch = cuda
    from gadeon_b200 import GKV_ERR_CAPACITY, kv
    lib = kv.load_library()
    kvh, dh, P = 4, 256, 16
    k_pages = torch.zeros((64, kvh, P, dh), device="cuda", dtype=torch.float16)
    table = torch.zeros((2048, 1), device="cuda", dtype=torch.int32)
    q = torch.zeros((2048, 1, kvh * 4, dh), device="cuda", dtype=torch.float16)
    out = torch.zeros((2048, 1, kvh * 4, dh), device="cuda", dtype=torch.float32)
    # more sequences than the documented limit
    rc = _noalloc(lib, torch, k_pages, k_pages, table, [1] * 2048, 1, 4, q, out, 0.0625)
    assert rc == GKV_ERR_CAPACITY and b"limit" in lib.gkv_last_error()
    # more kv heads than the documented limit
    wide = torch.zeros((1, 65, P, 64), device="cuda", dtype=torch.float16)
    rc = _noalloc(lib, torch, wide, wide, table[:1], [1], 1, 1, q, out, 0.125)
    assert rc == GKV_ERR_CAPACITY and b"kv_heads" in lib.gkv_last_error()
