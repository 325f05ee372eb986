"""gkv_attend_noalloc: attention over caller-owned device memory that
allocates nothing.

It serves callers that may not call cudaMalloc while serving -- an engine
that reserves one device arena at start-up, or a language binding with its
own allocator -- so they keep K/V pages and block tables in their own
buffers.  Its scratch is a static device array inside the library.

This test owns all device memory itself (torch tensors standing in for the
caller's arena), calls the entry point through the C ABI twice in a row, and
checks each result against gkv_attend on a pool holding the same logical
K/V, within the parity tolerance of the other tests.  It lives in its own
file, collected last, so a failure here comes after every other test ran.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_attn_close

pytestmark = pytest.mark.gpu


def _noalloc(lib, torch, k_pages, v_pages, table, lens, n_q, G, q, out, scale):
    num_pages, kvh, P, dh = k_pages.shape
    L = np.ascontiguousarray(lens, dtype=np.int32)
    rc = lib.gkv_attend_noalloc(
        k_pages.data_ptr(), v_pages.data_ptr(), num_pages, kvh, dh, P,
        table.data_ptr(), table.shape[1], len(L), L.ctypes.data_as(C.POINTER(C.c_int32)),
        n_q, G, q.data_ptr(), out.data_ptr(), scale, torch.cuda.current_stream().cuda_stream)
    return rc


def test_noalloc_matches_pool_attend_two_calls(cuda):
    torch = cuda
    from gadeon_b200 import BlockPool, kv
    lib = kv.load_library()
    kvh, dh, P, G = 2, 256, 16, 4
    nH = kvh * G
    num_pages, stride = 700, 256
    lens = [37, 1024, 3001, 16, 2500, 4]
    gen = torch.Generator(device="cuda").manual_seed(1234)
    # the caller's own buffers: pages, block table (pages drawn from a permutation)
    k_pages = torch.randn((num_pages, kvh, P, dh), generator=gen, device="cuda", dtype=torch.float16)
    v_pages = torch.randn((num_pages, kvh, P, dh), generator=gen, device="cuda", dtype=torch.float16)
    perm = np.random.default_rng(5).permutation(num_pages).astype(np.int32)
    table_h = np.full((len(lens), stride), -1, dtype=np.int32)
    used = 0
    for i, n in enumerate(lens):
        npg = (n + P - 1) // P
        table_h[i, :npg] = perm[used:used + npg]
        used += npg
    table = torch.from_numpy(table_h).cuda()

    # the same logical K/V through the library's own pool and gkv_attend
    pool = BlockPool(kvh, dh, P, num_pages, len(lens) + 1, stride, seed=3)
    ids = []
    for i, n in enumerate(lens):
        pids = torch.from_numpy(table_h[i, :(n + P - 1) // P].astype(np.int64)).cuda()
        K = k_pages[pids].permute(1, 0, 2, 3).reshape(kvh, -1, dh)[:, :n].contiguous()
        V = v_pages[pids].permute(1, 0, 2, 3).reshape(kvh, -1, dh)[:, :n].contiguous()
        s = pool.seq_create()
        pool.seed(s, K, V, n)
        ids.append(s)

    for call, n_q in enumerate([1, 4]):  # decode, then an MTP-verify-shaped call
        q = torch.randn((len(lens), n_q, nH, dh), generator=gen, device="cuda", dtype=torch.float16)
        want = pool.attend(ids, n_q, G, q, scale=dh ** -0.5)
        out = torch.full((len(lens), n_q, nH, dh), float("nan"), device="cuda", dtype=torch.float32)
        rc = _noalloc(lib, torch, k_pages, v_pages, table, lens, n_q, G, q, out, dh ** -0.5)
        assert rc == 0, lib.gkv_last_error().decode()
        torch.cuda.synchronize()
        assert_attn_close(out.cpu().numpy(), want.cpu().numpy(), f"no-alloc call {call}")


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
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
    # within the sequence limit but more split-K scratch than the static array holds
    rc = _noalloc(lib, torch, k_pages, k_pages, table[:1000], [1] * 1000, 1, 4, q[:1000], out[:1000], 0.0625)
    assert rc == GKV_ERR_CAPACITY and b"scratch" in lib.gkv_last_error()
