"""The reference's own layouts at the boundary (gkv_attend_ex /
gkv_append_attend_ex): q and attention output as [KVH, S, G, dh] per
sequence, verifyAttn's k/v rows as [KVH, S, dh], and fp16 output
(Engine.verifyAttn, LLM/src/CoreML/Engine.swift:2618-2646;
pagedFlashBatched, LLM/src/CoreML/PagedAttention.swift:370-416).

The kernels write those layouts themselves; the arithmetic is the one of the
token-major fp32 path, so a head-major result equals the token-major one
moved, bit for bit, and an fp16 result equals the fp32 one rounded to
nearest even, bit for bit.  Every path is also checked against the oracle
within the attention tolerance, and cache state after a head-major append
is bit-exact.  Covered: the split-K decode / verify kernel (direct and
merge outputs), its fused append, the unfused append (pages < 8 tokens) and
the tensor-core chunk kernel."""
import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair, dev_f16

pytestmark = pytest.mark.gpu


def to_head_major(a, kvh, G):
    """[n, S, KVH*G, dh] -> [n, KVH, S, G, dh]."""
    n, S, nH, dh = a.shape
    return np.ascontiguousarray(a.reshape(n, S, kvh, G, dh).transpose(0, 2, 1, 3, 4))


def rows_head_major(a, n, S, kvh):
    """token-major rows [n*S, KVH, dh] -> [n, KVH, S, dh]."""
    dh = a.shape[-1]
    return np.ascontiguousarray(a.reshape(n, S, kvh, dh).transpose(0, 2, 1, 3))


def f16_of(a):
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def check_layouts(pr, ids, n_q, G, what):
    """One attend in all four (layout, out type) combinations on the same
    pool: bit-identical up to the move and the rounding; within tolerance
    of the oracle."""
    torch = pr.torch
    q = pr.O.normal_f16(77, pr.stream, (len(ids), n_q, pr.kvh * G, pr.dh))
    pr.stream += 1
    qh = to_head_major(q, pr.kvh, G)
    scale = pr.dh ** -0.5
    tm32 = pr.gpu.attend(ids, n_q, G, dev_f16(torch, q), scale=scale).cpu().numpy()
    tm16 = pr.gpu.attend(ids, n_q, G, dev_f16(torch, q), scale=scale, out_f16=True).cpu().numpy()
    hm32 = pr.gpu.attend(ids, n_q, G, dev_f16(torch, qh), scale=scale, head_major=True).cpu().numpy()
    hm16 = pr.gpu.attend(ids, n_q, G, dev_f16(torch, qh), scale=scale, head_major=True,
                         out_f16=True).cpu().numpy()
    want = pr.orc.attend_causal(ids, n_q, q, G, scale, n_threads=8)
    assert_attn_close(tm32, want, f"{what}: token-major fp32")
    assert np.array_equal(hm32, to_head_major(tm32, pr.kvh, G)), f"{what}: head-major != moved token-major"
    assert np.array_equal(tm16.view(np.uint16), f16_of(tm32).view(np.uint16)), f"{what}: fp16 != rounded fp32"
    assert np.array_equal(hm16.view(np.uint16), f16_of(hm32).view(np.uint16)), f"{what}: head-major fp16"
    assert_attn_close(hm16.astype(np.float32), to_head_major(want, pr.kvh, G), f"{what}: head-major fp16 vs oracle")


@pytest.mark.parametrize("dh", [128, 256])
def test_layouts_decode_and_verify(cuda, oracle, dh):
    """Split-K kernel: a few short sequences (direct output) and two long
    ones spread over many CTAs (the merge writes the output)."""
    pr = Pair(cuda, oracle, kvh=2, dh=dh, P=16, num_pages=5000)
    ids = [pr.new_seq() for _ in range(5)]
    pr.append(ids, [4, 40, 300, 25000, 30000])
    for n_q, G in ((1, 4), (4, 4), (2, 8)):
        check_layouts(pr, ids, n_q, G, f"dh={dh} n_q={n_q} G={G}")


def test_layouts_chunk_kernel(cuda, oracle):
    """More than 16 rows per kv head: the tensor-core chunk kernel, single
    CTAs and CTA pairs (two or more query blocks)."""
    pr = Pair(cuda, oracle, kvh=4, dh=256, P=16, num_pages=3000)
    ids = [pr.new_seq() for _ in range(3)]
    pr.append(ids, [700, 2100, 300])
    check_layouts(pr, ids, 32, 4, "one query block")
    check_layouts(pr, ids, 300, 4, "CTA pairs")


@pytest.mark.parametrize("P", [16, 4])
def test_verify_attn_reference_layout(cuda, oracle, P):
    """gkv_append_attend_ex with the reference's verifyAttn layout: k/v
    [n, KVH, S, dh], q and fp16 out [n, KVH, S, G, dh].  P=16 appends inside
    the attend launch (fused), P=4 through the append kernel; a twin pool
    driven token-major gives the same output bits, and both pools' state
    matches the oracle bit for bit."""
    torch = cuda
    kvh, dh, G, S = 4, 256, 4, 4
    hm = Pair(torch, oracle, kvh=kvh, dh=dh, P=P, num_pages=3000)
    tm = Pair(torch, oracle, kvh=kvh, dh=dh, P=P, num_pages=3000)
    ids = [hm.new_seq() for _ in range(6)]
    assert [tm.new_seq() for _ in range(6)] == ids
    lens = [3, 15, 16, 130, 1000, 2047]
    for pr in (hm, tm):
        pr.append(ids, lens)
    for step in range(3):
        k, v = hm.rows(len(ids) * S, stream=500 + step)
        q = oracle.normal_f16(501, step, (len(ids), S, kvh * G, dh))
        got = hm.gpu.append_attend(ids, S, G, dev_f16(torch, rows_head_major(k, len(ids), S, kvh)),
                                   dev_f16(torch, rows_head_major(v, len(ids), S, kvh)),
                                   dev_f16(torch, to_head_major(q, kvh, G)), head_major=True,
                                   out_f16=True).cpu().numpy()
        ref = tm.gpu.append_attend(ids, S, G, dev_f16(torch, k), dev_f16(torch, v),
                                   dev_f16(torch, q)).cpu().numpy()
        for pr in (hm, tm):
            assert pr.orc.append(ids, [S] * len(ids), k, v) == 0
        assert np.array_equal(got.view(np.uint16), f16_of(to_head_major(ref, kvh, G)).view(np.uint16)), step
        want = hm.orc.attend_causal(ids, S, q, G, dh ** -0.5, n_threads=8)
        assert_attn_close(got.astype(np.float32), to_head_major(want, kvh, G), f"P={P} verify step {step}")
        hm.check_state()
        tm.check_state()


def test_reference_shaped_calls(cuda, oracle):
    """verify_attn and paged_flash_batched (PagePool-level, the Swift's
    shapes) against the oracle's per-token route."""
    torch = cuda
    from gadeon_b200 import BlockPool, PagePool, paged_flash_batched, verify_attn
    kvh, dh, P, G = 2, 256, 16, 4
    bp = BlockPool(kvh, dh, P, 400, 4, 400, seed=9)
    orc = oracle.OraclePool(kvh, dh, P, 400, 9)
    pool = PagePool(bp)
    s = orc.seq_create()
    assert s == pool.seq_id
    K = oracle.normal_f16(61, 0, (kvh, 777, dh))
    V = oracle.normal_f16(61, 1, (kvh, 777, dh))
    pool.seed(dev_f16(torch, K), dev_f16(torch, V), 777)
    assert orc.seed(s, K, V, 777) == 0
    # verify of L = 5 rows: append + causal attend, fp16 [KVH, L, G, dh]
    L = 5
    k = oracle.normal_f16(62, 0, (L, kvh, dh))
    v = oracle.normal_f16(62, 1, (L, kvh, dh))
    q = oracle.normal_f16(62, 2, (1, L, kvh * G, dh))
    got = verify_attn(pool, dev_f16(torch, k.transpose(1, 0, 2)), dev_f16(torch, v.transpose(1, 0, 2)),
                      dev_f16(torch, to_head_major(q, kvh, G)[0]), G).cpu().numpy()
    assert got.shape == (kvh, L, G, dh) and got.dtype == np.float16
    assert orc.append([s], [L], k, v) == 0
    want = orc.attend_causal([s], L, q, G, dh ** -0.5)
    assert_attn_close(got.astype(np.float32), to_head_major(want, kvh, G)[0], "verify_attn")
    # pagedFlashBatched over a chunk of S = 64 rows appended first
    S = 64
    k = oracle.normal_f16(63, 0, (S, kvh, dh))
    v = oracle.normal_f16(63, 1, (S, kvh, dh))
    q = oracle.normal_f16(63, 2, (1, S, kvh * G, dh))
    p0 = pool.length
    bp.append([pool.seq_id], [S], dev_f16(torch, k), dev_f16(torch, v))
    assert orc.append([s], [S], k, v) == 0
    got = paged_flash_batched(dev_f16(torch, to_head_major(q, kvh, G)[0]), pool, p0, S, G).cpu().numpy()
    assert got.shape == (kvh, S, G, dh) and got.dtype == np.float32
    want = orc.attend_causal([s], S, q, G, dh ** -0.5, n_threads=8)
    assert_attn_close(got, to_head_major(want, kvh, G)[0], "paged_flash_batched")


def test_named_entry_points_equal_gkv_attend(cuda, oracle):
    """gkv_attend_decode (n_q = 1) and gkv_attend_causal are gkv_attend under
    the names a caller binding the two forms separately uses: same bits."""
    import ctypes as C

    from gadeon_b200 import kv
    torch = cuda
    lib = kv.load_library()
    kvh, dh, G = 2, 256, 4
    pr = Pair(torch, oracle, kvh=kvh, dh=dh, P=16, num_pages=3000)
    ids = [pr.new_seq() for _ in range(4)]
    pr.append(ids, [90, 700, 2000, 5000])
    n = len(ids)
    cids = (C.c_int32 * n)(*ids)
    scale = dh ** -0.5
    for n_q in (1, 4, 64):
        q = dev_f16(torch, oracle.normal_f16(81, n_q, (n, n_q, kvh * G, dh)))
        ref = pr.gpu.attend(ids, n_q, G, q, scale=scale)
        got = torch.full_like(ref, float("nan"))
        if n_q == 1:
            rc = lib.gkv_attend_decode(pr.gpu._h, n, cids, G, q.data_ptr(), got.data_ptr(), scale, None)
            assert rc == 0, lib.gkv_last_error()
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int32), ref.view(torch.int32))
            got.fill_(float("nan"))
        rc = lib.gkv_attend_causal(pr.gpu._h, n, cids, n_q, G, q.data_ptr(), got.data_ptr(), scale, None)
        assert rc == 0, lib.gkv_last_error()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), ref.view(torch.int32)), n_q
