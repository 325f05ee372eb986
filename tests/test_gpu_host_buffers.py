"""Host buffers at the C ABI: page-locked memory in place, pageable memory staged.

The reference's callers hand the cache host arrays (hostFlashDecode takes q
and returns a [Float], LLM/src/CoreML/PagedAttention.swift:317-366).  Here q,
k, v and out of the hot-path calls may be page-locked host memory mapped into
the GPU's address space: the kernels read and write them in place over the
host link.  Results must equal those of the same calls with device buffers
bit for bit (same kernel, same arithmetic).  Pageable host memory -- which a
kernel cannot reach -- is staged by the library through the pool's device
memory, with the same results.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair, dev_f16

pytestmark = pytest.mark.gpu


def host_f16(torch, a):
    """uint16 fp16 bit patterns (numpy) -> page-locked torch.float16 CPU tensor."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.float16).pin_memory()


def test_pinned_host_buffers_match_device_buffers(cuda, oracle):
    """Two pools driven with the same calls, one with device buffers and one
    with page-locked host buffers: fused decode steps, a plain append, MTP
    verify rows and a chunk (tensor-core kernel) all agree bit for bit."""
    torch = cuda
    G, dh, P, kvh = 4, 256, 16, 2
    dev = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=400, seed=77)
    host = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=400, seed=77)
    ctx = [1, 15, 16, 33, 700, 1500]
    ids = [dev.new_seq() for _ in ctx]
    assert [host.new_seq() for _ in ctx] == ids
    # Host buffers stay referenced until the stream has finished with them:
    # torch's pinned-memory cache would hand a freed block to the next
    # pin_memory() while a kernel may still be reading it.
    k, v = dev.rows(sum(ctx))
    hk, hv = host_f16(torch, k), host_f16(torch, v)
    dev.gpu.append(ids, ctx, dev_f16(torch, k), dev_f16(torch, v))
    host.gpu.append(ids, ctx, hk, hv)
    torch.cuda.synchronize()
    assert dev.orc.append(ids, ctx, k, v) == 0
    assert host.orc.append(ids, ctx, k, v) == 0
    for step in range(20):  # crosses page boundaries: fresh pages in the fused path
        k, v = dev.rows(len(ids))
        q = oracle.normal_f16(61, step, (len(ids), 1, kvh * G, dh))
        got_d = dev.gpu.append_attend(ids, 1, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
        hk, hv, hq = host_f16(torch, k), host_f16(torch, v), host_f16(torch, q)
        got_h = host.gpu.append_attend(ids, 1, G, hk, hv, hq)
        torch.cuda.synchronize()
        assert not got_h.is_cuda and got_h.is_pinned()
        assert np.array_equal(got_d.cpu().numpy(), got_h.numpy()), f"step {step}"
        for pr in (dev, host):
            assert pr.orc.append(ids, [1] * len(ids), k, v) == 0
        want = dev.orc.attend_causal(ids, 1, q, G, dh ** -0.5)
        assert_attn_close(got_h.numpy(), want, f"host-buffer step {step}")
    for n_q in (4, 40):  # split-K verify rows, then the tcgen05 chunk kernel
        k, v = dev.rows(len(ids) * n_q)
        q = oracle.normal_f16(62, n_q, (len(ids), n_q, kvh * G, dh))
        out_h = torch.empty((len(ids), n_q, kvh * G, dh), dtype=torch.float32).pin_memory()
        got_d = dev.gpu.append_attend(ids, n_q, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
        hk, hv, hq = host_f16(torch, k), host_f16(torch, v), host_f16(torch, q)
        host.gpu.append_attend(ids, n_q, G, hk, hv, hq, out=out_h)
        torch.cuda.synchronize()
        assert np.array_equal(got_d.cpu().numpy(), out_h.numpy()), f"n_q={n_q}"
        for pr in (dev, host):
            assert pr.orc.append(ids, [n_q] * len(ids), k, v) == 0
        want = dev.orc.attend_causal(ids, n_q, q, G, dh ** -0.5)
        assert_attn_close(out_h.numpy(), want, f"host-buffer n_q={n_q}")
    dev.check_state()
    host.check_state()


def test_pageable_host_buffers_staged(cuda, oracle):
    """Plain (pageable) host arrays -- what a Swift [Float] or a numpy array
    is -- are staged by the library through a page-locked bounce buffer the
    pool owns: the call copies them in, the kernels read and write the
    bounce buffer in place, and the call returns with the output copied back
    in place.  Every hot-path call gives the same bits as with device
    buffers, and the cache state stays bit-exact."""
    import gadeon_b200 as gk
    torch = cuda
    G, dh, P, kvh = 4, 128, 16, 2
    nH = kvh * G
    dev = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=300, seed=5)
    host = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=300, seed=5)
    ids = [dev.new_seq() for _ in range(4)]
    assert [host.new_seq() for _ in range(4)] == ids
    lib = gk.load_library()
    idarr = np.array(ids, dtype=np.int32)
    pid = idarr.ctypes.data_as(C.POINTER(C.c_int32))
    scale = C.c_float(dh ** -0.5)

    def pageable(a):  # a fresh, plain numpy copy (malloc'd memory)
        return np.array(a, copy=True, order="C")

    # gkv_append from pageable k/v (the C ABI, numpy pointers)
    ctx = np.array([5, 17, 300, 40], dtype=np.int32)
    k, v = dev.rows(int(ctx.sum()))
    dev.gpu.append(ids, ctx, dev_f16(torch, k), dev_f16(torch, v))
    kp, vp = pageable(k), pageable(v)
    assert lib.gkv_append(host.gpu._h, 4, pid, ctx.ctypes.data_as(C.POINTER(C.c_int32)), kp.ctypes.data,
                          vp.ctypes.data, None) == 0, lib.gkv_last_error()
    for pr in (dev, host):
        assert pr.orc.append(ids, ctx, k, v) == 0
    # decode steps and an MTP verify through gkv_append_attend with pageable
    # k/v/q/out: out holds the result when the call returns
    for step, n_q in enumerate([1, 1, 4, 1, 40]):
        k, v = dev.rows(4 * n_q)
        q = oracle.normal_f16(71, step, (4, n_q, nH, dh))
        want = dev.gpu.append_attend(ids, n_q, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
        kp, vp, qp = pageable(k), pageable(v), pageable(q)
        outp = np.full((4, n_q, nH, dh), np.nan, dtype=np.float32)
        rc = lib.gkv_append_attend(host.gpu._h, 4, pid, n_q, G, kp.ctypes.data, vp.ctypes.data, qp.ctypes.data,
                                   outp.ctypes.data, scale, None)
        assert rc == 0, lib.gkv_last_error()
        assert np.array_equal(outp, want.cpu().numpy()), f"step {step}"
        for pr in (dev, host):
            assert pr.orc.append(ids, [n_q] * 4, k, v) == 0
    # gkv_attend: pageable q, device out; then device q, pageable out
    q = oracle.normal_f16(72, 0, (4, 1, nH, dh))
    want = dev.gpu.attend(ids, 1, G, dev_f16(torch, q)).cpu().numpy()
    outd = torch.empty((4, 1, nH, dh), dtype=torch.float32, device="cuda")
    qp = pageable(q)
    assert lib.gkv_attend(host.gpu._h, 4, pid, 1, G, qp.ctypes.data, outd.data_ptr(), scale, None) == 0
    assert np.array_equal(outd.cpu().numpy(), want)
    outp = np.zeros((4, 1, nH, dh), dtype=np.float32)
    assert lib.gkv_attend(host.gpu._h, 4, pid, 1, G, dev_f16(torch, q).data_ptr(), outp.ctypes.data, scale,
                          None) == 0
    assert np.array_equal(outp, want)
    # compact and tileAt into pageable buffers, fromCompact from them
    n = host.gpu.length(ids[2])
    Kp = np.zeros((kvh, n, dh), dtype=np.uint16)
    Vp = np.zeros_like(Kp)
    assert lib.gkv_compact_seq(host.gpu._h, ids[2], Kp.ctypes.data, Vp.ctypes.data, None) == 0
    oK, oV = host.orc.compact(ids[2])
    assert np.array_equal(Kp, oK) and np.array_equal(Vp, oV)
    Tk = np.full((kvh, 32, dh), 7, dtype=np.uint16)
    Tv = np.full_like(Tk, 7)
    assert lib.gkv_tile_at(host.gpu._h, ids[2], 16, 20, 32, Tk.ctypes.data, Tv.ctypes.data, None) == 0
    wk, wv = host.orc.tile_at(ids[2], 16, 20, 32)
    assert np.array_equal(Tk, wk) and np.array_equal(Tv, wv)
    new = C.c_int32(-1)
    assert lib.gkv_from_compact(host.gpu._h, Kp.ctypes.data, Vp.ctypes.data, n, C.byref(new), None) == 0
    assert host.orc.from_compact(oK, oV, n) == new.value
    host.seqs.append(new.value)
    # the Python layer passes plain CPU tensors through: the result comes back
    # as a plain CPU tensor
    q = oracle.normal_f16(73, 0, (4, 1, nH, dh))
    got = host.gpu.attend(ids, 1, G, torch.from_numpy(q.view(np.int16)).view(torch.float16))
    assert not got.is_cuda and not got.is_pinned()
    assert np.array_equal(got.numpy(), dev.gpu.attend(ids, 1, G, dev_f16(torch, q)).cpu().numpy())
    torch.cuda.synchronize()
    dev.check_state()
    host.check_state()


def test_pageable_megabyte_buffers(cuda, oracle):
    """Staged copies of a few MB (the bounce buffer grows to hold them): a
    6,000-row append from pageable k/v, a compact into pageable K/V, and a
    64-sequence decode with pageable q and out, each bit-exact against the
    oracle or the device-buffer call."""
    import gadeon_b200 as gk
    torch = cuda
    G, dh, P, kvh = 4, 256, 16, 2
    nH = kvh * G
    dev = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=2000, max_seqs=80, seed=9)
    host = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=2000, max_seqs=80, seed=9)
    ids = [dev.new_seq() for _ in range(64)]
    assert [host.new_seq() for _ in range(64)] == ids
    lib = gk.load_library()
    idarr = np.array(ids, dtype=np.int32)
    pid = idarr.ctypes.data_as(C.POINTER(C.c_int32))
    ctx = np.full(64, 8, dtype=np.int32)
    ctx[5] = 6000
    k, v = dev.rows(int(ctx.sum()))  # 6.4 MB each
    dev.gpu.append(ids, ctx, dev_f16(torch, k), dev_f16(torch, v))
    kp, vp = np.array(k, copy=True), np.array(v, copy=True)
    assert lib.gkv_append(host.gpu._h, 64, pid, ctx.ctypes.data_as(C.POINTER(C.c_int32)), kp.ctypes.data,
                          vp.ctypes.data, None) == 0, lib.gkv_last_error()
    for pr in (dev, host):
        assert pr.orc.append(ids, ctx, k, v) == 0
    Kp = np.zeros((kvh, 6000, dh), dtype=np.uint16)  # 6.1 MB each
    Vp = np.zeros_like(Kp)
    assert lib.gkv_compact_seq(host.gpu._h, ids[5], Kp.ctypes.data, Vp.ctypes.data, None) == 0
    oK, oV = host.orc.compact(ids[5])
    assert np.array_equal(Kp, oK) and np.array_equal(Vp, oV)
    q = oracle.normal_f16(74, 0, (64, 1, nH, dh))  # 256 KB in, 512 KB out
    want = dev.gpu.attend(ids, 1, G, dev_f16(torch, q)).cpu().numpy()
    qp = np.array(q, copy=True)
    outp = np.full((64, 1, nH, dh), np.nan, dtype=np.float32)
    assert lib.gkv_attend(host.gpu._h, 64, pid, 1, G, qp.ctypes.data, outp.ctypes.data,
                          C.c_float(dh ** -0.5), None) == 0, lib.gkv_last_error()
    assert np.array_equal(outp, want)
    torch.cuda.synchronize()
    dev.check_state(pages=False)
    host.check_state(pages=False)


def test_gdn_rollback_refuses_host_memory(cuda, oracle):
    """The GDN rollback kernels stream large state arrays and take device
    memory only: page-locked host memory is refused by the C ABI."""
    import gadeon_b200 as gk
    from gadeon_b200 import GKV_ERR_INVALID
    torch = cuda
    lib = gk.load_library()
    H, DK, DV, Cc = 1, 16, 16, 2
    m = np.array([1], dtype=np.int32)
    dev = [torch.zeros(n, dtype=torch.float32, device="cuda") for n in (DK * DV, Cc * DV, Cc * DK, Cc, DK * DV)]
    host_s0 = torch.zeros(DK * DV, dtype=torch.float32).pin_memory()
    args = [t.data_ptr() for t in dev]
    args[0] = host_s0.data_ptr()
    rc = lib.gkv_mtp_rollback(1, m.ctypes.data_as(C.POINTER(C.c_int32)), H, DK, DV, Cc, *args, None)
    assert rc == GKV_ERR_INVALID
    assert "host memory" in lib.gkv_last_error().decode()
