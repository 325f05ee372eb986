"""Host buffers at the C ABI: page-locked memory in place, pageable memory refused.

The reference's callers hand the cache host arrays (hostFlashDecode takes q
and returns a [Float], LLM/src/CoreML/PagedAttention.swift:317-366).  Here q,
k, v and out of the hot-path calls may be page-locked host memory mapped into
the GPU's address space: the kernels read and write them in place over the
host link.  Results must equal those of the same calls with device buffers
bit for bit (same kernel, same arithmetic), and pageable host memory -- which
a kernel cannot reach -- must be refused before anything is launched or the
pool changes.
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


def test_pageable_host_memory_refused(cuda, oracle):
    """Pointers into plain (pageable) host memory are refused with
    GKV_ERR_INVALID by the C ABI itself, before any launch: lengths, tables,
    free list and pages stay as they were."""
    import gadeon_b200 as gk
    from gadeon_b200 import GKV_ERR_INVALID, GkvError
    torch = cuda
    G, dh, kvh = 4, 128, 2
    pr = Pair(cuda, oracle, kvh=kvh, dh=dh, P=16, num_pages=40, seed=3)
    s = pr.new_seq()
    pr.append([s], [20])
    torch.cuda.synchronize()
    lib = gk.load_library()
    ids = np.array([s], dtype=np.int32)
    pid = ids.ctypes.data_as(C.POINTER(C.c_int32))
    # 16-byte aligned pageable buffers
    q = np.zeros(kvh * G * dh + 64, dtype=np.float16)
    kv = np.zeros(kvh * dh + 64, dtype=np.float16)
    out = np.zeros(kvh * G * dh + 64, dtype=np.float32)

    def aligned(a):
        p = a.ctypes.data
        return p + (-p) % 16

    qd = dev_f16(torch, oracle.normal_f16(1, 1, (1, 1, kvh * G, dh)))
    outd = torch.empty((1, 1, kvh * G, dh), dtype=torch.float32, device="cuda")
    one = np.array([1], dtype=np.int32)
    calls = [
        lambda: lib.gkv_attend(pr.gpu._h, 1, pid, 1, G, aligned(q), outd.data_ptr(), C.c_float(0.1), None),
        lambda: lib.gkv_attend(pr.gpu._h, 1, pid, 1, G, qd.data_ptr(), aligned(out), C.c_float(0.1), None),
        lambda: lib.gkv_append_attend(pr.gpu._h, 1, pid, 1, G, aligned(kv), aligned(kv), qd.data_ptr(),
                                      outd.data_ptr(), C.c_float(0.1), None),
        lambda: lib.gkv_append(pr.gpu._h, 1, pid, one.ctypes.data_as(C.POINTER(C.c_int32)), aligned(kv),
                               aligned(kv), None),
    ]
    for call in calls:
        assert call() == GKV_ERR_INVALID
        assert "pageable" in lib.gkv_last_error().decode()
    # the Python layer refuses an unpinned CPU tensor too
    with pytest.raises(GkvError) as ei:
        pr.gpu.attend([s], 1, G, torch.zeros((1, 1, kvh * G, dh), dtype=torch.float16))
    assert ei.value.code == GKV_ERR_INVALID
    torch.cuda.synchronize()
    assert pr.gpu.length(s) == 20
    pr.check_state()


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
