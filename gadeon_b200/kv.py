"""Python binding of libgadeonkv.so (include/gadeon_kv.h) over ctypes.

Two layers:

* :class:`BlockPool` -- one attention layer's physical page pool on one GPU
  (``gkv_pool``): batched append / attend / truncate / clone / compact over
  many sequences at once, the shape a batching server drives.
* :class:`PagePool` -- the reference's per-sequence cache object
  (leok7v/gadeon ``PagePool``, LLM/src/CoreML/PagedAttention.swift:21-287):
  ``append(k, v)``, ``seed``, ``truncate(to)``, ``clone()``, ``compact()``,
  ``from_compact``, ``tile_at``, ``k_page`` / ``v_page``, ``floats32``,
  ``length``, ``page_count``; and :func:`host_flash_decode`,
  the drop-in for ``hostFlashDecode(q:pool:G:)`` (:317-366).

Device tensors are torch CUDA tensors (torch is the device-memory and stream
plumbing); fp16 data is passed as ``torch.float16`` or as raw ``int16``/
``uint16`` bit patterns.  Failures raise :class:`GkvError`, the counterpart of
the reference's ``throws`` (allocation) and ``precondition`` (shape) paths.
There is no CPU fallback: without the built library or a GPU every call
fails loudly.
"""
from __future__ import annotations

import ctypes as C
import math
import os
from typing import Iterable, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgadeonkv.so")

GKV_OK = 0
GKV_ERR_INVALID = 1
GKV_ERR_NO_PAGES = 2
GKV_ERR_CUDA = 3
GKV_ERR_BAD_SEQ = 4
GKV_ERR_UNSUPPORTED = 5
GKV_ERR_CAPACITY = 6

# gkv_attend_ex / gkv_append_attend_ex flags
GKV_ATTEND_HEAD_MAJOR = 1  # q / out [n, kv_heads, n_q, group, head_dim]; k / v [n, kv_heads, n_q, head_dim]
GKV_ATTEND_OUT_F16 = 2     # out fp16, rounded to nearest even
GKV_ATTEND_P_F16 = 4       # chunk path: softmax weights rounded once to fp16 (the Metal attn_batch_mm arithmetic)

# Every entry point include/gadeon_kv.h declares.
EXPORTED = (
    "gkv_last_error", "gkv_version", "gkv_pool_create", "gkv_pool_destroy", "gkv_seq_create",
    "gkv_seq_release", "gkv_seq_length", "gkv_seq_page_count", "gkv_free_page_count",
    "gkv_append", "gkv_seed", "gkv_attend", "gkv_append_attend", "gkv_truncate",
    "gkv_clone_seq", "gkv_compact_seq", "gkv_from_compact", "gkv_export_table",
    "gkv_export_free_list", "gkv_page_refcount", "gkv_export_page", "gkv_device_status",
    "gkv_attend_noalloc", "gkv_mtp_rollback", "gkv_conv_rollback", "gkv_attn_step",
    "gkv_rope_table", "gkv_serialize", "gkv_deserialize", "gkv_state_header", "gkv_state_read_header",
    "gkv_rewind_append", "gkv_mtp_rollback_f16", "gkv_conv_rollback_f16", "gkv_check_bounded_wait",
    "gkv_tile_at", "gkv_gdn_rollback_f16", "gkv_gdn_rollback", "gkv_noalloc_status",
    "gkv_attend_ex", "gkv_append_attend_ex", "gkv_attend_decode", "gkv_attend_causal",
)


class GkvError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"gkv error {code}: {message}")
        self.code = code


class _PoolConfig(C.Structure):
    _fields_ = [
        ("device", C.c_int32), ("kv_heads", C.c_int32), ("head_dim", C.c_int32),
        ("page_tokens", C.c_int32), ("num_pages", C.c_int32), ("max_seqs", C.c_int32),
        ("max_pages_per_seq", C.c_int32), ("seed", C.c_uint64),
    ]


_lib = None


def load_library(path: str = LIB_PATH):
    """Load libgadeonkv.so and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is not built: run `python -m gadeon_b200.build`")
    L = C.CDLL(path)
    P = C.c_void_p
    i32, i64, f32 = C.c_int32, C.c_int64, C.c_float
    i32p, i64p = C.POINTER(C.c_int32), C.POINTER(C.c_int64)
    sig = {
        "gkv_last_error": (C.c_char_p, []),
        "gkv_version": (C.c_char_p, []),
        "gkv_pool_create": (C.c_int, [C.POINTER(_PoolConfig), C.POINTER(P)]),
        "gkv_pool_destroy": (C.c_int, [P]),
        "gkv_seq_create": (C.c_int, [P, i32p]),
        "gkv_seq_release": (C.c_int, [P, i32]),
        "gkv_seq_length": (C.c_int, [P, i32, i64p]),
        "gkv_seq_page_count": (C.c_int, [P, i32, i32p]),
        "gkv_free_page_count": (C.c_int, [P, i32p]),
        "gkv_append": (C.c_int, [P, i32, i32p, i32p, P, P, P]),
        "gkv_seed": (C.c_int, [P, i32, P, P, i64, P]),
        "gkv_attend": (C.c_int, [P, i32, i32p, i32, i32, P, P, f32, P]),
        "gkv_attend_decode": (C.c_int, [P, i32, i32p, i32, P, P, f32, P]),
        "gkv_attend_causal": (C.c_int, [P, i32, i32p, i32, i32, P, P, f32, P]),
        "gkv_append_attend": (C.c_int, [P, i32, i32p, i32, i32, P, P, P, P, f32, P]),
        "gkv_attend_ex": (C.c_int, [P, i32, i32p, i32, i32, P, P, f32, C.c_uint32, P]),
        "gkv_append_attend_ex": (C.c_int, [P, i32, i32p, i32, i32, P, P, P, P, f32, C.c_uint32, P]),
        "gkv_truncate": (C.c_int, [P, i32, i32p, i64p]),
        "gkv_rewind_append": (C.c_int, [P, i32, i32p, i64p, i32p, P, P, P]),
        "gkv_clone_seq": (C.c_int, [P, i32, i32p, P]),
        "gkv_compact_seq": (C.c_int, [P, i32, P, P, P]),
        "gkv_from_compact": (C.c_int, [P, P, P, i64, i32p, P]),
        "gkv_export_table": (C.c_int, [P, i32, i32p, i32, i32p]),
        "gkv_export_free_list": (C.c_int, [P, i32p, i32, i32p]),
        "gkv_page_refcount": (C.c_int, [P, i32, i32p]),
        "gkv_export_page": (C.c_int, [P, i32, P, P]),
        "gkv_device_status": (C.c_int, [P, i32p]),
        "gkv_attend_noalloc": (C.c_int, [P, P, i32, i32, i32, i32, P, i32, i32, i32p, i32, i32, P, P,
                                         f32, P]),
        "gkv_noalloc_status": (C.c_int, [P, i32p]),
        "gkv_mtp_rollback": (C.c_int, [i32, i32p, i32, i32, i32, i32, P, P, P, P, P, P]),
        "gkv_attn_step": (C.c_int, [P, i32, i32p, i32, P, P, P, P, P, f32, P, P, i32, f32, P, P]),
        "gkv_rope_table": (C.c_int, [i32, f32, i32, i64p, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
        "gkv_serialize": (C.c_int, [i32, C.POINTER(P), i32p, i32p, P, i64, i64p, P]),
        "gkv_deserialize": (C.c_int, [i32, C.POINTER(P), P, i64, i32p, i32p, i64p, P]),
        "gkv_state_header": (C.c_int, [P, i64, i64p]),
        "gkv_state_read_header": (C.c_int, [P, i64, i64p]),
        "gkv_conv_rollback": (C.c_int, [i32, i32p, i32, i32, i32, P, P, P, P]),
        "gkv_mtp_rollback_f16": (C.c_int, [i32, i32p, i32, i32, i32, i32, P, P, P, P, P, P]),
        "gkv_conv_rollback_f16": (C.c_int, [i32, i32p, i32, i32, i32, P, P, P, P]),
        "gkv_check_bounded_wait": (C.c_int, [i32, i64, i32p]),
        "gkv_tile_at": (C.c_int, [P, i32, i64, i64, i32, P, P, P]),
        "gkv_gdn_rollback_f16": (C.c_int, [i32, i32p, i32, i32, i32, i32, P, P, P, P, P, i32, i32, P, P, P, P]),
        "gkv_gdn_rollback": (C.c_int, [i32, i32p, i32, i32, i32, i32, P, P, P, P, P, i32, i32, P, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(rc: int):
    if rc != GKV_OK:
        raise GkvError(rc, _lib.gkv_last_error().decode())


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32).reshape(-1))


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64).reshape(-1))


def _p32(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def _p64(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_int64))


def _dev_ptr(t) -> Optional[int]:
    """Address of a contiguous torch tensor (or None): a CUDA tensor, a
    page-locked CPU tensor (``pin_memory()``), which the kernels read and
    write in place over the host link, or a plain CPU tensor, which the
    library stages through device memory (the call returns with its output
    in place).  The library checks each address again and refuses host
    memory where an argument must be device memory.  A page-locked buffer
    must stay referenced and unchanged until the stream has finished with
    it: torch's pinned-memory cache can hand a freed block to the next
    pin_memory() at once."""
    if t is None:
        return None
    if not t.is_cuda and t.device.type != "cpu":
        raise GkvError(GKV_ERR_INVALID, "tensor must live on the GPU or in host memory")
    if not t.is_contiguous():
        raise GkvError(GKV_ERR_INVALID, "tensor must be contiguous")
    return t.data_ptr()


def _gpu_ptr(t) -> Optional[int]:
    """Address of a contiguous CUDA tensor, for the entry points that take
    device memory only (the GDN rollback)."""
    if t is not None and not t.is_cuda:
        raise GkvError(GKV_ERR_INVALID, "tensor must live on the GPU (this call takes device memory only)")
    return _dev_ptr(t)


def _empty_f32(shape, like):
    """fp32 output beside `like`: on its GPU, or in host memory of its kind
    (page-locked or plain)."""
    import torch
    if like.is_cuda:
        return torch.empty(shape, dtype=torch.float32, device=like.device)
    out = torch.empty(shape, dtype=torch.float32)
    return out.pin_memory() if like.is_pinned() else out


def _check_shape(name, t, shape, dtypes):
    """The C ABI takes raw device pointers; refuse a tensor whose size or type
    differs from what the kernel will read or write."""
    if t is None:
        return
    if tuple(t.shape) != tuple(shape) and t.numel() != int(np.prod(shape)):
        raise GkvError(GKV_ERR_INVALID, f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
    if str(t.dtype).replace("torch.", "") not in dtypes:
        raise GkvError(GKV_ERR_INVALID, f"{name}: dtype {t.dtype}, expected one of {dtypes}")


_F16 = ("float16", "int16", "uint16")


def _stream_ptr(stream) -> Optional[int]:
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def _attend_flags(head_major: bool, out_f16: bool, p_f16: bool) -> int:
    return ((GKV_ATTEND_HEAD_MAJOR if head_major else 0) | (GKV_ATTEND_OUT_F16 if out_f16 else 0)
            | (GKV_ATTEND_P_F16 if p_f16 else 0))


class BlockPool:
    """One full-attention layer's page pool on one GPU (``gkv_pool``)."""

    def __init__(self, kv_heads: int, head_dim: int, page_tokens: int, num_pages: int,
                 max_seqs: int, max_pages_per_seq: int, seed: int = 0, device: int = 0):
        L = load_library()
        self.kv_heads, self.head_dim, self.page_tokens = kv_heads, head_dim, page_tokens
        self.num_pages, self.max_seqs, self.max_pages_per_seq = num_pages, max_seqs, max_pages_per_seq
        self.device = device
        cfg = _PoolConfig(device, kv_heads, head_dim, page_tokens, num_pages, max_seqs,
                          max_pages_per_seq, seed & (2**64 - 1))
        h = C.c_void_p()
        _check(L.gkv_pool_create(C.byref(cfg), C.byref(h)))
        self._h = h

    # ------------------------------------------------------------ lifetime
    def close(self):
        if getattr(self, "_h", None):
            _lib.gkv_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ------------------------------------------------------------ sequences
    def seq_create(self) -> int:
        out = C.c_int32()
        _check(_lib.gkv_seq_create(self._h, C.byref(out)))
        return out.value

    def seq_release(self, seq: int):
        _check(_lib.gkv_seq_release(self._h, seq))

    def length(self, seq: int) -> int:
        out = C.c_int64()
        _check(_lib.gkv_seq_length(self._h, seq, C.byref(out)))
        return out.value

    def page_count(self, seq: int) -> int:
        out = C.c_int32()
        _check(_lib.gkv_seq_page_count(self._h, seq, C.byref(out)))
        return out.value

    def free_page_count(self) -> int:
        out = C.c_int32()
        _check(_lib.gkv_free_page_count(self._h, C.byref(out)))
        return out.value

    # ------------------------------------------------------------ hot path
    def append(self, seq_ids: Sequence[int], n_new: Sequence[int], k, v, stream=None):
        """k, v: token-major [sum(n_new), kv_heads, head_dim] fp16 on the GPU."""
        ids, nn = _i32(seq_ids), _i32(n_new)
        rows = int(np.maximum(nn, 0).sum())
        for name, t in (("k", k), ("v", v)):
            _check_shape(name, t, (rows, self.kv_heads, self.head_dim), _F16)
        _check(_lib.gkv_append(self._h, len(ids), _p32(ids), _p32(nn), _dev_ptr(k), _dev_ptr(v),
                               _stream_ptr(stream)))

    def seed(self, seq: int, K, V, count: int, stream=None):
        """K, V: head-major [kv_heads, count, head_dim] fp16; the sequence must be empty."""
        for name, t in (("K", K), ("V", V)):
            _check_shape(name, t, (self.kv_heads, count, self.head_dim), _F16)
        _check(_lib.gkv_seed(self._h, seq, _dev_ptr(K), _dev_ptr(V), count, _stream_ptr(stream)))

    def _qo_shape(self, n: int, n_q: int, group: int, head_major: bool):
        if head_major:
            return (n, self.kv_heads, n_q, group, self.head_dim)
        return (n, n_q, self.kv_heads * group, self.head_dim)

    def _out(self, out, shape, q, out_f16: bool):
        import torch
        dt = torch.float16 if out_f16 else torch.float32
        if out is None:
            out = torch.empty(shape, dtype=dt, device=q.device)
            if not q.is_cuda and q.is_pinned():
                out = out.pin_memory()
        _check_shape("out", out, shape, ("float16",) if out_f16 else ("float32",))
        return out

    def attend(self, seq_ids: Sequence[int], n_q: int, group: int, q, out=None,
               scale: Optional[float] = None, stream=None, head_major: bool = False,
               out_f16: bool = False, p_f16: bool = False):
        """q: [n, n_q, kv_heads*group, head_dim] fp16 (head_major: the
        reference's [n, kv_heads, n_q, group, head_dim]); returns the result
        in q's layout, fp32 (out_f16: fp16).  Row r of a sequence sees keys
        [0, length - n_q + r].  p_f16: the chunk path (n_q * group > 16)
        rounds the softmax weights once to fp16 (GKV_ATTEND_P_F16)."""
        ids = _i32(seq_ids)
        qshape = self._qo_shape(len(ids), n_q, group, head_major)
        _check_shape("q", q, qshape, _F16)
        out = self._out(out, qshape, q, out_f16)
        if scale is None:
            scale = self.head_dim ** -0.5
        flags = _attend_flags(head_major, out_f16, p_f16)
        _check(_lib.gkv_attend_ex(self._h, len(ids), _p32(ids), n_q, group, _dev_ptr(q),
                                  _dev_ptr(out), float(scale), flags, _stream_ptr(stream)))
        return out

    def append_attend(self, seq_ids: Sequence[int], n_q: int, group: int, k, v, q, out=None,
                      scale: Optional[float] = None, stream=None, head_major: bool = False,
                      out_f16: bool = False, p_f16: bool = False):
        """Append n_q rows per sequence, then attend those n_q query rows.
        k, v: [n * n_q, kv_heads, head_dim] (head_major: [n, kv_heads, n_q,
        head_dim]); q / out as for :meth:`attend`."""
        ids = _i32(seq_ids)
        n = len(ids)
        qshape = self._qo_shape(n, n_q, group, head_major)
        _check_shape("q", q, qshape, _F16)
        kshape = (n, self.kv_heads, n_q, self.head_dim) if head_major else (n * n_q, self.kv_heads, self.head_dim)
        for name, t in (("k", k), ("v", v)):
            _check_shape(name, t, kshape, _F16)
        out = self._out(out, qshape, q, out_f16)
        if scale is None:
            scale = self.head_dim ** -0.5
        flags = _attend_flags(head_major, out_f16, p_f16)
        _check(_lib.gkv_append_attend_ex(self._h, n, _p32(ids), n_q, group, _dev_ptr(k),
                                         _dev_ptr(v), _dev_ptr(q), _dev_ptr(out), float(scale), flags,
                                         _stream_ptr(stream)))
        return out

    def attn_step(self, seq_ids: Sequence[int], group: int, q_gate, k_raw, v_raw, q_norm, k_norm,
                  rope_cos, rope_sin, eps: float = 1e-6, out=None, scale: Optional[float] = None,
                  stream=None):
        """One decode token from raw fp32 projections (``gkv_attn_step``,
        the reference's ``Attn.step``): q|gate split, q/k RMSNorm, partial
        NEOX RoPE (n_rot = 2 * rope_cos.shape[-1]), append, attend, sigmoid
        output gate.  Returns out [n_seqs, kv_heads*group, head_dim] fp32."""
        import torch
        ids = _i32(seq_ids)
        n, KVH, dh = len(ids), self.kv_heads, self.head_dim
        half = int(rope_cos.shape[-1])
        _check_shape("q_gate", q_gate, (n, KVH * group, 2 * dh), ("float32",))
        _check_shape("k_raw", k_raw, (n, KVH, dh), ("float32",))
        _check_shape("v_raw", v_raw, (n, KVH, dh), ("float32",))
        _check_shape("q_norm", q_norm, (dh,), ("float32",))
        _check_shape("k_norm", k_norm, (dh,), ("float32",))
        _check_shape("rope_cos", rope_cos, (n, half), ("float32",))
        _check_shape("rope_sin", rope_sin, (n, half), ("float32",))
        if out is None:
            out = _empty_f32((n, KVH * group, dh), q_gate)
        _check_shape("out", out, (n, KVH * group, dh), ("float32",))
        if scale is None:
            scale = dh ** -0.5
        _check(_lib.gkv_attn_step(self._h, n, _p32(ids), group, _dev_ptr(q_gate), _dev_ptr(k_raw),
                                  _dev_ptr(v_raw), _dev_ptr(q_norm), _dev_ptr(k_norm), float(eps),
                                  _dev_ptr(rope_cos), _dev_ptr(rope_sin), 2 * half, float(scale),
                                  _dev_ptr(out), _stream_ptr(stream)))
        return out

    def truncate(self, seq_ids: Sequence[int], new_len: Sequence[int]):
        ids, nl = _i32(seq_ids), _i64(new_len)
        _check(_lib.gkv_truncate(self._h, len(ids), _p32(ids), _p64(nl)))

    def rewind_append(self, seq_ids: Sequence[int], base_len: Sequence[int], n_new: Sequence[int], k, v,
                      stream=None):
        """Truncate each sequence to base_len[i], then append n_new[i] rows
        (the drafter pool's per-cycle maintenance) in one call."""
        ids, bl, nn = _i32(seq_ids), _i64(base_len), _i32(n_new)
        rows = int(nn.sum()) if len(nn) else 0
        for name, t in (("k", k), ("v", v)):
            _check_shape(name, t, (rows, self.kv_heads, self.head_dim), _F16)
        _check(_lib.gkv_rewind_append(self._h, len(ids), _p32(ids), _p64(bl), _p32(nn), _dev_ptr(k), _dev_ptr(v),
                                      _stream_ptr(stream)))

    def clone(self, seq: int, stream=None) -> int:
        out = C.c_int32()
        _check(_lib.gkv_clone_seq(self._h, seq, C.byref(out), _stream_ptr(stream)))
        return out.value

    def compact(self, seq: int, stream=None):
        """(K, V) head-major [kv_heads, length, head_dim] fp16 device tensors."""
        import torch
        n = self.length(seq)
        dev = torch.device("cuda", self.device)
        K = torch.empty((self.kv_heads, n, self.head_dim), dtype=torch.float16, device=dev)
        V = torch.empty_like(K)
        _check(_lib.gkv_compact_seq(self._h, seq, _dev_ptr(K), _dev_ptr(V), _stream_ptr(stream)))
        return K, V

    def tile_at(self, seq: int, start: int, count: int, tile_p: int, stream=None):
        """``gkv_tile_at``: positions [start, start + count) as head-major
        [kv_heads, tile_p, head_dim] fp16 K and V device tensors, rows
        count..tile_p-1 zero."""
        import torch
        dev = torch.device("cuda", self.device)
        K = torch.empty((self.kv_heads, tile_p, self.head_dim), dtype=torch.float16, device=dev)
        V = torch.empty_like(K)
        _check(_lib.gkv_tile_at(self._h, seq, start, count, tile_p, _dev_ptr(K), _dev_ptr(V), _stream_ptr(stream)))
        return K, V

    def from_compact(self, K, V, length: int, stream=None) -> int:
        for name, t in (("K", K), ("V", V)):
            _check_shape(name, t, (self.kv_heads, length, self.head_dim), _F16)
        out = C.c_int32()
        _check(_lib.gkv_from_compact(self._h, _dev_ptr(K), _dev_ptr(V), length, C.byref(out),
                                     _stream_ptr(stream)))
        return out.value

    # ------------------------------------------------------------ state export
    def export_table(self, seq: int) -> np.ndarray:
        n = C.c_int32()
        _check(_lib.gkv_export_table(self._h, seq, None, 0, C.byref(n)))
        out = np.empty(n.value, dtype=np.int32)
        if n.value:
            _check(_lib.gkv_export_table(self._h, seq, _p32(out), n.value, C.byref(n)))
        return out

    def export_free_list(self) -> np.ndarray:
        n = C.c_int32()
        _check(_lib.gkv_export_free_list(self._h, None, 0, C.byref(n)))
        out = np.empty(n.value, dtype=np.int32)
        if n.value:
            _check(_lib.gkv_export_free_list(self._h, _p32(out), n.value, C.byref(n)))
        return out

    def page_refcount(self, pid: int) -> int:
        out = C.c_int32()
        _check(_lib.gkv_page_refcount(self._h, pid, C.byref(out)))
        return out.value

    def export_page(self, pid: int):
        """(K, V) of one physical page as uint16 [kv_heads, P, head_dim]."""
        shape = (self.kv_heads, self.page_tokens, self.head_dim)
        K = np.empty(shape, dtype=np.uint16)
        V = np.empty(shape, dtype=np.uint16)
        _check(_lib.gkv_export_page(self._h, pid, K.ctypes.data, V.ctypes.data))
        return K, V

    def device_status(self) -> int:
        out = C.c_int32()
        _check(_lib.gkv_device_status(self._h, C.byref(out)))
        return out.value


class PagePool:
    """The reference's per-layer, per-sequence cache object
    (``PagePool``, PagedAttention.swift:21-287) as a view of one sequence of a
    :class:`BlockPool`.  ``P``, ``kv_heads`` and ``dh`` mirror ``P``,
    ``kvHeads`` and ``dh`` (:22-24)."""

    def __init__(self, block_pool: BlockPool, seq_id: Optional[int] = None):
        self.block_pool = block_pool
        self.seq_id = block_pool.seq_create() if seq_id is None else seq_id

    @property
    def P(self) -> int:
        return self.block_pool.page_tokens

    @property
    def kv_heads(self) -> int:
        return self.block_pool.kv_heads

    @property
    def dh(self) -> int:
        return self.block_pool.head_dim

    @property
    def length(self) -> int:
        return self.block_pool.length(self.seq_id)

    @property
    def page_count(self) -> int:
        return self.block_pool.page_count(self.seq_id)

    def append(self, k, v, stream=None):
        """One position's K and V, [kv_heads, head_dim] fp16 each (:85-94)."""
        self.block_pool.append([self.seq_id], [1], k, v, stream)

    def seed(self, K, V, count: int, stream=None):
        """[kv_heads, count, head_dim] fp16 into fresh pages (:99-112)."""
        self.block_pool.seed(self.seq_id, K, V, count, stream)

    def truncate(self, to: int):
        """truncate(to:) (:181-189)."""
        self.block_pool.truncate([self.seq_id], [to])

    def clone(self, stream=None) -> "PagePool":
        """clone() (:199-210): shares full pages, copies a partial tail."""
        return PagePool(self.block_pool, self.block_pool.clone(self.seq_id, stream))

    def snapshot(self, stream=None) -> "PagePool":
        """MetalKVPool.snapshot() (MetalKVPool.swift:102-109): a bookmark that
        shares the full pages and owns a copy of a partial tail -- clone()."""
        return self.clone(stream)

    def restore(self, snap: "PagePool", stream=None):
        """MetalKVPool.restore(_:) (:110-120): this sequence becomes a copy of
        the snapshot (shared full pages, its own tail copy), so the snapshot
        stays intact and may be restored again.  The sequence id changes."""
        if snap.block_pool is not self.block_pool:
            raise GkvError(GKV_ERR_INVALID, "restore: the snapshot belongs to another BlockPool")
        new_id = self.block_pool.clone(snap.seq_id, stream)
        self.block_pool.seq_release(self.seq_id)
        self.seq_id = new_id

    def compact(self, stream=None):
        """compact() (:225-252): (k, v) [kv_heads, length, head_dim] fp16."""
        return self.block_pool.compact(self.seq_id, stream)

    def tile_at(self, start: int, count: int, tile_p: int, stream=None):
        """tileAt(_:_:_:) (:151-161): (K, V) [kv_heads, tile_p, head_dim] fp16,
        positions [start, start + count), rows past count zero."""
        return self.block_pool.tile_at(self.seq_id, start, count, tile_p, stream)

    def k_page(self, i: int):
        """kPage(_:) (:80): page i of the sequence as stored, uint16
        [kv_heads, P, head_dim] on the host (rows past the length included,
        as the pool holds them).  Waits for the device."""
        return self._page(i)[0]

    def v_page(self, i: int):
        """vPage(_:) (:81), as k_page."""
        return self._page(i)[1]

    def _page(self, i: int):
        table = self.block_pool.export_table(self.seq_id)
        if not 0 <= i < len(table):
            raise GkvError(GKV_ERR_INVALID, f"page {i} of a sequence with {len(table)} pages")
        return self.block_pool.export_page(int(table[i]))

    def floats32(self, stream=None):
        """floats32() (:46-62): (k, v), per kv head the sequence's rows as
        fp32, [kv_heads, length * head_dim] (numpy, host)."""
        K, V = self.compact(stream)
        n = self.kv_heads
        return (K.float().reshape(n, -1).cpu().numpy(), V.float().reshape(n, -1).cpu().numpy())

    @staticmethod
    def from_compact(block_pool: BlockPool, k, v, length: int, stream=None) -> "PagePool":
        """fromCompact(k:v:length:P:kvHeads:dh:) (:256-264)."""
        return PagePool(block_pool, block_pool.from_compact(k, v, length, stream))

    def release(self):
        self.block_pool.seq_release(self.seq_id)


def host_flash_decode(q, pool: PagePool, G: int, stream=None):
    """``hostFlashDecode(q:pool:G:)`` (PagedAttention.swift:317-366) on the GPU:
    q [kv_heads, G, head_dim] fp16 -> [kv_heads*G*head_dim] fp32, the newest
    query attending every one of the pool's ``length`` keys with
    scale = head_dim^-0.5.  An empty pool gives zeros, as the Swift (:323)."""
    bp = pool.block_pool
    if pool.length == 0:
        import torch
        return torch.zeros(bp.kv_heads * G * bp.head_dim, dtype=torch.float32, device=q.device)
    qq = q.reshape(1, 1, bp.kv_heads * G, bp.head_dim)
    out = bp.attend([pool.seq_id], 1, G, qq, scale=bp.head_dim ** -0.5, stream=stream)
    return out.reshape(-1)


def paged_flash_batched(q, pool: PagePool, s0_global_pos: int, s_count: int, G: int, out=None,
                        stream=None, p_f16: bool = False):
    """``pagedFlashBatched(q:pool:tile:s0GlobalPos:sCount:G:)``
    (PagedAttention.swift:376-416) on the GPU: the S = s_count query rows
    q [kv_heads, S, G, head_dim] fp16 at global positions s0_global_pos + s,
    each seeing keys [0, s0_global_pos + s] of the pool (the band mask of
    :512-529), scale = head_dim^-0.5.  Returns the normalized
    [kv_heads, S, G, head_dim] fp32 result (the Swift returns it flat).  The
    rows must be the pool's last S positions (the chunk appended first, as
    Engine.batchedAttn does, Engine.swift:1797-1820).  p_f16: the softmax
    weights rounded once to fp16 on the tensor-core path (GKV_ATTEND_P_F16,
    the arithmetic of the Metal attn_batch_mm)."""
    bp = pool.block_pool
    if s0_global_pos + s_count != pool.length:
        raise GkvError(GKV_ERR_INVALID, f"rows {s0_global_pos}..{s0_global_pos + s_count - 1} are not the "
                       f"last {s_count} positions of a pool of length {pool.length}")
    qq = q.reshape(1, bp.kv_heads, s_count, G, bp.head_dim)
    if out is not None:
        out = out.reshape(1, bp.kv_heads, s_count, G, bp.head_dim)
    res = bp.attend([pool.seq_id], s_count, G, qq, out=out, scale=bp.head_dim ** -0.5, stream=stream,
                    head_major=True, p_f16=p_f16)
    return res.reshape(bp.kv_heads, s_count, G, bp.head_dim)


def verify_attn(pool: PagePool, k, v, q, G: int, out=None, stream=None):
    """``Engine.verifyAttn`` (LLM/src/CoreML/Engine.swift:2620-2646) on the
    GPU: append the L rows k, v [kv_heads, L, head_dim] fp16 to the pool and
    attend query row s of q [kv_heads, L, G, head_dim] over the pool so far
    (causal among the rows), scale = head_dim^-0.5, in one launch.  Returns
    attn_out [kv_heads, L, G, head_dim] fp16 (each value rounded to nearest
    even, as the Swift stores Float16)."""
    bp = pool.block_pool
    L = int(k.shape[1])
    kk = k.reshape(1, bp.kv_heads, L, bp.head_dim)
    vv = v.reshape(1, bp.kv_heads, L, bp.head_dim)
    qq = q.reshape(1, bp.kv_heads, L, G, bp.head_dim)
    if out is not None:
        out = out.reshape(1, bp.kv_heads, L, G, bp.head_dim)
    res = bp.append_attend([pool.seq_id], L, G, kk, vv, qq, out=out, scale=bp.head_dim ** -0.5,
                           stream=stream, head_major=True, out_f16=True)
    return res.reshape(bp.kv_heads, L, G, bp.head_dim)


def mtp_rollback(m, s0, delta, k, gcum, out=None, stream=None):
    """``MtpRollback.stateAfter`` (LLM/src/CoreML/MtpRollback.swift:47-60) on the
    GPU for a batch of items (sequence x GDN layer): s0 [n, H, DK, DV],
    delta [n, H, C, DV], k [n, H, C, DK], gcum [n, H, C] CUDA tensors,
    m = accepted prefix per item (1..C).  Returns S_m [n, H, DK, DV] in s0's
    dtype: fp32, or fp16 -- the reference's state storage
    (``gkv_mtp_rollback_f16``: widened, computed in fp32, rounded)."""
    import torch
    L = load_library()
    n, H, DK, DV = (int(x) for x in s0.shape)
    Cw = int(gcum.shape[-1])
    f16 = str(s0.dtype) == "torch.float16"
    _check_shape("s0", s0, (n, H, DK, DV), ("float16",) if f16 else ("float32",))
    _check_shape("delta", delta, (n, H, Cw, DV), ("float32",))
    _check_shape("k", k, (n, H, Cw, DK), ("float32",))
    _check_shape("gcum", gcum, (n, H, Cw), ("float32",))
    if out is None:
        out = torch.empty_like(s0)
    _check_shape("out", out, (n, H, DK, DV), ("float16",) if f16 else ("float32",))
    mm = _i32(m)
    if len(mm) != n:
        raise GkvError(GKV_ERR_INVALID, f"m has {len(mm)} entries for {n} items")
    fn = L.gkv_mtp_rollback_f16 if f16 else L.gkv_mtp_rollback
    _check(fn(n, _p32(mm), H, DK, DV, Cw, _gpu_ptr(s0), _gpu_ptr(delta), _gpu_ptr(k),
              _gpu_ptr(gcum), _gpu_ptr(out), _stream_ptr(stream)))
    return out


def conv_rollback(m, proj, pre, out=None, stream=None):
    """``Engine.convFromProj`` (LLM/src/CoreML/Engine.swift:2719-2740) on the GPU
    for a batch: proj [n, C, CD] fp32, pre [n, CD, taps] -> [n, CD, taps] in
    pre's dtype (fp32, or fp16 as the reference stores the conv tail)."""
    import torch
    L = load_library()
    n, Cw, CD = (int(x) for x in proj.shape)
    taps = int(pre.shape[-1])
    f16 = str(pre.dtype) == "torch.float16"
    dt = ("float16",) if f16 else ("float32",)
    _check_shape("proj", proj, (n, Cw, CD), ("float32",))
    _check_shape("pre", pre, (n, CD, taps), dt)
    if out is None:
        out = torch.empty_like(pre)
    _check_shape("out", out, (n, CD, taps), dt)
    mm = _i32(m)
    if len(mm) != n:
        raise GkvError(GKV_ERR_INVALID, f"m has {len(mm)} entries for {n} items")
    fn = L.gkv_conv_rollback_f16 if f16 else L.gkv_conv_rollback
    _check(fn(n, _p32(mm), CD, taps, Cw, _gpu_ptr(proj), _gpu_ptr(pre), _gpu_ptr(out), _stream_ptr(stream)))
    return out


def gdn_rollback(m, s0, delta, k, gcum, proj, pre, out=None, conv_out=None, stream=None):
    """``gkv_gdn_rollback_f16`` / ``gkv_gdn_rollback``: Engine.rollbackGDN
    (Engine.swift:2678-2716) for a batch in one launch -- :func:`mtp_rollback`
    of the state and :func:`conv_rollback` of the conv tail, the same items and
    m; fp16 storage (the reference's) or fp32, as s0 and pre are.
    Returns (state_out, conv_out)."""
    import torch
    L = load_library()
    n, H, DK, DV = (int(x) for x in s0.shape)
    Cw = int(gcum.shape[-1])
    CD, T = int(pre.shape[1]), int(pre.shape[2])
    sd = ("float16",) if str(s0.dtype) == "torch.float16" else ("float32",)
    _check_shape("s0", s0, (n, H, DK, DV), sd)
    _check_shape("delta", delta, (n, H, Cw, DV), ("float32",))
    _check_shape("k", k, (n, H, Cw, DK), ("float32",))
    _check_shape("gcum", gcum, (n, H, Cw), ("float32",))
    _check_shape("proj", proj, (n, Cw, CD), ("float32",))
    _check_shape("pre", pre, (n, CD, T), sd)
    if out is None:
        out = torch.empty_like(s0)
    if conv_out is None:
        conv_out = torch.empty_like(pre)
    _check_shape("out", out, (n, H, DK, DV), sd)
    _check_shape("conv_out", conv_out, (n, CD, T), sd)
    mm = _i32(m)
    if len(mm) != n:
        raise GkvError(GKV_ERR_INVALID, f"m has {len(mm)} entries for {n} items")
    fn = L.gkv_gdn_rollback_f16 if sd == ("float16",) else L.gkv_gdn_rollback
    _check(fn(n, _p32(mm), H, DK, DV, Cw, _gpu_ptr(s0), _gpu_ptr(delta), _gpu_ptr(k), _gpu_ptr(gcum), _gpu_ptr(out),
              CD, T, _gpu_ptr(proj), _gpu_ptr(pre), _gpu_ptr(conv_out), _stream_ptr(stream)))
    return out, conv_out


def check_bounded_wait(device: int = 0, limit_ns: int = 50_000_000) -> int:
    """``gkv_check_bounded_wait``: one device wait on a barrier nothing
    arrives on; returns the status bits it left (1 = the wait ran out and
    gave up, as designed)."""
    L = load_library()
    st = C.c_int32()
    _check(L.gkv_check_bounded_wait(int(device), int(limit_ns), C.byref(st)))
    return st.value


def rope_table(n_rot: int, base: float, positions) -> tuple:
    """``gkv_rope_table``: cos and sin tables [n, n_rot/2] (numpy fp32) for
    the given token positions, angle = pos * base^(-2i/n_rot) in fp32."""
    L = load_library()
    pos = _i64(positions)
    cos = np.empty((len(pos), n_rot // 2), dtype=np.float32)
    sin = np.empty_like(cos)
    _check(L.gkv_rope_table(n_rot, float(base), len(pos), _p64(pos),
                            cos.ctypes.data_as(C.POINTER(C.c_float)), sin.ctypes.data_as(C.POINTER(C.c_float))))
    return cos, sin


def serialize(pools: Sequence["BlockPool"], layer_ids: Sequence[int], seq_ids: Sequence[int], stream=None) -> bytes:
    """``gkv_serialize``: Engine.serialize's pool section for sequence
    seq_ids[i] of pools[i] under layer id layer_ids[i] (layers ascending)."""
    L = load_library()
    n = len(pools)
    hs = (C.c_void_p * n)(*[p._h.value for p in pools])
    lids, sids = _i32(layer_ids), _i32(seq_ids)
    size = C.c_int64()
    _check(L.gkv_serialize(n, hs, _p32(lids), _p32(sids), None, 0, C.byref(size), _stream_ptr(stream)))
    buf = (C.c_uint8 * size.value)()
    _check(L.gkv_serialize(n, hs, _p32(lids), _p32(sids), buf, size.value, C.byref(size), _stream_ptr(stream)))
    return bytes(buf)


def deserialize(pools: Sequence["BlockPool"], data: bytes, stream=None):
    """``gkv_deserialize``: rebuild each layer's sequence; returns
    (layer_ids, seq_ids, bytes consumed)."""
    L = load_library()
    n = len(pools)
    hs = (C.c_void_p * n)(*[p._h.value for p in pools])
    lids = np.zeros(n, dtype=np.int32)
    sids = np.zeros(n, dtype=np.int32)
    used = C.c_int64()
    raw = (C.c_uint8 * len(data)).from_buffer_copy(data) if data else (C.c_uint8 * 1)()
    _check(L.gkv_deserialize(n, hs, raw, len(data), _p32(lids), _p32(sids), C.byref(used), _stream_ptr(stream)))
    return lids.tolist(), sids.tolist(), used.value


def state_header() -> bytes:
    """``gkv_state_header``: the StateBytes "GDNS" v1 header (12 bytes)."""
    L = load_library()
    size = C.c_int64()
    buf = (C.c_uint8 * 12)()
    _check(L.gkv_state_header(buf, 12, C.byref(size)))
    return bytes(buf[: size.value])


def read_state_header(data: bytes) -> Optional[int]:
    """``gkv_state_read_header``: payload offset when data starts with the
    GDNS v1 header, else None."""
    L = load_library()
    off = C.c_int64()
    raw = (C.c_uint8 * max(1, len(data))).from_buffer_copy(data.ljust(1, b"\0"))
    rc = L.gkv_state_read_header(raw, len(data), C.byref(off))
    return off.value if rc == GKV_OK else None
