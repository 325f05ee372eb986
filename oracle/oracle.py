"""ctypes wrapper over oracle/liboracle.so -- the CPU oracle for the paged
KV-cache path.

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's
``cpu_baseline`` / ``--impl reference`` legs import this module, as the
checker or as the timed CPU baseline.  The product (``gadeon_b200``) never
imports it.

The restated reference lines are cited in gkv_oracle.c's header:
``PagePool`` (LLM/src/CoreML/PagedAttention.swift:21-287) and
``hostFlashDecode`` (PagedAttention.swift:317-366), plus the explicit
block-pool / free-list model that the reference does not have.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

ORC_OK = 0
ORC_ERR_INVALID = 1
ORC_ERR_NO_PAGES = 2
ORC_ERR_BAD_SEQ = 4


def build() -> str:
    """Compile liboracle.so with gcc (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "gkv_oracle.c"))
    ):
        build()
    L = C.CDLL(_LIB_PATH)
    P = C.c_void_p
    i32p = C.POINTER(C.c_int32)
    i64p = C.POINTER(C.c_int64)
    u16p = C.POINTER(C.c_uint16)
    f32p = C.POINTER(C.c_float)
    sig = {
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
        "orc_fill_normal_f16": (None, [C.c_uint64, C.c_uint64, u16p, C.c_int64]),
        "orc_permutation": (None, [C.c_uint64, C.c_int32, i32p]),
        "orc_pool_create": (P, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64]),
        "orc_pool_destroy": (None, [P]),
        "orc_seq_create": (C.c_int, [P]),
        "orc_seq_release": (C.c_int, [P, C.c_int]),
        "orc_append": (C.c_int, [P, C.c_int, i32p, i32p, u16p, u16p]),
        "orc_seed": (C.c_int, [P, C.c_int, u16p, u16p, C.c_int64]),
        "orc_truncate": (C.c_int, [P, C.c_int, i32p, i64p]),
        "orc_clone": (C.c_int, [P, C.c_int]),
        "orc_compact": (C.c_int, [P, C.c_int, u16p, u16p]),
        "orc_tile_at": (C.c_int, [P, C.c_int, C.c_int64, C.c_int64, C.c_int, u16p, u16p]),
        "orc_from_compact": (C.c_int, [P, u16p, u16p, C.c_int64]),
        "orc_seq_length": (C.c_int64, [P, C.c_int]),
        "orc_seq_pages": (C.c_int32, [P, C.c_int, i32p]),
        "orc_free_list": (C.c_int32, [P, i32p]),
        "orc_page_ref": (C.c_int32, [P, C.c_int32]),
        "orc_page_k": (u16p, [P, C.c_int32]),
        "orc_page_v": (u16p, [P, C.c_int32]),
        "orc_flash_decode": (C.c_int, [P, C.c_int, u16p, C.c_int, C.c_float, f32p]),
        "orc_attend_causal": (
            C.c_int, [P, C.c_int, i32p, C.c_int, u16p, C.c_int, C.c_float, f32p, C.c_int]),
        "orc_attend_rows": (
            C.c_int, [P, C.c_int, i32p, C.c_int, i32p, C.c_int, u16p, C.c_int, C.c_float, f32p, C.c_int]),
        "orc_seq_drop_mirror": (C.c_int, [P, C.c_int]),
        "orc_mtp_rollback": (None, [C.c_int, i32p, C.c_int, C.c_int, C.c_int, C.c_int, f32p, f32p, f32p,
                                    f32p, f32p]),
        "orc_conv_rollback": (None, [C.c_int, i32p, C.c_int, C.c_int, C.c_int, f32p, f32p, f32p]),
        "orc_rmsnorm_rows": (None, [f32p, C.c_int, C.c_int, f32p, C.c_float]),
        "orc_rope_neox": (None, [f32p, C.c_int, C.c_int, C.c_int, f32p, f32p]),
        "orc_rope_table": (None, [C.c_int, C.c_float, C.c_int, i64p, f32p, f32p]),
        "orc_gate": (None, [f32p, f32p, C.c_int64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(C.POINTER(ct))


# ---------------------------------------------------------------- helpers

def normal_f16(seed: int, stream: int, shape) -> np.ndarray:
    """N(0,1) draws as fp16 bit patterns (uint16): splitmix64 -> Box-Muller
    in double -> float -> fp16 round-to-nearest-even."""
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.uint16)
    lib().orc_fill_normal_f16(seed & (2**64 - 1), stream & (2**64 - 1), _ptr(out, C.c_uint16), n)
    return out.reshape(shape)


def permutation(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib().orc_permutation(seed & (2**64 - 1), n, _ptr(out, C.c_int32))
    return out


def f16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint16).view(np.float16).astype(np.float32)


class OraclePool:
    """The oracle's block pool for one attention layer: PagePool semantics per
    sequence over one physical pool with a seeded LIFO free list."""

    def __init__(self, kv_heads: int, head_dim: int, page_tokens: int, num_pages: int, seed: int):
        self.kv_heads, self.head_dim, self.P, self.num_pages = kv_heads, head_dim, page_tokens, num_pages
        self._h = lib().orc_pool_create(kv_heads, head_dim, page_tokens, num_pages, seed & (2**64 - 1))
        if not self._h:
            raise ValueError("orc_pool_create rejected the geometry")

    def close(self):
        if self._h:
            lib().orc_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- sequences
    def seq_create(self) -> int:
        return lib().orc_seq_create(self._h)

    def seq_release(self, seq: int) -> int:
        return lib().orc_seq_release(self._h, seq)

    def append(self, seq_ids, n_new, k: np.ndarray, v: np.ndarray) -> int:
        ids = np.ascontiguousarray(seq_ids, dtype=np.int32)
        nn = np.ascontiguousarray(n_new, dtype=np.int32)
        k = np.ascontiguousarray(k, dtype=np.uint16)
        v = np.ascontiguousarray(v, dtype=np.uint16)
        return lib().orc_append(self._h, len(ids), _ptr(ids, C.c_int32), _ptr(nn, C.c_int32),
                                _ptr(k, C.c_uint16), _ptr(v, C.c_uint16))

    def seed(self, seq: int, K: np.ndarray, V: np.ndarray, count: int) -> int:
        K = np.ascontiguousarray(K, dtype=np.uint16)
        V = np.ascontiguousarray(V, dtype=np.uint16)
        return lib().orc_seed(self._h, seq, _ptr(K, C.c_uint16), _ptr(V, C.c_uint16), count)

    def truncate(self, seq_ids, new_len) -> int:
        ids = np.ascontiguousarray(seq_ids, dtype=np.int32)
        nl = np.ascontiguousarray(new_len, dtype=np.int64)
        return lib().orc_truncate(self._h, len(ids), _ptr(ids, C.c_int32), _ptr(nl, C.c_int64))

    def clone(self, seq: int) -> int:
        return lib().orc_clone(self._h, seq)

    def compact(self, seq: int):
        n = self.length(seq)
        K = np.zeros((self.kv_heads, n, self.head_dim), dtype=np.uint16)
        V = np.zeros_like(K)
        rc = lib().orc_compact(self._h, seq, _ptr(K, C.c_uint16), _ptr(V, C.c_uint16))
        if rc:
            raise ValueError(f"orc_compact rc={rc}")
        return K, V

    def tile_at(self, seq: int, start: int, count: int, tile_p: int):
        """PagePool.tileAt (PagedAttention.swift:151-161): (K, V) tiles
        [KVH, tile_p, dh], rows >= count zero; raises on a bad window."""
        K = np.zeros((self.kv_heads, tile_p, self.head_dim), dtype=np.uint16)
        V = np.zeros_like(K)
        rc = lib().orc_tile_at(self._h, seq, start, count, tile_p, _ptr(K, C.c_uint16), _ptr(V, C.c_uint16))
        if rc:
            raise ValueError(f"orc_tile_at rc={rc}")
        return K, V

    def from_compact(self, K: np.ndarray, V: np.ndarray, length: int) -> int:
        K = np.ascontiguousarray(K, dtype=np.uint16)
        V = np.ascontiguousarray(V, dtype=np.uint16)
        return lib().orc_from_compact(self._h, _ptr(K, C.c_uint16), _ptr(V, C.c_uint16), length)

    # -- state
    def length(self, seq: int) -> int:
        return int(lib().orc_seq_length(self._h, seq))

    def pages(self, seq: int) -> np.ndarray:
        n = lib().orc_seq_pages(self._h, seq, None)
        out = np.empty(max(n, 0), dtype=np.int32)
        if n > 0:
            lib().orc_seq_pages(self._h, seq, _ptr(out, C.c_int32))
        return out

    def free_list(self) -> np.ndarray:
        n = lib().orc_free_list(self._h, None)
        out = np.empty(n, dtype=np.int32)
        if n:
            lib().orc_free_list(self._h, _ptr(out, C.c_int32))
        return out

    def page_ref(self, pid: int) -> int:
        return int(lib().orc_page_ref(self._h, pid))

    def page_bytes(self, pid: int):
        """(K, V) of one physical page as uint16 [KVH, P, dh] copies."""
        n = self.kv_heads * self.P * self.head_dim
        kp = lib().orc_page_k(self._h, pid)
        vp = lib().orc_page_v(self._h, pid)
        K = np.ctypeslib.as_array(kp, shape=(n,)).copy().reshape(self.kv_heads, self.P, self.head_dim)
        V = np.ctypeslib.as_array(vp, shape=(n,)).copy().reshape(self.kv_heads, self.P, self.head_dim)
        return K, V

    # -- attention
    def flash_decode(self, seq: int, q: np.ndarray, G: int, scale: float) -> np.ndarray:
        """hostFlashDecode: q [KVH, G, dh] fp16 bits -> [KVH*G*dh] fp32."""
        q = np.ascontiguousarray(q, dtype=np.uint16)
        out = np.zeros(self.kv_heads * G * self.head_dim, dtype=np.float32)
        rc = lib().orc_flash_decode(self._h, seq, _ptr(q, C.c_uint16), G, scale, _ptr(out, C.c_float))
        if rc:
            raise ValueError(f"orc_flash_decode rc={rc}")
        return out

    def attend_causal(self, seq_ids, n_q: int, q: np.ndarray, G: int, scale: float,
                      n_threads: int = 1) -> np.ndarray:
        """q [n, n_q, KVH*G, dh] fp16 bits -> same shape fp32; row r of
        sequence b sees keys [0, len_b - n_q + r]."""
        ids = np.ascontiguousarray(seq_ids, dtype=np.int32)
        q = np.ascontiguousarray(q, dtype=np.uint16)
        out = np.zeros(q.shape, dtype=np.float32)
        rc = lib().orc_attend_causal(self._h, len(ids), _ptr(ids, C.c_int32), n_q,
                                     _ptr(q, C.c_uint16), G, scale, _ptr(out, C.c_float), n_threads)
        if rc:
            raise ValueError(f"orc_attend_causal rc={rc}")
        return out


    def attend_rows(self, seq_ids, n_q: int, rows, q: np.ndarray, G: int, scale: float,
                    n_threads: int = 1) -> np.ndarray:
        """attend_causal for chosen rows of each sequence's last n_q
        positions: q [n, len(rows), KVH*G, dh] fp16 bits (those rows only)
        -> same shape fp32; row rows[i] sees keys [0, len - n_q + rows[i]]."""
        ids = np.ascontiguousarray(seq_ids, dtype=np.int32)
        rr = np.ascontiguousarray(rows, dtype=np.int32)
        q = np.ascontiguousarray(q, dtype=np.uint16)
        out = np.zeros(q.shape, dtype=np.float32)
        rc = lib().orc_attend_rows(self._h, len(ids), _ptr(ids, C.c_int32), n_q, _ptr(rr, C.c_int32), len(rr),
                                   _ptr(q, C.c_uint16), G, scale, _ptr(out, C.c_float), n_threads)
        if rc:
            raise ValueError(f"orc_attend_rows rc={rc}")
        return out

    def drop_mirror(self, seq: int):
        """Free the sequence's fp32 mirror (host memory); results unchanged."""
        if lib().orc_seq_drop_mirror(self._h, seq):
            raise ValueError(f"unknown sequence {seq}")


def mtp_rollback(m, s0, delta, k, gcum) -> np.ndarray:
    """MtpRollback.stateAfter restated (gkv_oracle.c): s0 [n,H,DK,DV],
    delta [n,H,C,DV], k [n,H,C,DK], gcum [n,H,C] fp32; m per item."""
    s0 = np.ascontiguousarray(s0, dtype=np.float32)
    delta = np.ascontiguousarray(delta, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    gcum = np.ascontiguousarray(gcum, dtype=np.float32)
    n, H, DK, DV = s0.shape
    Cw = gcum.shape[-1]
    mm = np.ascontiguousarray(m, dtype=np.int32)
    out = np.empty_like(s0)
    lib().orc_mtp_rollback(n, _ptr(mm, C.c_int32), H, DK, DV, Cw, _ptr(s0, C.c_float), _ptr(delta, C.c_float),
                           _ptr(k, C.c_float), _ptr(gcum, C.c_float), _ptr(out, C.c_float))
    return out


def mtp_rollback_f16(m, s0_f16, delta, k, gcum) -> np.ndarray:
    """The reference's storage boundary around stateAfter
    (LLM/src/CoreML/Engine.swift:2697-2705): the fp16 state widened exactly
    (floats()), rebuilt in fp32, stored back rounded to nearest even
    (fp16Array).  s0_f16 / result: float16 [n,H,DK,DV]."""
    s0 = np.asarray(s0_f16, dtype=np.float16).astype(np.float32)
    return mtp_rollback(m, s0, delta, k, gcum).astype(np.float16)


def conv_rollback_f16(m, proj, pre_f16) -> np.ndarray:
    """convFromProj with the fp16 conv tail (Engine.swift:2719-2740: the pre
    tail read through floats(), each tap stored as Float16(val))."""
    pre = np.asarray(pre_f16, dtype=np.float16).astype(np.float32)
    return conv_rollback(m, proj, pre).astype(np.float16)


def conv_rollback(m, proj, pre) -> np.ndarray:
    """Engine.convFromProj restated: proj [n,C,CD], pre [n,CD,taps] -> [n,CD,taps]."""
    proj = np.ascontiguousarray(proj, dtype=np.float32)
    pre = np.ascontiguousarray(pre, dtype=np.float32)
    n, Cw, CD = proj.shape
    taps = pre.shape[-1]
    mm = np.ascontiguousarray(m, dtype=np.int32)
    out = np.empty_like(pre)
    lib().orc_conv_rollback(n, _ptr(mm, C.c_int32), CD, taps, Cw, _ptr(proj, C.c_float), _ptr(pre, C.c_float),
                            _ptr(out, C.c_float))
    return out


def rmsnorm_rows(x, w, eps) -> np.ndarray:
    """Kern.rmsnormRows restated: every row of the last axis normalised."""
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    w = np.ascontiguousarray(w, dtype=np.float32)
    d = x.shape[-1]
    lib().orc_rmsnorm_rows(_ptr(x, C.c_float), d, x.size // d, _ptr(w, C.c_float), float(eps))
    return x


def rope_neox(x, n_rot, cos_row, sin_row) -> np.ndarray:
    """Kern.ropeNeox restated with one token's cos / sin row; x [n_head, head_dim]."""
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    cs = np.ascontiguousarray(cos_row, dtype=np.float32)
    sn = np.ascontiguousarray(sin_row, dtype=np.float32)
    lib().orc_rope_neox(_ptr(x, C.c_float), x.shape[-1], x.size // x.shape[-1], int(n_rot), _ptr(cs, C.c_float),
                        _ptr(sn, C.c_float))
    return x


def rope_table(n_rot, base, positions):
    pos = np.ascontiguousarray(positions, dtype=np.int64)
    cs = np.empty((len(pos), n_rot // 2), dtype=np.float32)
    sn = np.empty_like(cs)
    lib().orc_rope_table(int(n_rot), float(base), len(pos), _ptr(pos, C.c_int64), _ptr(cs, C.c_float),
                         _ptr(sn, C.c_float))
    return cs, sn


def gate(x, g) -> np.ndarray:
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    g = np.ascontiguousarray(g, dtype=np.float32)
    lib().orc_gate(_ptr(x, C.c_float), _ptr(g, C.c_float), x.size)
    return x
