"""Generate the golden fixtures in tests/golden/ from the CPU oracle.

The reference repository commits no golden vectors for the paged-KV path
(its MetalGolden writes them at run time only, LLM/src/Metal/MetalGolden.swift
:1-21), so these fixtures pin the oracle against regressions and give the GPU
tests fixed expected outputs.  Inputs come from a restatement of the
reference's deterministic test fill -- a hashed LCG over the index giving
floats in [-1, 1) (MetalSelfTest.fill, LLM/src/Metal/MetalSelfTest.swift:
10-21) -- cast to fp16 round-to-nearest-even.  Shapes follow the reference's
own paged-attention tests:

  metal_golden_p8   P=8,  T=40, nH=2, nKV=1, hd=256, scale 0.125
                    (MetalGolden attn_head cases, MetalGolden.swift:269-325)
  gemma_p32_hd512   P=32, T=40, nH=2, nKV=1, hd=512, scale 1.0
                    (GemmaMetalKernelTests.swift:205-271)
  verify_p16        KVH=4, G=4, 4 draft rows causal over 100 keys, P=16
  chunk_p16         KVH=2, G=4, a 48-row chunk over 92 prior keys, P=16
  rollback_p4       append / truncate / clone / append sequence on P=4 pages:
                    block tables and free list after every step

Run:  python tests/golden/make_golden.py   (rewrites tests/golden/*.npz)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

MASK64 = (1 << 64) - 1


def reference_fill(n: int, seed: int) -> np.ndarray:
    """Floats in [-1, 1): s = seed + 0x9E3779B97F4A7C15; per index
    s = s * 6364136223846793005 + 1442695040888963407 (mod 2^64);
    bits = (s >> 33) as uint32; value = float(bits) / float(2^32 - 1) * 2 - 1,
    in single precision."""
    out = np.empty(n, dtype=np.float32)
    s = (seed + 0x9E3779B97F4A7C15) & MASK64
    den = np.float32(4294967295.0)
    for i in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & MASK64
        bits = np.float32((s >> 33) & 0xFFFFFFFF)
        out[i] = bits / den * np.float32(2.0) - np.float32(1.0)
    return out


def f16(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float16).view(np.uint16)


def attend_case(name, kvh, G, dh, P, prior, n_q, scale, seed):
    num_pages = (prior + n_q + P - 1) // P + 8
    pool = O.OraclePool(kvh, dh, P, num_pages, seed)
    s = pool.seq_create()
    total = prior + n_q
    k = f16(reference_fill(total * kvh * dh, seed + 1)).reshape(total, kvh, dh)
    v = f16(reference_fill(total * kvh * dh, seed + 2)).reshape(total, kvh, dh)
    q = f16(reference_fill(n_q * kvh * G * dh, seed + 3)).reshape(1, n_q, kvh * G, dh)
    assert pool.append([s], [total], k, v) == 0
    out = pool.attend_causal([s], n_q, q, G, scale, n_threads=4)
    return dict(kind="attend", kvh=kvh, G=G, dh=dh, P=P, prior=prior, n_q=n_q, scale=np.float32(scale),
                seed=seed, num_pages=num_pages, k=k, v=v, q=q, out=out,
                table=pool.pages(s), free=pool.free_list())


def rollback_case(seed=77):
    kvh, dh, P, num_pages = 2, 64, 4, 24
    pool = O.OraclePool(kvh, dh, P, num_pages, seed)
    ops = []  # (op, args) replayed by the tests
    rows = f16(reference_fill(200 * kvh * dh, seed)).reshape(200, kvh, dh)
    used = 0
    a, b = pool.seq_create(), pool.seq_create()
    script = [("append", [a, b], [6, 9]), ("truncate", [a, b], [5, 2]), ("append", [b, a], [7, 3]),
              ("clone", a), ("truncate", [2], [3]), ("append", [2, a], [5, 1]), ("release", b),
              ("append", [a], [13])]
    tables, frees = [], []
    for op in script:
        if op[0] == "append":
            n = int(sum(op[2]))
            assert pool.append(op[1], op[2], rows[used:used + n], rows[used:used + n]) == 0
            used += n
        elif op[0] == "truncate":
            assert pool.truncate(op[1], op[2]) == 0
        elif op[0] == "clone":
            assert pool.clone(op[1]) == 2
        elif op[0] == "release":
            assert pool.seq_release(op[1]) == 0
        ops.append(repr(op))
        tables.append(repr({sid: pool.pages(sid).tolist() for sid in (0, 1, 2) if pool.length(sid) >= 0}))
        frees.append(pool.free_list())
    return dict(kind="rollback", kvh=kvh, dh=dh, P=P, num_pages=num_pages, seed=seed, rows=rows,
                ops=np.array(ops), tables=np.array(tables),
                frees=np.array([np.pad(f, (0, num_pages - len(f)), constant_values=-1) for f in frees]),
                nfree=np.array([len(f) for f in frees]))


CASES = {
    "metal_golden_p8": lambda: attend_case("metal_golden_p8", 1, 2, 256, 8, 39, 1, 0.125, 11),
    "gemma_p32_hd512": lambda: attend_case("gemma_p32_hd512", 1, 2, 512, 32, 39, 1, 1.0, 12),
    "verify_p16": lambda: attend_case("verify_p16", 4, 4, 256, 16, 96, 4, 0.0625, 13),
    "chunk_p16": lambda: attend_case("chunk_p16", 2, 4, 256, 16, 92, 48, 0.0625, 14),
    "rollback_p4": rollback_case,
}


def main():
    for name, fn in CASES.items():
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **fn())
        print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
