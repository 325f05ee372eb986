"""Golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py):
the CPU oracle must reproduce them, and the CUDA path must match them
(outputs within the parity tolerance, cache state bit-exact)."""
import ast
import os

import numpy as np
import pytest

from conftest import assert_attn_close

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ATTEND = ["metal_golden_p8", "gemma_p32_hd512", "verify_p16", "chunk_p16"]


def load(name):
    return dict(np.load(os.path.join(HERE, name + ".npz")))


def test_reference_fill_restatement():
    """The restated MetalSelfTest.fill against a direct big-integer evaluation."""
    import sys
    sys.path.insert(0, HERE)
    from make_golden import reference_fill
    seed = 5
    s = (seed + 0x9E3779B97F4A7C15) % 2**64
    want = []
    for _ in range(6):
        s = (s * 6364136223846793005 + 1442695040888963407) % 2**64
        want.append(np.float32(np.float32(s >> 33) / np.float32(2**32 - 1) * np.float32(2) - np.float32(1)))
    got = reference_fill(6, seed)
    assert np.array_equal(got, np.array(want, dtype=np.float32))
    assert (got >= -1).all() and (got < 1).all()


@pytest.mark.parametrize("name", ATTEND)
def test_oracle_reproduces_golden(oracle, name):
    g = load(name)
    kvh, G, dh, P = int(g["kvh"]), int(g["G"]), int(g["dh"]), int(g["P"])
    pool = oracle.OraclePool(kvh, dh, P, int(g["num_pages"]), int(g["seed"]))
    s = pool.seq_create()
    assert pool.append([s], [g["k"].shape[0]], g["k"], g["v"]) == 0
    out = pool.attend_causal([s], int(g["n_q"]), g["q"], G, float(g["scale"]), n_threads=2)
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-6)
    assert np.array_equal(pool.pages(s), g["table"])
    assert np.array_equal(pool.free_list(), g["free"])


def replay_rollback(pool, g, rows_to):
    """Replay the rollback script on an oracle or GPU pool; yield after each op."""
    rows = g["rows"]
    used = 0
    for op_s in g["ops"]:
        op = ast.literal_eval(str(op_s))
        if op[0] == "append":
            n = int(sum(op[2]))
            pool.append(op[1], op[2], rows_to(rows[used:used + n]), rows_to(rows[used:used + n]))
            used += n
        elif op[0] == "truncate":
            pool.truncate(op[1], op[2])
        elif op[0] == "clone":
            assert pool.clone(op[1]) == 2
        elif op[0] == "release":
            pool.seq_release(op[1])
        yield op


def test_oracle_reproduces_rollback_golden(oracle):
    g = load("rollback_p4")
    pool = oracle.OraclePool(int(g["kvh"]), int(g["dh"]), int(g["P"]), int(g["num_pages"]), int(g["seed"]))
    a, b = pool.seq_create(), pool.seq_create()
    for i, _ in enumerate(replay_rollback(pool, g, lambda x: x)):
        tables = {sid: pool.pages(sid).tolist() for sid in (0, 1, 2) if pool.length(sid) >= 0}
        assert repr(tables) == str(g["tables"][i])
        assert np.array_equal(pool.free_list(), g["frees"][i][: g["nfree"][i]])


@pytest.mark.gpu
@pytest.mark.parametrize("name", ATTEND)
def test_gpu_matches_golden(cuda, name):
    from gadeon_b200 import BlockPool
    from test_gpu_parity import dev_f16
    g = load(name)
    kvh, G, dh, P = int(g["kvh"]), int(g["G"]), int(g["dh"]), int(g["P"])
    pool = BlockPool(kvh, dh, P, int(g["num_pages"]), 2, int(g["num_pages"]), seed=int(g["seed"]))
    s = pool.seq_create()
    pool.append([s], [g["k"].shape[0]], dev_f16(cuda, g["k"]), dev_f16(cuda, g["v"]))
    out = pool.attend([s], int(g["n_q"]), G, dev_f16(cuda, g["q"]), scale=float(g["scale"]))
    assert_attn_close(out.cpu().numpy(), g["out"], name)
    assert np.array_equal(pool.export_table(s), g["table"])
    assert np.array_equal(pool.export_free_list(), g["free"])


@pytest.mark.gpu
def test_gpu_matches_rollback_golden(cuda):
    from gadeon_b200 import BlockPool
    from test_gpu_parity import dev_f16
    g = load("rollback_p4")
    n = int(g["num_pages"])
    pool = BlockPool(int(g["kvh"]), int(g["dh"]), int(g["P"]), n, 4, n, seed=int(g["seed"]))
    a, b = pool.seq_create(), pool.seq_create()
    for i, _ in enumerate(replay_rollback(pool, g, lambda x: dev_f16(cuda, x))):
        alive = [sid for sid in (0, 1, 2) if _alive(pool, sid)]
        tables = {sid: pool.export_table(sid).tolist() for sid in alive}
        assert repr(tables) == str(g["tables"][i])
        assert np.array_equal(pool.export_free_list(), g["frees"][i][: g["nfree"][i]])
    assert pool.device_status() == 0


def _alive(pool, sid):
    try:
        pool.length(sid)
        return True
    except Exception:
        return False
