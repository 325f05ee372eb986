"""The MTP drafter pool's cycle (Engine.decodeSpecStep,
LLM/src/CoreML/Engine.swift:2742-2812): n draft steps, each an append of one
row plus decode attention over the drafter pool (mtpForward, :2452-2475),
then mtpPool.truncate(to: mtpBase) and the m committed positions appended
again (:2788-2797) -- here one gkv_rewind_append.  State bit-exact against the
oracle's truncate + append after every cycle; draft outputs within the
attention tolerance."""
import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair, dev_f16

pytestmark = pytest.mark.gpu


def draft_step(pr, ids, G):
    """mtpForward's cache work for every sequence: append 1 row, attend it."""
    k, v = pr.rows(len(ids))
    q = pr.O.normal_f16(31, pr.stream, (len(ids), 1, pr.kvh * G, pr.dh))
    pr.stream += 1
    T = pr.torch
    got = pr.gpu.append_attend(ids, 1, G, dev_f16(T, k), dev_f16(T, v), dev_f16(T, q)).cpu().numpy()
    assert pr.orc.append(ids, [1] * len(ids), k, v) == 0
    want = pr.orc.attend_causal(ids, 1, q, G, pr.dh ** -0.5, n_threads=8)
    return got, want


def rewind_append(pr, ids, base, m):
    k, v = pr.rows(int(np.sum(m)))
    pr.gpu.rewind_append(ids, base, m, dev_f16(pr.torch, k), dev_f16(pr.torch, v))
    assert pr.orc.truncate(ids, base) == 0
    assert pr.orc.append(ids, m, k, v) == 0


@pytest.mark.parametrize("P", [8, 16])
def test_drafter_cycles(cuda, oracle, P):
    pr = Pair(cuda, oracle, kvh=4, dh=256, P=P, num_pages=2000 // P * 4, seed=5 + P)
    ids = [pr.new_seq() for _ in range(6)]
    pr.append(ids, [1, 14, 15, 16, 100, 257])
    rng = np.random.default_rng(P)
    n_draft, G = 3, 4
    for cycle in range(6):
        base = [pr.orc.length(s) for s in ids]
        for d in range(n_draft):
            got, want = draft_step(pr, ids, G)
            assert_attn_close(got, want, f"cycle {cycle} draft {d}")
        m = rng.integers(1, n_draft + 2, size=len(ids)).tolist()  # accepted + 1
        rewind_append(pr, ids, base, m)
        pr.check_state()
        assert [pr.gpu.length(s) for s in ids] == [b + x for b, x in zip(base, m)]


def test_rewind_append_matches_truncate_then_append(cuda, oracle):
    """Same seed, same calls: one pool takes gkv_rewind_append, the other
    gkv_truncate + gkv_append; tables, free lists and pages are identical."""
    from gadeon_b200 import BlockPool
    torch = cuda
    a = BlockPool(2, 128, 8, 300, 8, 200, seed=9)
    b = BlockPool(2, 128, 8, 300, 8, 200, seed=9)
    g = torch.Generator(device="cuda").manual_seed(0)
    ids = []
    for n in (40, 9, 64):
        k = torch.randn((n, 2, 128), generator=g, device="cuda", dtype=torch.float16)
        sa, sb = a.seq_create(), b.seq_create()
        a.append([sa], [n], k, k)
        b.append([sb], [n], k, k)
        ids.append(sa)
    for base, m in (([40, 9, 64], [3, 0, 7]), ([17, 9, 60], [1, 20, 5]), ([0, 1, 2], [8, 8, 8])):
        k = torch.randn((sum(m), 2, 128), generator=g, device="cuda", dtype=torch.float16)
        a.rewind_append(ids, base, m, k, k)
        b.truncate(ids, base)
        b.append(ids, m, k, k)
        assert np.array_equal(a.export_free_list(), b.export_free_list())
        for s in ids:
            assert np.array_equal(a.export_table(s), b.export_table(s))
            for pid in a.export_table(s):
                ka, va = a.export_page(int(pid))
                kb, vb = b.export_page(int(pid))
                assert np.array_equal(ka, kb) and np.array_equal(va, vb)


def test_rewind_append_refused_changes_nothing(cuda, oracle):
    import gadeon_b200 as gk
    pr = Pair(cuda, oracle, kvh=1, dh=256, P=16, num_pages=10, seed=3)
    ids = [pr.new_seq(), pr.new_seq()]
    pr.append(ids, [70, 60])  # 5 + 4 pages: one page free
    before = (pr.gpu.export_free_list().copy(), [pr.gpu.export_table(s).copy() for s in ids],
              [pr.gpu.length(s) for s in ids])
    k = cuda.zeros((80, 1, 256), dtype=cuda.float16, device="cuda")
    # rewinding seq 0 to 33 frees 2 pages (3 free); 80 new rows need 5 more pages
    with pytest.raises(gk.GkvError) as e:
        pr.gpu.rewind_append(ids, [33, 60], [40, 40], k, k)
    assert e.value.code == gk.GKV_ERR_NO_PAGES
    after = (pr.gpu.export_free_list(), [pr.gpu.export_table(s) for s in ids], [pr.gpu.length(s) for s in ids])
    assert np.array_equal(before[0], after[0])
    assert all(np.array_equal(x, y) for x, y in zip(before[1], after[1]))
    assert before[2] == after[2]
    pr.check_state()
    with pytest.raises(gk.GkvError) as e:
        pr.gpu.rewind_append(ids, [71, 60], [1, 1], k[:2], k[:2])  # base past the length
    assert e.value.code == gk.GKV_ERR_BAD_SEQ
