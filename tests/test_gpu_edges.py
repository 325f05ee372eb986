"""Edge cases of the path on the GPU, vs the oracle: the longest context of
the BASELINE configs (config 5 draws up to 131,072 tokens), empty batches on
every entry point, a sequence reaching its block-table row's capacity, and
zero-row entries inside a batch.  Cache state stays bit-exact with the
oracle's PagePool restatement (LLM/src/CoreML/PagedAttention.swift:21-287)
and outputs within the BASELINE tolerance of hostFlashDecode (:317-366)."""
import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair, dev_f16

pytestmark = pytest.mark.gpu


def test_longest_context_decode_and_verify(cuda, oracle):
    """One sequence at 131,072 tokens (config 5's upper bound) beside a
    short one: fused decode steps across the page boundary, then a verify
    of 4 drafts; the split-K merge spans many CTAs."""
    torch = cuda
    kvh, dh, P, G = 4, 256, 16, 4
    L = 131072
    pr = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=L // P + 64, max_pps=L // P + 8, seed=131)
    a, b = pr.new_seq(), pr.new_seq()
    pr.seed(a, L - 2)
    pr.append([b], [5])
    for step in range(3):  # L-1, L (fills the page), L+1 (fresh page)
        k, v = pr.rows(2)
        q = oracle.normal_f16(91, step, (2, 1, kvh * G, dh))
        got = pr.gpu.append_attend([a, b], 1, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
        assert pr.orc.append([a, b], [1, 1], k, v) == 0
        want = pr.orc.attend_causal([a, b], 1, q, G, dh ** -0.5, n_threads=8)
        assert_attn_close(got.cpu().numpy(), want, f"131K decode step {step}")
    assert pr.gpu.length(a) == L + 1
    k, v = pr.rows(8)
    q = oracle.normal_f16(92, 0, (2, 4, kvh * G, dh))
    got = pr.gpu.append_attend([a, b], 4, G, dev_f16(torch, k), dev_f16(torch, v), dev_f16(torch, q))
    assert pr.orc.append([a, b], [4, 4], k, v) == 0
    want = pr.orc.attend_causal([a, b], 4, q, G, dh ** -0.5, n_threads=8)
    assert_attn_close(got.cpu().numpy(), want, "131K verify")
    pr.check_state(pages=False)
    # the pages written this test, bit for bit
    for pid in pr.gpu.export_table(a)[-2:]:
        gk_, gv = pr.gpu.export_page(int(pid))
        ok, ov = pr.orc.page_bytes(int(pid))
        assert np.array_equal(gk_, ok) and np.array_equal(gv, ov)


def test_empty_batches_are_no_ops(cuda, oracle):
    """n_seqs = 0 on every batched entry point returns OK, launches nothing
    and changes nothing."""
    torch = cuda
    kvh, dh, G = 2, 128, 4
    pr = Pair(cuda, oracle, kvh=kvh, dh=dh, P=16, num_pages=32, seed=5)
    s = pr.new_seq()
    pr.append([s], [20])
    torch.cuda.synchronize()
    e16 = torch.empty((0, kvh, dh), dtype=torch.float16, device="cuda")
    q0 = torch.empty((0, 1, kvh * G, dh), dtype=torch.float16, device="cuda")
    pr.gpu.append([], [], e16, e16)
    out = pr.gpu.attend([], 1, G, q0)
    assert out.shape[0] == 0
    out = pr.gpu.append_attend([], 1, G, e16, e16, q0)
    assert out.shape[0] == 0
    pr.gpu.truncate([], [])
    pr.gpu.rewind_append([], [], [], e16, e16)
    torch.cuda.synchronize()
    assert pr.gpu.length(s) == 20
    pr.check_state()


def test_table_row_capacity(cuda, oracle):
    """A sequence may grow to exactly max_pages_per_seq pages; one row more
    is refused with GKV_ERR_CAPACITY and the pool stays as it was."""
    from gadeon_b200 import GKV_ERR_CAPACITY, GkvError
    torch = cuda
    kvh, dh, P = 2, 128, 16
    pr = Pair(cuda, oracle, kvh=kvh, dh=dh, P=P, num_pages=64, max_pps=4, seed=6)
    s = pr.new_seq()
    pr.append([s], [4 * P - 1])
    pr.append([s], [1])  # exactly 4 pages
    k, v = pr.rows(1)
    with pytest.raises(GkvError) as e:
        pr.gpu.append([s], [1], dev_f16(torch, k), dev_f16(torch, v))
    assert e.value.code == GKV_ERR_CAPACITY
    assert pr.gpu.length(s) == 4 * P
    pr.check_state()


def test_zero_row_entries_in_a_batch(cuda, oracle):
    """Entries appending zero rows sit between real ones: nothing is
    written for them and the row offsets of the others stay right."""
    pr = Pair(cuda, oracle, kvh=2, dh=256, P=8, num_pages=64, seed=7)
    ids = [pr.new_seq() for _ in range(4)]
    pr.append(ids, [3, 0, 9, 0])
    pr.append(ids, [0, 5, 0, 8])
    pr.check_state()
    got, want = pr.attend([ids[0], ids[1], ids[2], ids[3]], 1, 2)
    assert_attn_close(got, want, "after zero-row entries")


def test_pools_driven_from_threads(cuda, oracle):
    """Four host threads, each with its own pool, seeding, appending and
    running fused decode steps at the same time (the library's host code
    runs concurrently: ctypes releases the interpreter lock); every pool's
    state and outputs match its own oracle."""
    import threading
    errors = []

    def worker(t):
        try:
            pr = Pair(cuda, oracle, kvh=2, dh=128, P=16, num_pages=120, seed=300 + t)
            ids = [pr.new_seq() for _ in range(4)]
            for s, n in zip(ids, (17, 33, 64, 90)):
                pr.seed(s, n)
            for step in range(12):
                k, v = pr.rows(len(ids))
                q = oracle.normal_f16(300 + t, step, (len(ids), 1, 8, 128))
                got = pr.gpu.append_attend(ids, 1, 4, dev_f16(cuda, k), dev_f16(cuda, v), dev_f16(cuda, q))
                assert pr.orc.append(ids, [1] * len(ids), k, v) == 0
                want = pr.orc.attend_causal(ids, 1, q, 4, 128 ** -0.5)
                assert_attn_close(got.cpu().numpy(), want, f"thread {t} step {step}")
            pr.check_state()
        except BaseException as e:  # reported by the main thread
            errors.append((t, e))

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(4)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not any(th.is_alive() for th in threads), "a worker did not finish"
    assert not errors, errors
