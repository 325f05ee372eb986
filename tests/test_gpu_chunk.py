"""GPU parity of the prefill-chunk path (n_q * G > 16 query rows per kv
head: the tcgen05 chunk kernel) against the oracle's per-token route --
append row s, then hostFlashDecode over keys [0, p0 + s]
(LLM/src/CoreML/Engine.swift:1220-1224, :2620-2646), which is what the
reference's batched flash with its band mask computes
(LLM/src/CoreML/PagedAttention.swift:376-416, :512-529)."""
import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair, dev_f16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dh", [64, 128, 256])
def test_chunk_head_dims(cuda, oracle, dh):
    pr = Pair(cuda, oracle, kvh=2, dh=dh, P=16, num_pages=400)
    ids = [pr.new_seq() for _ in range(2)]
    pr.append(ids, [100, 37])
    pr.append(ids, [40, 40])
    got, want = pr.attend(ids, 40, 4)
    assert_attn_close(got, want, f"chunk dh={dh}")


@pytest.mark.parametrize("G", [1, 2, 3, 4, 6, 8, 16])
def test_chunk_groups(cuda, oracle, G):
    """qtok = 128 // G tokens per CTA; G that does not divide 128 pads rows."""
    pr = Pair(cuda, oracle, kvh=1, dh=128, P=16, num_pages=300)
    s = pr.new_seq()
    pr.append([s], [70])
    n_q = max(17, 300 // G)
    pr.append([s], [n_q])
    got, want = pr.attend([s], n_q, G)
    assert_attn_close(got, want, f"chunk G={G}")


@pytest.mark.parametrize("P", [8, 16, 32, 64, 128, 512])
def test_chunk_page_sizes(cuda, oracle, P):
    pr = Pair(cuda, oracle, kvh=2, dh=256, P=P, num_pages=max(16, 6000 // P))
    ids = [pr.new_seq() for _ in range(3)]
    pr.append(ids, [0, 5, 333])
    pr.append(ids, [200, 130, 77])  # ragged rows are not allowed: use equal n_q below
    pr.append(ids, [64, 64, 64])
    got, want = pr.attend(ids, 64, 4)
    assert_attn_close(got, want, f"chunk P={P}")
    pr.check_state(pages=False)


def test_chunk_from_empty_prefill(cuda, oracle):
    """p0 = 0: a whole prompt ingested in one chunk (pagedFlashCarrySingle's case)."""
    pr = Pair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=200)
    s = pr.new_seq()
    pr.append([s], [512])
    got, want = pr.attend([s], 512, 4)
    assert_attn_close(got, want, "prefill from empty")


def test_config4_shape_scaled(cuda, oracle):
    """Config 4 geometry (16 q heads, 4 KV heads, dh=256, P=16): sequences with
    an existing seeded context ingest a chunk and attend causally over prior +
    new; several query blocks per sequence and per kv head."""
    pr = Pair(cuda, oracle, kvh=4, dh=256, P=16, num_pages=800)
    ids = [pr.new_seq() for _ in range(3)]
    for s, c in zip(ids, [1024, 640, 2000]):
        pr.seed(s, c)
    pr.append(ids, [256, 256, 256])
    got, want = pr.attend(ids, 256, 4)
    assert_attn_close(got, want, "config4 scaled")
    pr.check_state(pages=False)


def test_chunk_matches_decode_kernel_on_overlap(cuda, oracle):
    """A wide verify (n_q*G = 32 rows, chunk kernel) and a narrow one
    (n_q*G = 16, split-K kernel) agree on the rows they share."""
    torch = cuda
    pr = Pair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=200)
    s = pr.new_seq()
    pr.append([s], [700])
    q = oracle.normal_f16(9, 9, (1, 8, 8, 256))
    wide = pr.gpu.attend([s], 8, 4, dev_f16(torch, q)).cpu().numpy()
    narrow = pr.gpu.attend([s], 4, 4, dev_f16(torch, np.ascontiguousarray(q[:, 4:]))).cpu().numpy()
    assert_attn_close(wide[:, 4:], narrow, "chunk vs split-K")
