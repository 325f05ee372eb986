"""Speculative decoding leaves the cache exactly where plain decoding would.

The reference checks its MTP path end to end by comparing speculative and
plain greedy token streams (gadeon-cli --verify-mtp, cli/Probes.swift:285-337).
At the cache level the same property is: cycles of "append n drafts and
verify them, then truncate the rejected suffix" (Engine.decodeSpecStep,
LLM/src/CoreML/Engine.swift:2742-2812) must leave the compacted K/V of a
sequence byte-identical to single-token decoding of the committed tokens
(PagePool.append + hostFlashDecode per token, PagedAttention.swift:85-94,
:317-366), and the verify rows of the committed tokens must see exactly the
keys their plain decode saw.  Checked on the oracle (CPU) and through the C
ABI on the GPU, where the drafts ride in the attend launch.
"""
import numpy as np
import pytest

from conftest import assert_attn_close


def _cycles(seed, n_cycles, n_draft):
    """Accepted prefix per cycle (1..n_draft: the engine always commits at
    least the verified token)."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(1, n_draft + 1, size=n_cycles)]


def _run_oracle(O, kvh, dh, P, G, ctx, accepts, n_draft, seed):
    """Plain route on sequence a, speculative route on sequence b of one
    oracle pool; returns both routes' committed-row outputs and the pool."""
    pool = O.OraclePool(kvh, dh, P, 4096, seed)
    a, b = pool.seq_create(), pool.seq_create()
    K = O.normal_f16(seed, 0, (kvh, ctx, dh))
    V = O.normal_f16(seed, 1, (kvh, ctx, dh))
    assert pool.seed(a, K, V, ctx) == 0 and pool.seed(b, K, V, ctx) == 0
    plain, spec = [], []
    for c, m in enumerate(accepts):
        k = O.normal_f16(seed, 10 + 3 * c, (n_draft, 1, kvh, dh))
        v = O.normal_f16(seed, 11 + 3 * c, (n_draft, 1, kvh, dh))
        q = O.normal_f16(seed, 12 + 3 * c, (1, n_draft, kvh * G, dh))
        for r in range(m):  # plain: one committed token at a time
            assert pool.append([a], [1], k[r], v[r]) == 0
            plain.append(pool.attend_causal([a], 1, q[:, r:r + 1], G, dh ** -0.5)[0, 0])
        before = pool.length(b)
        assert pool.append([b], [n_draft], k[:, 0], v[:, 0]) == 0
        out = pool.attend_causal([b], n_draft, q, G, dh ** -0.5)
        spec.extend(out[0, r] for r in range(m))
        assert pool.truncate([b], [before + m]) == 0
    return pool, a, b, np.array(plain), np.array(spec)


@pytest.mark.parametrize("P,ctx", [(16, 37), (8, 64)])
def test_oracle_spec_equals_plain(oracle, P, ctx):
    kvh, dh, G, n_draft = 2, 64, 4, 4
    accepts = _cycles(P, 12, n_draft)
    pool, a, b, plain, spec = _run_oracle(oracle, kvh, dh, P, G, ctx, accepts, n_draft, 5 + P)
    assert pool.length(a) == pool.length(b) == ctx + sum(accepts)
    ka, va = pool.compact(a)
    kb, vb = pool.compact(b)
    assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    # same keys, same arithmetic order in the restatement: identical outputs
    assert np.array_equal(plain, spec)


@pytest.mark.gpu
@pytest.mark.parametrize("P,dh,G", [(16, 256, 4), (8, 128, 2)])
def test_gpu_spec_equals_plain(cuda, oracle, P, dh, G):
    """The GPU runs both routes (fused single-token decode; fused n-draft
    verify + truncate): compacted K/V identical byte for byte, committed rows'
    outputs within tolerance of each other and of the oracle's plain route."""
    from gadeon_b200 import BlockPool
    torch = cuda
    kvh, n_draft, ctx = 2, 4, 300
    accepts = _cycles(dh + P, 16, n_draft)
    seed = 7 + P
    _, _, _, plain_orc, _ = _run_oracle(oracle, kvh, dh, P, G, ctx, accepts, n_draft, seed)

    def dev(x):
        return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda().view(torch.float16)

    gpu = BlockPool(kvh, dh, P, 2048, 4, 512, seed=seed)
    a, b = gpu.seq_create(), gpu.seq_create()
    K = oracle.normal_f16(seed, 0, (kvh, ctx, dh))
    V = oracle.normal_f16(seed, 1, (kvh, ctx, dh))
    gpu.seed(a, dev(K), dev(V), ctx)
    gpu.seed(b, dev(K), dev(V), ctx)
    plain, spec = [], []
    for c, m in enumerate(accepts):
        k = oracle.normal_f16(seed, 10 + 3 * c, (n_draft, 1, kvh, dh))
        v = oracle.normal_f16(seed, 11 + 3 * c, (n_draft, 1, kvh, dh))
        q = oracle.normal_f16(seed, 12 + 3 * c, (1, n_draft, kvh * G, dh))
        for r in range(m):
            out = gpu.append_attend([a], 1, G, dev(k[r]), dev(v[r]), dev(q[:, r:r + 1]))
            plain.append(out.cpu().numpy()[0, 0])
        before = gpu.length(b)
        out = gpu.append_attend([b], n_draft, G, dev(k[:, 0]), dev(v[:, 0]), dev(q))
        o = out.cpu().numpy()
        spec.extend(o[0, r] for r in range(m))
        gpu.truncate([b], [before + m])
    assert gpu.length(a) == gpu.length(b) == ctx + sum(accepts)
    ka, va = gpu.compact(a)
    kb, vb = gpu.compact(b)
    assert torch.equal(ka.view(torch.int16), kb.view(torch.int16))
    assert torch.equal(va.view(torch.int16), vb.view(torch.int16))
    plain, spec = np.array(plain), np.array(spec)
    assert_attn_close(spec, plain, "speculative vs plain route")
    assert_attn_close(plain, plain_orc, "plain route vs oracle")
    assert gpu.device_status() == 0
    gpu.close()
