"""gkv_attn_step: one decode token of a Qwen3.5 full-attention layer from
its raw projections (Attn.step, LLM/src/SIMD/Attention.swift:72-139) --
q|gate split, q/k RMSNorm (Kernels.swift:26-37), partial NEOX RoPE
(Kernels.swift:66-84), append, attention, sigmoid output gate
(Attention.swift:133-135) -- against the oracle's restatement of each step
followed by its append and hostFlashDecode.

Outputs within the attention tolerance.  Block tables, the free list and
page bytes are bit-exact, the producer-built K rows included: the GPU forms
RMSNorm's sum of squares in the reference's sequential order."""
import numpy as np
import pytest

from conftest import assert_attn_close


def f16_bits(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32).astype(np.float16)).view(np.uint16)


# ---------------------------------------------------------------- CPU: oracle

def test_oracle_rmsnorm_matches_float64(oracle):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((6, 256)) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    got = oracle.rmsnorm_rows(x, w, 1e-6)
    x64 = x.astype(np.float64)
    want = x64 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-6)


def test_oracle_rope_properties(oracle):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    c0, s0 = oracle.rope_table(256, 1e7, [0])
    assert np.array_equal(oracle.rope_neox(x, 256, c0[0], s0[0]), x)  # position 0: identity
    c, s = oracle.rope_table(64, 1e7, [12345])
    y = oracle.rope_neox(x, 64, c[0], s[0])
    assert np.array_equal(y[:, 64:], x[:, 64:])  # past n_rot untouched
    # pair (i, i+32) rotated by the table's angle
    cc, ss = c[0].astype(np.float64), s[0].astype(np.float64)
    a, b = x[:, :32].astype(np.float64), x[:, 32:64].astype(np.float64)
    np.testing.assert_allclose(y[:, :32], a * cc - b * ss, atol=2e-6)
    np.testing.assert_allclose(y[:, 32:64], a * ss + b * cc, atol=2e-6)
    np.testing.assert_allclose(cc ** 2 + ss ** 2, 1.0, atol=1e-6)
    # the table's angle is pos * base^(-2i/n_rot) evaluated in fp32; at a
    # small position its rounding is below 1e-6
    c5, s5 = oracle.rope_table(64, 1e7, [5])
    ang = 5 * (1e7 ** (-2 * np.arange(32) / 64.0))
    np.testing.assert_allclose(c5[0], np.cos(ang), atol=1e-6)
    np.testing.assert_allclose(s5[0], np.sin(ang), atol=1e-6)


def test_oracle_gate(oracle):
    rng = np.random.default_rng(3)
    x, g = rng.standard_normal(100).astype(np.float32), (4 * rng.standard_normal(100)).astype(np.float32)
    np.testing.assert_allclose(oracle.gate(x, g), x / (1 + np.exp(-g.astype(np.float64))), rtol=1e-6)


def test_library_rope_table_matches_oracle(oracle):
    """Host helper of the C ABI (no device work): same fp32 formula, same bits."""
    import gadeon_b200 as gk
    pos = [0, 1, 7, 4095, 131071, 1 << 20]
    for n_rot, base in ((64, 1e7), (128, 10000.0), (256, 1e6)):
        c, s = gk.rope_table(n_rot, base, pos)
        oc, os_ = oracle.rope_table(n_rot, base, pos)
        assert np.array_equal(c, oc) and np.array_equal(s, os_)


# ---------------------------------------------------------------- GPU

class StepPair:
    """GPU pool + oracle pool driven by identical attention steps."""

    def __init__(self, torch, O, kvh, dh, P, num_pages, G, n_rot, base=1e7, eps=1e-6, seed=77):
        from test_gpu_parity import Pair
        self.pr = Pair(torch, O, kvh=kvh, dh=dh, P=P, num_pages=num_pages, seed=seed)
        self.torch, self.O = torch, O
        self.kvh, self.dh, self.G, self.n_rot, self.base, self.eps = kvh, dh, G, n_rot, base, eps
        rng = np.random.default_rng(seed)
        self.q_norm = (1 + 0.1 * rng.standard_normal(dh)).astype(np.float32)
        self.k_norm = (1 + 0.1 * rng.standard_normal(dh)).astype(np.float32)
        self.rng = rng

    def dev(self, a):
        return self.torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()

    def step(self, ids):
        """One gkv_attn_step on the GPU, the restated producer + append +
        hostFlashDecode + gate on the oracle; returns (got, want)."""
        O, pr, rng = self.O, self.pr, self.rng
        n, KVH, dh, G = len(ids), self.kvh, self.dh, self.G
        nH = KVH * G
        q_gate = rng.standard_normal((n, nH, 2 * dh)).astype(np.float32)
        k_raw = (3 * rng.standard_normal((n, KVH, dh))).astype(np.float32)
        v_raw = rng.standard_normal((n, KVH, dh)).astype(np.float32)
        pos = [pr.orc.length(s) for s in ids]  # the new token's position
        cos, sin = O.rope_table(self.n_rot, self.base, pos)
        got = pr.gpu.attn_step(ids, G, self.dev(q_gate), self.dev(k_raw), self.dev(v_raw), self.dev(self.q_norm),
                               self.dev(self.k_norm), self.dev(cos), self.dev(sin), eps=self.eps)
        got = got.cpu().numpy()
        qs = np.empty((n, 1, nH, dh), dtype=np.uint16)
        ks = np.empty((n, KVH, dh), dtype=np.uint16)
        for i in range(n):
            q = O.rope_neox(O.rmsnorm_rows(q_gate[i, :, :dh], self.q_norm, self.eps), self.n_rot, cos[i], sin[i])
            k = O.rope_neox(O.rmsnorm_rows(k_raw[i], self.k_norm, self.eps), self.n_rot, cos[i], sin[i])
            qs[i, 0] = f16_bits(q)
            ks[i] = f16_bits(k)
        assert pr.orc.append(ids, [1] * n, ks, f16_bits(v_raw)) == 0
        want = pr.orc.attend_causal(ids, 1, qs, G, dh ** -0.5, n_threads=8)[:, 0]
        self.last_ungated = want.copy()
        for i in range(n):
            want[i] = O.gate(want[i], q_gate[i, :, dh:])
        return got, want

    def check_state(self):
        """Tables, free list, lengths, refcounts and page bytes bit-exact --
        the producer-built K rows included (RMSNorm's sum of squares in the
        reference's sequential order, every product and sum rounded)."""
        pr = self.pr
        pr.check_state(pages=False)
        for s in pr.seqs:
            for pid in pr.gpu.export_table(s):
                gk, gv = pr.gpu.export_page(int(pid))
                ok, ov = pr.orc.page_bytes(int(pid))
                assert np.array_equal(gv, ov), f"V page {pid}"
                d = np.abs(gk.astype(np.int32) - ok.astype(np.int32))
                assert np.array_equal(gk, ok), f"K page {pid}: {(d > 0).sum()} values differ, max {d.max()} ulp"


@pytest.mark.gpu
def test_attn_step_fused_config2_geometry(cuda, oracle):
    """nH=8, KVH=2, dh=256, P=16, partial rope 64 of 256 (Qwen3.5): every
    step appends through the attend kernel's prologue; contexts straddle
    page boundaries (fresh pages zero-filled)."""
    sp = StepPair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=400, G=4, n_rot=64)
    ids = [sp.pr.new_seq() for _ in range(5)]
    sp.pr.append(ids, [0, 15, 16, 31, 300])
    sp.pr.check_state()
    for step in range(3):
        got, want = sp.step(ids)
        assert_attn_close(got, want, f"step {step}")
        sp.check_state()


@pytest.mark.gpu
@pytest.mark.parametrize("dh,G,n_rot", [(128, 1, 16), (128, 8, 128), (128, 16, 64), (256, 2, 256), (256, 6, 32)])
def test_attn_step_geometries(cuda, oracle, dh, G, n_rot):
    sp = StepPair(cuda, oracle, kvh=2, dh=dh, P=16, num_pages=300, G=G, n_rot=n_rot, base=10000.0)
    ids = [sp.pr.new_seq() for _ in range(3)]
    sp.pr.append(ids, [1, 40, 700])
    got, want = sp.step(ids)
    assert_attn_close(got, want, f"dh={dh} G={G} n_rot={n_rot}")
    sp.check_state()


@pytest.mark.gpu
def test_attn_step_copy_on_write_route(cuda, oracle):
    """A bookmark shares the tail page: the step takes the unfused route
    (producer kernel, append with copy-on-write, attend with the producer's
    q and gate) and leaves the bookmark's page untouched."""
    sp = StepPair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=200, G=4, n_rot=64)
    pr = sp.pr
    s = pr.new_seq()
    pr.append([s], [37])
    c = pr.gpu.clone(s)
    assert pr.orc.clone(s) == c
    pr.seqs.append(c)
    got, want = sp.step([c])
    assert_attn_close(got, want, "after clone")
    sp.check_state()
    got, want = sp.step([s, c])
    assert_attn_close(got, want, "both")
    sp.check_state()


@pytest.mark.gpu
def test_attn_step_small_pages(cuda, oracle):
    """P=4: no TMA boxes; the rows are produced, appended, then attended
    with the cp.async loader."""
    sp = StepPair(cuda, oracle, kvh=1, dh=256, P=4, num_pages=100, G=4, n_rot=64)
    ids = [sp.pr.new_seq() for _ in range(2)]
    sp.pr.append(ids, [3, 41])
    for _ in range(2):
        got, want = sp.step(ids)
        assert_attn_close(got, want, "P=4")
        sp.check_state()


@pytest.mark.gpu
def test_attn_step_anti_vacuity(cuda, oracle):
    """The gate and the norms matter: dropping the gate on the oracle side
    moves the output far outside the tolerance."""
    sp = StepPair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=100, G=4, n_rot=64)
    ids = [sp.pr.new_seq()]
    sp.pr.append(ids, [50])
    got, want = sp.step(ids)
    assert_attn_close(got, want, "baseline")
    assert np.abs(got).max() > 0.05
    assert np.abs(sp.last_ungated - got).max() > 5e-2  # the gate is applied


@pytest.mark.gpu
def test_attn_step_rejects_bad_arguments(cuda, oracle):
    import gadeon_b200 as gk
    torch = cuda
    pool = gk.BlockPool(2, 256, 16, 64, 8, 64, seed=1)
    s = pool.seq_create()
    f = lambda *shape: torch.zeros(shape, dtype=torch.float32, device="cuda")  # noqa: E731
    args = dict(q_gate=f(1, 8, 512), k_raw=f(1, 2, 256), v_raw=f(1, 2, 256), q_norm=f(256), k_norm=f(256))
    for half, G, code in ((4, 4, gk.GKV_ERR_INVALID), (32, 17, gk.GKV_ERR_INVALID), (256, 4, gk.GKV_ERR_INVALID)):
        qg = f(1, 2 * G, 512)
        with pytest.raises(gk.GkvError) as e:
            pool.attn_step([s], G, qg, args["k_raw"], args["v_raw"], args["q_norm"], args["k_norm"],
                           f(1, half), f(1, half))
        assert e.value.code == code
    assert pool.length(s) == 0  # a refused step changes nothing
    small = gk.BlockPool(2, 64, 16, 64, 8, 64, seed=1)
    t = small.seq_create()
    with pytest.raises(gk.GkvError) as e:
        small.attn_step([t], 4, f(1, 8, 128), f(1, 2, 64), f(1, 2, 64), f(64), f(64), f(1, 16), f(1, 16))
    assert e.value.code == gk.GKV_ERR_UNSUPPORTED


@pytest.mark.gpu
@pytest.mark.parametrize("seed,P,dh,G,n_rot", [(61, 16, 256, 4, 64), (62, 8, 128, 2, 128), (63, 32, 128, 4, 32)])
def test_attn_step_random_mix(cuda, oracle, seed, P, dh, G, n_rot):
    """gkv_attn_step interleaved with the operations that reshape the cache
    -- plain appends, truncates into shared pages, clones, releases -- so
    that steps meet fresh pages, page boundaries and copy-on-write tails
    (the unfused route) in every combination; state and outputs checked
    after every step against the oracle's producer + append + decode."""
    from test_gpu_parity import dev_f16
    sp = StepPair(cuda, oracle, kvh=2, dh=dh, P=P, num_pages=160, G=G, n_rot=n_rot, seed=seed)
    pr, rng = sp.pr, np.random.default_rng(seed)
    live = [pr.new_seq() for _ in range(3)]
    pr.append(live, [int(x) for x in rng.integers(1, 3 * P, size=3)])
    ops = ["step", "step", "step", "append", "truncate", "clone", "release", "new"]
    for i in range(60):
        op = ops[int(rng.integers(len(ops)))]
        if op == "step":
            ids = [int(x) for x in rng.choice(live, size=int(rng.integers(1, len(live) + 1)), replace=False)]
            got, want = sp.step(ids)
            assert_attn_close(got, want, f"step {i}")
        elif op == "append":
            ids = [int(x) for x in rng.choice(live, size=int(rng.integers(1, len(live) + 1)), replace=False)]
            pr.append(ids, [int(x) for x in rng.integers(0, 2 * P, size=len(ids))])
        elif op == "truncate":
            ids = [int(x) for x in rng.choice(live, size=int(rng.integers(1, len(live) + 1)), replace=False)]
            pr.truncate(ids, [int(rng.integers(1, pr.gpu.length(s) + 1)) if pr.gpu.length(s) else 0 for s in ids])
        elif op == "clone" and len(live) < 8:
            src = int(rng.choice(live))
            c = pr.gpu.clone(src)
            assert pr.orc.clone(src) == c
            pr.seqs.append(c)
            live.append(c)
        elif op == "release" and len(live) > 2:
            s = int(rng.choice(live))
            pr.gpu.seq_release(s)
            assert pr.orc.seq_release(s) == 0
            live.remove(s)
            pr.seqs.remove(s)
        elif op == "new" and len(live) < 8:
            live.append(pr.new_seq())
        if i % 6 == 5:
            sp.check_state()
        else:
            pr.check_state(pages=False)
    sp.check_state()
