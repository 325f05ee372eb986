"""GDN rollback after an accepted speculative prefix: the recurrent-state
reconstruction (MtpRollback.stateAfter, LLM/src/CoreML/MtpRollback.swift:47-60)
and the conv tail (Engine.convFromProj, LLM/src/CoreML/Engine.swift:2719-2740).

The oracle restatement is pinned by the reference's own known answers
(LLM/tests/MtpRollbackTests.swift, tolerance 1e-3) and by a numpy evaluation
of the closed form; the CUDA path is checked against both.  The conv tail is
a pure gather, so it must match bit for bit."""
import math

import numpy as np
import pytest

# MtpRollbackTests.swift:11-13 (one head, DK=DV=C=2) and :44-47 (C=5)
S0 = np.array([1, 0, 0, 1], dtype=np.float32)
K2 = np.array([1, 2, 5, 6], dtype=np.float32)
D2 = np.array([3, 4, 7, 8], dtype=np.float32)
K5 = np.array([1, 2, 5, 6, 1, 1, 2, 0, 1, 1], dtype=np.float32)
D5 = np.array([3, 4, 7, 8, 1, 1, 0, 3, 2, 2], dtype=np.float32)
KAT_TOL = 1e-3


def kat_cases():
    """(name, m, C, k, delta, gcum, want) -- the reference's six known answers."""
    eM, w0 = math.exp(-1.5), math.exp(-0.5)
    g4 = [-1, -1.5, -1.8, -2.0, -2.1]
    o = [[3, 4, 6, 8], [35, 40, 42, 48], [1, 1, 1, 1], [0, 6, 0, 0]]
    m4 = [math.exp(g4[3]) * S0[i] + sum(math.exp(g4[3] - g4[t]) * o[t][i] for t in range(4)) for i in range(4)]
    return [
        ("full_prefix_no_decay", 2, 2, K2, D2, [0, 0], [39, 44, 48, 57]),
        ("partial_prefix_no_decay", 1, 2, K2, D2, [0, 0], [4, 4, 6, 9]),
        ("decay_weighting", 2, 2, K2, D2, [-1, -1.5],
         [eM + w0 * 3 + 35, w0 * 4 + 40, w0 * 6 + 42, eM + w0 * 8 + 48]),
        ("m4_no_decay", 4, 5, K5, D5, [0] * 5, [40, 51, 49, 58]),
        ("m5_no_decay", 5, 5, K5, D5, [0] * 5, [42, 53, 51, 60]),
        ("m4_decay", 4, 5, K5, D5, g4, m4),
    ]


def kat_arrays(m, C, k, d, g):
    return (np.array([m], dtype=np.int32), S0.reshape(1, 1, 2, 2), d.reshape(1, 1, C, 2),
            k.reshape(1, 1, C, 2), np.array(g, dtype=np.float32).reshape(1, 1, C))


def closed_form(m, s0, delta, k, gcum):
    """S_m = exp(g[m-1]) S0 + sum_{t<m} exp(g[m-1]-g[t]) outer(k_t, delta_t), float64."""
    n, H = s0.shape[:2]
    out = np.empty(s0.shape, dtype=np.float64)
    for it in range(n):
        mm = int(m[it])
        for h in range(H):
            g = gcum[it, h].astype(np.float64)
            w = np.exp(g[mm - 1] - g[:mm])
            out[it, h] = math.exp(g[mm - 1]) * s0[it, h] + np.einsum(
                "t,ti,tj->ij", w, k[it, h, :mm].astype(np.float64), delta[it, h, :mm].astype(np.float64))
    return out


def random_batch(seed, n, H, DK, DV, C, m=None):
    """Shapes and value ranges of a Qwen3.5 GDN layer's verify ingredients:
    state entries O(0.1), unit-norm-ish keys, gates = negative cumsums."""
    rng = np.random.default_rng(seed)
    s0 = (rng.standard_normal((n, H, DK, DV)) * 0.1).astype(np.float32)
    k = (rng.standard_normal((n, H, C, DK)) / math.sqrt(DK)).astype(np.float32)
    delta = (rng.standard_normal((n, H, C, DV)) * 0.5).astype(np.float32)
    gcum = np.cumsum(-rng.uniform(0.0, 0.7, (n, H, C)), axis=-1).astype(np.float32)
    if m is None:
        m = rng.integers(1, C + 1, n).astype(np.int32)
    return np.asarray(m, dtype=np.int32), s0, delta, k, gcum


def conv_closed_form(m, proj, pre):
    n, C, CD = proj.shape
    taps = pre.shape[-1]
    out = np.empty_like(pre)
    for it in range(n):
        for t in range(taps):
            pos = int(m[it]) - taps + t
            out[it, :, t] = proj[it, pos] if pos >= 0 else pre[it, :, int(m[it]) + t]
    return out


# ---------------------------------------------------------------- CPU: oracle

@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c[0])
def test_oracle_reference_known_answers(oracle, case):
    _, m, C, k, d, g, want = case
    got = oracle.mtp_rollback(*kat_arrays(m, C, k, d, g))
    np.testing.assert_allclose(got.reshape(-1), np.array(want, dtype=np.float64), rtol=0, atol=KAT_TOL)


def test_oracle_matches_closed_form(oracle):
    m, s0, delta, k, gcum = random_batch(3, 6, 4, 16, 12, 5)
    got = oracle.mtp_rollback(m, s0, delta, k, gcum)
    want = closed_form(m, s0, delta, k, gcum)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


def half_ulp_f16(x):
    """Half the spacing of fp16 numbers at |x| (the error of one rounding)."""
    x = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(x, 2.0 ** -14)))
    return 2.0 ** (e - 10) / 2


@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c[0])
def test_oracle_f16_storage_known_answers(oracle, case):
    """The reference stores the state in fp16 (Engine.swift:2697-2705): with
    S0 and the result in fp16 the known answers hold to their tolerance plus
    one fp16 rounding."""
    _, m, C, k, d, g, want = case
    mm, s0, delta, kk, gcum = kat_arrays(m, C, k, d, g)
    got = oracle.mtp_rollback_f16(mm, s0.astype(np.float16), delta, kk, gcum)
    assert got.dtype == np.float16
    want = np.array(want, dtype=np.float64)
    assert np.all(np.abs(got.reshape(-1).astype(np.float64) - want) <= KAT_TOL + half_ulp_f16(want))


def test_oracle_conv_tail_f16(oracle):
    rng = np.random.default_rng(6)
    n, C, CD, taps = 5, 5, 16, 3
    proj = rng.standard_normal((n, C, CD)).astype(np.float32)
    pre = rng.standard_normal((n, CD, taps)).astype(np.float16)
    m = np.array([1, 2, 3, 4, 5], dtype=np.int32)
    got = oracle.conv_rollback_f16(m, proj, pre)
    assert np.array_equal(got, conv_closed_form(m, proj, pre.astype(np.float32)).astype(np.float16))


def test_oracle_conv_tail(oracle):
    rng = np.random.default_rng(4)
    n, C, CD, taps = 7, 5, 24, 3
    proj = rng.standard_normal((n, C, CD)).astype(np.float32)
    pre = rng.standard_normal((n, CD, taps)).astype(np.float32)
    m = np.array([1, 2, 3, 4, 5, 1, 5], dtype=np.int32)
    assert np.array_equal(oracle.conv_rollback(m, proj, pre), conv_closed_form(m, proj, pre))
    # a 1-token commit keeps the two newest carried taps and adds proj row 0
    one = oracle.conv_rollback(m[:1], proj[:1], pre[:1])
    assert np.array_equal(one[0, :, :2], pre[0, :, 1:]) and np.array_equal(one[0, :, 2], proj[0, 0])


# ---------------------------------------------------------------- GPU

def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c[0])
def test_gpu_reference_known_answers(cuda, case):
    import gadeon_b200 as gk
    torch = cuda
    _, m, C, k, d, g, want = case
    mm, s0, delta, kk, gcum = kat_arrays(m, C, k, d, g)
    out = gk.mtp_rollback(mm, _dev(torch, s0), _dev(torch, delta), _dev(torch, kk), _dev(torch, gcum))
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy().reshape(-1), np.array(want, dtype=np.float64), rtol=0,
                               atol=KAT_TOL)


@pytest.mark.gpu
@pytest.mark.parametrize("H,DK,DV,C", [
    (16, 128, 128, 5), (32, 128, 128, 4), (2, 256, 96, 8),  # register-resident path (C <= 8)
    (4, 64, 96, 17), (2, 8, 4, 64), (2, 300, 8, 3),          # float4 path
    (3, 5, 6, 7),                                            # scalar path (DV % 4 != 0)
])
def test_gpu_matches_oracle(cuda, oracle, H, DK, DV, C):
    """Batch of items with their own accepted lengths (every m in 1..C met)."""
    import gadeon_b200 as gk
    torch = cuda
    n = max(C, 6)
    m = (np.arange(n) % C + 1).astype(np.int32)
    m, s0, delta, k, gcum = random_batch(10 + C, n, H, DK, DV, C, m)
    want = oracle.mtp_rollback(m, s0, delta, k, gcum)
    got = gk.mtp_rollback(m, _dev(torch, s0), _dev(torch, delta), _dev(torch, k), _dev(torch, gcum))
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    # fp32 with the reference's operation order; only expf may differ by an ulp
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got, closed_form(m, s0, delta, k, gcum), rtol=1e-4, atol=1e-5)


@pytest.mark.gpu
def test_gpu_many_items_cross_launch_chunks(cuda, oracle):
    """More items than one launch carries (2048 accepted lengths per parameter block)."""
    import gadeon_b200 as gk
    torch = cuda
    n, H, DK, DV, C = 2100, 40, 4, 8, 3
    m, s0, delta, k, gcum = random_batch(21, n, H, DK, DV, C)
    want = oracle.mtp_rollback(m, s0, delta, k, gcum)
    got = gk.mtp_rollback(m, _dev(torch, s0), _dev(torch, delta), _dev(torch, k), _dev(torch, gcum))
    torch.cuda.synchronize()
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
def test_gpu_conv_tail_bit_exact(cuda, oracle):
    import gadeon_b200 as gk
    torch = cuda
    rng = np.random.default_rng(5)
    n, C, CD, taps = 2500, 5, 96, 3
    proj = rng.standard_normal((n, C, CD)).astype(np.float32)
    pre = rng.standard_normal((n, CD, taps)).astype(np.float32)
    m = rng.integers(1, C + 1, n).astype(np.int32)
    got = gk.conv_rollback(m, _dev(torch, proj), _dev(torch, pre))
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), oracle.conv_rollback(m, proj, pre))


@pytest.mark.gpu
def test_gpu_rollback_rejects_bad_arguments(cuda):
    import gadeon_b200 as gk
    torch = cuda
    m, s0, delta, k, gcum = random_batch(1, 2, 2, 8, 8, 4)
    args = [_dev(torch, x) for x in (s0, delta, k, gcum)]
    for bad_m in ([0, 1], [1, 5]):
        with pytest.raises(gk.GkvError) as e:
            gk.mtp_rollback(bad_m, *args)
        assert e.value.code == gk.GKV_ERR_INVALID
    with pytest.raises(gk.GkvError):
        gk.mtp_rollback([1], *args)  # m count != items
    m2, s2, d2, k2, g2 = random_batch(2, 1, 1, 8, 8, 65)
    with pytest.raises(gk.GkvError) as e:
        gk.mtp_rollback(m2, *[_dev(torch, x) for x in (s2, d2, k2, g2)])
    assert e.value.code == gk.GKV_ERR_UNSUPPORTED
    proj = torch.zeros(2, 4, 8, device="cuda")
    pre = torch.zeros(2, 8, 3, device="cuda")
    with pytest.raises(gk.GkvError) as e:
        gk.conv_rollback([0, 1], proj, pre)
    assert e.value.code == gk.GKV_ERR_INVALID


# ---------------------------------------------------------------- GPU: fp16 state storage

F16_SHAPES = [
    (32, 128, 128, 5), (16, 128, 128, 8), (2, 256, 64, 3),  # fast path (DV % 8 == 0, C <= 8)
    (4, 64, 96, 17), (2, 8, 12, 4), (3, 5, 6, 7),           # element-wise path
]


@pytest.mark.gpu
@pytest.mark.parametrize("H,DK,DV,C", F16_SHAPES)
def test_gpu_f16_state_is_the_rounded_fp32_rollback(cuda, oracle, H, DK, DV, C):
    """gkv_mtp_rollback_f16 == fp16(gkv_mtp_rollback(fp32(s0))) bit for bit:
    the same fp32 arithmetic in the same order, one rounding at the store;
    and within one fp16 ulp of the oracle (whose expf may differ by an ulp)."""
    import gadeon_b200 as gk
    torch = cuda
    n = max(C, 6)
    m = (np.arange(n) % C + 1).astype(np.int32)
    m, s0, delta, k, gcum = random_batch(40 + C, n, H, DK, DV, C, m)
    s16 = s0.astype(np.float16)
    dev = [_dev(torch, x) for x in (delta, k, gcum)]
    got = gk.mtp_rollback(m, _dev(torch, s16), *dev)
    ref32 = gk.mtp_rollback(m, _dev(torch, s16.astype(np.float32)), *dev)
    torch.cuda.synchronize()
    assert got.dtype == torch.float16
    got = got.cpu().numpy()
    assert np.array_equal(got.view(np.uint16), ref32.cpu().numpy().astype(np.float16).view(np.uint16))
    want = oracle.mtp_rollback_f16(m, s16, delta, k, gcum).astype(np.float64)
    got = got.astype(np.float64)
    # one fp16 ulp at the larger magnitude (values that round to +0 / -0 compare equal)
    diff = np.abs(got - want)
    assert np.all(diff <= 2 * half_ulp_f16(np.maximum(np.abs(got), np.abs(want)))), diff.max()
    assert (diff > 0).mean() < 0.01, (diff > 0).mean()


@pytest.mark.gpu
@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c[0])
def test_gpu_f16_reference_known_answers(cuda, case):
    import gadeon_b200 as gk
    torch = cuda
    _, m, C, k, d, g, want = case
    mm, s0, delta, kk, gcum = kat_arrays(m, C, k, d, g)
    out = gk.mtp_rollback(mm, _dev(torch, s0.astype(np.float16)), _dev(torch, delta), _dev(torch, kk),
                          _dev(torch, gcum))
    torch.cuda.synchronize()
    want = np.array(want, dtype=np.float64)
    got = out.cpu().numpy().reshape(-1).astype(np.float64)
    assert np.all(np.abs(got - want) <= KAT_TOL + half_ulp_f16(want)), (got, want)


@pytest.mark.gpu
def test_gpu_conv_tail_f16_bit_exact(cuda, oracle):
    import gadeon_b200 as gk
    torch = cuda
    rng = np.random.default_rng(7)
    n, C, CD, taps = 2100, 5, 104, 3
    proj = rng.standard_normal((n, C, CD)).astype(np.float32)
    pre = rng.standard_normal((n, CD, taps)).astype(np.float16)
    m = rng.integers(1, C + 1, n).astype(np.int32)
    got = gk.conv_rollback(m, _dev(torch, proj), _dev(torch, pre))
    torch.cuda.synchronize()
    assert got.dtype == torch.float16
    assert np.array_equal(got.cpu().numpy().view(np.uint16), oracle.conv_rollback_f16(m, proj, pre).view(np.uint16))


@pytest.mark.gpu
@pytest.mark.parametrize("CD,taps", [(96, 1), (96, 2), (64, 4), (20, 3), (64, 5)])
@pytest.mark.parametrize("f16", [False, True])
def test_gpu_conv_tail_shapes(cuda, oracle, CD, taps, f16):
    """Vector path (conv_dim % 8 == 0, taps <= 4) for every tap count, the
    element-wise path otherwise; m from 1 to C covers all-carried, mixed and
    all-projected tails.  Bit for bit with the oracle."""
    import gadeon_b200 as gk
    torch = cuda
    rng = np.random.default_rng(CD * 10 + taps)
    n, C = 300, 6
    proj = rng.standard_normal((n, C, CD)).astype(np.float32)
    pre = rng.standard_normal((n, CD, taps)).astype(np.float16 if f16 else np.float32)
    m = (np.arange(n) % C + 1).astype(np.int32)
    got = gk.conv_rollback(m, _dev(torch, proj), _dev(torch, pre))
    torch.cuda.synchronize()
    want = oracle.conv_rollback_f16(m, proj, pre) if f16 else oracle.conv_rollback(m, proj, pre)
    assert np.array_equal(got.cpu().numpy().view(np.uint16 if f16 else np.uint32),
                          want.view(np.uint16 if f16 else np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("in_place", [False, True])
def test_gpu_f16_many_heads(cuda, oracle, in_place):
    """fp16 state, 128 x 128 heads at C = 5 over a batch of 5,120 heads (far
    more CTAs than fit on the GPU at once), with and without out == s0:
    equal bit for bit to the fp32-storage path rounded once; a slice of the
    items against the oracle."""
    import gadeon_b200 as gk
    torch = cuda
    n, H, DK, DV, C = 160, 32, 128, 128, 5   # 5,120 heads
    rng = np.random.default_rng(11 + in_place)
    m = rng.integers(1, C + 1, n).astype(np.int32)
    m, s0, delta, k, gcum = random_batch(77, n, H, DK, DV, C, m)
    s16 = s0.astype(np.float16)
    dev = [_dev(torch, x) for x in (delta, k, gcum)]
    ref32 = gk.mtp_rollback(m, _dev(torch, s16.astype(np.float32)), *dev).cpu().numpy().astype(np.float16)
    d16 = _dev(torch, s16)
    got = gk.mtp_rollback(m, d16, *dev, out=d16 if in_place else None)
    torch.cuda.synchronize()
    if in_place:
        assert got.data_ptr() == d16.data_ptr()
    got = got.cpu().numpy()
    assert np.array_equal(got.view(np.uint16), ref32.view(np.uint16))
    sl = slice(0, 4)
    want = oracle.mtp_rollback_f16(m[sl], s16[sl], delta[sl], k[sl], gcum[sl]).astype(np.float64)
    diff = np.abs(got[sl].astype(np.float64) - want)
    assert np.all(diff <= 2 * half_ulp_f16(np.maximum(np.abs(got[sl]), np.abs(want)))), diff.max()


@pytest.mark.gpu
def test_gpu_f16_unaligned_state_takes_the_elementwise_kernel(cuda, oracle):
    """A state array 8 bytes off a 16-byte boundary cannot be moved in
    16-byte columns: the call falls back to the element-wise kernel, same
    bits."""
    import gadeon_b200 as gk
    torch = cuda
    n, H, DK, DV, C = 6, 4, 128, 128, 5
    m = (np.arange(n) % C + 1).astype(np.int32)
    m, s0, delta, k, gcum = random_batch(78, n, H, DK, DV, C, m)
    s16 = s0.astype(np.float16)
    dev = [_dev(torch, x) for x in (delta, k, gcum)]
    flat = torch.zeros(s16.size + 4, dtype=torch.float16, device="cuda")
    flat[4:] = _dev(torch, s16).reshape(-1)
    odd = flat[4:].view(s16.shape)
    assert odd.data_ptr() % 16 == 8
    got = gk.mtp_rollback(m, odd, *dev)
    aligned = gk.mtp_rollback(m, _dev(torch, s16), *dev)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy().view(np.uint16), aligned.cpu().numpy().view(np.uint16))


@pytest.mark.gpu
@pytest.mark.parametrize("H,DK,DV,C,CD,taps", [
    (32, 128, 128, 5, 8192, 3),   # Qwen3.5 GDN layer at the MTP verify width: one fused launch
    (16, 128, 128, 8, 1024, 4),   # wide verify, 4 taps: fused
    (4, 128, 128, 5, 256, 1),     # 1 tap, a conv block a quarter full: fused
    (4, 64, 64, 3, 136, 2),       # 2 taps, 17 channel groups: fused
    (4, 8, 12, 5, 64, 2),         # DV % 8 != 0: the two separate launches
    (4, 128, 128, 5, 20, 3),      # conv_dim % 8 != 0: the two separate launches
])
def test_gpu_gdn_rollback_fused_equals_two_calls(cuda, oracle, H, DK, DV, C, CD, taps):
    """gkv_gdn_rollback_f16 (Engine.rollbackGDN in one call) gives the state
    and conv tail of gkv_mtp_rollback_f16 and gkv_conv_rollback_f16 bit for
    bit, in place too, over a batch with every m; the conv tail also matches
    the oracle bit for bit."""
    import gadeon_b200 as gk
    torch = cuda
    n = 3 * C + 1
    m = (np.arange(n) % C + 1).astype(np.int32)
    m, s0, delta, k, gcum = random_batch(90 + C, n, H, DK, DV, C, m)
    rng = np.random.default_rng(91)
    proj = rng.standard_normal((n, C, CD)).astype(np.float32)
    pre = rng.standard_normal((n, CD, taps)).astype(np.float16)
    d16, dpre = _dev(torch, s0.astype(np.float16)), _dev(torch, pre)
    dev = [_dev(torch, x) for x in (delta, k, gcum)]
    dproj = _dev(torch, proj)
    want_s = gk.mtp_rollback(m, d16, *dev)
    want_c = gk.conv_rollback(m, dproj, dpre)
    got_s, got_c = gk.gdn_rollback(m, d16, *dev, dproj, dpre)
    torch.cuda.synchronize()
    u16 = lambda t: t.cpu().numpy().view(np.uint16)
    assert np.array_equal(u16(got_s), u16(want_s))
    assert np.array_equal(u16(got_c), u16(want_c))
    assert np.array_equal(u16(got_c), oracle.conv_rollback_f16(m, proj, pre).view(np.uint16))
    gk.gdn_rollback(m, d16, *dev, dproj, dpre, out=d16, conv_out=dpre)  # in place
    torch.cuda.synchronize()
    assert np.array_equal(u16(d16), u16(want_s)) and np.array_equal(u16(dpre), u16(want_c))


@pytest.mark.gpu
def test_gpu_gdn_rollback_fused_across_launch_chunks(cuda):
    """2,100 items: the fused call splits at the 2,048 items a parameter
    block holds; both launches equal the separate calls bit for bit."""
    import gadeon_b200 as gk
    torch = cuda
    n, H, DK, DV, C, CD, taps = 2100, 2, 128, 128, 5, 64, 3
    m, s0, delta, k, gcum = random_batch(93, n, H, DK, DV, C)
    rng = np.random.default_rng(94)
    proj = _dev(torch, rng.standard_normal((n, C, CD)).astype(np.float32))
    pre = _dev(torch, rng.standard_normal((n, CD, taps)).astype(np.float16))
    d16 = _dev(torch, s0.astype(np.float16))
    dev = [_dev(torch, x) for x in (delta, k, gcum)]
    want_s, want_c = gk.mtp_rollback(m, d16, *dev), gk.conv_rollback(m, proj, pre)
    got_s, got_c = gk.gdn_rollback(m, d16, *dev, proj, pre)
    torch.cuda.synchronize()
    u16 = lambda t: t.cpu().numpy().view(np.uint16)
    assert np.array_equal(u16(got_s), u16(want_s)) and np.array_equal(u16(got_c), u16(want_c))


@pytest.mark.gpu
@pytest.mark.parametrize("H,DK,DV,C,CD,taps", [
    (32, 128, 128, 5, 8192, 3),   # fp32 state at the MTP verify width: one fused launch
    (8, 128, 128, 8, 2056, 1),    # wide verify, 1 tap, a conv block partly filled: fused
    (4, 8, 6, 5, 64, 2),          # DV % 4 != 0: the two separate launches
])
def test_gpu_gdn_rollback_f32_fused_equals_two_calls(cuda, oracle, H, DK, DV, C, CD, taps):
    """gkv_gdn_rollback (fp32 storage) equals gkv_mtp_rollback +
    gkv_conv_rollback bit for bit; state within rtol 1e-5 of the oracle
    (expf may differ by an ulp), conv tail bit-exact with it."""
    import gadeon_b200 as gk
    torch = cuda
    n = 3 * C + 1
    m = (np.arange(n) % C + 1).astype(np.int32)
    m, s0, delta, k, gcum = random_batch(95 + C, n, H, DK, DV, C, m)
    rng = np.random.default_rng(96)
    proj = rng.standard_normal((n, C, CD)).astype(np.float32)
    pre = rng.standard_normal((n, CD, taps)).astype(np.float32)
    ds, dpre, dproj = _dev(torch, s0), _dev(torch, pre), _dev(torch, proj)
    dev = [_dev(torch, x) for x in (delta, k, gcum)]
    want_s, want_c = gk.mtp_rollback(m, ds, *dev), gk.conv_rollback(m, dproj, dpre)
    got_s, got_c = gk.gdn_rollback(m, ds, *dev, dproj, dpre)
    torch.cuda.synchronize()
    assert got_s.dtype == torch.float32
    u32 = lambda t: t.cpu().numpy().view(np.uint32)
    assert np.array_equal(u32(got_s), u32(want_s)) and np.array_equal(u32(got_c), u32(want_c))
    np.testing.assert_allclose(got_s.cpu().numpy(), oracle.mtp_rollback(m, s0, delta, k, gcum), rtol=1e-5, atol=1e-6)
    assert np.array_equal(got_c.cpu().numpy(), oracle.conv_rollback(m, proj, pre))
