"""GKV_ATTEND_P_F16: the tensor-core chunk path with the softmax weights
rounded once to fp16 (one P.V per key tile), the arithmetic of the
reference's Metal attn_batch_mm (a half P tile times half V into fp32,
LLM/metal/Kernels.metal:1891-1912).

Rounding a weight p to fp16 moves it by at most 2^-11 of itself, so each
output element moves by at most 2^-11 x sum_i w_i |V_i| -- B, the same
attention over |V| -- from the exact result.  The tests hold every element
within 2^-10 x B + 1e-5 of the oracle's fp32 result (the extra factor and
the constant cover the two sides' fp32 accumulation orders), with B
computed by the oracle on a twin pool whose V rows have their sign bits
cleared.  They also check that the flag changes the chunk path's result
(the default keeps ~22 bits of every weight), that the decode / verify
path ignores it (bit for bit), and that it composes with the reference's
head-major layout and fp16 output."""
import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import dev_f16

pytestmark = pytest.mark.gpu


class Twin:
    """A GPU pool and two oracle pools (V and |V|) seeded with the same
    rows."""

    def __init__(self, torch, O, kvh, dh, P, lens, seed):
        from gadeon_b200 import BlockPool
        self.torch, self.O, self.kvh, self.dh = torch, O, kvh, dh
        pages = sum((n + P - 1) // P for n in lens) + 8 * len(lens) + 8
        self.gpu = BlockPool(kvh, dh, P, pages, len(lens) + 1, pages, seed=seed)
        self.orc = O.OraclePool(kvh, dh, P, pages, seed)
        self.absorc = O.OraclePool(kvh, dh, P, pages, seed)
        self.ids = []
        for i, n in enumerate(lens):
            K = O.normal_f16(seed, 2 * i, (kvh, n, dh))
            V = O.normal_f16(seed, 2 * i + 1, (kvh, n, dh))
            s = self.gpu.seq_create()
            assert self.orc.seq_create() == s and self.absorc.seq_create() == s
            self.gpu.seed(s, dev_f16(torch, K), dev_f16(torch, V), n)
            assert self.orc.seed(s, K, V, n) == 0
            assert self.absorc.seed(s, K, V & np.uint16(0x7FFF), n) == 0
            self.ids.append(s)

    def check(self, n_q, G, seed, what):
        scale = self.dh ** -0.5
        q = self.O.normal_f16(seed, 0, (len(self.ids), n_q, self.kvh * G, self.dh))
        qd = dev_f16(self.torch, q)
        fast = self.gpu.attend(self.ids, n_q, G, qd, scale=scale, p_f16=True).cpu().numpy()
        full = self.gpu.attend(self.ids, n_q, G, qd, scale=scale).cpu().numpy()
        want = self.orc.attend_causal(self.ids, n_q, q, G, scale, n_threads=8)
        bound = self.absorc.attend_causal(self.ids, n_q, q, G, scale, n_threads=8)
        err = np.abs(fast - want)
        lim = 2.0 ** -10 * bound + 1e-5
        worst = np.unravel_index(np.argmax(err - lim), err.shape)
        assert np.all(err <= lim), (f"{what}: |d| {err[worst]:.3g} > {lim[worst]:.3g} at {worst} "
                                    f"(max |d| / B = {np.max(err / np.maximum(bound, 1e-30)):.3g})")
        assert_attn_close(full, want, f"{what}: default")
        assert not np.array_equal(fast, full), f"{what}: the flag changed nothing"
        assert self.gpu.device_status() == 0
        return q, fast


@pytest.mark.parametrize("kvh,dh,G,lens,n_q", [
    (4, 256, 4, [700, 2100, 300], 300),   # CTA pairs, several query blocks
    (4, 256, 4, [40, 1500], 32),          # one query block (the pair's odd CTA idle)
    (2, 128, 8, [3000, 129, 800], 64),    # dh 128 pairs
    (2, 128, 4, [500, 64], 32),           # dh 128, one CTA
    (2, 64, 4, [900, 2000], 100),         # dh 64
])
def test_p_f16_within_its_bound(cuda, oracle, kvh, dh, G, lens, n_q):
    tw = Twin(cuda, oracle, kvh, dh, 16, lens, seed=7100 + dh + n_q)
    tw.check(n_q, G, 7200 + n_q, f"kvh={kvh} dh={dh} G={G} n_q={n_q}")


def test_p_f16_head_major_fp16_out(cuda, oracle):
    """The flag with the reference's [KVH, S, G, dh] layout and fp16 output:
    the same arithmetic, so the result is the token-major one moved and
    rounded, bit for bit."""
    torch = cuda
    kvh, dh, G, n_q = 4, 256, 4, 64
    tw = Twin(torch, oracle, kvh, dh, 16, [300, 1000], seed=7301)
    q, fast = tw.check(n_q, G, 7302, "token-major")
    n = len(tw.ids)
    qh = np.ascontiguousarray(q.reshape(n, n_q, kvh, G, dh).transpose(0, 2, 1, 3, 4))
    hm = tw.gpu.attend(tw.ids, n_q, G, dev_f16(torch, qh), head_major=True, out_f16=True,
                       p_f16=True).cpu().numpy()
    moved = np.ascontiguousarray(fast.reshape(n, n_q, kvh, G, dh).transpose(0, 2, 1, 3, 4))
    assert np.array_equal(hm.view(np.uint16), moved.astype(np.float16).view(np.uint16))


def test_decode_and_verify_ignore_the_flag(cuda, oracle):
    """n_q * G <= 16 runs the split-K kernel, whose compensated P costs no
    MMA: the flag leaves its result unchanged, bit for bit."""
    torch = cuda
    kvh, dh = 2, 256
    tw = Twin(torch, oracle, kvh, dh, 16, [20, 3000, 9000], seed=7401)
    for n_q, G in ((1, 4), (4, 4), (2, 8)):
        q = oracle.normal_f16(7402, n_q, (len(tw.ids), n_q, kvh * G, dh))
        qd = dev_f16(torch, q)
        a = tw.gpu.attend(tw.ids, n_q, G, qd, p_f16=True).cpu().numpy()
        b = tw.gpu.attend(tw.ids, n_q, G, qd).cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (n_q, G)


def test_unknown_flag_bits_are_refused(cuda):
    import ctypes as C

    from gadeon_b200 import GKV_ERR_INVALID, BlockPool, kv
    torch = cuda
    lib = kv.load_library()
    bp = BlockPool(2, 128, 16, 64, 4, 64, seed=1)
    s = bp.seq_create()
    bp.seed(s, torch.zeros((2, 16, 128), device="cuda", dtype=torch.float16),
            torch.zeros((2, 16, 128), device="cuda", dtype=torch.float16), 16)
    q = torch.zeros((1, 1, 8, 128), device="cuda", dtype=torch.float16)
    out = torch.zeros((1, 1, 8, 128), device="cuda", dtype=torch.float32)
    ids = (C.c_int32 * 1)(s)
    rc = lib.gkv_attend_ex(bp._h, 1, ids, 1, 4, q.data_ptr(), out.data_ptr(), 0.0884, 8, None)
    assert rc == GKV_ERR_INVALID and b"flags" in lib.gkv_last_error()
