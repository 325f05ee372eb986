"""CPU tests of the algorithmic byte and FLOP counts that every roofline
fraction in bench.py divides by (gadeon_b200/workload.py, bench.chunk_flops),
against closed forms written out here and the configurations' published
shapes."""
import os
import sys

import numpy as np

from gadeon_b200.workload import CONFIGS, GDN, append_bytes, decode_bytes, rollback_bytes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_decode_bytes_closed_form():
    """One attend launch: every K and V byte of the context once, q read
    (fp16), out written (fp32), one 4-byte table entry per page."""
    cfg = CONFIGS[2]  # KVH=2, dh=256, nH=8, P=16, n_q=1
    c = 1000
    want = c * 2 * 256 * 2 * 2 + 1 * 8 * 256 * (2 + 4) + 4 * 63  # ceil(1000/16) = 63 pages
    assert decode_bytes([c], cfg) == want
    assert decode_bytes([c, c], cfg) == 2 * want
    # config 3's verify: 4 query rows per sequence, KVH=4, nH=16
    cfg3 = CONFIGS[3]
    assert decode_bytes([8196], cfg3) == 8196 * 4 * 256 * 2 * 2 + 4 * 16 * 256 * 6 + 4 * 513


def test_config2_step_bytes_near_the_published_estimate():
    """Config 2 at its mean context (~17.5K) moves ~2.3 GB per layer: 6
    layers ~13.8 GB per step, the order of the per-step estimate (13.3 GB at
    a mean of 16,896)."""
    cfg = CONFIGS[2]
    per_layer = decode_bytes([16896] * 64, cfg) + append_bytes(64, cfg)
    assert abs(6 * per_layer / 1e9 - 13.3) < 0.2


def test_append_bytes():
    cfg = CONFIGS[2]
    assert append_bytes(1, cfg) == 2 * 256 * 2 * 2 * 2  # K and V rows, read and written


def test_chunk_flops_config4():
    """Row s of a 4,096-token chunk over 16,384 prior tokens sees 16,385 + s
    keys; QK^T and P.V are 2 flops per multiply-add each, every query head:
    3.958e13 per launch, 3.17e14 per 8-layer step."""
    sys.path.insert(0, ROOT)
    import bench
    cfg = CONFIGS[4]
    fl = bench.chunk_flops([16384] * 32, 4096, cfg)
    want = 32 * 16 * (4096 * 16384 + 4096 * 4097 / 2) * 4 * 256
    assert fl == want
    assert abs(fl / 3.958e13 - 1) < 1e-3 and abs(8 * fl / 3.17e14 - 1) < 2e-3


def test_rollback_bytes_closed_form():
    """Per item and value head: the state read and written once, the m
    accepted rows of k and delta (fp32), the C gate values; conv tail
    written once with each tap read once (projection rows fp32, carried taps
    in the storage type)."""
    g = GDN
    assert g.conv_dim == (2 * 16 + 32) * 128 == 8192
    H, D = g.value_heads, g.head_dim
    for sb in (2, 4):
        state, conv = rollback_bytes([2], g, sb)
        assert state == H * (2 * D * D * sb + 2 * 2 * D * 4 + g.chunk * 4)
        # m = 2 < taps = 3: two taps from the projection rows, one carried
        assert conv == g.conv_dim * (3 * sb + 2 * 4 + 1 * sb)
    state5, conv5 = rollback_bytes([5], g, 2)
    assert conv5 == g.conv_dim * (3 * 2 + 3 * 4)  # every tap from the projection rows
    s, c = rollback_bytes(np.array([1, 5]), g, 2)
    assert (s, c) == tuple(a + b for a, b in zip(rollback_bytes([1], g, 2), rollback_bytes([5], g, 2)))
