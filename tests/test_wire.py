"""The park / restore wire format: the pool section of Engine.serialize /
deserialize (LLM/src/CoreML/Engine.swift:1062-1119) and the StateBytes
"GDNS" header (LLM/src/Shared/StateBytes.swift:12-40).

The expected bytes are restated here from the Swift framing (little-endian
Int64 counts, fp16 payloads, layers ascending) over the oracle's compact
K/V, so the library's output is checked byte for byte."""
import struct

import numpy as np
import pytest


def engine_pool_section(sections):
    """Engine.serialize's pool loop (Engine.swift:1078-1087) over
    (layer, length, K, V) with K/V head-major compact uint16 arrays."""
    out = struct.pack("<q", len(sections))
    for layer, length, K, V in sorted(sections, key=lambda s: s[0]):
        out += struct.pack("<qq", layer, length)
        out += struct.pack("<q", K.size) + np.ascontiguousarray(K, dtype="<u2").tobytes()
        out += struct.pack("<q", V.size) + np.ascontiguousarray(V, dtype="<u2").tobytes()
    return out


# ---------------------------------------------------------------- CPU

def test_state_header_bytes():
    import gadeon_b200 as gk
    h = gk.state_header()
    assert h == b"GDNS" + struct.pack("<q", 1)
    assert gk.read_state_header(h + b"payload") == 12
    assert gk.read_state_header(h) == 12
    assert gk.read_state_header(b"GDNS" + struct.pack("<q", 2)) is None  # other version
    assert gk.read_state_header(b"GDNT" + struct.pack("<q", 1)) is None  # other magic
    assert gk.read_state_header(h[:11]) is None                          # short
    assert gk.read_state_header(b"") is None


def test_engine_section_restatement_layout():
    """The restated framing itself: count, then per layer 4 Int64 fields
    (layer, length, n, n) and two fp16 payloads (guards the expected-bytes
    helper the GPU test uses)."""
    K = np.arange(2 * 3 * 4, dtype=np.uint16).reshape(2, 3, 4)
    b = engine_pool_section([(7, 3, K, K + 1), (2, 0, K[:, :0], K[:, :0])])
    assert struct.unpack_from("<q", b, 0)[0] == 2
    assert struct.unpack_from("<qqq", b, 8) == (2, 0, 0)      # layer 2 first
    assert struct.unpack_from("<q", b, 32)[0] == 0
    assert struct.unpack_from("<qqq", b, 40) == (7, 3, 24)
    assert struct.unpack_from("<q", b, 64 + 48)[0] == 24
    assert len(b) == 8 + 2 * 32 + 4 * 24


# ---------------------------------------------------------------- GPU

def _layers(cuda, oracle, n_layers=3):
    from test_gpu_parity import Pair
    prs = [Pair(cuda, oracle, kvh=2, dh=256, P=16, num_pages=300, seed=40 + i) for i in range(n_layers)]
    for pr in prs:
        a, b = pr.new_seq(), pr.new_seq()
        pr.append([a, b], [75, 300])
        pr.truncate([b], [123])  # a stale tail past the length must not travel
    return prs


@pytest.mark.gpu
def test_serialize_bytes_match_engine_framing(cuda, oracle):
    import gadeon_b200 as gk
    prs = _layers(cuda, oracle)
    layer_ids = [11, 3, 7]  # unsorted on purpose: the data lists layers ascending
    data = gk.serialize([pr.gpu for pr in prs], layer_ids, [1, 1, 1])
    sections = []
    for pr, lid in zip(prs, layer_ids):
        K, V = pr.orc.compact(1)
        sections.append((lid, pr.orc.length(1), K, V))
    assert data == engine_pool_section(sections)


@pytest.mark.gpu
def test_deserialize_round_trip(cuda, oracle):
    import gadeon_b200 as gk
    from gadeon_b200 import BlockPool
    torch = cuda
    prs = _layers(cuda, oracle)
    data = gk.state_header() + gk.serialize([pr.gpu for pr in prs], [0, 4, 8], [0, 0, 0])
    off = gk.read_state_header(data)
    assert off == 12
    fresh = [BlockPool(2, 256, 16, 200, 8, 100, seed=900 + i) for i in range(3)]
    for f in fresh:  # occupy id 0 so new ids differ from the originals
        f.seq_create()
    lids, sids, used = gk.deserialize(fresh, data[off:])
    assert lids == [0, 4, 8] and used == len(data) - off
    for pr, f, s in zip(prs, fresh, sids):
        assert f.length(s) == pr.gpu.length(0) == 75
        Kg, Vg = f.compact(s)
        Ko, Vo = pr.orc.compact(0)
        assert np.array_equal(Kg.cpu().numpy().view(np.uint16), Ko)
        assert np.array_equal(Vg.cpu().numpy().view(np.uint16), Vo)
        q = torch.randn((1, 1, 8, 256), device="cuda", dtype=torch.float16)
        a = pr.gpu.attend([0], 1, 4, q).cpu().numpy()
        b = f.attend([s], 1, 4, q).cpu().numpy()
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-6)
    # re-serialising the restored sequences reproduces the payload
    assert gk.serialize(fresh, lids, sids) == data[off:]


@pytest.mark.gpu
def test_deserialize_rejects_bad_data_and_changes_nothing(cuda, oracle):
    import gadeon_b200 as gk
    from gadeon_b200 import BlockPool
    prs = _layers(cuda, oracle, 2)
    data = gk.serialize([pr.gpu for pr in prs], [1, 2], [1, 1])
    fresh = [BlockPool(2, 256, 16, 200, 8, 100, seed=7) for _ in range(2)]
    before = [f.free_page_count() for f in fresh]
    for bad in (data[:-1], data[:40], struct.pack("<q", 3) + data[8:], b""):
        with pytest.raises(gk.GkvError) as e:
            gk.deserialize(fresh, bad)
        assert e.value.code == gk.GKV_ERR_INVALID
    wrong_geometry = [BlockPool(1, 256, 16, 200, 8, 100, seed=7), fresh[1]]
    with pytest.raises(gk.GkvError):
        gk.deserialize(wrong_geometry, data)
    assert [f.free_page_count() for f in fresh] == before
    small = [BlockPool(2, 256, 16, 4, 8, 100, seed=7), fresh[1]]  # 8 pages needed
    with pytest.raises(gk.GkvError) as e:
        gk.deserialize(small, data)
    assert e.value.code == gk.GKV_ERR_NO_PAGES
    assert [f.free_page_count() for f in fresh] == before
