import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


# Tolerance for attention outputs (fp16 storage, fp32 accumulate): max-abs
# 2e-3 and max-rel 1e-2, both element-wise.  Every element must satisfy
# |got - want| <= ATOL, and every element whose oracle value has magnitude
# >= REL_FLOOR must also satisfy |got - want| <= RTOL * |want| (below the
# floor a relative error says nothing: the value is within rounding of 0).
ATOL = 2e-3
RTOL = 1e-2
REL_FLOOR = 2e-3


def attn_errors(got, want):
    """(max-abs, max-rel) over the elements; max-rel only where |want| >= REL_FLOOR."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    diff = np.abs(got - want)
    max_abs = float(diff.max()) if diff.size else 0.0
    big = np.abs(want) >= REL_FLOOR
    max_rel = float((diff[big] / np.abs(want[big])).max()) if big.any() else 0.0
    return max_abs, max_rel


def assert_attn_close(got, want, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    max_abs, max_rel = attn_errors(got, want)
    msg = f"{what}: max-abs {max_abs:.3e} (limit {ATOL}), max-rel {max_rel:.3e} (limit {RTOL}, |want| >= {REL_FLOOR})"
    assert max_abs <= ATOL and max_rel <= RTOL, msg
    return max_abs, max_rel


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from gadeon_b200 import build
    build.build()
    return torch
