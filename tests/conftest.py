import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


# BASELINE tolerance for attention outputs (fp16 storage, fp32 accumulate):
# max-abs 2e-3 and max-rel 1e-2, the relative error taken as the L2 norm of
# the difference over the L2 norm of the oracle's output.
ATOL = 2e-3
RTOL = 1e-2


def assert_attn_close(got, want, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    diff = np.abs(got - want)
    max_abs = float(diff.max()) if diff.size else 0.0
    rel = float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)) if diff.size else 0.0
    assert max_abs <= ATOL, f"{what}: max-abs {max_abs:.3e} > {ATOL}"
    assert rel <= RTOL, f"{what}: rel {rel:.3e} > {RTOL}"
    return max_abs, rel


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
