"""Failure detection on the GPU without a fault.

Every wait of this library's kernels on an mbarrier (TMA completion, MMA
completion, the hand-offs between warps) is bounded by %globaltimer; when a
wait runs out the kernel records DEV_ERR_WAIT_TIMEOUT in a status word the
host reads, raises its CTA's abort flag and returns, so the context stays
usable.  gkv_check_bounded_wait runs that same bounded wait on a barrier
nothing ever arrives on: the wait must give up after its limit, report the
timeout, and leave the device working (a pool built afterwards must still
match the oracle).  No fault, trap or hang is provoked.
"""
import time

import numpy as np
import pytest

from conftest import assert_attn_close
from test_gpu_parity import Pair

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports(cuda, oracle):
    import gadeon_b200 as gk
    torch = cuda
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    st = gk.check_bounded_wait(0, 30_000_000)  # 30 ms limit
    dt = time.perf_counter() - t0
    assert st == 1, f"status {st}: the wait should have run out (DEV_ERR_WAIT_TIMEOUT)"
    assert 0.025 <= dt < 5.0, dt
    # twice in a row: the probe leaves nothing behind
    assert gk.check_bounded_wait(0, 5_000_000) == 1
    # the context is still usable: a fresh pool decodes correctly
    pr = Pair(cuda, oracle, kvh=2, dh=128, P=16, num_pages=64, seed=9)
    s = pr.new_seq()
    pr.append([s], [50])
    got, want = pr.attend([s], 1, 4)
    assert_attn_close(got, want, "after the bounded-wait probe")
    pr.check_state()


def test_bounded_wait_rejects_bad_arguments(cuda):
    import gadeon_b200 as gk
    for dev, lim in [(0, 10), (0, 20_000_000_000), (-1, 5_000_000), (999, 5_000_000)]:
        with pytest.raises(gk.GkvError) as e:
            gk.check_bounded_wait(dev, lim)
        assert e.value.code == gk.GKV_ERR_INVALID
