"""CPU test of bench.py's interleaved timing (no GPU): a fake torch records
what interleaved_blocks runs, so the order the GPU line depends on is
pinned -- W warm-up steps of the first variant, one untimed call of each
other variant, then rounds that time one block of exactly K steps of every
variant in turn, with the state rewound after every block -- and the
per-block times come back per variant."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class FakeEvent:
    clock = [0.0]

    def __init__(self, enable_timing=False):
        self.t = None

    def record(self):
        self.t = FakeEvent.clock[0]

    def elapsed_time(self, other):
        return other.t - self.t


class FakeCuda:
    Event = FakeEvent

    @staticmethod
    def synchronize():
        pass


class FakeTorch:
    cuda = FakeCuda
    float64 = "float64"

    @staticmethod
    def device(kind, index):
        return (kind, index)

    class _T(list):
        def tolist(self):
            return [list(r) for r in self]

    @staticmethod
    def tensor(data, device=None, dtype=None):
        return FakeTorch._T([list(r) for r in data])


class NoClocks:
    def __init__(self, idx):
        pass

    def start(self):
        pass

    def stop(self):
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}


def test_interleaved_blocks_order_and_times(monkeypatch):
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setattr(bench, "ClockSampler", NoClocks)
    monkeypatch.setattr(bench.time, "sleep", lambda s: None)
    log = []
    cost = {"a": 1.0, "b": 2.0, "c": 3.0}  # fake ms per step of each variant

    def leg(name):
        def step(i, ti):
            log.append((name, i, ti))
            FakeEvent.clock[0] += cost[name]
        return step

    def rewind():
        log.append(("rewind",))

    W, K, R = 3, 4, 2
    times, clk = bench.interleaved_blocks(FakeTorch, None, 1, W, K, [leg("a"), leg("b"), leg("c")], 0, R, rewind)
    want = [("a", i, None) for i in range(W)]
    want += [("b", W, 0), ("rewind",), ("c", W, 0), ("rewind",)]
    for _ in range(R):
        for name in "abc":
            want += [(name, W + i, i) for i in range(K)] + [("rewind",)]
    assert log == want
    assert times == [[1.0] * R, [2.0] * R, [3.0] * R]
    assert clk["reasons"] == ["unavailable"]
