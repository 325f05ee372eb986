"""CPU test of bench.py's reference arm (`--impl reference`, the oracle port
of the reference's CPU path on the host cores): it runs without a GPU and
prints exactly one JSON line carrying the contract's keys, with the same
metric, unit and config object as the GPU arm, complete timed steps, and an
e2e entry that moves no bytes.  A reduced job (--seqs, --layers) keeps the
run short."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    sys.path.insert(0, ROOT)
    import bench
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1", "--seqs", "8", "--layers", "2"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [line for line in r.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT
    assert d["value"] > 0 and d["higher_is_better"] is True and (d["steps"], d["warmup"]) == (1, 1)
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # one GPU: rank 0's shard is the whole job, timed in complete steps with nothing scaled
    assert d["config"] == bench.config2_dict(8, 2, 1, bench.weak_rank_contexts(2, bench.parse_args([]).seed, 8, 1, 0),
                                             bench.CONFIGS[2])
    assert d["job_ms_per_step"] == d["ms_per_step"] and "no scaling" in cb["sample"]
    assert abs(d["value"] - 8 / (d["ms_per_step"] * 1e-3)) < 1e-6 * d["value"]


def test_reference_arm_under_torchrun_prints_once():
    """Launched like the driver's scaling run (torchrun, 2 ranks, 127.0.0.1):
    rank 0 alone prints one line, for the whole 2-GPU job; every rank exits 0."""
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", "29541", os.path.join(ROOT, "bench.py"),
                        "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1",
                        "--seqs", "8", "--layers", "2"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [line for line in r.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["config"]["seqs_per_gpu"] == 8
    # rank 0's shard is timed; one host runs the whole job, so the job's step is ~2x the shard's
    assert 1.8 < d["job_ms_per_step"] / d["ms_per_step"] < 2.2
    assert abs(d["value"] - 16 / (d["job_ms_per_step"] * 1e-3)) < 1e-6 * d["value"]
