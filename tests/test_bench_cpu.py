"""The reference arm of bench.py (the reference's CPU golden, restated) keeps the
bench contract: one JSON line with the metric, its unit, the timing fields, the
CPU-baseline description and an e2e block without host transfers; under
torchrun only rank 0 prints. Runs on the host cores, on the small MLP workload."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env=None, *args):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                          capture_output=True, text=True, env=env, timeout=300, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    r = _run(None, "--workload", "mlp_block_small", "--steps", "2", "--warmup", "1", "--ref-rows", "64")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["value"] > 0
    for key in ("metric", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling", "vs_baseline",
                "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 2 and d["warmup"] == 1 and d["higher_is_better"] is True
    assert d["scaling"] == "strong"  # the same config as the GPU arm: the workload's rows split over the GPUs
    assert d["config"]["workload"] == "mlp_block_small"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--workload", "mlp_block_small", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_traffic_table_names_real_workloads():
    """The per-launch DRAM traffic the GPU arm reports (from the ncu captures in profiles/) is keyed by workload
    name: every key must be a workload, and each figure must lie between a quarter of the step's algorithmic bytes
    and ten times them (a misplaced decimal or a figure for the wrong workload would fall outside)."""
    sys.path[:0] = [str(ROOT), str(ROOT / "tt-flow_b200")]
    import bench
    from tfb200 import workloads as W

    assert bench.TRAFFIC_BYTES_PER_LAUNCH
    for name, traffic in bench.TRAFFIC_BYTES_PER_LAUNCH.items():
        assert name in W.WORKLOADS, name
        step_bytes = W.algorithmic_bytes(name)
        assert step_bytes / 4 < traffic < 10 * step_bytes, (name, traffic, step_bytes)
