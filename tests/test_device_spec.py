"""The B200 device entry (tt-flow_b200/spec/devices.json, in the layout of the
reference's spec/devices.json) is the source of the planner's device figures
and time model: the plan JSON's device block and its time estimate must follow
from the entry, every figure group names a listed source, and the derived
figures agree with each other."""

import json
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SPEC = json.loads((ROOT / "tt-flow_b200" / "spec" / "devices.json").read_text())
B200 = SPEC["devices"]["b200"]
OPT = ROOT / "tt-flow_b200" / "bin" / "tfb200-opt"


@pytest.fixture(scope="module", autouse=True)
def tool():
    if not OPT.exists():
        subprocess.run(["make", "-C", str(ROOT / "tt-flow_b200"), "bin/tfb200-opt"], check=True, capture_output=True)


def _plan(lit_name):
    r = subprocess.run([str(OPT), "--tensixflow-device=b200", "--tensixflow-fuse-rmsnorm-matmul",
                        "--tensixflow-plan-noc-sharding", "--tensixflow-to-json", str(ROOT / "tests" / "lit" / lit_name)],
                       capture_output=True, text=True, check=True)
    return json.loads(r.stdout)


def test_every_group_names_a_listed_source():
    ids = {s["id"] for s in SPEC["sources"]}
    assert SPEC["default_device"] == "b200"
    for group, src in B200["sources"].items():
        assert group in B200, group
        assert src in ids, (group, src)
    assert ids == set(B200["sources"].values())  # no unused source


def test_derived_figures_agree():
    assert B200["die"]["sms"] == B200["die"]["dies"] * B200["die"]["sms_per_die"] == 148
    assert B200["compute"]["grid_x"] * B200["compute"]["grid_y"] == B200["die"]["sms"]
    assert B200["tmem"]["bytes_per_sm"] == B200["tmem"]["columns"] * B200["tmem"]["lanes"] * 4
    assert B200["l1"]["usable_bytes"] <= B200["l1"]["nominal_bytes"]
    peak = B200["matrix_unit"]["flops_per_cycle_per_core"] * B200["die"]["sms"] * 1.855e9  # boost clock of the rating
    assert abs(peak / B200["matrix_unit"]["dense_bf16_flops_per_second"] - 1) < 0.01
    m = B200["measured"]
    assert m["bf16_flops_per_second_sustained"] < m["bf16_flops_per_second"] < B200["matrix_unit"]["dense_bf16_flops_per_second"]
    assert m["hbm_bytes_per_second"] < B200["dram"]["bandwidth_bytes_per_second"]


@pytest.mark.parametrize("lit", ["b200_plan_mlp.mlir", "b200_plan_rmsnorm_matmul.mlir", "b200_plan_decode.mlir"])
def test_plan_device_block_and_time_model_follow_the_entry(lit):
    plan = _plan(lit)
    dev = plan["device"]
    assert dev["name"] == "b200" and dev["arch"] == B200["arch"]
    assert dev["grid_x"] == B200["compute"]["grid_x"] and dev["grid_y"] == B200["compute"]["grid_y"]
    assert dev["l1_usable_bytes"] == B200["l1"]["usable_bytes"]
    assert dev["flops_per_cycle_per_core"] == B200["matrix_unit"]["flops_per_cycle_per_core"]
    assert dev["dram_bandwidth_bytes_per_second"] == B200["dram"]["bandwidth_bytes_per_second"]
    assert f"B of {B200['l1']['usable_bytes']}" in plan["viz"]["cb_usage"]
    assert f"TMEM" in plan["viz"]["cb_usage"] and f"of {B200['tmem']['columns']} columns" in plan["viz"]["cb_usage"]
    # Time estimate: max(FLOPs / (measured bf16 x efficiency), HBM bytes / (measured copy bandwidth x efficiency))
    # + launches x launch time, in cycles of the entry's SM clock.
    shapes = {t["name"]: t["shape"] for t in plan["tensors"]}
    rows = 1
    for d in shapes["input"][:-1]:
        rows *= d
    k = shapes["input"][-1]
    if plan["fusion"] == "fused_mlp":
        h, n = shapes["w1"][1], shapes["w2"][1]
        flops = 2 * rows * k * h + 2 * rows * h * n
    else:
        flops = 2 * rows * k * shapes["weight"][1]
    hbm = plan["emission"]["dram_read_bytes"] + plan["emission"]["dram_write_bytes"]
    launches = int(re.match(r"(\d+) launches", plan["viz"]["timeline"]).group(1))
    model, meas = SPEC["model"], B200["measured"]
    est = max(flops / (meas["bf16_flops_per_second"] * model["tensor_efficiency"]),
              hbm / (meas["hbm_bytes_per_second"] * model["hbm_efficiency"])) + launches * model["launch_seconds"]
    assert abs(plan["perf"]["est_cycles"] - est * B200["clock_hz"]) <= 1


def test_python_lookup_reads_the_same_entry():
    import sys

    sys.path.insert(0, str(ROOT / "tt-flow_b200"))
    from tfb200 import devices

    d = devices.lookup("b200")
    assert devices.DEFAULT_DEVICE == "b200" and devices.lookup("hgx-b200") is d
    assert d.total_cores == 148 and d.cb_budget() == B200["l1"]["usable_bytes"]
    assert d.flops_per_cycle_per_core == B200["matrix_unit"]["flops_per_cycle_per_core"]
    assert d.measured_bf16_flops_per_second == B200["measured"]["bf16_flops_per_second"]
    assert devices.all_devices() == (d,)
    with pytest.raises(KeyError, match="valid devices: b200"):
        devices.lookup("n150")
