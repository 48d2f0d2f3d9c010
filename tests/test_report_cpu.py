"""The plan report of the B200 backend (tfb200-report), with the contract of the
reference's report tool (tensixflow tools/tensixflow-report, tested by
python/tensixflow/tests/test_report.py): it validates a plan document by
re-deriving the emission block from the plan's own tensors and fusion, renders
a self-contained HTML page with a "Projected Emitted Path" section when they
agree, and refuses (non-zero exit, the field named on stderr, nothing written) a
stale emission byte count, an unknown mapping, or a plan without an emission
block. Plans come from tfb200-opt on this repository's lit inputs."""

import json
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
BIN = ROOT / "tt-flow_b200" / "bin"
LIT = ROOT / "tests" / "lit"


@pytest.fixture(scope="module", autouse=True)
def tools():
    if not (BIN / "tfb200-report").exists() or not (BIN / "tfb200-opt").exists():
        subprocess.run(["make", "-C", str(ROOT / "tt-flow_b200"), "bin/tfb200-opt", "bin/tfb200-report"],
                       check=True, capture_output=True)


def _plan(lit_name: str) -> dict:
    r = subprocess.run([str(BIN / "tfb200-opt"), "--tensixflow-device=b200", "--tensixflow-fuse-rmsnorm-matmul",
                        "--tensixflow-plan-noc-sharding", "--tensixflow-allocate-circular-buffers",
                        "--tensixflow-to-json", str(LIT / lit_name)], capture_output=True, text=True, check=True)
    return json.loads(r.stdout)


def _report(tmp_path: Path, plan: dict, name: str):
    plan_path = tmp_path / f"{name}.json"
    plan_path.write_text(json.dumps(plan))
    html = tmp_path / f"{name}.html"
    r = subprocess.run([str(BIN / "tfb200-report"), "--in", str(plan_path), "--out", str(html)],
                       capture_output=True, text=True)
    return r, html


@pytest.fixture(scope="module")
def rms_plan():
    return _plan("b200_plan_rmsnorm_matmul.mlir")


def test_report_renders_the_emitted_path_section(tmp_path, rms_plan):
    r, html = _report(tmp_path, rms_plan, "ok")
    assert r.returncode == 0, r.stderr
    page = html.read_text()
    assert "Projected Emitted Path" in page and "emitted-path item" in page
    assert rms_plan["emission"]["mapping"] in page


def test_report_rejects_a_stale_emitted_byte_count(tmp_path, rms_plan):
    stale = json.loads(json.dumps(rms_plan))
    stale["emission"]["dram_read_bytes"] += 1
    r, html = _report(tmp_path, stale, "stale")
    assert r.returncode != 0
    assert "emission.dram_read_bytes" in r.stderr
    assert not html.exists()


def test_report_rejects_an_unknown_emission_mapping(tmp_path, rms_plan):
    unknown = json.loads(json.dumps(rms_plan))
    unknown["emission"]["mapping"] = "mystery"
    r, html = _report(tmp_path, unknown, "unknown")
    assert r.returncode != 0
    assert "mapping" in r.stderr and "mystery" in r.stderr
    assert not html.exists()


def test_report_rejects_a_plan_without_an_emission_block(tmp_path, rms_plan):
    stripped = json.loads(json.dumps(rms_plan))
    del stripped["emission"]
    r, html = _report(tmp_path, stripped, "stripped")
    assert r.returncode != 0
    assert "emission" in r.stderr
    assert not html.exists()


def test_report_rejects_an_edited_feasibility(tmp_path, rms_plan):
    edited = json.loads(json.dumps(rms_plan))
    edited["emission"]["fused_feasible"] = not edited["emission"]["fused_feasible"]
    r, html = _report(tmp_path, edited, "edited")
    assert r.returncode != 0 and "emission.fused_feasible" in r.stderr
    assert not html.exists()


def test_report_refuses_a_plan_for_another_device(tmp_path, rms_plan):
    other = json.loads(json.dumps(rms_plan))
    other["device"]["name"] = "n150"
    r, html = _report(tmp_path, other, "other")
    assert r.returncode != 0 and "n150" in r.stderr
    assert not html.exists()


@pytest.mark.parametrize("lit_name,mapping", [("b200_plan_mlp.mlir", "persistent-cta-pair-tiles"),
                                              ("b200_plan_decode.mlir", "stream-k-swap-ab"),
                                              ("b200_plan_rmsnorm_matmul.mlir", "persistent-cta-pair-tiles")])
def test_report_accepts_every_planned_fused_path(tmp_path, lit_name, mapping):
    plan = _plan(lit_name)
    assert plan["emission"]["mapping"] == mapping
    r, html = _report(tmp_path, plan, lit_name)
    assert r.returncode == 0, r.stderr
    assert mapping in html.read_text()


def test_a_reference_plan_replanned_for_b200_passes_the_report(tmp_path):
    """A plan the reference wrote for an n150 (its translate tool names the tensors arg0..argN) is refused as it
    stands and accepted once tfb200_plan has re-planned it for the B200."""
    import ctypes
    import sys

    sys.path.insert(0, str(ROOT / "tt-flow_b200"))
    from tfb200 import _lib as L

    shapes = [[8192, 4096], [4096], [4096, 16384], [16384], [16384, 4096], [8192, 4096]]
    doc = {"graph_id": "g", "device": {"name": "n150", "arch": "wormhole_b0", "grid_x": 8, "grid_y": 8},
           "fusion": "fused_mlp", "emission": {"mapping": "blocked-reuse"},
           "tensors": [{"name": f"arg{i}", "shape": s, "dtype": "bf16", "placement": "DRAM"}
                       for i, s in enumerate(shapes)]}
    r, html = _report(tmp_path, doc, "n150")
    assert r.returncode != 0 and not html.exists()
    lib = L.lib()
    need = ctypes.c_size_t(0)
    assert lib.tfb200_plan(json.dumps(doc).encode(), None, 0, ctypes.byref(need)) == L.TFB200_ENOSPC
    buf = ctypes.create_string_buffer(need.value)
    assert lib.tfb200_plan(json.dumps(doc).encode(), buf, need.value, None) == L.TFB200_OK
    r, html = _report(tmp_path, json.loads(buf.value.decode()), "replanned")
    assert r.returncode == 0, r.stderr
    assert "persistent-cta-pair-tiles" in html.read_text()


def test_translate_name_reads_planned_ir_from_stdin():
    """tensixflow-translate --tensixflow-to-json reads the planned module on stdin; tfb200-translate (the same
    tool under that name, for TENSIXFLOW_TRANSLATE_BIN) gives the plan JSON tfb200-opt gives."""
    if not (BIN / "tfb200-translate").exists():
        subprocess.run(["make", "-C", str(ROOT / "tt-flow_b200"), "bin/tfb200-translate"], check=True,
                       capture_output=True)
    lit = LIT / "b200_plan_mlp.mlir"
    planned = subprocess.run([str(BIN / "tfb200-opt"), "--tensixflow-device=b200", "--tensixflow-fuse-rmsnorm-matmul",
                              "--tensixflow-plan-noc-sharding", "--tensixflow-allocate-circular-buffers", str(lit)],
                             capture_output=True, text=True, check=True).stdout
    via_translate = subprocess.run([str(BIN / "tfb200-translate"), "--tensixflow-to-json"], input=planned,
                                   capture_output=True, text=True, check=True).stdout
    assert json.loads(via_translate) == _plan("b200_plan_mlp.mlir")
