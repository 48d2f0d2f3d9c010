"""The tensixflow front end on the B200 backend (CPU only).

* The reference's own lit tests for the dialect, the verifiers and the fusion
  passes run unchanged through `tfb200-opt` and FileCheck (when the
  environment variable TENSIXFLOW_REFERENCE names a tt-flow source tree; they
  are skipped otherwise).
* This backend's lit tests (tests/lit) pin the B200 planner's schedule and
  emission attributes, device selection and the fused_mlp verifier.
* The plan JSON matches the reference's plan schema (required keys, no extra
  keys, JSON types, enums), through a digest of that schema committed in
  tests/golden (tests/golden/make_schema_digest.py).
* The planner's time model agrees with the measured kernels.
"""

import ctypes
import json
import os
import subprocess
from pathlib import Path

import pytest

import litrun

ROOT = Path(__file__).resolve().parents[1]
# The reference's lit files are read from a tt-flow source tree named by
# TENSIXFLOW_REFERENCE (its root directory); those tests are skipped without it.
_REF_ROOT = os.environ.get("TENSIXFLOW_REFERENCE")
REF_TESTS = Path(_REF_ROOT) / "test" / "Tensixflow" if _REF_ROOT else None
# Reference lit files whose RUN lines exercise what this backend implements
# (parsing/printing, verifiers, fusion passes, bare-TTIR import). RUN lines with
# flags this backend does not implement (--tensixflow-infer-tile-layout, the
# Tensix tile layouts of the n150 family) are skipped by the runner.
# plan_noc_sharding.mlir checks n150 Tensix planner numbers, which the B200
# planner replaces; the other files test Tenstorrent lowering or TT-Metalium
# emission.
REF_FILES = ["attrs.mlir", "dialect_parse.mlir", "smoke.mlir", "ops.mlir", "matmul.mlir", "rmsnorm.mlir",
             "shape_inference.mlir", "fused_ops.mlir", "fuse_rmsnorm_matmul.mlir", "fuse_mlp.mlir",
             "fusion_tracking.mlir", "import_ttir.mlir", "import_ttir_negative.mlir", "canonicalize.mlir"]


@pytest.fixture(scope="module", autouse=True)
def tool():
    if not litrun.TOOL.exists():
        subprocess.run(["make", "-C", str(ROOT / "tt-flow_b200"), "bin/tfb200-opt"], check=True, capture_output=True)
    if litrun.filecheck() is None:
        pytest.skip("FileCheck (shipped with triton) not available")
    return litrun.TOOL


@pytest.mark.parametrize("name", REF_FILES)
def test_reference_lit_file(name):
    if REF_TESTS is None:
        pytest.skip("TENSIXFLOW_REFERENCE (a tt-flow source tree) is not set")
    path = REF_TESTS / name
    if not path.exists():
        pytest.skip(f"{path} is not present")
    r = litrun.run_file(path)
    assert r["ran"] > 0
    assert not r["failed"], r["failed"]


@pytest.mark.parametrize("path", sorted((ROOT / "tests" / "lit").glob("*.mlir")), ids=lambda p: p.name)
def test_b200_lit_file(path):
    r = litrun.run_file(path)
    assert r["ran"] > 0 and not r["skipped"], r
    assert not r["failed"], r["failed"]


def _opt(text, *flags):
    p = subprocess.run([str(litrun.TOOL), *flags], input=text, capture_output=True, text=True)
    return p.returncode, p.stdout, p.stderr


def _check(value, schema, where="plan"):
    t = schema.get("type")
    pytypes = {"object": dict, "array": list, "string": str, "boolean": bool, "number": (int, float),
               "integer": int}
    if t:
        assert isinstance(value, pytypes[t]) and not (t == "integer" and isinstance(value, bool)), where
    if "enum" in schema:
        assert value in schema["enum"], (where, value)
    if t == "object":
        for k in schema["required"]:
            assert k in value, f"{where}: missing {k}"
        if schema["additional"] is False:
            extra = set(value) - set(schema["properties"])
            assert not extra, f"{where}: unexpected keys {extra}"
        for k, v in value.items():
            if k in schema["properties"]:
                _check(v, schema["properties"][k], f"{where}.{k}")
    if t == "array" and "items" in schema:
        for i, v in enumerate(value):
            _check(v, schema["items"], f"{where}[{i}]")


@pytest.mark.parametrize("lit", ["b200_plan_rmsnorm_matmul.mlir", "b200_plan_mlp.mlir", "b200_plan_decode.mlir"])
def test_plan_json_matches_reference_schema(lit):
    text = (ROOT / "tests" / "lit" / lit).read_text()
    rc, out, err = _opt(text, "--tensixflow-fuse-rmsnorm-matmul", "--tensixflow-to-json")
    assert rc == 0, err
    plan = json.loads(out)
    schema = json.loads((ROOT / "tests" / "golden" / "plan_schema_digest.json").read_text())
    _check(plan, schema)
    assert plan["device"]["name"] == "b200" and plan["emission"]["fused_feasible"] is True
    assert plan["noc"]["multicast_bytes"] == 0


def test_unfusable_graph_plans_unfused():
    text = """tensixflow.func @lone(%a: tensor<4096x4096xbf16>, %b: tensor<4096x4096xbf16>) -> tensor<4096x4096xbf16> {
  %0 = tensixflow.matmul %a, %b : tensor<4096x4096xbf16> x tensor<4096x4096xbf16> -> tensor<4096x4096xbf16>
  tensixflow.return %0 : tensor<4096x4096xbf16>
}"""
    rc, out, err = _opt(text, "--tensixflow-fuse-rmsnorm-matmul", "--tensixflow-to-json")
    assert rc == 0, err
    plan = json.loads(out)
    assert plan["fusion"] == "none" and plan["estimated_dram_reads_saved"] == 0
    assert plan["perf"]["bottleneck"] == "compute"


def test_parse_errors_are_reported():
    rc, out, err = _opt("tensixflow.func @f(%a: tensor<4xbf16>) -> tensor<4xbf16> {\n  %0 = tensixflow.gelu %b : tensor<4xbf16>\n}")
    assert rc != 0 and "undefined value" in err


def test_c_abi_matches_tool():
    from tfb200 import _lib as L

    lib = L.lib()
    text = (ROOT / "tests" / "lit" / "b200_plan_mlp.mlir").read_text()
    flags = "--tensixflow-fuse-rmsnorm-matmul --tensixflow-plan-noc-sharding --tensixflow-allocate-circular-buffers"
    need = ctypes.c_size_t(0)
    assert lib.tfb200_opt(text.encode(), flags.encode(), None, 0, ctypes.byref(need)) == L.TFB200_ENOSPC
    buf = ctypes.create_string_buffer(need.value)
    assert lib.tfb200_opt(text.encode(), flags.encode(), buf, need.value, None) == L.TFB200_OK
    rc, out, _ = _opt(text, *flags.split())
    assert rc == 0 and buf.value.decode() == out
    assert lib.tfb200_opt(b"tensixflow.func @f(", b"", None, 0, None) == L.TFB200_EINVAL
    assert b"error" in lib.tfb200_last_error()


def _plan(doc: str):
    from tfb200 import _lib as L

    lib = L.lib()
    need = ctypes.c_size_t(0)
    rc = lib.tfb200_plan(doc.encode(), None, 0, ctypes.byref(need))
    if rc != L.TFB200_ENOSPC:
        return rc, None, lib.tfb200_last_error().decode()
    buf = ctypes.create_string_buffer(need.value)
    rc = lib.tfb200_plan(doc.encode(), buf, need.value, None)
    return rc, buf.value.decode(), lib.tfb200_last_error().decode()


@pytest.mark.parametrize("lit", ["b200_plan_rmsnorm_matmul.mlir", "b200_plan_mlp.mlir", "b200_plan_decode.mlir"])
def test_plan_json_round_trips_through_tfb200_plan(lit):
    """A plan written by this front end, re-planned from its JSON, comes back unchanged."""
    text = (ROOT / "tests" / "lit" / lit).read_text()
    rc, out, err = _opt(text, "--tensixflow-fuse-rmsnorm-matmul", "--tensixflow-to-json")
    assert rc == 0, err
    rc2, again, err2 = _plan(out)
    assert rc2 == 0, err2
    assert again == out


def _reference_style_doc(fusion, shapes):
    """A plan document as the reference's translate tool writes it for an n150: function arguments arg0..argN."""
    tensors = [{"name": f"arg{i}", "shape": s, "dtype": "bf16", "placement": "DRAM"} for i, s in enumerate(shapes)]
    doc = {"graph_id": "g", "device": {"name": "n150", "arch": "wormhole_b0", "grid_x": 8, "grid_y": 8,
                                        "l1_usable_bytes": 1499136, "flops_per_cycle_per_core": 2048,
                                        "dram_bandwidth_bytes_per_second": 288000000000},
           "tensors": tensors, "layout": {"activation_sharding": "row-major", "weight_strategy": "replicate"},
           "shard_grid": {"grid_y": 8, "grid_x": 8}, "cb_specs": [], "noc": {}, "emission": {}, "perf": {}, "viz": {}}
    if fusion:
        doc["fusion"] = fusion
    return json.dumps(doc)


@pytest.mark.parametrize("fusion,shapes,want", [
    ("fused_mlp", [[8192, 4096], [4096], [4096, 16384], [16384], [16384, 4096], [8192, 4096]], "fused_mlp"),
    (None, [[8192, 4096], [4096], [4096, 16384], [16384], [16384, 4096], [8192, 4096]], "fused_mlp"),
    ("fused_rmsnorm_matmul", [[2, 4096, 4096], [4096], [4096, 6144]], "fused_rmsnorm_matmul"),
    (None, [[8192, 4096], [4096], [4096, 6144]], "fused_rmsnorm_matmul"),
    (None, [[256, 512], [512, 1024]], "none"),
    ("fused_mlp", [[32, 8192], [8192], [8192, 28672], [28672], [28672, 8192], [32, 8192]], "fused_mlp"),
])
def test_tfb200_plan_replans_reference_documents(fusion, shapes, want):
    rc, out, err = _plan(_reference_style_doc(fusion, shapes))
    assert rc == 0, err
    plan = json.loads(out)
    schema = json.loads((ROOT / "tests" / "golden" / "plan_schema_digest.json").read_text())
    _check(plan, schema)
    assert plan["device"]["name"] == "b200" and plan["fusion"] == want
    assert [t["name"] for t in plan["tensors"]] == [f"arg{i}" for i in range(len(shapes))]
    assert plan["emission"]["fused_feasible"] is True
    if shapes[0][0] == 32:
        assert plan["emission"]["mapping"] == "stream-k-swap-ab"


@pytest.mark.parametrize("doc,msg", [
    ('{"tensors": [1, 2', "1:18"),
    ('[]', "not an object"),
    ('{"graph_id": "g"}', "tensors"),
    ('{"tensors": [{"name": "arg0", "shape": [4, 8]}, {"name": "arg1", "shape": [9, 3]}], "fusion": "fused_mlp"}',
     "fused_mlp needs"),
    ('{"tensors": [{"name": "arg0", "shape": [4, 8]}, {"name": "arg1", "shape": [8, 3]}], "fusion": "bogus"}',
     "unknown fusion"),
    ('{"tensors": [{"name": "arg0", "shape": [4, 8.5]}]}', "not a non-negative integer"),
])
def test_tfb200_plan_rejects_bad_documents(doc, msg):
    from tfb200 import _lib as L

    rc, _, err = _plan(doc)
    assert rc == L.TFB200_EINVAL and msg in err, err


# Measured on B200 with CUDA events (bench.py, one CUDA graph of the timed steps): fused MLP
# 8192x4096x16384 1.506-1.715 ms per step (box to box), fused RMSNorm+QKV 8192x4096x6144
# 0.292-0.298 ms, decode MLP 32x8192x28672 0.154-0.158 ms.
MEASURED_S = {"b200_plan_mlp.mlir": 1.56e-3, "b200_plan_rmsnorm_matmul.mlir": 0.295e-3,
              "b200_plan_decode.mlir": 0.156e-3}


@pytest.mark.parametrize("lit", sorted(MEASURED_S))
def test_time_model_tracks_measurement(lit):
    text = (ROOT / "tests" / "lit" / lit).read_text()
    rc, out, err = _opt(text, "--tensixflow-fuse-rmsnorm-matmul", "--tensixflow-to-json")
    assert rc == 0, err
    plan = json.loads(out)
    est_s = plan["perf"]["est_cycles"] / 1.965e9
    assert abs(est_s / MEASURED_S[lit] - 1.0) < 0.15, (est_s, MEASURED_S[lit])


# Kernel time per step from the ncu captures summarised in profiles/ (every kernel of the step, serialised,
# cold L2): fused MLP 8192x4096x16384 = k_gemm_pair (8285.4 + 8274.3) us / 12 steps + k_rms_prep_reg 246.9 us
# / 12 steps; decode MLP 32x8192x28672 = k_stream 91.2 + 85.7 us + k_rms_prep_rows 6.5 us.
NCU_S = {"b200_plan_mlp.mlir": (8285.4 + 8274.3 + 246.9) / 12 * 1e-6, "b200_plan_decode.mlir": (91.2 + 85.7 + 6.5) * 1e-6}


@pytest.mark.parametrize("lit", sorted(NCU_S))
def test_time_model_tracks_ncu(lit):
    """The roofline model against the ncu-measured kernel time of the same step."""
    text = (ROOT / "tests" / "lit" / lit).read_text()
    rc, out, err = _opt(text, "--tensixflow-fuse-rmsnorm-matmul", "--tensixflow-to-json")
    assert rc == 0, err
    est_s = json.loads(out)["perf"]["est_cycles"] / 1.965e9
    assert abs(est_s / NCU_S[lit] - 1.0) < 0.15, (est_s, NCU_S[lit])


def test_lit_runner_not_inverts_only_the_tool(tmp_path):
    """`not tool | FileCheck` must still fail when FileCheck fails: a wrong CHECK is reported."""
    bad = tmp_path / "bad.mlir"
    bad.write_text("// RUN: not tensixflow-opt --allow-unregistered-dialect --tensixflow-import-ttir %s 2>&1 | "
                   "FileCheck %s\n// CHECK: this text is not in the diagnostic\n"
                   "func.func @f(%arg0: tensor<?x4xbf16>) -> tensor<?x4xbf16> {\n  return %arg0 : tensor<?x4xbf16>\n}\n")
    r = litrun.run_file(bad)
    assert r["ran"] == 1 and len(r["failed"]) == 1
    good = tmp_path / "good.mlir"
    good.write_text(bad.read_text().replace("this text is not in the diagnostic", "has a dynamic shape"))
    r = litrun.run_file(good)
    assert r["ran"] == 1 and not r["failed"], r


def _emit(tmp_path, lit, *extra):
    out = tmp_path / "project"
    text = (ROOT / "tests" / "lit" / lit).read_text()
    rc, _, err = _opt(text, "--tensixflow-fuse-rmsnorm-matmul", *extra, f"--tensixflow-emit-cuda=output-dir={out}")
    return rc, out, err


@pytest.mark.parametrize("lit", ["b200_plan_mlp.mlir", "b200_plan_rmsnorm_matmul.mlir", "b200_plan_decode.mlir"])
def test_emit_cuda_project_writes_a_buildable_project(tmp_path, lit):
    rc, out, err = _emit(tmp_path, lit, "--tensixflow-plan-noc-sharding")
    assert rc == 0, err
    for f in ("host.cpp", "Makefile", "run.sh", "README.md", "plan.json"):
        assert (out / f).stat().st_size > 0, f
    host = (out / "host.cpp").read_text()
    assert "TENSIXFLOW_RESULT" in host and "kPccThreshold" in host and "std::mt19937" in host
    assert "tfb200_fused_" in host
    assert "fused_feasible | true" in (out / "README.md").read_text()
    assert json.loads((out / "plan.json").read_text())["emission"]["fused_feasible"] is True
    assert 'TENSIXFLOW_RESULT {"status"' in (out / "run.sh").read_text()
    # The host program compiles and links against the library without a GPU.
    import shutil

    if shutil.which("g++") and Path("/usr/local/cuda/include/cuda_runtime.h").exists():
        r = subprocess.run(["make", "-s", "-C", str(out), "host", f"TFB200_ROOT={ROOT}"], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        assert (out / "host").exists()


def test_emit_cuda_refuses_an_unplanned_module(tmp_path):
    rc, out, err = _emit(tmp_path, "b200_plan_mlp.mlir")
    assert rc != 0 and "run --tensixflow-plan-noc-sharding before" in err
    assert not out.exists()


def test_emit_metalium_flag_names_the_cuda_project_for_b200(tmp_path):
    out = tmp_path / "p2"
    text = (ROOT / "tests" / "lit" / "b200_plan_rmsnorm_matmul.mlir").read_text()
    rc, _, err = _opt(text, "--tensixflow-plan-noc-sharding", f"--tensixflow-emit-metalium=output-dir={out}")
    assert rc == 0, err
    assert (out / "host.cpp").exists()
    rc, _, err = _opt(text, "--tensixflow-plan-noc-sharding", "--tensixflow-emit-cuda=dir=x")
    assert rc != 0 and "expects output-dir=" in err


def test_emit_cuda_refuses_an_infeasible_plan(tmp_path):
    text = """tensixflow.func @dyn(%x: tensor<?x4096xbf16>, %gamma: tensor<4096xbf16>, %w: tensor<4096x6144xbf16>) -> tensor<?x6144xbf16> {
  %0 = tensixflow.rmsnorm %x, %gamma {epsilon = 1.0e-05 : f32} : tensor<?x4096xbf16>, tensor<4096xbf16> -> tensor<?x4096xbf16>
  %1 = tensixflow.matmul %0, %w : tensor<?x4096xbf16> x tensor<4096x6144xbf16> -> tensor<?x6144xbf16>
  tensixflow.return %1 : tensor<?x6144xbf16>
}"""
    out = tmp_path / "never"
    rc, _, err = _opt(text, "--tensixflow-plan-noc-sharding", f"--tensixflow-emit-cuda=output-dir={out}")
    assert rc != 0 and "not fused_feasible" in err
    assert not out.exists()
