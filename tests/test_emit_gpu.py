"""Projects emitted by `tfb200-opt --tensixflow-emit-cuda` build and pass on the GPU.

Each case plans a small graph of one kind (fused MLP, streamed decode MLP, fused
RMSNorm+MatMul, plain matmul), emits the project, and runs its run.sh: the
host program's TENSIXFLOW_RESULT must say pass and run.sh must print
{"status":"pass","backend":"b200",...} with exit status 0.
"""

import json
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
TOOL = ROOT / "tt-flow_b200" / "bin" / "tfb200-opt"

CASES = {
    "mlp": """tensixflow.func @mlp(%x: tensor<512x768xbf16>, %g: tensor<768xbf16>, %w1: tensor<768x1536xbf16>, %b1: tensor<1536xbf16>, %w2: tensor<1536x768xbf16>, %r: tensor<512x768xbf16>) -> tensor<512x768xbf16> {
  %0 = tensixflow.fused_mlp %x, %g, %w1, %b1, %w2, %r {epsilon = 1.0e-05 : f32} : tensor<512x768xbf16>, tensor<768xbf16>, tensor<768x1536xbf16>, tensor<1536xbf16>, tensor<1536x768xbf16>, tensor<512x768xbf16> -> tensor<512x768xbf16>
  tensixflow.return %0 : tensor<512x768xbf16>
}""",
    "decode": """tensixflow.func @decode(%x: tensor<16x1024xbf16>, %g: tensor<1024xbf16>, %w1: tensor<1024x4096xbf16>, %b1: tensor<4096xbf16>, %w2: tensor<4096x1024xbf16>, %r: tensor<16x1024xbf16>) -> tensor<16x1024xbf16> {
  %0 = tensixflow.fused_mlp %x, %g, %w1, %b1, %w2, %r {epsilon = 1.0e-05 : f32} : tensor<16x1024xbf16>, tensor<1024xbf16>, tensor<1024x4096xbf16>, tensor<4096xbf16>, tensor<4096x1024xbf16>, tensor<16x1024xbf16> -> tensor<16x1024xbf16>
  tensixflow.return %0 : tensor<16x1024xbf16>
}""",
    "rmsnorm_matmul": """tensixflow.func @rm(%x: tensor<300x512xbf16>, %g: tensor<512xbf16>, %w: tensor<512x640xbf16>) -> tensor<300x640xbf16> {
  %0 = tensixflow.rmsnorm %x, %g {epsilon = 1.0e-05 : f32} : tensor<300x512xbf16>, tensor<512xbf16> -> tensor<300x512xbf16>
  %1 = tensixflow.matmul %0, %w : tensor<300x512xbf16> x tensor<512x640xbf16> -> tensor<300x640xbf16>
  tensixflow.return %1 : tensor<300x640xbf16>
}""",
    "matmul": """tensixflow.func @mm(%a: tensor<256x512xbf16>, %b: tensor<512x1024xbf16>) -> tensor<256x1024xbf16> {
  %0 = tensixflow.matmul %a, %b : tensor<256x512xbf16> x tensor<512x1024xbf16> -> tensor<256x1024xbf16>
  tensixflow.return %0 : tensor<256x1024xbf16>
}""",
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_emitted_project_passes_on_gpu(tmp_path, name):
    src = tmp_path / f"{name}.mlir"
    src.write_text(CASES[name])
    out = tmp_path / "project"
    r = subprocess.run([str(TOOL), "--tensixflow-fuse-rmsnorm-matmul", "--tensixflow-plan-noc-sharding",
                        f"--tensixflow-emit-cuda=output-dir={out}", str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run(["bash", str(out / "run.sh")], capture_output=True, text=True, timeout=600,
                       env={"TFB200_ROOT": str(ROOT), "PATH": "/usr/bin:/bin:/usr/local/cuda/bin"})
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    last = json.loads(r.stdout.strip().splitlines()[-1])
    assert last["status"] == "pass" and last["backend"] == "b200" and last["pcc"] >= 0.9999
