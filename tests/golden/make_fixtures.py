"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that has the tensixflow sources (the reference's Python
package is imported unmodified from ``<reference>/python``):

    python tests/golden/make_fixtures.py --reference <tt-flow source tree>

It writes ``golden_vectors.npz`` holding, for every workload:

* the sha256 of each seeded input tensor (bf16 encodings), which pins the
  workload generator in ``tt-flow_b200/tfb200/workloads.py``;
* the reference's fp32 golden output (``golden.fused_rmsnorm_matmul``,
  ``golden.fused_mlp`` with exact-erf GELU, or ``golden.matmul``) for the whole
  output on the small workloads and for a few rows on the large ones (rows are
  independent in this computation, so a row of the full workload is a full
  check of that row);

and ``rounding_vectors.npz``: the reference's ``rounding.to_bf16`` applied to
its 1000-value consistency vector and to the special values its tests use.

Nothing on the GPU box reads the reference: the tests only read these files.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "tt-flow_b200"))

from tfb200 import workloads as W  # noqa: E402

# Rows of the large workloads whose golden output is stored.
SAMPLE_ROWS = {
    "matmul_256x512x1024": [0, 1, 127, 255],
    "qkv_8192x4096x6144": [0, 1, 4097, 8191],
    "mlp_8192x4096x16384": [0, 3, 5000, 8191],
    "decode_mlp_32x8192x28672": [0, 7, 16, 31],
}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TENSIXFLOW_REFERENCE"),
                    help="root of a tt-flow source tree (default: $TENSIXFLOW_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the tt-flow source tree with --reference or TENSIXFLOW_REFERENCE")
    sys.path.insert(0, str(Path(args.reference) / "python"))
    from tensixflow import golden as G  # the reference, unmodified
    from tensixflow import rounding as R

    f32 = W.bf16_to_f32
    out: dict[str, np.ndarray] = {}
    for name, wl in W.WORKLOADS.items():
        t = W.generate(name)
        for k, v in t.items():
            out[f"{name}/sha/{k}"] = np.frombuffer(bytes.fromhex(sha(v)), dtype=np.uint8)
        rows = SAMPLE_ROWS.get(name)
        eps = wl.eps
        if wl.kind == "matmul":
            a = f32(t["a"])
            if rows is not None:
                a = a[rows]
            y = G.matmul(a, f32(t["b"]))
        elif wl.kind == "fused_rmsnorm_matmul":
            x = f32(t["x"])
            if rows is not None:
                x = x[rows]
            y = G.fused_rmsnorm_matmul(x, f32(t["gamma"]), f32(t["w"]), eps)
        else:
            x = f32(t["x"])
            if rows is not None:
                x = x[rows]
            y = G.fused_mlp(x, f32(t["gamma"]), f32(t["w1"]), f32(t["b1"]), f32(t["w2"]), x, eps)
        out[f"{name}/golden"] = np.asarray(y, dtype=np.float32)
        out[f"{name}/rows"] = np.asarray(rows if rows is not None else [], dtype=np.int64)
        print(name, y.shape, float(np.abs(y).max()))
    np.savez_compressed(HERE / "golden_vectors.npz", **out)

    cons = R.consistency_inputs()
    specials = np.array([0x3F800000, 0x3F000000, 0xC0000000, 0x3FC00000, 0x40000000, 0x00000000,
                         0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00001, 0x7F800001,
                         0x3F808000, 0x3F818000, 0x3F80D1B7, 0x7F7FFFFF, 0x00000001, 0x807FFFFF],
                        dtype=np.uint32)
    np.savez_compressed(
        HERE / "rounding_vectors.npz",
        consistency_in=cons,
        consistency_out=R.float_to_bits(R.to_bf16(R.bits_to_float(cons))),
        specials_in=specials,
        specials_out=R.float_to_bits(R.to_bf16(R.bits_to_float(specials))),
    )
    # The reference's hand-computed vectors (python/tensixflow/tests/test_golden.py:34-65),
    # re-evaluated through the reference golden so the fixture holds its exact bits.
    kat = {
        "rmsnorm_x": np.array([[1.0, 1.0], [2.0, 2.0]], np.float32),
        "rmsnorm_gamma": np.array([3.0, 1.0], np.float32),
        "matmul_a": np.array([[1.0, 2.0], [3.0, 4.0]], np.float32),
        "matmul_b": np.array([[5.0, 6.0], [7.0, 8.0]], np.float32),
        "gelu_x": np.array([0.0, 1.0, -1.0, 2.0, -3.5, 0.125, 6.0, -0.7], np.float32),
    }
    kat["rmsnorm_out"] = G.rmsnorm(kat["rmsnorm_x"], kat["rmsnorm_gamma"], eps=0.0)
    kat["matmul_out"] = G.matmul(kat["matmul_a"], kat["matmul_b"])
    kat["gelu_out"] = G.gelu(kat["gelu_x"])
    rng = np.random.default_rng(2026)
    fx = rng.standard_normal((5, 12)).astype(np.float32)
    fg = rng.standard_normal(12).astype(np.float32)
    fw1 = rng.standard_normal((12, 20)).astype(np.float32)
    fb1 = rng.standard_normal(20).astype(np.float32)
    fw2 = rng.standard_normal((20, 12)).astype(np.float32)
    fr = rng.standard_normal((5, 12)).astype(np.float32)
    kat.update(mlp_x=fx, mlp_gamma=fg, mlp_w1=fw1, mlp_b1=fb1, mlp_w2=fw2, mlp_res=fr,
               mlp_out=G.fused_mlp(fx, fg, fw1, fb1, fw2, fr, 1e-6),
               frm_out=G.fused_rmsnorm_matmul(fx, fg, fw1, 1e-6))
    np.savez_compressed(HERE / "kat_vectors.npz", **kat)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
