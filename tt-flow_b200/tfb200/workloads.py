"""Seeded synthetic workloads for the fused RMSNorm+MatMul and fused MLP path.

There is no public dataset behind these shapes; seeded synthetic tensors with the
stated shapes and distributions stand in for real activations and weights.

Generation rule (shared by the tests, the fixtures and the benchmark):
``rng = numpy.random.default_rng(seed)``; tensors are drawn in the listed order,
normals as ``rng.standard_normal(shape, dtype=float32) * std`` and uniforms as
``lo + (hi - lo) * rng.random(shape, dtype=float32)``, then rounded to bf16
(round to nearest even). Tensors are returned as uint16 bf16 encodings, row-major.
The residual of every MLP workload is X itself.

Workloads (names used throughout the repository):

* ``rmsnorm_matmul_small``  X[128,128] N(0,1), gamma[128] U(0.5,1.5),
  W[128,256] N(0,1/sqrt(128)), eps 1e-5, seed 0  (the reference's
  ``examples/rmsnorm_matmul_small.mlir`` shape)
* ``matmul_256x512x1024``   A[256,512] N(0,1), B[512,1024] N(0,1/sqrt(512)), seed 1
* ``matmul_padded``         A[100,50], B[50,100] drawn next from the same generator
  (the reference's ``examples/matmul_padded.mlir`` shape)
* ``qkv_8192x4096x6144``    X[8192,4096] N(0,1), gamma[4096] U(0.5,1.5),
  W[4096,6144] N(0,1/64), eps 1e-5, seed 2
* ``mlp_8192x4096x16384``   X[8192,4096], gamma[4096], W1[4096,16384] N(0,1/64),
  b1[16384] N(0,0.02), W2[16384,4096] N(0,1/128), tanh GELU, eps 1e-5, seed 3
* ``decode_mlp_32x8192x28672`` X[32,8192], gamma[8192], W1[8192,28672] N(0,1/90.5),
  b1[28672] N(0,0.02), W2[28672,8192] N(0,1/169), tanh GELU, eps 1e-5, seed 4
* ``mlp_block_small``       the reference's ``examples/mlp_block_small.mlir`` shape
  (M=K=H=N=128), same distributions as the MLP workload, seed 5
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

__all__ = ["Workload", "WORKLOADS", "generate", "bf16_bits", "bf16_to_f32", "flops", "algorithmic_bytes"]


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 encodings (uint16), round to nearest even, NaN kept quiet."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    lsb = (u >> 16) & 1
    r = ((u + np.uint32(0x7FFF) + lsb) >> 16).astype(np.uint16)
    q = ((u >> 16) & 0x8000 | 0x7FC0).astype(np.uint16)
    return np.where(nan, q, r)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    """bf16 encodings (uint16) -> fp32, exact."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass(frozen=True)
class Workload:
    name: str
    kind: str                      # "fused_rmsnorm_matmul" | "matmul" | "fused_mlp"
    seed: int
    dims: dict                     # M, K, N (and H for the MLP)
    eps: float = 1e-5
    gelu: str = "tanh"
    extra: dict = field(default_factory=dict)


WORKLOADS: dict[str, Workload] = {
    "rmsnorm_matmul_small": Workload("rmsnorm_matmul_small", "fused_rmsnorm_matmul", 0,
                                     {"M": 128, "K": 128, "N": 256}),
    "matmul_256x512x1024": Workload("matmul_256x512x1024", "matmul", 1, {"M": 256, "K": 512, "N": 1024}),
    "matmul_padded": Workload("matmul_padded", "matmul", 1, {"M": 100, "K": 50, "N": 100}),
    "qkv_8192x4096x6144": Workload("qkv_8192x4096x6144", "fused_rmsnorm_matmul", 2,
                                   {"M": 8192, "K": 4096, "N": 6144}),
    "mlp_8192x4096x16384": Workload("mlp_8192x4096x16384", "fused_mlp", 3,
                                    {"M": 8192, "K": 4096, "H": 16384, "N": 4096}),
    "decode_mlp_32x8192x28672": Workload("decode_mlp_32x8192x28672", "fused_mlp", 4,
                                         {"M": 32, "K": 8192, "H": 28672, "N": 8192}),
    "mlp_block_small": Workload("mlp_block_small", "fused_mlp", 5,
                                {"M": 128, "K": 128, "H": 128, "N": 128}),
}

_STD = {
    "mlp_8192x4096x16384": (1 / 64, 1 / 128),
    "decode_mlp_32x8192x28672": (1 / 90.5, 1 / 169),
}


def _normal(rng, shape, std):
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(std)


def _uniform(rng, shape, lo, hi):
    return np.float32(lo) + np.float32(hi - lo) * rng.random(shape, dtype=np.float32)


def generate(name: str, rows: tuple[int, int] | None = None) -> dict[str, np.ndarray]:
    """Draw a workload's tensors (bf16 encodings, uint16, row-major).

    ``rows`` = (start, stop) keeps only those rows of X (and of the residual) after
    drawing everything, so a row sample sees exactly the full workload's values.
    """
    w = WORKLOADS[name]
    d = w.dims
    rng = np.random.default_rng(w.seed)
    out: dict[str, np.ndarray] = {}
    if w.kind == "fused_rmsnorm_matmul":
        out["x"] = _normal(rng, (d["M"], d["K"]), 1.0)
        out["gamma"] = _uniform(rng, (d["K"],), 0.5, 1.5)
        out["w"] = _normal(rng, (d["K"], d["N"]), 1.0 / np.sqrt(d["K"]))
    elif w.kind == "matmul":
        a = _normal(rng, (256, 512), 1.0)
        b = _normal(rng, (512, 1024), 1.0 / np.sqrt(512))
        if name == "matmul_256x512x1024":
            out["a"], out["b"] = a, b
        else:
            out["a"] = _normal(rng, (100, 50), 1.0)
            out["b"] = _normal(rng, (50, 100), 1.0 / np.sqrt(50))
    elif w.kind == "fused_mlp":
        s1, s2 = _STD.get(name, (1.0 / np.sqrt(d["K"]), 1.0 / np.sqrt(d["H"])))
        out["x"] = _normal(rng, (d["M"], d["K"]), 1.0)
        out["gamma"] = _uniform(rng, (d["K"],), 0.5, 1.5)
        out["w1"] = _normal(rng, (d["K"], d["H"]), s1)
        out["b1"] = _normal(rng, (d["H"],), 0.02)
        out["w2"] = _normal(rng, (d["H"], d["N"]), s2)
    else:
        raise ValueError(w.kind)
    res = {k: bf16_bits(v) for k, v in out.items()}
    if w.kind == "fused_mlp":
        res["residual"] = res["x"]
    if rows is not None:
        lo, hi = rows
        for k in ("x", "residual", "a"):
            if k in res:
                res[k] = np.ascontiguousarray(res[k][lo:hi])
    return res


def flops(name: str) -> int:
    """Algorithmic FLOPs of one pass (2*M*N*K per GEMM; elementwise work excluded,
    as in the reference's cost model, docs/performance.md)."""
    w = WORKLOADS[name]
    d = w.dims
    if w.kind == "fused_mlp":
        return 2 * d["M"] * d["K"] * d["H"] + 2 * d["M"] * d["H"] * d["N"]
    return 2 * d["M"] * d["K"] * d["N"]


def algorithmic_bytes(name: str) -> int:
    """Bytes of one pass if every tensor crosses HBM exactly once (bf16)."""
    w = WORKLOADS[name]
    d = w.dims
    if w.kind == "fused_mlp":
        M, K, H, N = d["M"], d["K"], d["H"], d["N"]
        # the residual is X itself, so X is counted once
        return 2 * (M * K + K + K * H + H + H * N + M * N)
    if w.kind == "matmul":
        return 2 * (d["M"] * d["K"] + d["K"] * d["N"] + d["M"] * d["N"])
    return 2 * (d["M"] * d["K"] + d["K"] + d["K"] * d["N"] + d["M"] * d["N"])
