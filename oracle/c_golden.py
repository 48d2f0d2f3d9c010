"""ctypes wrapper of oracle/_build/liboracle.so, the C restatement of the
reference's emitted host golden (goldenRmsnorm / goldenMatmul / goldenMlp in
tensixflow lib/tensixflow/Codegen/EmitHost.cpp:727-762, 1176-1227).

Test infrastructure only. Build with ``make -C oracle``.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_build" / "liboracle.so"
_L = None


def _lib():
    global _L
    if _L is None:
        if not LIB.exists():
            raise RuntimeError(f"{LIB} missing: run `make -C {LIB.parents[1]}`")
        _L = ctypes.CDLL(str(LIB))
        P = ctypes.POINTER(ctypes.c_float)
        i64 = ctypes.c_int64
        _L.tfo_rmsnorm_bf16.argtypes = [P, P, i64, i64, ctypes.c_float, P]
        _L.tfo_matmul_bf16.argtypes = [P, P, i64, i64, i64, P]
        _L.tfo_mlp_bf16.argtypes = [P, P, P, P, P, P, i64, i64, i64, i64, ctypes.c_float, ctypes.c_int, P]
        _L.tfo_bf16_round.argtypes = [P, P, i64]
    return _L


def _p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rmsnorm_bf16(x, gamma, eps):
    x, g = _f(x), _f(gamma)
    out = np.empty_like(x)
    _lib().tfo_rmsnorm_bf16(_p(x), _p(g), x.shape[0], x.shape[1], eps, _p(out))
    return out


def matmul_bf16(a, b):
    a, b = _f(a), _f(b)
    out = np.empty((a.shape[0], b.shape[1]), np.float32)
    _lib().tfo_matmul_bf16(_p(a), _p(b), a.shape[0], a.shape[1], b.shape[1], _p(out))
    return out


def fused_rmsnorm_matmul_bf16(x, gamma, w, eps):
    """The emitted host golden of the fused RMSNorm+MatMul program."""
    return matmul_bf16(rmsnorm_bf16(x, gamma, eps), w)


def mlp_bf16(x, gamma, w1, b1, w2, residual, eps, gelu="erf"):
    """The emitted host golden of the fused MLP program (goldenMlp)."""
    x, g, w1, w2, r = _f(x), _f(gamma), _f(w1), _f(w2), _f(residual)
    b = _f(b1) if b1 is not None else None
    m, k = x.shape
    h, n = w1.shape[1], w2.shape[1]
    out = np.empty((m, n), np.float32)
    _lib().tfo_mlp_bf16(_p(x), _p(g), _p(w1), _p(b) if b is not None else None, _p(w2), _p(r), m, k, h, n, eps,
                        0 if gelu == "erf" else 1, _p(out))
    return out


def bf16_round(a):
    a = _f(a)
    out = np.empty_like(a)
    _lib().tfo_bf16_round(_p(a), _p(out), a.size)
    return out
