"""CPU oracle for the fused RMSNorm+MatMul and fused MLP path (test infrastructure).

This module is the checker, not the product: only the tests, the smoke check in
``__graft_entry__`` and the ``cpu_baseline`` leg of ``bench.py`` may import it.
The product path (the CUDA kernels behind ``libtfb200.so``) never calls it.

It restates, in numpy, the reference's fp32 golden and its bf16 rounding rule:

* ``rmsnorm``       follows tensixflow ``python/tensixflow/golden.py:41-53``
* ``matmul``        follows ``golden.py:56-60`` (numpy ``@`` in fp32)
* ``gelu`` (erf)    follows ``golden.py:63-77`` (libm ``math.erf`` per element,
                    evaluated in double and stored as fp32)
* ``fused_rmsnorm_matmul`` follows ``golden.py:97-102``
* ``fused_mlp``     follows ``golden.py:105-122`` (all intermediates fp32)
* ``to_bf16``       follows ``python/tensixflow/rounding.py:54-67,91-99``
                    (round to nearest even, NaN made a sign-keeping quiet NaN)

Two additions that the reference does not have, both marked as such:

* ``gelu_tanh`` -- the tanh form of GELU that the benchmark's MLP workloads ask
  for; the reference only implements the exact-erf form.
* ``emulate_device_*`` -- the same algebra with the bf16 roundings placed where
  the device kernels place them (x*gamma rounded to bf16 before the matmul, the
  GELU output rounded to bf16 between the GEMMs). It follows the reference's
  emitted host golden (``lib/tensixflow/Codegen/EmitHost.cpp:1176-1227``), which
  also rounds its intermediates. It is used to predict the kernel's error, never
  as the parity target.

Parity is pinned: ``tests/golden/`` holds vectors produced by importing the
reference's own ``golden.py`` and ``rounding.py`` (script committed beside them),
and ``tests/test_oracle.py`` checks this restatement against them bit for bit.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32
U32 = np.uint32

__all__ = [
    "to_bf16",
    "to_bf16_bits",
    "bf16_bits_to_f32",
    "rmsnorm",
    "matmul",
    "gelu",
    "gelu_fast",
    "gelu_tanh",
    "fused_rmsnorm_matmul",
    "fused_mlp",
    "emulate_device_fused_rmsnorm_matmul",
    "emulate_device_fused_mlp",
    "lcg_u32",
]


# --------------------------------------------------------------------------- bf16


def _nan_mask(bits: np.ndarray) -> np.ndarray:
    exp_all_ones = (bits & U32(0x7F800000)) == U32(0x7F800000)
    return exp_all_ones & ((bits & U32(0x007FFFFF)) != 0)


def _rne_bits(bits: np.ndarray) -> np.ndarray:
    """fp32 bit patterns -> bf16 (kept in the high half), round to nearest even.

    Same rule as rounding.py:54-67: a tie goes to the candidate whose bf16
    mantissa LSB is zero; NaN becomes (sign | 0x7FC00000); inf and -0 survive.
    Implemented here as an explicit round-up decision on the discarded half.
    """
    bits = np.asarray(bits, dtype=U32)
    keep = bits & U32(0xFFFF0000)
    dropped = bits & U32(0x0000FFFF)
    odd = (bits >> U32(16)) & U32(1)
    up = (dropped > U32(0x8000)) | ((dropped == U32(0x8000)) & (odd == U32(1)))
    out = np.where(up, keep + U32(0x10000), keep).astype(U32)
    quiet = (bits & U32(0x80000000)) | U32(0x7FC00000)
    return np.where(_nan_mask(bits), quiet, out).astype(U32)


def to_bf16(x) -> np.ndarray:
    """Round fp32 values to bf16 precision; the result is fp32 (rounding.py:91-99)."""
    a = np.asarray(x, dtype=F32)
    r = _rne_bits(a.view(U32)).view(F32)
    return r.reshape(a.shape)


def to_bf16_bits(x) -> np.ndarray:
    """bf16 encodings (uint16) of fp32 values, rounded to nearest even."""
    a = np.asarray(x, dtype=F32)
    return (_rne_bits(a.view(U32)) >> U32(16)).astype(np.uint16).reshape(a.shape)


def bf16_bits_to_f32(b) -> np.ndarray:
    """uint16 bf16 encodings -> fp32 values (exact)."""
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(U32) << U32(16)).view(F32)


def lcg_u32(n: int, seed: int) -> np.ndarray:
    """The 32-bit LCG (Numerical Recipes constants) of rounding.py:125-137, used by
    the reference's rounding consistency vector (seed 0x5EED2026, 1000 values)."""
    out = np.empty(n, dtype=U32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = s
    return out


# ---------------------------------------------------------------- fp32 golden ops


def rmsnorm(x, gamma, eps: float = 1e-6) -> np.ndarray:
    """x * (1 / sqrt(mean_k(x^2) + eps)) * gamma, every step in fp32 (golden.py:41-53)."""
    x = np.asarray(x, dtype=F32)
    g = np.asarray(gamma, dtype=F32)
    k = x.shape[-1]
    ms = np.sum(x * x, axis=-1, keepdims=True) / F32(k)
    inv = F32(1.0) / np.sqrt(ms + F32(eps))
    return x * inv * g


def matmul(a, b) -> np.ndarray:
    """fp32 a @ b (golden.py:56-60)."""
    return np.asarray(a, dtype=F32) @ np.asarray(b, dtype=F32)


def _erf_libm(v: np.ndarray) -> np.ndarray:
    flat = v.ravel()
    out = np.fromiter((math.erf(float(t)) for t in flat), dtype=F32, count=flat.size)
    return out.reshape(v.shape)


def gelu(x) -> np.ndarray:
    """Exact-erf GELU 0.5*x*(1+erf(x/sqrt(2))) in fp32 (golden.py:63-77).

    erf is libm's, evaluated per element in double and stored as fp32, as the
    reference does. O(n) Python calls: use for the sizes the tests need.
    """
    x = np.asarray(x, dtype=F32)
    arg = x / F32(math.sqrt(2.0))
    return (F32(0.5) * x * (F32(1.0) + _erf_libm(arg))).astype(F32)


def gelu_fast(x) -> np.ndarray:
    """gelu() with scipy's vectorised erf in place of the per-element libm loop.

    Not in the reference: used only where the libm loop would take minutes
    (row samples of the largest workloads). scipy's erf and libm's erf agree to a
    few fp32 ulp; tests/test_oracle.py bounds the gap.
    """
    from scipy.special import erf as _erf

    x = np.asarray(x, dtype=F32)
    arg = x / F32(math.sqrt(2.0))
    e = _erf(arg.astype(np.float64)).astype(F32)
    return (F32(0.5) * x * (F32(1.0) + e)).astype(F32)


def gelu_tanh(x) -> np.ndarray:
    """tanh-form GELU 0.5*x*(1+tanh(sqrt(2/pi)*(x+0.044715*x^3))), fp32.

    Not in the reference (which implements only the erf form): the MLP
    workloads of the benchmark specify this form, so the oracle carries it.
    tanh is evaluated in double and stored as fp32, mirroring how gelu() treats erf.
    """
    x = np.asarray(x, dtype=F32)
    c = F32(math.sqrt(2.0 / math.pi))
    inner = c * (x + F32(0.044715) * x * x * x)
    t = np.tanh(inner.astype(np.float64)).astype(F32)
    return (F32(0.5) * x * (F32(1.0) + t)).astype(F32)


def _gelu_by_mode(h: np.ndarray, mode: str) -> np.ndarray:
    if mode == "erf":
        return gelu(h)
    if mode == "erf_fast":
        return gelu_fast(h)
    if mode == "tanh":
        return gelu_tanh(h)
    raise ValueError(f"unknown gelu mode {mode!r}")


def fused_rmsnorm_matmul(x, gamma, w, eps: float = 1e-6) -> np.ndarray:
    """matmul(rmsnorm(x, gamma, eps), w) with the fp32 intermediate (golden.py:97-102)."""
    return matmul(rmsnorm(x, gamma, eps), w)


def fused_mlp(x, gamma, w1, b1, w2, residual, eps: float = 1e-6, gelu_mode: str = "erf") -> np.ndarray:
    """(gelu(rmsnorm(x)@w1 + b1) @ w2) + residual, all fp32 (golden.py:105-122).

    ``gelu_mode`` "erf" is the reference; "tanh" is the benchmark's variant;
    "erf_fast" is the erf form with scipy's vectorised erf.
    """
    normed = rmsnorm(x, gamma, eps)
    hidden = matmul(normed, w1) + np.asarray(b1, dtype=F32)
    act = _gelu_by_mode(hidden.astype(F32), gelu_mode)
    return (matmul(act, w2) + np.asarray(residual, dtype=F32)).astype(F32)


# ------------------------------------------------ device-numerics emulation (extra)


def emulate_device_fused_rmsnorm_matmul(x, gamma, w, eps: float = 1e-6) -> np.ndarray:
    """What the kernel computes: bf16(x*gamma) @ w in fp32, scaled per row by
    1/rms(x), rounded to bf16. Predicts the kernel's error against the golden."""
    x = np.asarray(x, dtype=F32)
    g = np.asarray(gamma, dtype=F32)
    k = x.shape[-1]
    inv = F32(1.0) / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) / F32(k) + F32(eps))
    xg = to_bf16(x * g)
    return to_bf16((xg @ np.asarray(w, dtype=F32)) * inv)


def emulate_device_fused_mlp(x, gamma, w1, b1, w2, residual, eps: float = 1e-6,
                             gelu_mode: str = "erf") -> np.ndarray:
    """Kernel numerics for the MLP: hidden = bf16(gelu(inv*(bf16(x*gamma)@w1) + b1)),
    y = bf16(hidden@w2 + residual)."""
    x = np.asarray(x, dtype=F32)
    g = np.asarray(gamma, dtype=F32)
    k = x.shape[-1]
    inv = F32(1.0) / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) / F32(k) + F32(eps))
    xg = to_bf16(x * g)
    h = (xg @ np.asarray(w1, dtype=F32)) * inv + np.asarray(b1, dtype=F32)
    h = to_bf16(_gelu_by_mode(h.astype(F32), gelu_mode))
    return to_bf16(h @ np.asarray(w2, dtype=F32) + np.asarray(residual, dtype=F32))
