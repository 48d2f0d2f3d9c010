"""The reference's operator interface on the B200 backend.

Same names, argument order and meaning as the reference golden
(tensixflow ``python/tensixflow/golden.py``): ``matmul(a, b)`` (:56-60),
``fused_rmsnorm_matmul(x, gamma, w, eps=1e-6)`` (:97-102) and
``fused_mlp(x, gamma, w1, b1, w2, residual, eps=1e-6)`` (:105-122), plus a
``gelu`` keyword ("erf", the reference's exact form, or "tanh").

Inputs are CUDA bf16 torch tensors, row-major; leading dimensions of ``x`` /
``a`` / ``residual`` are flattened into rows as the reference's lowering does
(``LowerToTTKernelPass.cpp:181-189``). The result is a bf16 tensor of shape
``[..., N]``. Every call runs the sm_100a kernels of libtfb200.so through its C
ABI; there is no other code path. Shape errors raise ``ValueError`` (numpy's
``@`` raises the same class in the reference); backend errors raise
``TFB200Error``.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib as L

__all__ = ["matmul", "fused_rmsnorm_matmul", "fused_mlp", "fused_mlp_partial", "fused_mlp_tp", "residual_add",
           "mlp_workspace_bytes",
           "rmsnorm_matmul_workspace_bytes", "mat", "stream_ptr"]


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _rows2d(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16 (got {t.dtype})")
    if t.dim() < 2:
        raise ValueError(f"{name} must have at least 2 dimensions")
    t2 = t.reshape(math.prod(t.shape[:-1]), t.shape[-1])
    if t2.stride(-1) != 1:
        t2 = t2.contiguous()
    return t2


def mat(t: torch.Tensor) -> L.Mat:
    """tfb200_mat view of a 2-D row-major tensor (unit column stride)."""
    assert t.dim() == 2 and (t.stride(1) == 1 or t.shape[1] <= 1)
    ld = t.stride(0) if t.shape[0] > 1 else max(t.shape[1], 1)
    return L.Mat(t.data_ptr(), t.shape[0], t.shape[1], max(ld, t.shape[1], 1), L.TFB200_BF16)


def _vec(t: torch.Tensor | None, n: int, name: str):
    if t is None:
        return None
    if not t.is_cuda or t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be a CUDA bfloat16 tensor")
    t = t.reshape(-1)
    if t.numel() != n:
        raise ValueError(f"{name} has {t.numel()} elements, expected {n}")
    return t.contiguous()


def matmul(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``a @ b`` with fp32 accumulation and a bf16 result (golden.matmul)."""
    a2 = _rows2d(a, "a")
    b2 = _rows2d(b, "b")
    if a2.shape[1] != b2.shape[0]:
        raise ValueError(f"matmul: inner dimensions differ ({a2.shape[1]} vs {b2.shape[0]})")
    dev = _device_of(("a", a), ("b", b), ("out", out))
    y = out if out is not None else torch.empty(a2.shape[0], b2.shape[1], dtype=torch.bfloat16, device=a.device)
    with torch.cuda.device(dev):
        L.check(L.lib().tfb200_matmul(ctypes.byref(mat(a2)), ctypes.byref(mat(b2)), ctypes.byref(mat(y)),
                                      ctypes.c_void_p(stream_ptr())))
    return y.reshape(*a.shape[:-1], b2.shape[1]) if out is None else y


def rmsnorm_matmul_workspace_bytes(m: int, k: int, n: int) -> int:
    return int(L.lib().tfb200_fused_rmsnorm_matmul_workspace_size(m, k, n))


def _workspace(need: int, ws: torch.Tensor | None, device) -> torch.Tensor:
    """The caller's workspace, checked, or (when none is given) a new one. A workspace that is given but too small
    is an error, not a silent reallocation: callers pass one precisely to keep allocations out of their loop."""
    if ws is None:
        return torch.empty(max(need, 256), dtype=torch.uint8, device=device)
    if not ws.is_cuda or ws.device != device:
        raise ValueError(f"workspace must be on {device} (got {ws.device})")
    if not ws.is_contiguous():
        raise ValueError("workspace must be contiguous")
    if ws.numel() * ws.element_size() < need:
        raise ValueError(f"workspace holds {ws.numel() * ws.element_size()} bytes; this call needs {need}")
    return ws


def _device_of(*named) -> torch.device:
    """The one CUDA device of every operand given (name, tensor-or-None); the call then runs on that device's
    current stream."""
    dev = None
    for name, t in named:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise TypeError(f"{name} must be a CUDA tensor")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{name} is on {t.device}; the other operands are on {dev}")
    return dev


def fused_rmsnorm_matmul(x: torch.Tensor, gamma: torch.Tensor, w: torch.Tensor, eps: float = 1e-6,
                         out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``matmul(rmsnorm(x, gamma, eps), w)`` (golden.fused_rmsnorm_matmul)."""
    x2 = _rows2d(x, "x")
    w2 = _rows2d(w, "w")
    K = x2.shape[1]
    if w2.shape[0] != K:
        raise ValueError(f"fused_rmsnorm_matmul: x has K={K} but w has {w2.shape[0]} rows")
    g = _vec(gamma, K, "gamma")
    dev = _device_of(("x", x), ("gamma", gamma), ("w", w), ("out", out))
    y = out if out is not None else torch.empty(x2.shape[0], w2.shape[1], dtype=torch.bfloat16, device=x.device)
    ws = _workspace(rmsnorm_matmul_workspace_bytes(x2.shape[0], K, w2.shape[1]), workspace, dev)
    with torch.cuda.device(dev):
        L.check(L.lib().tfb200_fused_rmsnorm_matmul(ctypes.byref(mat(x2)), ctypes.c_void_p(g.data_ptr()),
                                                    ctypes.byref(mat(w2)), ctypes.c_float(eps), ctypes.byref(mat(y)),
                                                    ctypes.c_void_p(stream_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                                    ctypes.c_size_t(ws.numel() * ws.element_size())))
    return y.reshape(*x.shape[:-1], w2.shape[1]) if out is None else y


def mlp_workspace_bytes(m: int, k: int, h: int, n: int) -> int:
    return int(L.lib().tfb200_fused_mlp_workspace_size(m, k, h, n))


_GELU = {"erf": L.TFB200_GELU_ERF, "tanh": L.TFB200_GELU_TANH}


def fused_mlp(x: torch.Tensor, gamma: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor | None,
              w2: torch.Tensor, residual: torch.Tensor, eps: float = 1e-6, gelu: str = "erf",
              out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``(gelu(rmsnorm(x) @ w1 + b1) @ w2) + residual`` (golden.fused_mlp).

    ``b1`` is the 1-D ``[H]`` bias the dialect's verifier accepts
    (TensixflowOps.cpp:329-335); a full-rank bias whose rows are all equal may be
    passed and is reduced to its first row.
    """
    x2 = _rows2d(x, "x")
    W1 = _rows2d(w1, "w1")
    W2 = _rows2d(w2, "w2")
    r2 = _rows2d(residual, "residual")
    M, K = x2.shape
    H = W1.shape[1]
    N = W2.shape[1]
    if W1.shape[0] != K or W2.shape[0] != H:
        raise ValueError("fused_mlp: shapes do not chain (x[M,K] @ w1[K,H] @ w2[H,N])")
    if r2.shape != (M, N):
        raise ValueError(f"fused_mlp: residual must be [{M},{N}] (got {tuple(r2.shape)})")
    if b1 is not None and b1.dim() > 1:
        b1 = b1.reshape(-1, b1.shape[-1])[0]
    b = _vec(b1, H, "b1")
    g = _vec(gamma, K, "gamma")
    if gelu not in _GELU:
        raise ValueError(f"gelu must be 'erf' or 'tanh' (got {gelu!r})")
    dev = _device_of(("x", x), ("gamma", gamma), ("w1", w1), ("b1", b1), ("w2", w2), ("residual", residual),
                     ("out", out))
    y = out if out is not None else torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    workspace = _workspace(mlp_workspace_bytes(M, K, H, N), workspace, dev)
    with torch.cuda.device(dev):
        L.check(L.lib().tfb200_fused_mlp(
            ctypes.byref(mat(x2)), ctypes.c_void_p(g.data_ptr()), ctypes.byref(mat(W1)),
            ctypes.c_void_p(b.data_ptr() if b is not None else None), ctypes.byref(mat(W2)), ctypes.byref(mat(r2)),
            ctypes.c_float(eps), ctypes.c_int(_GELU[gelu]), ctypes.byref(mat(y)), ctypes.c_void_p(stream_ptr()),
            ctypes.c_void_p(workspace.data_ptr()), ctypes.c_size_t(workspace.numel() * workspace.element_size())))
    return y.reshape(*x.shape[:-1], N) if out is None else y


def fused_mlp_partial(x: torch.Tensor, gamma: torch.Tensor, w1_shard: torch.Tensor, b1_shard: torch.Tensor | None,
                      w2_shard: torch.Tensor, eps: float = 1e-6, gelu: str = "erf",
                      out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One GPU's share of a tensor-parallel MLP: fp32 ``gelu(rmsnorm(x) @ w1_shard + b1_shard) @ w2_shard``
    (W1 split by columns, W2 by rows). Sum over GPUs, then ``residual_add``."""
    x2 = _rows2d(x, "x")
    W1 = _rows2d(w1_shard, "w1_shard")
    W2 = _rows2d(w2_shard, "w2_shard")
    M, K = x2.shape
    H, N = W1.shape[1], W2.shape[1]
    if W1.shape[0] != K or W2.shape[0] != H:
        raise ValueError("fused_mlp_partial: shapes do not chain")
    b = _vec(b1_shard, H, "b1_shard")
    g = _vec(gamma, K, "gamma")
    if gelu not in _GELU:
        raise ValueError(f"gelu must be 'erf' or 'tanh' (got {gelu!r})")
    dev = _device_of(("x", x), ("gamma", gamma), ("w1_shard", w1_shard), ("b1_shard", b1_shard),
                     ("w2_shard", w2_shard), ("out", out))
    y = out if out is not None else torch.empty(M, N, dtype=torch.float32, device=x.device)
    ws = _workspace(int(L.lib().tfb200_fused_mlp_partial_workspace_size(M, K, H, N)), workspace, dev)
    with torch.cuda.device(dev):
        L.check(L.lib().tfb200_fused_mlp_partial(
            ctypes.byref(mat(x2)), ctypes.c_void_p(g.data_ptr()), ctypes.byref(mat(W1)),
            ctypes.c_void_p(b.data_ptr() if b is not None else None), ctypes.byref(mat(W2)), ctypes.c_float(eps),
            ctypes.c_int(_GELU[gelu]), ctypes.c_void_p(y.data_ptr()), ctypes.c_int64(y.stride(0)),
            ctypes.c_void_p(stream_ptr()), ctypes.c_void_p(ws.data_ptr()),
            ctypes.c_size_t(ws.numel() * ws.element_size())))
    return y


def fused_mlp_tp(x: torch.Tensor, gamma: torch.Tensor, w1_shard: torch.Tensor, b1_shard: torch.Tensor | None,
                 w2_shard: torch.Tensor, residual: torch.Tensor, comm: L.TpComm, eps: float = 1e-6,
                 gelu: str = "erf", workspace: torch.Tensor | None = None) -> None:
    """One rank's call of the tensor-parallel MLP whose all-reduce is fused into the down-projection kernel
    (``tfb200_fused_mlp_tp``). The result lands in every rank's ``comm.out`` buffer; ``tp.TPDecodeMLPFused``
    owns the buffers and the epoch."""
    x2 = _rows2d(x, "x")
    W1 = _rows2d(w1_shard, "w1_shard")
    W2 = _rows2d(w2_shard, "w2_shard")
    r2 = _rows2d(residual, "residual")
    M, K = x2.shape
    H, N = W1.shape[1], W2.shape[1]
    if W1.shape[0] != K or W2.shape[0] != H:
        raise ValueError("fused_mlp_tp: shapes do not chain")
    if tuple(r2.shape) != (M, N):
        raise ValueError(f"fused_mlp_tp: residual must be [{M},{N}] (got {tuple(r2.shape)})")
    if gelu not in _GELU:
        raise ValueError(f"gelu must be 'erf' or 'tanh' (got {gelu!r})")
    b = _vec(b1_shard, H, "b1_shard")
    g = _vec(gamma, K, "gamma")
    dev = _device_of(("x", x), ("gamma", gamma), ("w1_shard", w1_shard), ("b1_shard", b1_shard),
                     ("w2_shard", w2_shard), ("residual", residual))
    ws = _workspace(int(L.lib().tfb200_fused_mlp_partial_workspace_size(M, K, H, N)), workspace, dev)
    with torch.cuda.device(dev):
        L.check(L.lib().tfb200_fused_mlp_tp(
            ctypes.byref(mat(x2)), ctypes.c_void_p(g.data_ptr()), ctypes.byref(mat(W1)),
            ctypes.c_void_p(b.data_ptr() if b is not None else None), ctypes.byref(mat(W2)), ctypes.byref(mat(r2)),
            ctypes.c_float(eps), ctypes.c_int(_GELU[gelu]), ctypes.byref(comm), ctypes.c_void_p(stream_ptr()),
            ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel() * ws.element_size())))


def residual_add(partial: torch.Tensor, residual: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``bf16(partial + residual)``: the tail of the tensor-parallel MLP."""
    if partial.dtype != torch.float32 or partial.dim() != 2 or partial.stride(1) != 1:
        raise TypeError("partial must be a row-major fp32 matrix")
    r2 = _rows2d(residual, "residual")
    if tuple(r2.shape) != tuple(partial.shape):
        raise ValueError("residual and partial shapes differ")
    dev = _device_of(("partial", partial), ("residual", residual), ("out", out))
    y = out if out is not None else torch.empty(r2.shape, dtype=torch.bfloat16, device=partial.device)
    with torch.cuda.device(dev):
        L.check(L.lib().tfb200_residual_add(ctypes.c_void_p(partial.data_ptr()), ctypes.c_int64(partial.stride(0)),
                                            ctypes.byref(mat(r2)), ctypes.byref(mat(y)),
                                            ctypes.c_void_p(stream_ptr())))
    return y
