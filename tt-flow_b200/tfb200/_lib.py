"""ctypes binding of libtfb200.so (the C ABI in include/tfb200.h).

The library is built in-tree (``make -C tt-flow_b200`` or
``__graft_entry__.build()``) to ``tt-flow_b200/lib/libtfb200.so``. There is no
fallback: if the library is missing, ``lib()`` raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]
LIB_PATH = Path(os.environ.get("TFB200_LIB", PKG_ROOT / "lib" / "libtfb200.so"))

TFB200_OK = 0
TFB200_EINVAL = -1
TFB200_EUNSUPPORTED = -2
TFB200_ECUDA = -3
TFB200_ETIMEOUT = -4
TFB200_EWORKSPACE = -5
TFB200_ENOSPC = -6
TFB200_BF16 = 0
TFB200_F32 = 1
TFB200_GELU_ERF = 0
TFB200_GELU_TANH = 1
TFB200_NOALLOC_SCRATCH_BYTES = 8 * 1024 * 1024

# Every symbol include/tfb200.h declares (checked by tests/test_abi.py).
EXPORTS = (
    "tfb200_version",
    "tfb200_last_error",
    "tfb200_matmul",
    "tfb200_fused_rmsnorm_matmul_workspace_size",
    "tfb200_fused_rmsnorm_matmul",
    "tfb200_fused_mlp_workspace_size",
    "tfb200_fused_mlp",
    "tfb200_fused_mlp_noalloc",
    "tfb200_fused_mlp_partial_workspace_size",
    "tfb200_fused_mlp_partial",
    "tfb200_tp_buffer_bytes",
    "tfb200_tp_output",
    "tfb200_fused_mlp_tp",
    "tfb200_ipc_get",
    "tfb200_ipc_open",
    "tfb200_ipc_close",
    "tfb200_residual_add",
    "tfb200_device_status",
    "tfb200_clear_device_status",
    "tfb200_opt",
    "tfb200_plan",
    "tfb200_selftest_bounded_wait",
    "tfb200_set_wait_limit_ns",
    "tfb200_launch_count",
)


class Mat(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("ld", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
    ]


MAX_TP = 8


class TpComm(ctypes.Structure):
    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("max_rows", ctypes.c_int64),
        ("peer_buf", ctypes.c_void_p * MAX_TP),
    ]


class TFB200Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"tfb200 error {code}: {msg}")
        self.code = code


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {PKG_ROOT}`")
    L = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.POINTER(Mat)
    vp, sz, f32, i32, u64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_int, ctypes.c_uint64
    sig = {
        "tfb200_version": ([], i32),
        "tfb200_last_error": ([], ctypes.c_char_p),
        "tfb200_matmul": ([P, P, P, vp], i32),
        "tfb200_fused_rmsnorm_matmul_workspace_size": ([ctypes.c_int64] * 3, sz),
        "tfb200_fused_rmsnorm_matmul": ([P, vp, P, f32, P, vp, vp, sz], i32),
        "tfb200_fused_mlp_workspace_size": ([ctypes.c_int64] * 4, sz),
        "tfb200_fused_mlp": ([P, vp, P, vp, P, P, f32, i32, P, vp, vp, sz], i32),
        "tfb200_fused_mlp_noalloc": ([P, vp, P, vp, P, P, f32, i32, P, vp], i32),
        "tfb200_fused_mlp_partial_workspace_size": ([ctypes.c_int64] * 4, sz),
        "tfb200_fused_mlp_partial": ([P, vp, P, vp, P, f32, i32, vp, ctypes.c_int64, vp, vp, sz], i32),
        "tfb200_residual_add": ([vp, ctypes.c_int64, P, P, vp], i32),
        "tfb200_tp_buffer_bytes": ([ctypes.c_int64, ctypes.c_int64, ctypes.c_int32], sz),
        "tfb200_tp_output": ([ctypes.POINTER(TpComm), ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p)], i32),
        "tfb200_fused_mlp_tp": ([P, vp, P, vp, P, P, f32, i32, ctypes.POINTER(TpComm), vp, vp, sz], i32),
        "tfb200_ipc_get": ([vp, vp, ctypes.POINTER(ctypes.c_size_t)], i32),
        "tfb200_ipc_open": ([vp, ctypes.POINTER(ctypes.c_void_p)], i32),
        "tfb200_ipc_close": ([vp], i32),
        "tfb200_device_status": ([], i32),
        "tfb200_clear_device_status": ([], i32),
        "tfb200_opt": ([ctypes.c_char_p, ctypes.c_char_p, vp, sz, ctypes.POINTER(ctypes.c_size_t)], i32),
        "tfb200_plan": ([ctypes.c_char_p, vp, sz, ctypes.POINTER(ctypes.c_size_t)], i32),
        "tfb200_selftest_bounded_wait": ([u64, vp], i32),
        "tfb200_set_wait_limit_ns": ([u64], None),
        "tfb200_launch_count": ([], u64),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _LIB = L
    return L


def check(code: int) -> None:
    if code != TFB200_OK:
        raise TFB200Error(code, lib().tfb200_last_error().decode(errors="replace"))
