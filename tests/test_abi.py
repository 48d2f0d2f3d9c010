"""The C ABI library loads and exports every symbol include/tfb200.h declares.

CPU only: calls here are restricted to those that never touch a device
(version, workspace sizing, host-side argument validation).
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tfb200.h"


@pytest.fixture(scope="module")
def L():
    from tfb200 import _lib

    if not _lib.LIB_PATH.exists():
        subprocess.run(["make", "-C", str(_lib.PKG_ROOT)], check=True, capture_output=True)
    return _lib


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(tfb200_\w+)\s*\(", text, re.M)))


def test_header_lists_the_binding_exports(L):
    assert declared() == sorted(L.EXPORTS)


def test_library_exports_every_declared_symbol(L):
    lib = ctypes.CDLL(str(L.LIB_PATH))
    for name in declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(L.LIB_PATH)], capture_output=True, text=True).stdout
    for name in declared():
        assert re.search(rf"\bT {name}$", out, re.M), name


def test_version_and_workspace(L):
    lib = L.lib()
    assert lib.tfb200_version() == 1
    # Above 128 rows the CTA-pair GEMM may split the tail of its last wave over idle pairs: the workspace adds
    # the split's flags (128 slots x 64 int32, per GEMM) and up to 128 fp32 slots of 2 x 128 x 256 (or 4 per tile).
    flags, slot = 128 * 64 * 4, 2 * 128 * 256 * 4
    # hidden block + staged bf16(x * gamma) + per-row inverse RMS, each 256-byte aligned
    base = 8192 * 16384 * 2 + 8192 * 4096 * 2 + 8192 * 4
    assert lib.tfb200_fused_mlp_workspace_size(8192, 4096, 16384, 4096) == base + 2 * flags + 128 * slot
    assert lib.tfb200_fused_mlp_workspace_size(0, 4096, 16384, 4096) == 0
    # few rows: the streamed path adds the streaming kernel's partial-sum slots (one fp32 [m, 128] per column block
    # plus one per CTA beyond the first, up to 160 CTAs) and the column-block counters with the phase barrier
    streamed = 256 + 512 + (1 + 160 - 1) * 3 * 128 * 4 + 256
    assert lib.tfb200_fused_mlp_workspace_size(3, 8, 5, 8) == streamed
    assert lib.tfb200_fused_mlp_partial_workspace_size(3, 8, 5, 8) == streamed
    # 128 rows run on the one-CTA kernel: no split region
    assert lib.tfb200_fused_mlp_workspace_size(128, 128, 128, 128) == 128 * 128 * 2 + 128 * 128 * 2 + 512
    assert lib.tfb200_fused_rmsnorm_matmul_workspace_size(8192, 4096, 6144) == (8192 * 4096 * 2 + 8192 * 4 + flags
                                                                               + 128 * slot)
    # one 256 x 256 tile: at most 4 parts
    assert lib.tfb200_fused_rmsnorm_matmul_workspace_size(200, 64, 256) == 200 * 64 * 2 + 1024 + flags + 4 * slot
    # the staged block's leading dimension is rounded up to 8 elements for TMA
    assert lib.tfb200_fused_rmsnorm_matmul_workspace_size(100, 50, 7) == 11264 + 512  # 100*56*2 -> 11264
    # absurd sizes saturate instead of wrapping around
    assert lib.tfb200_fused_mlp_workspace_size(1 << 40, 4096, 16384, 4096) == 2 ** 64 - 1
    assert lib.tfb200_fused_rmsnorm_matmul_workspace_size(4096, 1 << 40, 64) == 2 ** 64 - 1


def test_host_validation_needs_no_device(L):
    lib = L.lib()
    a = L.Mat(None, 4, 8, 8, L.TFB200_BF16)
    b = L.Mat(None, 9, 8, 8, L.TFB200_BF16)  # inner dims disagree
    c = L.Mat(None, 4, 8, 8, L.TFB200_BF16)
    assert lib.tfb200_matmul(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None) == L.TFB200_EINVAL
    assert b"null data" in lib.tfb200_last_error() or b"shapes" in lib.tfb200_last_error()
    bad = L.Mat(None, 4, 8, 4, L.TFB200_BF16)  # ld < cols
    assert lib.tfb200_matmul(ctypes.byref(bad), ctypes.byref(a), ctypes.byref(c), None) == L.TFB200_EINVAL
    f32 = L.Mat(None, 4, 8, 8, L.TFB200_F32)
    assert lib.tfb200_matmul(ctypes.byref(f32), ctypes.byref(a), ctypes.byref(c), None) == L.TFB200_EINVAL
    assert lib.tfb200_fused_mlp(None, None, None, None, None, None, 1e-5, 0, None, None, None, 0) == L.TFB200_EINVAL


def test_tp_buffer_sizes():
    """One rank's tensor-parallel buffer: local sums, counters, a slot per rank, arrivals, output, done word."""
    from tfb200 import _lib as L

    lib = L.lib()
    al = lambda b: (b + 255) // 256 * 256  # noqa: E731
    for rows, n, world in [(32, 8192, 2), (64, 8192, 8), (1, 8, 1), (7, 1000, 3)]:
        blocks = (n + 127) // 128
        want = (al(rows * n * 4) + al(blocks * 4) + world * al(rows * n * 4) + al(blocks * 4) + al(rows * n * 2)
                + 256)
        assert lib.tfb200_tp_buffer_bytes(rows, n, world) == want
    assert lib.tfb200_tp_buffer_bytes(65, 8192, 2) == 0
    assert lib.tfb200_tp_buffer_bytes(32, 8192, 9) == 0
    assert lib.tfb200_tp_buffer_bytes(32, 8192, 0) == 0
