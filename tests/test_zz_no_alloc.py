"""The fused MLP entry point that allocates nothing (tfb200_fused_mlp_noalloc).

Some callers cannot call cudaMalloc or let a library allocate for them: plugin
hosts and inference servers that own all of the GPU's memory, and
latency-critical loops that must not risk the synchronisation an allocation can
bring. For them tfb200_fused_mlp_noalloc keeps the hidden block in a fixed
device array of the library instead of a caller workspace. This test calls it
through the C ABI, twice in a row with different inputs, and checks each result
against tfb200_fused_mlp on the same inputs with the parity tolerance the other
tests use; it also checks that an oversized problem is refused before any launch.

The file name makes pytest collect it last, so a run that stops at the first
failure has run every other test before this one. It also passes on its own in
a fresh process (its first call then performs the per-device set-up).
"""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import golden as O  # noqa: E402
from tfb200 import _lib as L  # noqa: E402
from tfb200 import workloads as W  # noqa: E402
from tfb200.metrics import parity  # noqa: E402

pytestmark = pytest.mark.gpu


def _case(seed, m, k, h, n):
    rng = np.random.default_rng(seed)
    t = {
        "x": rng.standard_normal((m, k), dtype=np.float32),
        "gamma": 0.5 + rng.random(k, dtype=np.float32),
        "w1": rng.standard_normal((k, h), dtype=np.float32) / np.float32(np.sqrt(k)),
        "b1": 0.02 * rng.standard_normal(h, dtype=np.float32),
        "w2": rng.standard_normal((h, n), dtype=np.float32) / np.float32(np.sqrt(h)),
    }
    return {key: W.bf16_bits(v) for key, v in t.items()}


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.bfloat16)


def _mat(t):
    return L.Mat(t.data_ptr(), t.shape[0], t.shape[1], t.stride(0), L.TFB200_BF16)


def _run(lib, t, gelu, use_noalloc):
    x, g, w1, b1, w2 = (_dev(t[key]) for key in ("x", "gamma", "w1", "b1", "w2"))  # residual = x (N == K)
    y = torch.empty(x.shape[0], w2.shape[1], dtype=torch.bfloat16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [ctypes.byref(_mat(x)), ctypes.c_void_p(g.data_ptr()), ctypes.byref(_mat(w1)),
            ctypes.c_void_p(b1.data_ptr()), ctypes.byref(_mat(w2)), ctypes.byref(_mat(x)), ctypes.c_float(1e-5),
            ctypes.c_int(gelu), ctypes.byref(_mat(y)), stream]
    if use_noalloc:
        rc = lib.tfb200_fused_mlp_noalloc(*args)
    else:
        need = lib.tfb200_fused_mlp_workspace_size(x.shape[0], x.shape[1], w1.shape[1], w2.shape[1])
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        rc = lib.tfb200_fused_mlp(*args, ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(need))
    assert rc == L.TFB200_OK, lib.tfb200_last_error()
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    assert torch.cuda.is_available()
    lib = L.lib()
    cases = [(_case(101, 192, 256, 1024, 256), L.TFB200_GELU_TANH),
             (_case(202, 64, 512, 2048, 512), L.TFB200_GELU_ERF)]
    for t, gelu in cases:  # two calls in a row; the second sees the first's leftover scratch
        got = _run(lib, t, gelu, use_noalloc=True)
        want = _run(lib, t, gelu, use_noalloc=False)
        m = parity(got, want)
        assert m["ok"], m
        x = W.bf16_to_f32(t["x"])
        golden = O.fused_mlp(x, W.bf16_to_f32(t["gamma"]), W.bf16_to_f32(t["w1"]), W.bf16_to_f32(t["b1"]),
                             W.bf16_to_f32(t["w2"]), x, 1e-5, "tanh" if gelu == L.TFB200_GELU_TANH else "erf")
        assert parity(got, golden)["ok"]
    assert lib.tfb200_device_status() == L.TFB200_OK


def test_noalloc_call_takes_no_device_memory():
    """After the first call on the device (which may commit the scratch under lazy module loading), a call takes no
    device memory: the device's free bytes are the same before and after it."""
    lib = L.lib()
    t = _case(303, 96, 256, 1024, 256)
    x, g, w1, b1, w2 = (_dev(t[key]) for key in ("x", "gamma", "w1", "b1", "w2"))
    y = torch.empty(x.shape[0], w2.shape[1], dtype=torch.bfloat16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [ctypes.byref(_mat(x)), ctypes.c_void_p(g.data_ptr()), ctypes.byref(_mat(w1)),
            ctypes.c_void_p(b1.data_ptr()), ctypes.byref(_mat(w2)), ctypes.byref(_mat(x)), ctypes.c_float(1e-5),
            ctypes.c_int(L.TFB200_GELU_TANH), ctypes.byref(_mat(y)), stream]
    assert lib.tfb200_fused_mlp_noalloc(*args) == L.TFB200_OK, lib.tfb200_last_error()
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    assert lib.tfb200_fused_mlp_noalloc(*args) == L.TFB200_OK, lib.tfb200_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert lib.tfb200_device_status() == L.TFB200_OK


def test_noalloc_refuses_problems_beyond_its_scratch():
    lib = L.lib()
    m, k, h, n = 1024, 64, 8192, 64  # hidden block 16 MiB > 8 MiB
    x = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    w1 = torch.zeros(k, h, dtype=torch.bfloat16, device="cuda")
    w2 = torch.zeros(h, n, dtype=torch.bfloat16, device="cuda")
    g = torch.ones(k, dtype=torch.bfloat16, device="cuda")
    y = torch.full((m, n), 7.0, dtype=torch.bfloat16, device="cuda")
    before = lib.tfb200_launch_count()
    rc = lib.tfb200_fused_mlp_noalloc(ctypes.byref(_mat(x)), ctypes.c_void_p(g.data_ptr()), ctypes.byref(_mat(w1)),
                                      None, ctypes.byref(_mat(w2)), ctypes.byref(_mat(y)), ctypes.c_float(1e-5),
                                      ctypes.c_int(L.TFB200_GELU_TANH), ctypes.byref(_mat(y)),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == L.TFB200_EINVAL
    assert b"scratch" in lib.tfb200_last_error()
    assert lib.tfb200_launch_count() == before
    assert bool((y == 7.0).all())
