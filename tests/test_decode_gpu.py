"""The streamed (decode-shaped) fused MLP and its tensor-parallel split on one GPU.

The tensor-parallel split is emulated on one device: each shard's partial is
computed by the real kernels, the partials are summed, and the residual kernel
finishes; the multi-process NCCL version runs the same steps per GPU.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import golden as O  # noqa: E402
from tfb200 import workloads as W  # noqa: E402
from tfb200.metrics import parity  # noqa: E402

pytestmark = pytest.mark.gpu
f32 = W.bf16_to_f32


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.bfloat16)


def _case(m, k, h, seed=3):
    rng = np.random.default_rng(seed + m)
    t = {"x": rng.standard_normal((m, k), dtype=np.float32), "gamma": 0.5 + rng.random(k, dtype=np.float32),
         "w1": rng.standard_normal((k, h), dtype=np.float32) / np.float32(np.sqrt(k)),
         "b1": 0.02 * rng.standard_normal(h, dtype=np.float32),
         "w2": rng.standard_normal((h, k), dtype=np.float32) / np.float32(np.sqrt(h))}
    return {key: W.bf16_bits(v) for key, v in t.items()}


def _golden(t, gelu):
    x = f32(t["x"])
    return O.fused_mlp(x, f32(t["gamma"]), f32(t["w1"]), f32(t["b1"]), f32(t["w2"]), x, 1e-5,
                       "tanh" if gelu == "tanh" else "erf")


@pytest.mark.parametrize("m", [1, 7, 32, 33, 64])
@pytest.mark.parametrize("gelu", ["tanh", "erf"])
def test_streamed_mlp_rows(m, gelu):
    from tfb200 import ops

    t = _case(m, 1024, 3072)
    x = dev(t["x"])
    y = ops.fused_mlp(x, dev(t["gamma"]), dev(t["w1"]), dev(t["b1"]), dev(t["w2"]), x, 1e-5, gelu=gelu)
    got = y.float().cpu().numpy()
    m_ = parity(got, _golden(t, gelu))
    assert m_["ok"], m_


@pytest.mark.parametrize("m,k,h", [(32, 512, 2048), (32, 8192, 28672), (5, 1000, 3000)])
def test_streamed_mlp_bit_identical_calls(m, k, h):
    """Two calls on one workspace give the same result bit for bit: the CTAs' partial sums of a column block are
    added in CTA order, whatever order they arrive in (and the counters are cleared between calls). The second
    shape is the decode workload's; the third has a width that is not a multiple of 128."""
    from tfb200 import ops

    t = _case(m, k, h)
    x = dev(t["x"])
    args = (x, dev(t["gamma"]), dev(t["w1"]), dev(t["b1"]), dev(t["w2"]), x, 1e-5)
    ws = torch.empty(ops.mlp_workspace_bytes(m, k, h, k), dtype=torch.uint8, device="cuda")
    a = ops.fused_mlp(*args, gelu="tanh", workspace=ws)
    b = ops.fused_mlp(*args, gelu="tanh", workspace=ws)
    assert torch.equal(a, b)
    assert parity(a.float().cpu().numpy(), _golden(t, "tanh"))["ok"]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_split_on_one_gpu(world):
    from tfb200 import ops
    from tfb200.tp import shard_mlp

    t = _case(32, 1024, 4096)
    x, g = dev(t["x"]), dev(t["gamma"])
    w1, b1, w2 = dev(t["w1"]), dev(t["b1"]), dev(t["w2"])
    total = torch.zeros(32, 1024, dtype=torch.float32, device="cuda")
    for r in range(world):
        s = shard_mlp(w1, b1, w2, r, world)
        total += ops.fused_mlp_partial(x, g, s.w1, s.b1, s.w2, 1e-5, "tanh")
    y = ops.residual_add(total, x).float().cpu().numpy()
    m_ = parity(y, _golden(t, "tanh"))
    assert m_["ok"], m_


def test_bounded_wait_reports_timeout_and_context_survives():
    """A kernel waits on a barrier nothing completes; its bounded wait gives up,
    the status word says TFB200_ETIMEOUT, and the device keeps working."""
    import ctypes

    from tfb200 import _lib as L
    from tfb200 import ops

    lib = L.lib()
    assert lib.tfb200_clear_device_status() == L.TFB200_OK
    rc = lib.tfb200_selftest_bounded_wait(ctypes.c_uint64(20_000_000), ctypes.c_void_p(ops.stream_ptr()))
    assert rc == L.TFB200_OK
    torch.cuda.synchronize()
    assert lib.tfb200_device_status() == L.TFB200_ETIMEOUT
    assert lib.tfb200_clear_device_status() == L.TFB200_OK
    t = _case(8, 256, 512)
    x = dev(t["x"])
    y = ops.fused_mlp(x, dev(t["gamma"]), dev(t["w1"]), dev(t["b1"]), dev(t["w2"]), x, 1e-5, gelu="tanh")
    assert parity(y.float().cpu().numpy(), _golden(t, "tanh"))["ok"]
    assert lib.tfb200_device_status() == L.TFB200_OK


def test_single_launch_mode_matches_two_launches_bit_for_bit(tmp_path):
    """The streamed MLP runs as two launches by default; TFB200_STREAM_LAUNCHES=1 runs both GEMMs in one
    cooperative launch with a grid barrier between them (measured slower, kept as an option). Both add the CTAs'
    partial sums in the same order, so with the same grid they give the same bits. The L2 prefetch of the next
    weights (TFB200_STREAM_PREFETCH=0 turns it off) changes timing only. Run in child processes (the switches are
    read once per process)."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    script = tmp_path / "run.py"
    script.write_text(
        "import sys\n"
        f"sys.path[:0] = [{str(root)!r}, {str(root / 'tt-flow_b200')!r}]\n"
        "import numpy as np, torch\n"
        "from tfb200 import ops\n"
        "g = torch.Generator(device='cuda').manual_seed(7)\n"
        "def r(*s, std=1.0):\n"
        "    return (torch.randn(*s, generator=g, device='cuda') * std).to(torch.bfloat16)\n"
        "x, gm = r(16, 4096), (0.5 + torch.rand(4096, generator=g, device='cuda')).to(torch.bfloat16)\n"
        "w1, b1, w2 = r(4096, 12288, std=1 / 64), r(12288, std=0.02), r(12288, 4096, std=1 / 111)\n"
        "y = ops.fused_mlp(x, gm, w1, b1, w2, x, 1e-5, gelu='tanh')\n"
        "np.save(sys.argv[1], y.view(torch.int16).cpu().numpy())\n")
    outs = []
    for i, extra in enumerate(({}, {"TFB200_STREAM_LAUNCHES": "1"}, {"TFB200_STREAM_PREFETCH": "0"})):
        out = tmp_path / f"y{i}.npy"
        env = dict(os.environ, **extra)
        r = subprocess.run([sys.executable, str(script), str(out)], env=env, capture_output=True, text=True,
                           timeout=300)
        assert r.returncode == 0, r.stderr
        outs.append(np.load(out))
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(outs[0], outs[2])
