"""The fused calls captured in a CUDA graph and replayed, as a serving loop runs them.

Every launch of a call is stream-ordered (kernels launched with cluster and
programmatic-serialization attributes; the staging launch also clears the
counters and flags the later launches use), so a call can be recorded once with
torch.cuda.graph and replayed with new inputs copied into the captured buffers.
The first eager call on a device does the per-device set-up (function
attributes, occupancy query, status word), so it comes before the capture. Both
paths add their partial sums in a fixed order (the CTA-pair path's tail-split
parts, the streamed path's per-CTA slots in CTA order), so every replay must
give the eager call's bits, besides meeting the parity bar against the oracle.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import golden as O  # noqa: E402
from tfb200 import workloads as W  # noqa: E402
from tfb200.metrics import parity  # noqa: E402

pytestmark = pytest.mark.gpu

f32 = W.bf16_to_f32


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.bfloat16)


def _inputs(seed, m, k, h, n):
    rng = np.random.default_rng(seed)
    return {
        "x": W.bf16_bits(rng.standard_normal((m, k), dtype=np.float32)),
        "gamma": W.bf16_bits(0.5 + rng.random(k, dtype=np.float32)),
        "w1": W.bf16_bits(rng.standard_normal((k, h), dtype=np.float32) / np.float32(np.sqrt(k))),
        "b1": W.bf16_bits(0.02 * rng.standard_normal(h, dtype=np.float32)),
        "w2": W.bf16_bits(rng.standard_normal((h, n), dtype=np.float32) / np.float32(np.sqrt(h))),
    }


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available()
    from tfb200 import ops as _ops

    return _ops


@pytest.mark.parametrize("m", [32, 512])  # streamed decode path, CTA-pair path
def test_fused_mlp_replays_from_a_cuda_graph(ops, m):
    k = n = 512
    h = 1024
    t = _inputs(7 + m, m, k, h, n)
    G, W1, B1, W2 = (_dev(t[key]) for key in ("gamma", "w1", "b1", "w2"))
    batches = [W.bf16_bits(np.random.default_rng(100 + i).standard_normal((m, k), dtype=np.float32))
               for i in range(3)]
    X = _dev(batches[0])
    Y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    WS = torch.empty(ops.mlp_workspace_bytes(m, k, h, n), dtype=torch.uint8, device="cuda")

    def call():
        ops.fused_mlp(X, G, W1, B1, W2, X, 1e-5, gelu="tanh", out=Y, workspace=WS)

    eager = []
    for b in batches:
        X.copy_(_dev(b))
        call()
        torch.cuda.synchronize()
        eager.append(Y.clone())

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        call()  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()

    for rep in range(2):
        for i, b in enumerate(batches):
            X.copy_(_dev(b))
            Y.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            got = Y.float().cpu().numpy()
            xf = f32(b)
            want = O.fused_mlp(xf, f32(t["gamma"]), f32(t["w1"]), f32(t["b1"]), f32(t["w2"]), xf, 1e-5, "tanh")
            res = parity(got, want)
            assert res["ok"], (rep, i, res)
            assert torch.equal(Y, eager[i]), f"replay {rep} of batch {i} differs from the eager call"
    del graph


def test_fused_rmsnorm_matmul_replays_from_a_cuda_graph(ops):
    m, k, n = 640, 1024, 768
    t = _inputs(3, m, k, n, n)
    G, Wt = _dev(t["gamma"]), _dev(t["w1"])
    X = _dev(t["x"])
    Y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    WS = torch.empty(ops.rmsnorm_matmul_workspace_bytes(m, k, n), dtype=torch.uint8, device="cuda")

    def call():
        ops.fused_rmsnorm_matmul(X, G, Wt, 1e-5, out=Y, workspace=WS)

    call()
    torch.cuda.synchronize()
    eager = Y.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        call()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    Y.zero_()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(Y, eager)
    want = O.fused_rmsnorm_matmul(f32(t["x"]), f32(t["gamma"]), f32(t["w1"]), 1e-5)
    assert parity(Y.float().cpu().numpy(), want)["ok"]
    del graph
