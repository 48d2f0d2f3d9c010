"""Tensor-parallel decode MLP with the all-reduce fused into the down-projection kernel.

With one rank the same kernel path runs on one GPU (owner of every column block
is rank 0, the peer buffers are this process's own). With two or more GPUs
visible, one process per GPU exchanges CUDA IPC handles and every rank's output
must match the unsharded oracle and be identical across ranks (each block is
written to all ranks by the one finisher). Ranks are never emulated as several
processes on one GPU: their kernels wait on one another.
"""

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

from oracle import golden as O  # noqa: E402
from tfb200 import workloads as W  # noqa: E402
from tfb200.metrics import parity  # noqa: E402

pytestmark = pytest.mark.gpu
f32 = W.bf16_to_f32


def _case(m, k, h, seed=5):
    rng = np.random.default_rng(seed + 31 * m)
    t = {"x": rng.standard_normal((m, k), dtype=np.float32), "gamma": 0.5 + rng.random(k, dtype=np.float32),
         "w1": rng.standard_normal((k, h), dtype=np.float32) / np.float32(np.sqrt(k)),
         "b1": 0.02 * rng.standard_normal(h, dtype=np.float32),
         "w2": rng.standard_normal((h, k), dtype=np.float32) / np.float32(np.sqrt(h))}
    return {key: W.bf16_bits(v) for key, v in t.items()}


def _golden(t, gelu):
    x = f32(t["x"])
    return O.fused_mlp(x, f32(t["gamma"]), f32(t["w1"]), f32(t["b1"]), f32(t["w2"]), x, 1e-5, gelu)


def _dev(a, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device).view(torch.bfloat16)


K, H = 1024, 4096
ROWS = [1, 7, 32, 64, 33]


def test_fused_tp_single_rank_many_calls():
    """Calls of different row counts on one set of buffers; every result matches the oracle."""
    from tfb200 import _lib as L
    from tfb200.tp import TPDecodeMLPFused

    lib = L.lib()
    assert lib.tfb200_clear_device_status() == L.TFB200_OK
    full = _case(64, K, H)
    w1, b1, w2, g = _dev(full["w1"]), _dev(full["b1"]), _dev(full["w2"]), _dev(full["gamma"])
    for gelu in ("tanh", "erf"):
        mlp = TPDecodeMLPFused(w1, b1, w2, g, rank=0, world=1, max_rows=64, eps=1e-5, gelu=gelu)
        for m in ROWS:
            t = dict(full, x=_case(m, K, H)["x"])
            x = _dev(t["x"])
            y = mlp(x, x).float().cpu().numpy()
            res = parity(y, _golden(t, gelu))
            assert res["ok"], (gelu, m, res)
        assert mlp.calls == len(ROWS)
    torch.cuda.synchronize()
    assert lib.tfb200_device_status() == L.TFB200_OK


def test_fused_tp_rejects_bad_communicator():
    import ctypes

    from tfb200 import _lib as L
    from tfb200 import ops

    t = _case(4, K, H)
    x, g, w1, b1, w2 = (_dev(t[k]) for k in ("x", "gamma", "w1", "b1", "w2"))
    comm = L.TpComm()
    comm.rank, comm.world = 2, 2
    with pytest.raises(L.TFB200Error):
        ops.fused_mlp_tp(x, g, w1, b1, w2, x, comm)
    comm.rank, comm.world, comm.max_rows = 0, 1, 64  # peer buffers missing
    with pytest.raises(L.TFB200Error):
        ops.fused_mlp_tp(x, g, w1, b1, w2, x, comm)
    comm.max_rows = 2  # fewer rows than the call has
    with pytest.raises(L.TFB200Error):
        ops.fused_mlp_tp(x, g, w1, b1, w2, x, comm)
    assert ctypes.c_size_t(L.lib().tfb200_tp_buffer_bytes(0, 8, 1)).value == 0
    assert ctypes.c_size_t(L.lib().tfb200_tp_buffer_bytes(65, 8, 1)).value == 0


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from tfb200 import _lib as L
    from tfb200.tp import TPDecodeMLP, TPDecodeMLPFused

    full = _case(64, K, H)
    dev = f"cuda:{rank}"
    w1, b1, w2, g = (_dev(full[k], dev) for k in ("w1", "b1", "w2", "gamma"))
    fused = TPDecodeMLPFused(w1, b1, w2, g, rank=rank, world=world, max_rows=64, eps=1e-5, gelu="tanh")
    nccl = TPDecodeMLP(w1, b1, w2, g, rank=rank, world=world, eps=1e-5, gelu="tanh")
    got = {}
    for i, m in enumerate(ROWS * 2):
        x = _dev(_case(m, K, H)["x"], dev)
        y = fused(x, x).clone()
        ref = nccl(x, x)
        got[f"y{i}"] = y.view(torch.int16).cpu().numpy()
        got[f"n{i}"] = ref.view(torch.int16).cpu().numpy()
    torch.cuda.synchronize()
    got["status"] = np.array([L.lib().tfb200_device_status()])
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **got)
    dist.barrier()
    fused.close()
    dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_tp_across_gpus(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (ranks on one GPU would wait on one another)")
    from tfb200 import _lib as L

    port = 31000 + (os.getpid() % 1000)
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    outs = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for o in outs:
        assert int(o["status"][0]) == L.TFB200_OK
    for i, m in enumerate(ROWS * 2):
        want = _golden(dict(_case(64, K, H), x=_case(m, K, H)["x"]), "tanh")
        ys = [o[f"y{i}"] for o in outs]
        for y in ys[1:]:
            assert np.array_equal(y, ys[0]), f"ranks disagree at call {i}"
        res = parity(f32(ys[0].view(np.uint16)), want)
        assert res["ok"], (i, m, res)
        res_n = parity(f32(outs[0][f"n{i}"].view(np.uint16)), want)
        assert res_n["ok"], (i, m, res_n)


def _timeout_rank(rank, world, port, out_dir):
    """Rank body of the timeout test: call 0 on every rank, call 1 on rank 0 only (rank 1 skips it, with no
    kernel of its own in flight), then recovery and call 2 on every rank."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from tfb200 import _lib as L
    from tfb200.tp import TPDecodeMLPFused

    lib = L.lib()
    lib.tfb200_set_wait_limit_ns(50_000_000)  # 50 ms: the waits of the skipped call run out quickly
    full = _case(64, K, H)
    dev = f"cuda:{rank}"
    w1, b1, w2, g = (_dev(full[k], dev) for k in ("w1", "b1", "w2", "gamma"))
    fused = TPDecodeMLPFused(w1, b1, w2, g, rank=rank, world=world, max_rows=64, eps=1e-5, gelu="tanh")
    x = _dev(_case(32, K, H)["x"], dev)
    got = {}
    got["y0"] = fused(x, x).clone().view(torch.int16).cpu().numpy()
    torch.cuda.synchronize()
    got["s0"] = np.array([lib.tfb200_device_status()])
    dist.barrier()
    if rank == 0:  # rank 1 leaves this step out
        fused(x, x)
        torch.cuda.synchronize()
    got["s1"] = np.array([lib.tfb200_device_status()])
    dist.barrier()
    # Recovery: the buffers are in an unknown state after a timeout; zero them and clear the status word.
    fused.buf.zero_()
    torch.cuda.synchronize()
    lib.tfb200_clear_device_status()
    dist.barrier()
    x2 = _dev(_case(7, K, H)["x"], dev)
    got["y2"] = fused(x2, x2).clone().view(torch.int16).cpu().numpy()
    torch.cuda.synchronize()
    got["s2"] = np.array([lib.tfb200_device_status()])
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **got)
    dist.barrier()
    fused.close()
    dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_fused_tp_times_out_when_a_rank_skips_a_call(tmp_path):
    """Failure detection across GPUs: a rank that does not make a call leaves the other rank's cross-GPU waits
    (the owner of a column block waiting for the other ranks' partial sums, and the wait for every block's
    arrival) without a partner. The waits are bounded: the kernel gives up, records TFB200_ETIMEOUT in the
    device status word and returns; nothing faults or hangs, and after zeroing the buffers and clearing the
    status both ranks compute the next call correctly. The reference's counterpart is its host-side failure
    contract (scripts/run_generated.sh:17-23: a failed run is reported, not hung)."""
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (ranks on one GPU would wait on one another)")
    from tfb200 import _lib as L

    port = 32000 + (os.getpid() % 1000)
    mp.start_processes(_timeout_rank, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    outs = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    assert [int(o["s0"][0]) for o in outs] == [L.TFB200_OK] * world
    assert int(outs[0]["s1"][0]) == L.TFB200_ETIMEOUT  # rank 0 waited for rank 1 and gave up
    assert int(outs[1]["s1"][0]) == L.TFB200_OK  # rank 1 launched nothing
    assert [int(o["s2"][0]) for o in outs] == [L.TFB200_OK] * world
    full = _case(64, K, H)
    for key, m in (("y0", 32), ("y2", 7)):
        ys = [o[key] for o in outs]
        assert np.array_equal(ys[0], ys[1]), f"ranks disagree on {key}"
        want = _golden(dict(full, x=_case(m, K, H)["x"]), "tanh")
        res = parity(f32(ys[0].view(np.uint16)), want)
        assert res["ok"], (key, res)
