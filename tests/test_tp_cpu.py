"""Host logic of the tensor-parallel decode MLP on two CPU ranks (gloo).

Each rank shards the weights, computes its partial sum with the oracle standing
in for the GPU kernel (no device here), the partials are all-reduced over gloo,
and the residual is added; the result must equal the unsharded oracle.
"""

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _case():
    rng = np.random.default_rng(9)
    m, k, h, n = 4, 32, 48, 32
    return dict(x=rng.standard_normal((m, k)).astype(np.float32), g=(0.5 + rng.random(k)).astype(np.float32),
                w1=(rng.standard_normal((k, h)) / np.sqrt(k)).astype(np.float32),
                b1=(0.02 * rng.standard_normal(h)).astype(np.float32),
                w2=(rng.standard_normal((h, n)) / np.sqrt(h)).astype(np.float32))


def _worker(rank, world, port, out_path):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "tt-flow_b200")]
    from oracle import golden as O
    from tfb200.tp import shard_mlp, tp_forward

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    c = _case()
    sh = shard_mlp(c["w1"], c["b1"], c["w2"], rank, world)

    def partial(x, s):
        hid = O.matmul(O.rmsnorm(x, c["g"], 1e-5), s.w1) + s.b1
        return torch.from_numpy(O.matmul(O.gelu_tanh(hid), s.w2))

    def all_reduce(t):
        dist.all_reduce(t, op=dist.ReduceOp.SUM)

    y = tp_forward(c["x"], c["x"], sh, partial, all_reduce, lambda p, r: p.numpy() + r)
    if rank == 0:
        np.save(out_path, y)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_sharding_matches_unsharded_oracle(tmp_path, world):
    from oracle import golden as O

    port = 29500 + (os.getpid() % 1000)
    out = str(tmp_path / "y.npy")
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
    c = _case()
    want = O.fused_mlp(c["x"], c["g"], c["w1"], c["b1"], c["w2"], c["x"], 1e-5, "tanh")
    got = np.load(out)
    assert np.allclose(got, want, rtol=1e-5, atol=1e-5)


def test_shard_rejects_uneven_split():
    from tfb200.tp import shard_mlp

    c = _case()
    with pytest.raises(ValueError):
        shard_mlp(c["w1"], c["b1"], c["w2"], 0, 5)


def test_shards_cover_hidden_dimension_once():
    from tfb200.tp import shard_mlp

    c = _case()
    shards = [shard_mlp(c["w1"], c["b1"], c["w2"], r, 4) for r in range(4)]
    assert np.array_equal(np.concatenate([s.w1 for s in shards], axis=1), c["w1"])
    assert np.array_equal(np.concatenate([s.w2 for s in shards], axis=0), c["w2"])
    assert np.array_equal(np.concatenate([s.b1 for s in shards]), c["b1"])


def _exchange_worker(rank, world, port, out_path):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "tt-flow_b200")]
    from tfb200.tp import exchange_handles

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    local = (bytes([rank]) * 64, 256 * rank)

    def gather(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    peers = exchange_handles(local, rank, world, gather)
    if rank == 0:
        np.save(out_path, np.array([[h[0], o] for h, o in peers]))
    dist.barrier()
    dist.destroy_process_group()


def test_ipc_handle_exchange_in_rank_order(tmp_path):
    """Each rank's IPC handle and offset reach every rank in rank order (gloo stands in for NCCL)."""
    world = 3
    port = 30500 + (os.getpid() % 1000)
    out = str(tmp_path / "peers.npy")
    mp.start_processes(_exchange_worker, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
    got = np.load(out)
    assert got.tolist() == [[r, 256 * r] for r in range(world)]


def test_exchange_rejects_misordered_gather():
    from tfb200.tp import exchange_handles

    with pytest.raises(RuntimeError):
        exchange_handles((b"a", 0), 0, 2, lambda obj: [(b"b", 0), obj])
    with pytest.raises(RuntimeError):
        exchange_handles((b"a", 0), 0, 2, lambda obj: [obj])
