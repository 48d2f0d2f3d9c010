"""Tensor-parallel decode MLP over the GPUs of one node.

The reference has no multi-device path: its two-chip n300 card exists only as a
multiplier in the planner's arithmetic (tensixflow include/tensixflow/Generated/
DeviceSpecs.h CoreGrid::totalCores). Here the decode-shaped MLP block is split
the standard way: W1 by columns and b1 alongside, W2 by rows. Each GPU runs the
streamed kernels on its shard (``ops.fused_mlp_partial``, fp32 [M, N] partial
sum), one all-reduce sums the partials (NCCL over NVLink / NVSwitch through
``torch.distributed``), and ``ops.residual_add`` adds the residual and rounds.
RMSNorm is computed redundantly on every GPU from the full X.

``TPDecodeMLPFused`` drops the separate all-reduce: the down-projection kernel
adds its fp32 partial sums straight into the owning rank's accumulator over
NVLink peer memory (CUDA IPC between the processes), and the last contributor to
each 128-column block finishes it (residual, bf16) and writes it to every rank.

The host logic takes its partial, all-reduce and finish steps as arguments so
that the sharding and reduction order can be checked on CPU ranks (gloo).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

__all__ = ["Shard", "shard_mlp", "tp_forward", "TPDecodeMLP", "TPDecodeMLPFused", "exchange_handles"]


@dataclass
class Shard:
    w1: object   # [K, H / world] columns of W1
    b1: object   # [H / world] slice of b1 (or None)
    w2: object   # [H / world, N] rows of W2
    cols: tuple  # (first, stop) hidden columns owned


def shard_mlp(w1, b1, w2, rank: int, world: int) -> Shard:
    """This rank's slice of the MLP weights (numpy arrays or torch tensors).

    H must divide evenly by the world size, and each shard is made contiguous.
    """
    H = w1.shape[1]
    if w2.shape[0] != H:
        raise ValueError("w1 columns and w2 rows differ")
    if H % world:
        raise ValueError(f"hidden width {H} is not divisible by {world} ranks")
    hs = H // world
    lo, hi = rank * hs, (rank + 1) * hs

    def cont(t):
        return t.contiguous() if hasattr(t, "contiguous") else t.copy()

    return Shard(cont(w1[:, lo:hi]), cont(b1[lo:hi]) if b1 is not None else None, cont(w2[lo:hi, :]), (lo, hi))


def tp_forward(x, residual, shard: Shard, partial_fn: Callable, all_reduce_fn: Callable, finish_fn: Callable):
    """partial on this shard -> all-reduce (sum) in place -> residual add."""
    part = partial_fn(x, shard)
    all_reduce_fn(part)
    return finish_fn(part, residual)


class TPDecodeMLP:
    """The decode MLP block on `world` GPUs of one node (one process per GPU)."""

    def __init__(self, w1, b1, w2, gamma, rank: int, world: int, eps: float = 1e-5, gelu: str = "tanh",
                 group=None):
        import torch

        from . import _lib as L
        from . import ops

        self.ops = ops
        self.L = L
        self.shard = shard_mlp(w1, b1, w2, rank, world)
        self.gamma = gamma
        self.eps = eps
        self.gelu = gelu
        self.group = group
        self.world = world
        self._ws = None
        self._part = None
        self.torch = torch

    def partial(self, x, shard: Shard):
        M, N = x.shape[0], shard.w2.shape[1]
        if self._part is None or tuple(self._part.shape) != (M, N):
            self._part = self.torch.empty(M, N, dtype=self.torch.float32, device=x.device)
        K, H = shard.w1.shape
        need = int(self.L.lib().tfb200_fused_mlp_partial_workspace_size(M, K, H, N))
        if self._ws is None or self._ws.numel() < need:  # allocated once per shape growth, not per call
            self._ws = self.torch.empty(max(need, 256), dtype=self.torch.uint8, device=x.device)
        return self.ops.fused_mlp_partial(x, self.gamma, shard.w1, shard.b1, shard.w2, self.eps, self.gelu,
                                          out=self._part, workspace=self._ws)

    def all_reduce(self, t):
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def __call__(self, x, residual, out=None):
        return tp_forward(x, residual, self.shard, self.partial, self.all_reduce,
                          lambda p, r: self.ops.residual_add(p, r, out=out))


def exchange_handles(local: tuple, rank: int, world: int, gather_fn: Callable) -> list:
    """Every rank's (handle bytes, offset) pair, in rank order. ``gather_fn(obj)`` returns the list of
    all ranks' objects (``torch.distributed.all_gather_object`` on GPUs, a gloo group on CPU)."""
    got = gather_fn(local)
    if len(got) != world:
        raise RuntimeError(f"handle exchange returned {len(got)} entries for {world} ranks")
    if tuple(got[rank]) != tuple(local):
        raise RuntimeError("handle exchange returned another rank's entry in this rank's slot")
    return [tuple(g) for g in got]


class TPDecodeMLPFused:
    """The decode MLP on `world` GPUs with the all-reduce inside the down-projection kernel.

    Every rank allocates one zero-filled buffer (local sums and counters, one receive slot per rank, arrival
    counters, bf16 output, done counter) for up to ``max_rows`` token rows and shares it with CUDA IPC. All ranks
    must make the same calls in the same order. ``__call__`` returns a view of this rank's output buffer, valid
    until the next call. After a device timeout the buffers are in an unknown state: build a new instance.
    """

    def __init__(self, w1, b1, w2, gamma, rank: int, world: int, max_rows: int = 64, eps: float = 1e-5,
                 gelu: str = "tanh", group=None):
        import ctypes

        import torch

        from . import _lib as L
        from . import ops

        if not 1 <= world <= L.MAX_TP:
            raise ValueError(f"world size {world} outside 1..{L.MAX_TP}")
        self.L, self.ops, self.torch, self.ctypes = L, ops, torch, ctypes
        self.shard = shard_mlp(w1, b1, w2, rank, world)
        self.gamma, self.eps, self.gelu = gamma, eps, gelu
        self.rank, self.world, self.max_rows = rank, world, max_rows
        self.N = w2.shape[1]
        self.calls = 0
        lib = L.lib()
        nbytes = int(lib.tfb200_tp_buffer_bytes(max_rows, self.N, world))
        if nbytes == 0:
            raise ValueError("tfb200_tp_buffer_bytes: bad shape (max_rows must be 1..64)")
        # 256-byte aligned, zero-filled (the caching allocator returns 512-byte aligned blocks)
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=w1.device)
        torch.cuda.synchronize(w1.device)
        self._opened = []
        bases = [0] * world
        bases[rank] = self.buf.data_ptr()
        if world > 1:
            import torch.distributed as dist

            handle = (ctypes.c_char * 64)()
            off = ctypes.c_size_t()
            L.check(lib.tfb200_ipc_get(ctypes.c_void_p(self.buf.data_ptr()), handle, ctypes.byref(off)))

            def gather(obj):
                out = [None] * world
                dist.all_gather_object(out, obj, group=group)
                return out

            peers = exchange_handles((bytes(handle), off.value), rank, world, gather)
            for r, (h, o) in enumerate(peers):
                if r == rank:
                    continue
                base = ctypes.c_void_p()
                L.check(lib.tfb200_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(base)))
                self._opened.append(base.value)
                bases[r] = base.value + o
        self.comm = L.TpComm()
        self.comm.rank, self.comm.world, self.comm.max_rows = rank, world, max_rows
        for r in range(world):
            self.comm.peer_buf[r] = bases[r]
        out = ctypes.c_void_p()
        L.check(lib.tfb200_tp_output(ctypes.byref(self.comm), self.N, ctypes.byref(out)))
        o = out.value - self.buf.data_ptr()
        self._out_flat = self.buf[o:o + max_rows * self.N * 2].view(torch.bfloat16)
        self._ws = None
        # Every rank's buffer is zero before any rank's first call.
        if world > 1:
            torch.distributed.barrier(group=group)

    def __call__(self, x, residual):
        M = x.reshape(-1, x.shape[-1]).shape[0]
        if M > self.max_rows:
            raise ValueError(f"{M} token rows, this instance was built for at most {self.max_rows}")
        if self._ws is None:
            K, H = self.shard.w1.shape
            need = int(self.L.lib().tfb200_fused_mlp_partial_workspace_size(self.max_rows, K, H, self.N))
            self._ws = self.torch.empty(max(need, 256), dtype=self.torch.uint8, device=x.device)
        self.ops.fused_mlp_tp(x, self.gamma, self.shard.w1, self.shard.b1, self.shard.w2, residual, self.comm,
                              self.eps, self.gelu, workspace=self._ws)
        self.calls += 1
        return self._out_flat[:M * self.N].view(M, self.N)

    def close(self):
        for base in self._opened:
            self.L.lib().tfb200_ipc_close(self.ctypes.c_void_p(base))
        self._opened = []
