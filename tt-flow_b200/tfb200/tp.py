"""Tensor-parallel decode MLP over the GPUs of one node.

The reference has no multi-device path: its two-chip n300 card exists only as a
multiplier in the planner's arithmetic (tensixflow include/tensixflow/Generated/
DeviceSpecs.h CoreGrid::totalCores). Here the decode-shaped MLP block is split
the standard way: W1 by columns and b1 alongside, W2 by rows. Each GPU runs the
streamed kernels on its shard (``ops.fused_mlp_partial``, fp32 [M, N] partial
sum), one all-reduce sums the partials (NCCL over NVLink / NVSwitch through
``torch.distributed``), and ``ops.residual_add`` adds the residual and rounds.
RMSNorm is computed redundantly on every GPU from the full X.

The host logic takes its partial, all-reduce and finish steps as arguments so
that the sharding and reduction order can be checked on CPU ranks (gloo).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

__all__ = ["Shard", "shard_mlp", "tp_forward", "TPDecodeMLP"]


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

        from . import ops

        self.ops = ops
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
        return self.ops.fused_mlp_partial(x, self.gamma, shard.w1, shard.b1, shard.w2, self.eps, self.gelu,
                                          out=self._part, workspace=self._ws)

    def all_reduce(self, t):
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def __call__(self, x, residual, out=None):
        return tp_forward(x, residual, self.shard, self.partial, self.all_reduce,
                          lambda p, r: self.ops.residual_add(p, r, out=out))
