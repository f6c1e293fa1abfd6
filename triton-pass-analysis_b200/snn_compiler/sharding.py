"""Batch-sharded data-parallel inference across the GPUs of one node.

The reference has no multi-GPU code; the scaling layer here is the minimum the path
needs: one process per GPU, each running its own copy of the engine on a contiguous
slice of the global batch, and one all-gather of the per-sample results (logits) in
rank order.  Inputs never cross GPUs; the only collective is that all-gather (NCCL over
NVLink on B200 nodes, gloo on CPU for tests).
"""
from __future__ import annotations

import torch


def shard_range(global_batch: int, rank: int, world: int):
    """[start, stop) of rank's contiguous slice; the first (global_batch % world) ranks take
    one extra sample, so slices differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class ShardedInference:
    """Runs `engine(x_local) -> [B_local, ...]` on this rank's slice and all-gathers the
    results of every rank into [global_batch, ...] (rank order = batch order).

    Slices of unequal size are padded to the largest slice for the collective and the
    padding is dropped afterwards, so any global batch works.
    """

    def __init__(self, engine, group=None):
        import torch.distributed as dist
        self.engine = engine
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def local_slice(self, x_global: torch.Tensor, batch_dim: int = 0) -> torch.Tensor:
        s, e = shard_range(x_global.shape[batch_dim], self.rank, self.world)
        return x_global.narrow(batch_dim, s, e - s)

    def gather(self, y_local: torch.Tensor, global_batch: int) -> torch.Tensor:
        if self.world == 1:
            return y_local
        per = -(-global_batch // self.world)
        pad = torch.zeros((per,) + tuple(y_local.shape[1:]), dtype=y_local.dtype,
                          device=y_local.device)
        pad[:y_local.shape[0]] = y_local
        out = torch.empty((per * self.world,) + tuple(y_local.shape[1:]), dtype=y_local.dtype,
                          device=y_local.device)
        self.dist.all_gather_into_tensor(out, pad, group=self.group)
        parts = []
        for r in range(self.world):
            s, e = shard_range(global_batch, r, self.world)
            parts.append(out[r * per: r * per + (e - s)])
        return torch.cat(parts, 0)

    def __call__(self, x_global: torch.Tensor, batch_dim: int = 0) -> torch.Tensor:
        y = self.engine(self.local_slice(x_global, batch_dim))
        return self.gather(y, x_global.shape[batch_dim])
