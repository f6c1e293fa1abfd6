"""Batch-sharded data-parallel inference across the GPUs of one node.

The reference has no multi-GPU code; the scaling layer here is the minimum the path
needs: one process per GPU, each running its own copy of the engine on a contiguous
slice of the global batch, and one all-gather of the per-sample results (logits) in
rank order.  Inputs never cross GPUs; the only collective is that all-gather (NCCL over
NVLink on B200 nodes, gloo on CPU for tests).

The all-gather can run off the critical path: ``submit`` issues the engine's forward on
the caller's stream and the all-gather on a side stream that waits only for that forward,
so the next ``submit``'s forward overlaps it.  Results land in preallocated slots (two by
default), so a steady serving loop allocates nothing per call.
"""
from __future__ import annotations

import inspect

import torch


def shard_range(global_batch: int, rank: int, world: int):
    """[start, stop) of rank's contiguous slice; the first (global_batch % world) ranks take
    one extra sample, so slices differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class Pending:
    """Result of ShardedInference.submit.  ``wait()`` makes the caller's current stream wait
    for the all-gather and returns the [global_batch, ...] result (a view into the slot,
    valid until the slot is reused ``slots`` submits later).  With ``defer=True`` the
    all-gather is issued by ``start()`` (or by ``wait()``), so a caller can place it after
    work it issues later (e.g. to overlap it with the next forward only)."""

    def __init__(self, owner=None, args=None, result=None, event=None):
        self._owner, self._args = owner, args
        self._result, self._event = result, event

    def start(self, after: "torch.cuda.Event | None" = None) -> "Pending":
        if self._args is not None:
            self._result, self._event = self._owner._gather_async(*self._args, after=after)
            self._args = None
        return self

    @property
    def done_event(self):
        return self._event

    def wait(self) -> torch.Tensor:
        self.start()
        if self._event is not None:
            torch.cuda.current_stream().wait_event(self._event)
        return self._result


class ShardedInference:
    """Runs `engine(x_local) -> [B_local, ...]` on this rank's slice and all-gathers the
    results of every rank into [global_batch, ...] (rank order = batch order).

    Slices of unequal size are padded to the largest slice for the collective and the
    padding is dropped afterwards, so any global batch of at least one sample per rank
    works; a global batch smaller than the world is rejected on every rank before any
    rank runs its engine or joins the collective (so no rank waits for a peer that
    raised).  If the engine accepts an ``out=`` keyword (SpikingVGG.forward does), it
    writes its result straight into the slot the all-gather sends from.
    """

    def __init__(self, engine, group=None, *, slots: int = 2):
        import torch.distributed as dist
        self.engine = engine
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.slots = max(1, int(slots))
        self._k = 0
        # (per, tail shape, dtype, device) -> [(send, recv, gathered event, forward event)]
        self._bufs = {}
        self._side = None
        self._index = {}
        try:
            self._engine_out = "out" in inspect.signature(engine).parameters
        except (TypeError, ValueError):
            self._engine_out = False

    # ---- batch split ----------------------------------------------------------------------
    def _check_batch(self, global_batch: int):
        if global_batch < self.world:
            raise ValueError(f"global batch {global_batch} is smaller than the world size "
                             f"{self.world}: every rank needs at least one sample")

    def local_slice(self, x_global: torch.Tensor, batch_dim: int = 0) -> torch.Tensor:
        s, e = shard_range(x_global.shape[batch_dim], self.rank, self.world)
        return x_global.narrow(batch_dim, s, e - s)

    def _slot(self, per, tail, dtype, device):
        key = (per, tuple(tail), dtype, str(device))
        if key not in self._bufs:
            self._bufs[key] = [
                (torch.zeros((per,) + tuple(tail), dtype=dtype, device=device),
                 torch.empty((per * self.world,) + tuple(tail), dtype=dtype, device=device),
                 torch.cuda.Event() if device.type == "cuda" else None,
                 torch.cuda.Event() if device.type == "cuda" else None)
                for _ in range(self.slots)]
        bufs = self._bufs[key]
        slot = bufs[self._k % len(bufs)]
        self._k += 1
        return slot

    def _result_view(self, recv, global_batch, per):
        if global_batch == per * self.world:
            return recv
        # drop each rank's padding rows: ranks >= extra hold one sample fewer
        key = (global_batch, per, str(recv.device))
        if key not in self._index:
            idx = []
            for r in range(self.world):
                s, e = shard_range(global_batch, r, self.world)
                idx.extend(r * per + i for i in range(e - s))
            self._index[key] = torch.tensor(idx, device=recv.device)
        return recv.index_select(0, self._index[key])

    # ---- synchronous form -----------------------------------------------------------------
    def gather(self, y_local: torch.Tensor, global_batch: int) -> torch.Tensor:
        """All-gather y_local [B_local, ...] of every rank into [global_batch, ...] on the
        current stream."""
        if self.world == 1:
            return y_local
        self._check_batch(global_batch)
        per = -(-global_batch // self.world)
        send, recv, _, _ = self._slot(per, y_local.shape[1:], y_local.dtype, y_local.device)
        if y_local.data_ptr() != send.data_ptr():
            send[:y_local.shape[0]].copy_(y_local)
        self.dist.all_gather_into_tensor(recv, send, group=self.group)
        return self._result_view(recv, global_batch, per)

    def __call__(self, x_global: torch.Tensor, batch_dim: int = 0) -> torch.Tensor:
        return self.submit(x_global, batch_dim, overlap=False).wait()

    # ---- asynchronous form ----------------------------------------------------------------
    def submit(self, x_global: torch.Tensor, batch_dim: int = 0, *, overlap: bool = True,
               out_shape=None, out_dtype=torch.float32, defer: bool = False) -> Pending:
        """Forward this rank's slice on the current stream; all-gather on a side stream (CUDA,
        overlap=True) that waits only for this forward, so the caller can issue the next
        forward at once.  ``out_shape`` (the per-sample result shape) lets an engine that
        takes ``out=`` write into the send slot directly.  A slot's send buffer is rewritten
        only after its previous all-gather has read it (the forward waits for that event)."""
        gb = x_global.shape[batch_dim]
        if self.world > 1:
            self._check_batch(gb)
        return self.submit_local(self.local_slice(x_global, batch_dim), gb, batch_dim,
                                 overlap=overlap, out_shape=out_shape, out_dtype=out_dtype,
                                 defer=defer)

    def submit_local(self, x: torch.Tensor, global_batch: int, batch_dim: int = 0, *,
                     overlap: bool = True, out_shape=None, out_dtype=torch.float32,
                     defer: bool = False) -> Pending:
        """``submit`` for a caller that already holds only this rank's slice ``x`` (rows
        shard_range(global_batch, rank, world) of the global batch)."""
        gb = global_batch
        if self.world == 1:
            return Pending(result=self.engine(x))
        self._check_batch(gb)
        s, e = shard_range(gb, self.rank, self.world)
        if x.shape[batch_dim] != e - s:
            raise ValueError(f"rank {self.rank} holds {x.shape[batch_dim]} samples, its slice "
                             f"of {gb} has {e - s}")
        per = -(-gb // self.world)
        dev = x.device
        on_gpu = dev.type == "cuda"
        cur = torch.cuda.current_stream(dev) if on_gpu else None
        direct = self._engine_out and out_shape is not None and x.shape[batch_dim] == per
        if direct:
            send, recv, done, fwd = self._slot(per, out_shape, out_dtype, dev)
            if on_gpu:
                cur.wait_event(done)             # the slot's last all-gather has read `send`
            y = self.engine(x, out=send)
        else:
            y = self.engine(x)
            send, recv, done, fwd = self._slot(per, y.shape[1:], y.dtype, dev)
            if on_gpu:
                cur.wait_event(done)
            send[:y.shape[0]].copy_(y)
        if not overlap or not on_gpu:
            self.dist.all_gather_into_tensor(recv, send, group=self.group)
            return Pending(result=self._result_view(recv, gb, per))
        fwd.record(cur)                          # this forward has written `send`
        p = Pending(self, (send, recv, done, fwd, gb, per))
        return p if defer else p.start()

    def _gather_async(self, send, recv, done, fwd, gb, per, after=None):
        if self._side is None:
            self._side = torch.cuda.Stream(device=send.device)
        self._side.wait_event(fwd)
        if after is not None:
            self._side.wait_event(after)
        with torch.cuda.stream(self._side):
            self.dist.all_gather_into_tensor(recv, send, group=self.group)
            res = self._result_view(recv, gb, per)
            done.record(self._side)
        return res, done
