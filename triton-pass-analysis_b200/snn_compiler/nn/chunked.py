"""T-chunked execution (reference snn_compiler/nn/chunked.py:33-79).

A network whose neurons carry their state across calls (StatefulLIFNode) runs over a
long [T, B, ...] sequence chunk by chunk: every chunk flows through all layers, the
layers' potentials are handed to the next chunk, and the chunk outputs are
concatenated along T.  Peak activation memory is then that of one chunk.
"""
from __future__ import annotations

from typing import Callable, List

import torch
import torch.nn as nn


def run_chunked(forward_fn: Callable[[torch.Tensor, dict | None], tuple[torch.Tensor, dict]],
                x_seq: torch.Tensor, *, chunk_t: int = 16) -> torch.Tensor:
    """forward_fn(x_chunk, state) -> (y_chunk, new_state), state None on the first chunk.
    Returns the chunk outputs concatenated along T (one call when chunk_t >= T)."""
    T = x_seq.shape[0]
    if chunk_t >= T:
        out, _ = forward_fn(x_seq, None)
        return out
    outs: List[torch.Tensor] = []
    state = None
    for t0 in range(0, T, chunk_t):
        y, state = forward_fn(x_seq[t0:t0 + min(chunk_t, T - t0)].contiguous(), state)
        outs.append(y)
    return torch.cat(outs, dim=0)


class ChunkedForward(nn.Module):
    """Wraps a model with ``forward_chunked(x_chunk, state) -> (y, state)``; calling the
    wrapper runs run_chunked with the fixed chunk length.  A model without that method
    is called directly (no chunking)."""

    def __init__(self, model: nn.Module, *, chunk_t: int = 16):
        super().__init__()
        self.model = model
        self.chunk_t = chunk_t

    def forward(self, x_seq):
        if not hasattr(self.model, "forward_chunked"):
            return self.model(x_seq)
        return run_chunked(self.model.forward_chunked, x_seq, chunk_t=self.chunk_t)
