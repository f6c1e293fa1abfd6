"""Bit packing and the popcount binary GEMM (K4), backed by libsnnb200.so.

Generalises the reference's packed K^T V (snn_compiler/kernels/attention.py:195-258:
_pack_N_kernel, _ktv_popcount_kernel, spike_ktv_popcount) to a tiled GEMM over
packed rows:
  mode 0  {0,1} x {0,1}      C = A @ B
  mode 1  {0,1} x {-1,+1}    C = A @ B       (2 popc(a & b) - popc(a))
  mode 2  {-1,+1} x {-1,+1}  C = A @ B       (K - 2 popc(a ^ b), the XNOR form)
Results are int32 and exact.
"""
from __future__ import annotations

import math

import torch

from .. import _lib


def packed_words(K: int) -> int:
    """Words per packed row: ceil(K/32) rounded up to a multiple of 4 (16-byte rows)."""
    return ((K + 31) // 32 + 3) // 4 * 4


def bitpack(x: torch.Tensor, *, positive: bool = False, ldw: int | None = None) -> torch.Tensor:
    """Pack the last axis of x into uint32 words (returned as int32), LSB first.
    positive=False: bit = x != 0 ({0,1});  positive=True: bit = x > 0 ({-1,+1})."""
    assert x.is_cuda and x.is_contiguous()
    if x.dtype == torch.int8:
        x = x.view(torch.uint8)
    K = x.shape[-1]
    rows = math.prod(x.shape[:-1])
    ldw = packed_words(K) if ldw is None else ldw
    out = torch.empty(*x.shape[:-1], ldw, device=x.device, dtype=torch.int32)
    st = _lib.lib().snnb_bitpack(_lib.ptr(x), _lib.dtype_code(x.dtype), rows, K, ldw,
                                 int(positive), _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_bitpack")
    return out


def bgemm(Ap: torch.Tensor, Bp: torch.Tensor, K: int, *, mode: int = 1, splits: int = 0,
          out: torch.Tensor | None = None) -> torch.Tensor:
    """C[M, N] int32 from packed A [M, ldw] and B [N, ldw] (see module doc for modes)."""
    assert Ap.is_cuda and Bp.is_cuda and Ap.dtype == torch.int32 and Bp.dtype == torch.int32
    assert Ap.is_contiguous() and Bp.is_contiguous() and Ap.shape[1] == Bp.shape[1]
    M, ldw = Ap.shape
    N = Bp.shape[0]
    C = out if out is not None else torch.empty(M, N, device=Ap.device, dtype=torch.int32)
    st = _lib.lib().snnb_bgemm(_lib.ptr(Ap), _lib.ptr(Bp), _lib.ptr(C), M, N, K, ldw, mode,
                               splits, _lib.stream_of(Ap))
    _lib.check(st, "snnb_bgemm")
    return C


def binary_matmul(A: torch.Tensor, B: torch.Tensor, *, mode: int = 1) -> torch.Tensor:
    """A [M, K] @ B [K, N] for binary operands (mode as in bgemm), exact int32.
    B is packed along K (its transpose's rows); for a fixed weight matrix pack it
    once with bitpack(B.t().contiguous(), positive=True) and call bgemm directly."""
    K = A.shape[1]
    Ap = bitpack(A.contiguous(), positive=(mode == 2))
    Bp = bitpack(B.t().contiguous(), positive=(mode != 0))
    return bgemm(Ap, Bp, K, mode=mode)
