"""Bit packing and popcount GEMM oracle (test infrastructure; see oracle/__init__.py).

Packing follows the reference's torch bit-pack
  snn_compiler/explore/attention/phase6b_bitpack.py:35-46   (bitpack_N)
and Triton pack kernel
  snn_compiler/kernels/attention.py:195-214                  (_pack_N_kernel):
32 consecutive elements of the packed axis go into one 32-bit word, element
32*w + i in bit i (LSB first); a ragged tail is zero-padded.

The popcount contraction follows
  snn_compiler/kernels/attention.py:217-233                  (_ktv_popcount_kernel):
  C[i, j] = sum_w popc(A[i, w] & B[j, w])                     ({0,1} x {0,1})
and its {0,1} x {-1,+1} generalisation (B bit = 1 <=> +1):
  C[i, j] = 2 * sum_w popc(A[i, w] & B[j, w]) - sum_w popc(A[i, w])
which equals the unpacked integer product A @ B exactly.
"""
from __future__ import annotations

import numpy as np


def pack_rows(bits) -> np.ndarray:
    """bits [..., K] (any dtype, nonzero = 1) -> uint32 [..., ceil(K/32)], LSB first."""
    b = np.asarray(bits) != 0
    K = b.shape[-1]
    W = (K + 31) // 32
    pad = W * 32 - K
    if pad:
        b = np.concatenate([b, np.zeros(b.shape[:-1] + (pad,), bool)], axis=-1)
    by = np.packbits(b, axis=-1, bitorder="little")          # [..., 4W] uint8
    return np.ascontiguousarray(by).view("<u4").reshape(b.shape[:-1] + (W,)).astype(np.uint32)


def unpack_rows(words, K) -> np.ndarray:
    w = np.ascontiguousarray(np.asarray(words, dtype=np.uint32)).view(np.uint8)
    bits = np.unpackbits(w.reshape(words.shape[:-1] + (-1,)), axis=-1, bitorder="little")
    return bits[..., :K]


def _popcount32(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.uint32)
    if hasattr(np, "bitwise_count"):
        return np.bitwise_count(x).astype(np.int64)
    x = x - ((x >> 1) & 0x55555555)
    x = (x & 0x33333333) + ((x >> 2) & 0x33333333)
    x = (x + (x >> 4)) & 0x0F0F0F0F
    return ((x * 0x01010101) & 0xFFFFFFFF) >> 24


def popc_and_gemm(Ap, Bp) -> np.ndarray:
    """C[i,j] = sum_w popc(Ap[i,w] & Bp[j,w]) for packed [M,W] and [N,W] (int64)."""
    Ap = np.asarray(Ap, np.uint32)
    Bp = np.asarray(Bp, np.uint32)
    M, W = Ap.shape
    N = Bp.shape[0]
    out = np.zeros((M, N), np.int64)
    for w in range(W):
        out += _popcount32(Ap[:, w:w + 1] & Bp[None, :, w])
    return out


def bgemm_01_pm1(Ap, Bp) -> np.ndarray:
    """{0,1} x {-1,+1} product from packed operands (int64)."""
    pa = _popcount32(np.asarray(Ap, np.uint32)).sum(axis=1)
    return 2 * popc_and_gemm(Ap, Bp) - pa[:, None]


def int_matmul(A, B) -> np.ndarray:
    """The unpacked reference product A @ B in int64 (BASELINE's bit-exact target)."""
    return np.asarray(A, np.int64) @ np.asarray(B, np.int64)


def bgemm_row_col_checksums(A01, Bpm1):
    """Size-independent checks for a full-size C = A @ B without forming C:
    row sums C @ 1 = A @ (B @ 1) and column sums 1^T C = (1^T A) @ B, both int64.
    A01 [M, K] {0,1}, Bpm1 [K, N] {-1,+1} (any integer dtype)."""
    A = np.asarray(A01, np.int64)
    B = np.asarray(Bpm1, np.int64)
    row = A @ B.sum(axis=1)
    col = A.sum(axis=0) @ B
    return row, col
