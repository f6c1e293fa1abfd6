"""Spiking-attention entry points (K3), same API as the reference.

Mirrors snn_compiler/kernels/attention.py of the reference:
  spike_av_lif(q, kv, *, scale, ...)   attention.py:107-137
  spike_ktv(k, v)                      attention.py:177-187
  spike_ktv_popcount(k, v)             attention.py:245-258
  HAS_POPC                             attention.py:26-36 (always True here)
and adds spike_attention, the fused K^T V + Q kv + LIF.  Every call is one launch of
snnb_spike_attention_core (libsnnb200.so); K^T V is a bit-packed AND + popcount.
Tensors are [T, B, heads, N, d]; spikes may be float32 / bf16 / fp16 {0,1}.
"""
from __future__ import annotations

import torch

from .. import _lib

HAS_POPC = True


def _bf16(x):
    return x if x.dtype == torch.bfloat16 and x.is_contiguous() else \
        x.to(torch.bfloat16).contiguous()


def _coeffs(tau, decay, decay_input):
    if decay is None:
        dec = 1.0 if tau is None else (1.0 - 1.0 / tau)
    else:
        dec = float(decay)
    sc = (1.0 / tau) if (decay_input and tau is not None) else 1.0
    return dec, sc


def _core(q, k, v, kv_in, want_kv, want_spikes, strides, out_strides, T, B, H, N, d, *,
          scale=1.0, tau=2.0, decay=None, decay_input=True, v_threshold=0.5, v_reset=0.0,
          soft_reset=False, out=None, device=None):
    dec, sc = _coeffs(tau, decay, decay_input)
    kv_out = torch.empty(T, B, H, d, d, device=device, dtype=torch.float32) if want_kv else None
    if want_spikes and out is None:
        out = torch.empty(T, B, H, N, d, device=device, dtype=torch.bfloat16)
    st, sb, sh, sn = strides
    ot, ob, oh, on = out_strides
    L = _lib.lib()
    s = _lib.stream_of(q if q is not None else k)
    rc = L.snnb_spike_attention_core(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), st, sb, sh, sn,
                                     _lib.ptr(kv_in), _lib.ptr(kv_out),
                                     _lib.ptr(out) if want_spikes else None, ot, ob, oh, on,
                                     T, B, H, N, d, float(dec), float(sc), float(scale),
                                     float(v_threshold), float(v_reset),
                                     0 if soft_reset else 1, s)
    _lib.check(rc, "snnb_spike_attention_core")
    return kv_out, out


def _std_strides(T, B, H, N, d):
    return (B * H * N * d, H * N * d, N * d, d)


def spike_ktv(k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """kv = k^T @ v for spikes k, v [T, B, heads, N, d] -> float32 [T, B, heads, d, d]."""
    assert k.is_cuda and v.is_cuda and k.shape == v.shape
    T, B, H, N, D = k.shape
    kb, vb = _bf16(k), _bf16(v)
    kv, _ = _core(None, kb, vb, None, True, False, _std_strides(T, B, H, N, D), (0, 0, 0, 0),
                  T, B, H, N, D, device=k.device)
    return kv


def spike_ktv_popcount(k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Bit-exact K^T V through bit-packing + popcount (the same kernel as spike_ktv)."""
    return spike_ktv(k, v)


def spike_av_lif(q, kv, *, scale, tau=2.0, decay=None, decay_input=True, v_threshold=0.5,
                 v_reset=0.0, soft_reset=False):
    """(q @ kv) * scale -> multi-step LIF; q [T, B, heads, N, d] spikes, kv [T, B, heads, d, d].
    Returns spikes [T, B, heads, N, d] of q's dtype."""
    assert q.is_cuda and kv.is_cuda
    T, B, H, N, D = q.shape
    qb = _bf16(q)
    kvf = kv.to(torch.float32).contiguous()
    st = _std_strides(T, B, H, N, D)
    _, out = _core(qb, None, None, kvf, False, True, st, st, T, B, H, N, D, scale=scale, tau=tau,
                   decay=decay, decay_input=decay_input, v_threshold=v_threshold,
                   v_reset=v_reset, soft_reset=soft_reset, device=q.device)
    return out.to(q.dtype)


def spike_attention(q, k, v, *, scale, tau=2.0, decay=None, decay_input=True, v_threshold=0.5,
                    v_reset=0.0, soft_reset=False):
    """Fused LIF((q @ (k^T @ v)) * scale) for spikes [T, B, heads, N, d] -> spikes (q's dtype)."""
    assert q.shape == k.shape == v.shape
    T, B, H, N, D = q.shape
    st = _std_strides(T, B, H, N, D)
    _, out = _core(_bf16(q), _bf16(k), _bf16(v), None, False, True, st, st, T, B, H, N, D,
                   scale=scale, tau=tau, decay=decay, decay_input=decay_input,
                   v_threshold=v_threshold, v_reset=v_reset, soft_reset=soft_reset,
                   device=q.device)
    return out.to(q.dtype)


def attention_from_qkv(qkv: torch.Tensor, heads: int, *, scale, tau=2.0, decay=None,
                       decay_input=True, v_threshold=0.5, v_reset=0.0, soft_reset=False,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused core on a token-major projection output qkv [T, B, N, 3D] bf16 (q | k | v along
    the last axis, head h at columns h*d..h*d+d-1 of each) -> spikes [T, B, N, D] bf16."""
    assert qkv.is_cuda and qkv.dtype == torch.bfloat16 and qkv.is_contiguous()
    T, B, N, D3 = qkv.shape
    D = D3 // 3
    d = D // heads
    if out is None:
        out = torch.empty(T, B, N, D, device=qkv.device, dtype=torch.bfloat16)
    strides = (B * N * D3, N * D3, d, D3)
    ostr = (B * N * D, N * D, d, D)
    _core(qkv, qkv[..., D:], qkv[..., 2 * D:], None, False, True, strides, ostr, T, B, heads, N,
          d, scale=scale, tau=tau, decay=decay, decay_input=decay_input, v_threshold=v_threshold,
          v_reset=v_reset, soft_reset=soft_reset, out=out, device=qkv.device)
    return out
