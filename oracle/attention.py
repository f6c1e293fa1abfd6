"""Spiking self-attention oracle (test infrastructure; see oracle/__init__.py).

Restates the reference's spiking self-attention block
  snn_compiler/tests/test_spike_attention.py:55-80   (_RefSSA: input LIF, Q/K/V =
      LIF(BN(Conv1d 1x1)), a = (q @ (k^T @ v)) * scale, attn LIF, proj Conv1d + BN)
  snn_compiler/nn/attention.py:133-164               (FusedSpikeAttention.forward)
  snn_compiler/kernels/attention.py:49-104           (_spike_av_lif_kernel: the attn
      LIF takes (q @ kv) with scale folded into its input scale)
on a token-major layout x [T, B, N, D] (a Conv1d 1x1 over channels is a Linear
over the feature axis).  Every LIF is multi-step, tau = 2, decay_input, hard
reset to 0, each with its own threshold.  Since q, k, v are {0,1}, k^T v and
q (k^T v) are exact integers in float32, so the product order (q k^T) v of the
benchmark description equals q (k^T v) exactly.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import bitops, neurons as _n
from .vgg import fold_conv_bn


def lif_tokens(y, bias=None, *, vth, tau=2.0):
    """Multi-step LIF over y [T, ...] with features on the last axis (bias per feature)."""
    T = y.shape[0]
    C = y.shape[-1]
    df, sc = _n.neuron_params("lif", tau=tau, decay_input=True)
    r = _n.lif_multistep(y.reshape(T, -1).contiguous().numpy(), df=df, sc=sc, hard_reset=True,
                         v_reset=0.0, thr=float(vth), C=C, HW=1,
                         bias=None if bias is None else bias.contiguous().numpy(),
                         channel_last=True)
    return torch.from_numpy(r["spikes"]).reshape(y.shape)


def _proj(x, p, fold):
    """Linear (+ folded or eval BN) -> (pre-activation, bias-for-LIF)."""
    if fold:
        w, b = fold_conv_bn(p["w"], p.get("b"), p["gamma"], p["beta"], p["mean"], p["var"], p["eps"])
        return F.linear(x, w, None), b
    y = F.linear(x, p["w"], p.get("b"))
    shp = y.shape
    y = F.batch_norm(y.reshape(-1, shp[-1]), p["mean"], p["var"], p["gamma"], p["beta"],
                     training=False, eps=p["eps"]).reshape(shp)
    return y, None


def ktv(k, v):
    """K^T V per (t, b, head): k, v [T,B,H,N,d] {0,1} -> [T,B,H,d,d] (float32 integers)."""
    return k.transpose(-2, -1) @ v


def ktv_popcount(k, v):
    """Same product through the packed popcount form (attention.py:245-258)."""
    T, B, H, N, d = k.shape
    kp = bitops.pack_rows(k.reshape(-1, N, d).transpose(1, 2).numpy())   # [TBH, d, W]
    vp = bitops.pack_rows(v.reshape(-1, N, d).transpose(1, 2).numpy())
    out = np.stack([bitops.popc_and_gemm(kp[i], vp[i]) for i in range(kp.shape[0])])
    return torch.from_numpy(out.astype(np.float32)).reshape(T, B, H, d, d)


def ssa_forward(x, P, *, heads, scale=0.125, in_vth=None, qkv_vth=0.3, attn_vth=0.5,
                out_vth=None, fold=True, collect=False):
    """x [T, B, N, D] -> output [T, B, N, D].

    in_vth  : threshold of the input LIF (None = input already spikes, no LIF).
    out_vth : threshold of an output LIF after proj+BN (None = return proj+BN).
    """
    T, B, N, D = x.shape
    d = D // heads
    h = x.to(torch.float32)
    if in_vth is not None:
        h = lif_tokens(h, vth=in_vth)
    qkv = []
    for nm in ("q", "k", "v"):
        y, b = _proj(h, P[nm], fold)
        s = lif_tokens(y, b, vth=qkv_vth)
        qkv.append(s.reshape(T, B, N, heads, d).permute(0, 1, 3, 2, 4).contiguous())
    q, k, v = qkv
    kv = ktv(k, v)
    a = q @ kv                                            # [T,B,H,N,d], exact integers
    attn = lif_tokens(a.permute(0, 1, 3, 2, 4).reshape(T, B, N, D) * scale, vth=attn_vth)
    y, b = _proj(attn, P["proj"], fold)
    if out_vth is not None:
        out = lif_tokens(y, b, vth=out_vth)
    else:
        out = y if b is None else y + b
    if collect:
        return out, {"q": q, "k": k, "v": v, "kv": kv, "attn": attn}
    return out


def ssa_params_from_ref_state(sd, C):
    """Map the reference _RefSSA state_dict (Conv1d k=1 + BatchNorm1d) to this layout."""
    P = {}
    for nm in ("q", "k", "v", "proj"):
        w = torch.as_tensor(sd[f"{nm}_conv.weight"]).reshape(C, C)
        b = sd.get(f"{nm}_conv.bias")
        P[nm] = {"w": w, "b": None if b is None else torch.as_tensor(b),
                 "gamma": torch.as_tensor(sd[f"{nm}_bn.weight"]),
                 "beta": torch.as_tensor(sd[f"{nm}_bn.bias"]),
                 "mean": torch.as_tensor(sd[f"{nm}_bn.running_mean"]),
                 "var": torch.as_tensor(sd[f"{nm}_bn.running_var"]), "eps": 1e-5}
    return P
