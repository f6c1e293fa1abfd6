"""Spiking self-attention block on the fused kernels (reference snn_compiler/nn/attention.py).

``SpikeAttentionBlock`` is the inference engine for a Spikformer / Spikingformer style
block on token-major spikes x [T, B, N, D]:

  (optional input LIF)                 snnb_neuron_multistep
  Q, K, V = LIF(BN(Linear(x)))         one snnb_linear_lif over the concatenated [3D, D]
                                       folded weights -> [T, B, N, 3D] spikes
  s = LIF((Q K^T V) * scale)           snnb_spike_attention_core (fused, v in registers)
  y = BN(Linear(s)) (+ optional LIF)   snnb_linear_f32 / snnb_linear_lif

BN is folded into the projections once (fold_conv_bn, snn_compiler/kernels/fused.py:585-599),
so results match the reference's fold_bn=True numerics.  ``FusedSpikeAttention`` keeps the
reference's constructor (from_reference on an SSA-style module with Conv1d 1x1 projections,
BatchNorm1d and LIF nodes exposing tau / v_threshold; nn/attention.py:62-164) and its
[T, B, C, H, W] forward.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..kernels import attention as KA
from ..kernels import conv as KC
from ..kernels.fused import fold_conv_bn
from ..kernels.neurons import neuron_multistep


def _fold(p):
    w = p["w"].detach().float()
    if w.ndim == 3:                       # Conv1d k=1 weight [out, in, 1]
        w = w[..., 0]
    b = p.get("b")
    return fold_conv_bn(w, None if b is None else b.detach().float(), p["gamma"].float(),
                        p["beta"].float(), p["mean"].float(), p["var"].float(), p["eps"])


class SpikeAttentionBlock:
    """Engine for one spiking self-attention block (see module doc)."""

    def __init__(self, P, *, heads: int, scale: float = 0.125, tau: float = 2.0,
                 in_vth: float | None = None, qkv_vth: float = 1.0, attn_vth: float = 0.5,
                 out_vth: float | None = 1.0, device="cuda", autotune: bool = True):
        self.heads, self.scale, self.tau = heads, float(scale), float(tau)
        self.in_vth, self.qkv_vth, self.attn_vth, self.out_vth = in_vth, qkv_vth, attn_vth, out_vth
        dev = torch.device(device)
        ws, bs = [], []
        for nm in ("q", "k", "v"):
            w, b = _fold(P[nm])
            ws.append(w)
            bs.append(b)
        self.w_qkv = torch.cat(ws, 0).to(torch.bfloat16).contiguous().to(dev)
        self.b_qkv = torch.cat(bs, 0).float().contiguous().to(dev)
        w, b = _fold(P["proj"])
        self.w_proj = w.to(torch.bfloat16).contiguous().to(dev)
        self.b_proj = b.float().contiguous().to(dev)
        self.D = self.w_proj.shape[0]
        self._bufs = {}
        self.autotune = autotune
        self.choice = {}          # (layer, T, rows) -> (variant, block_n, splits)
        self._workspace = None

    def _lin(self, name, x, w, b, vth, out):
        """linear + LIF through the fastest kernel configuration, timed on first use."""
        T, R, K = x.shape
        N = w.shape[0]
        key = (name, T, R)

        def launch(v, bn, sp):
            need = KC.split_workspace_bytes(T, R, 1, 1, N, sp)
            if need and (self._workspace is None or self._workspace.numel() * 4 < need):
                self._workspace = torch.empty(need // 4, device=x.device)
            return KC.linear_lif(x, w, b, tau=self.tau, v_threshold=vth, out=out, variant=v,
                                 block_n=bn, splits=sp,
                                 workspace=self._workspace if need else None)
        if key not in self.choice:
            self.choice[key] = KC.pick_fastest(launch, N, T, (K + 63) // 64) if self.autotune \
                else (0, 0, 1)
        return launch(*self.choice[key])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [T, B, N, D] spikes (or currents when an input LIF is configured) -> the
        block output [T, B, N, D]: bf16 spikes with an output LIF, else float32."""
        T, B, N, D = x.shape
        key = (T, B, N)
        if key not in self._bufs:
            dev = x.device
            self._bufs[key] = (
                torch.empty(T, B * N, 3 * D, device=dev, dtype=torch.bfloat16),
                torch.empty(T, B, N, D, device=dev, dtype=torch.bfloat16),
                torch.empty(T, B * N, D, device=dev,
                            dtype=torch.bfloat16 if self.out_vth is not None else torch.float32))
        qkv, s, y = self._bufs[key]
        h = x
        if self.in_vth is not None:
            h = neuron_multistep(x.contiguous(), decay_factor=1.0 - 1.0 / self.tau,
                                 input_scale=1.0 / self.tau, v_threshold=self.in_vth,
                                 spikes_dtype=torch.bfloat16)["spikes"]
        h = h.to(torch.bfloat16).contiguous().view(T, B * N, D)
        self._lin("qkv", h, self.w_qkv, self.b_qkv, self.qkv_vth, qkv)
        KA.attention_from_qkv(qkv.view(T, B, N, 3 * D), self.heads, scale=self.scale, tau=self.tau,
                              v_threshold=self.attn_vth, out=s)
        sv = s.view(T, B * N, D)
        if self.out_vth is not None:
            self._lin("proj", sv, self.w_proj, self.b_proj, self.out_vth, y)
        else:
            KC.linear_f32(sv, self.w_proj, self.b_proj, out=y)
        return y.view(T, B, N, D)

    __call__ = forward

    def stages(self, x: torch.Tensor):
        """(name, flops, launcher) per launch of forward(x), for profiling."""
        T, B, N, D = x.shape
        self.forward(x)
        qkv, s, y = self._bufs[(T, B, N)]
        h = x.to(torch.bfloat16).contiguous().view(T, B * N, D)
        M = T * B * N
        return [
            ("qkv_linear_lif", 2 * M * D * 3 * D,
             lambda: self._lin("qkv", h, self.w_qkv, self.b_qkv, self.qkv_vth, qkv)),
            ("attention_core", T * B * self.heads * 4 * N * (D // self.heads) ** 2,
             lambda: KA.attention_from_qkv(qkv.view(T, B, N, 3 * D), self.heads, scale=self.scale,
                                           tau=self.tau, v_threshold=self.attn_vth, out=s)),
            ("proj_linear", 2 * M * D * D,
             (lambda: self._lin("proj", s.view(T, B * N, D), self.w_proj, self.b_proj,
                                self.out_vth, y)) if self.out_vth is not None
             else (lambda: KC.linear_f32(s.view(T, B * N, D), self.w_proj, self.b_proj, out=y))),
        ]


def random_attention_params(seed: int = 1, *, D: int = 384):
    """Seeded synthetic block weights (host generator): projection weights N(0, 0.02), zero
    bias, BN gamma U(0.8, 1.2), beta N(0, 0.1), running mean N(0, 0.1), var U(0.5, 1.5)."""
    g = torch.Generator().manual_seed(int(seed))
    P = {}
    for nm in ("q", "k", "v", "proj"):
        P[nm] = {"w": torch.randn(D, D, generator=g) * 0.02, "b": torch.zeros(D),
                 "gamma": torch.rand(D, generator=g) * 0.4 + 0.8,
                 "beta": torch.randn(D, generator=g) * 0.1,
                 "mean": torch.randn(D, generator=g) * 0.1,
                 "var": torch.rand(D, generator=g) + 0.5, "eps": 1e-5}
    return P


def _has_lifs_and_core(m):
    return all(hasattr(m, n) for n in ("q_lif", "k_lif", "v_lif", "attn_lif", "q_conv", "k_conv",
                                       "v_conv", "proj_conv", "num_heads", "scale"))


def is_spiking_self_attention(m: nn.Module) -> bool:
    """Spikingformer SSA shape: Conv1d projections + BatchNorm1d + proj_lif (attention.py:46-49)."""
    return (_has_lifs_and_core(m) and isinstance(getattr(m, "q_conv"), nn.Conv1d)
            and hasattr(m, "q_bn") and hasattr(m, "proj_lif"))


def is_ms_attention(m: nn.Module) -> bool:
    """SDT-V2 MS block shape (attention.py:52-55); recognised but not fused here."""
    return (_has_lifs_and_core(m) and isinstance(getattr(m, "q_conv"), nn.Sequential)
            and hasattr(m, "head_lif"))


def is_spiking_attention(m: nn.Module) -> bool:
    return is_spiking_self_attention(m) or is_ms_attention(m)


def _lif_pv(node):
    return float(getattr(node, "tau", 2.0)), float(getattr(node, "v_threshold", 1.0))


class FusedSpikeAttention(nn.Module):
    """Drop-in for the reference's FusedSpikeAttention (SSA variant, BN folded).
    forward(x [T, B, C, H, W]) -> proj output [T, B, C, H, W] float32."""

    def __init__(self, num_heads, scale, variant="ssa", fold_bn=True, ktv_mode="popcount"):
        super().__init__()
        self.num_heads = num_heads
        self.scale = float(scale)
        self.variant = variant
        self.fold_bn = True
        self.ktv_mode = "popcount"
        self.block = None

    @classmethod
    def from_reference(cls, ref: nn.Module, *, fold_bn: bool = True, ktv_mode: str = "popcount"):
        if not is_spiking_self_attention(ref):
            raise TypeError(f"not a recognised SSA block: {type(ref).__name__}")
        self = cls(ref.num_heads, ref.scale, "ssa")
        in_tau, in_vth = _lif_pv(ref.proj_lif)
        q_tau, q_vth = _lif_pv(ref.q_lif)
        _, a_vth = _lif_pv(ref.attn_lif)
        P = {}
        for nm in ("q", "k", "v", "proj"):
            cv, bn = getattr(ref, f"{nm}_conv"), getattr(ref, f"{nm}_bn")
            P[nm] = {"w": cv.weight, "b": cv.bias, "gamma": bn.weight.detach(),
                     "beta": bn.bias.detach(), "mean": bn.running_mean.detach(),
                     "var": bn.running_var.detach(), "eps": bn.eps}
        dev = next(ref.parameters()).device
        self.block = SpikeAttentionBlock(P, heads=ref.num_heads, scale=ref.scale, tau=q_tau,
                                         in_vth=in_vth, qkv_vth=q_vth, attn_vth=a_vth,
                                         out_vth=None, device=dev)
        return self

    def forward(self, x):
        T, B, C, H, W = x.shape
        xt = x.flatten(3).transpose(2, 3).contiguous()          # [T, B, N, C]
        y = self.block.forward(xt)                               # [T, B, N, C] f32
        return y.transpose(2, 3).reshape(T, B, C, H, W)
