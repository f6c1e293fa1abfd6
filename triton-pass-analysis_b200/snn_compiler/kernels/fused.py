"""Bias / residual / rate-coded / stateful neuron entry points, same API as the reference.

Mirrors snn_compiler/kernels/fused.py of the reference:
  fused_bias_if_lif            fused.py:117-226
  fused_bias_if_lif_rate       fused.py:303-382
  fused_bias_if_lif_stateful   fused.py:444-507
  fold_conv_bn                 fused.py:585-599   (host-side, construction time)
  conv_neuron / linear_neuron / conv_bn_neuron     fused.py:513-611
Each neuron entry is one launch of ``snnb_neuron_multistep`` (K2); the conv
and linear entries run the fused tensor-core kernels of snn_compiler.kernels.conv.
"""
from __future__ import annotations

import torch

from .neurons import neuron_coeffs, neuron_multistep


def _check_layout(y_seq, layout):
    assert y_seq.is_cuda
    if not y_seq.is_contiguous():
        assert layout == "NHWC" and y_seq.ndim >= 4, \
            f"non-contiguous y_seq requires NHWC layout, got layout={layout} shape={tuple(y_seq.shape)}"


def fused_bias_if_lif(
    y_seq: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    residual: torch.Tensor | None = None,
    neuron: str = "if",
    tau: float = 2.0,
    decay: float | None = None,
    decay_input: bool = True,
    soft_reset: bool = False,
    v_threshold=1.0,
    v_reset: float = 0.0,
    layout: str = "NCHW",
) -> torch.Tensor:
    """v_t = decay*v + scale*(y_t + bias[c] (+ residual_t)) -> spikes (fused.py:117-226)."""
    _check_layout(y_seq, layout)
    df, sc = neuron_coeffs(neuron, tau, decay, decay_input)
    return neuron_multistep(y_seq, decay_factor=df, input_scale=sc, soft_reset=soft_reset,
                            v_threshold=v_threshold, v_reset=v_reset, bias=bias,
                            residual=residual)["spikes"]


def fused_bias_if_lif_rate(
    y_seq: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    neuron: str = "if",
    tau: float = 2.0,
    decay: float | None = None,
    decay_input: bool = True,
    soft_reset: bool = False,
    v_threshold=1.0,
    v_reset: float = 0.0,
    layout: str = "NCHW",
) -> torch.Tensor:
    """Rate-coded output: float32 spike count summed over T, shape y_seq.shape[1:]
    (fused.py:303-382).  Only the count is written to HBM."""
    _check_layout(y_seq, layout)
    df, sc = neuron_coeffs(neuron, tau, decay, decay_input)
    return neuron_multistep(y_seq, decay_factor=df, input_scale=sc, soft_reset=soft_reset,
                            v_threshold=v_threshold, v_reset=v_reset, bias=bias,
                            spikes=False, count=True)["count"]


def fused_bias_if_lif_stateful(
    y_seq: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    v_init: torch.Tensor | None = None,
    return_v: bool = False,
    neuron: str = "if",
    tau: float = 2.0,
    decay: float | None = None,
    decay_input: bool = True,
    soft_reset: bool = False,
    v_threshold: float = 1.0,
    v_reset: float = 0.0,
    layout: str = "NCHW",
):
    """T-chunked execution: optional v_init in, optional final v out (fused.py:444-507).
    Unlike the reference, tensor thresholds are accepted too."""
    _check_layout(y_seq, layout)
    df, sc = neuron_coeffs(neuron, tau, decay, decay_input)
    r = neuron_multistep(y_seq, decay_factor=df, input_scale=sc, soft_reset=soft_reset,
                         v_threshold=v_threshold, v_reset=v_reset, bias=bias,
                         v_init=v_init, v_out=return_v)
    if return_v:
        return r["spikes"], r["v"]
    return r["spikes"]


def fold_conv_bn(conv_w, conv_b, bn_w, bn_b, bn_mean, bn_var, bn_eps):
    """Fold eval-mode BN into the preceding conv / linear (fused.py:585-599):
    W' = W * gamma/sqrt(var+eps) (per output channel, cast to W's dtype);
    b' = (b - mean) * gamma/sqrt(var+eps) + beta."""
    inv_std = bn_w / torch.sqrt(bn_var + bn_eps)
    new_w = conv_w * inv_std.view(-1, *([1] * (conv_w.ndim - 1))).to(conv_w.dtype)
    if conv_b is None:
        conv_b = torch.zeros_like(bn_w)
    new_b = (conv_b - bn_mean) * inv_std + bn_b
    return new_w, new_b


from .conv import conv_bn_neuron, conv_neuron, linear_neuron  # noqa: E402  (conv imports fold_conv_bn)
