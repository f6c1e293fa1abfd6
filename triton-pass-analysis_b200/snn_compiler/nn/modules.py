"""nn.Module API (SpikingJelly-style multi-step neurons), same as the reference.

Mirrors snn_compiler/nn/modules.py of the reference:
  IFNode :26-49, LIFNode :52-85, CubaLIFNode :88-121, EIFNode :124-154,
  FusedAddNeuron :446-481, RateCodedLIFNode :487-522, RateCodedIFNode :525-547,
  StatefulLIFNode :553-586
plus PLIFNode (SpikingJelly ParametricLIFNode, in SpikingJelly's arithmetic: learnable w,
k = sigmoid(w), init_tau = 2 -> w = 0).  Every module takes x_seq [T, B, ...] and returns
[T, B, ...] spikes of x_seq's dtype; state is not kept between calls.
The conv / linear fused modules live in snn_compiler.nn.fused_layers.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..kernels.fused import (fused_bias_if_lif, fused_bias_if_lif_rate,
                             fused_bias_if_lif_stateful)
from ..kernels.neurons import cuba_lif, eif, if_lif, plif


def _store_threshold(mod, v_threshold):
    if isinstance(v_threshold, torch.Tensor):
        mod.register_buffer("v_threshold", v_threshold.float().contiguous())
    else:
        mod.v_threshold = float(v_threshold)


class IFNode(nn.Module):
    """Integrate-and-fire: v = decay*v + x (decay defaults to 1)."""

    def __init__(self, *, decay: float = 1.0, soft_reset: bool = False,
                 v_threshold=1.0, v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__()
        self.decay = decay
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        self.layout = layout
        _store_threshold(self, v_threshold)

    def forward(self, x_seq):
        return if_lif(x_seq if _dense(x_seq) else x_seq.contiguous(), neuron="if",
                      decay=self.decay, soft_reset=self.soft_reset,
                      v_threshold=self.v_threshold, v_reset=self.v_reset, layout=self.layout)


class LIFNode(nn.Module):
    """Leaky IF: v = (1-1/tau) v + x/tau (decay_input) -- SpikingJelly LIFNode semantics."""

    def __init__(self, *, tau: float = 2.0, decay: float | None = None,
                 decay_input: bool = True, soft_reset: bool = False, v_threshold=1.0,
                 v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__()
        self.tau = tau
        self.decay = decay
        self.decay_input = decay_input
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        self.layout = layout
        _store_threshold(self, v_threshold)

    def forward(self, x_seq):
        return if_lif(x_seq if _dense(x_seq) else x_seq.contiguous(), neuron="lif",
                      tau=self.tau, decay=self.decay, decay_input=self.decay_input,
                      soft_reset=self.soft_reset, v_threshold=self.v_threshold,
                      v_reset=self.v_reset, layout=self.layout)


class CubaLIFNode(nn.Module):
    """Current-based LIF (two states): i = alpha*i + input_scale*x, v = beta*v + i, with
    alpha = exp(-dt/tau_syn), beta = exp(-dt/tau_mem) unless decay_syn / decay_mem
    override them (decay_syn = 0 gives a one-state LIF, decay_mem = 1 no membrane leak)."""

    def __init__(self, *, tau_syn: float = 2.0, tau_mem: float = 4.0, dt: float = 1.0,
                 decay_syn: float | None = None, decay_mem: float | None = None,
                 input_scale: float = 1.0, soft_reset: bool = False,
                 v_threshold=1.0, v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__()
        self.tau_syn = tau_syn
        self.tau_mem = tau_mem
        self.dt = dt
        self.decay_syn = decay_syn
        self.decay_mem = decay_mem
        self.input_scale = input_scale
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        self.layout = layout
        _store_threshold(self, v_threshold)

    def forward(self, x_seq):
        return cuba_lif(x_seq.contiguous(), tau_syn=self.tau_syn, tau_mem=self.tau_mem,
                        dt=self.dt, decay_syn=self.decay_syn, decay_mem=self.decay_mem,
                        input_scale=self.input_scale, soft_reset=self.soft_reset,
                        v_threshold=self.v_threshold, v_reset=self.v_reset, layout=self.layout)


class EIFNode(nn.Module):
    """Exponential IF: v = decay*v + delta_T*exp(min((v - v_rh)/delta_T, 16)) + input_scale*x,
    decay = 1 - 1/tau unless given."""

    def __init__(self, *, tau: float = 2.0, decay: float | None = None,
                 delta_T: float = 1.0, v_rh: float = 0.5, input_scale: float = 1.0,
                 soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0,
                 layout: str = "NCHW"):
        super().__init__()
        self.tau = tau
        self.decay = decay
        self.delta_T = delta_T
        self.v_rh = v_rh
        self.input_scale = input_scale
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        self.layout = layout
        _store_threshold(self, v_threshold)

    def forward(self, x_seq):
        return eif(x_seq.contiguous(), tau=self.tau, decay=self.decay, delta_T=self.delta_T,
                   v_rh=self.v_rh, input_scale=self.input_scale, soft_reset=self.soft_reset,
                   v_threshold=self.v_threshold, v_reset=self.v_reset, layout=self.layout)


class PLIFNode(nn.Module):
    """Parametric LIF (SpikingJelly ParametricLIFNode, multi-step): learnable w with
    init_tau = 1 + exp(-w) (w = -log(init_tau - 1)), k = w.sigmoid(), and SpikingJelly's
    charge v = v + (x - (v - v_reset)) * k (decay_input; see kernels.neurons.plif for the
    other form), fire at v >= v_threshold, hard reset to v_reset (the neuron starts there)
    or soft reset (SpikingJelly's v_reset=None).  init_tau = 2 gives w = 0 and k = 0.5."""

    def __init__(self, *, init_tau: float = 2.0, decay_input: bool = True,
                 soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0,
                 layout: str = "NCHW"):
        super().__init__()
        self.w = nn.Parameter(torch.tensor([-math.log(init_tau - 1.0)], dtype=torch.float32))
        self.decay_input = decay_input
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        self.layout = layout
        _store_threshold(self, v_threshold)

    def forward(self, x_seq):
        return plif(x_seq if _dense(x_seq) else x_seq.contiguous(), self.w.detach(),
                    decay_input=self.decay_input, soft_reset=self.soft_reset,
                    v_threshold=self.v_threshold, v_reset=self.v_reset, layout=self.layout)


class FusedAddNeuron(nn.Module):
    """Two paths summed and fed to one neuron: v = decay*v + scale*(a_t + b_t)."""

    def __init__(self, *, neuron: str = "if", tau: float = 2.0, decay: float | None = None,
                 decay_input: bool = True, soft_reset: bool = False, v_threshold=1.0,
                 v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__()
        self.neuron = neuron
        self.tau = tau
        self.decay = decay
        self.decay_input = decay_input
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        self.layout = layout
        _store_threshold(self, v_threshold)

    def forward(self, a_seq, b_seq):
        return fused_bias_if_lif(a_seq, None, residual=b_seq, neuron=self.neuron, tau=self.tau,
                                 decay=self.decay, decay_input=self.decay_input,
                                 soft_reset=self.soft_reset, v_threshold=self.v_threshold,
                                 v_reset=self.v_reset, layout=self.layout)


class RateCodedLIFNode(nn.Module):
    """LIF that returns only the float32 spike count summed over T ([B, ...])."""

    def __init__(self, *, tau: float = 2.0, decay: float | None = None,
                 decay_input: bool = True, soft_reset: bool = False, v_threshold=1.0,
                 v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__()
        self.tau = tau
        self.decay = decay
        self.decay_input = decay_input
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        self.layout = layout
        _store_threshold(self, v_threshold)

    def forward(self, x_seq):
        return fused_bias_if_lif_rate(x_seq if _dense(x_seq) else x_seq.contiguous(), None,
                                      neuron="lif", tau=self.tau, decay=self.decay,
                                      decay_input=self.decay_input, soft_reset=self.soft_reset,
                                      v_threshold=self.v_threshold, v_reset=self.v_reset,
                                      layout=self.layout)


class RateCodedIFNode(nn.Module):
    """IF variant of RateCodedLIFNode."""

    def __init__(self, *, decay: float = 1.0, soft_reset: bool = False,
                 v_threshold=1.0, v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__()
        self.decay = decay
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        self.layout = layout
        _store_threshold(self, v_threshold)

    def forward(self, x_seq):
        return fused_bias_if_lif_rate(x_seq if _dense(x_seq) else x_seq.contiguous(), None,
                                      neuron="if", decay=self.decay, soft_reset=self.soft_reset,
                                      v_threshold=self.v_threshold, v_reset=self.v_reset,
                                      layout=self.layout)


class StatefulLIFNode(nn.Module):
    """LIF with v_init in and optional final v out, for T-chunked execution."""

    def __init__(self, *, tau: float = 2.0, decay: float | None = None,
                 decay_input: bool = True, soft_reset: bool = False,
                 v_threshold: float = 1.0, v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__()
        self.tau = tau
        self.decay = decay
        self.decay_input = decay_input
        self.soft_reset = soft_reset
        self.v_threshold = float(v_threshold)
        self.v_reset = v_reset
        self.layout = layout

    def forward(self, x_seq, v_init=None, return_v=False):
        return fused_bias_if_lif_stateful(
            x_seq if _dense(x_seq) else x_seq.contiguous(), None, v_init=v_init,
            return_v=return_v, neuron="lif", tau=self.tau, decay=self.decay,
            decay_input=self.decay_input, soft_reset=self.soft_reset,
            v_threshold=self.v_threshold, v_reset=self.v_reset, layout=self.layout)


def _dense(x):
    return x.is_contiguous() or (x.ndim == 5 and x.permute(0, 1, 3, 4, 2).is_contiguous())
