"""Multi-step IF / LIF / PLIF neuron entry points (K2), same API as the reference.

Mirrors snn_compiler/kernels/neurons.py of the reference:
  if_lif          neurons.py:311-376   (argument meaning, parameter derivation
                                        :349-356, threshold resolution :267-292,
                                        AssertionError / ValueError behaviour)
  cuba_lif, eif   neurons.py:379-457   (snnb_neuron_cuba_eif)
  NEURON_* / RESET_* / THR_* codes      neurons.py:58-68
and adds ``plif`` (SpikingJelly ParametricLIFNode semantics restated in the
reference's form: k = sigmoid(w), decay = 1 - k, input scale = k).

All work runs in ``snnb_neuron_multistep`` of libsnnb200.so (hand-written
sm_100a CUDA); there is no Triton and no CPU fallback.

Layout: the kernel walks memory order.  A tensor stored channels-last (a 5-D
[T,B,C,H,W] view of 4-D channels_last storage) uses channel index n % C, a
contiguous one (n // HW) % C; the choice is taken from the actual strides, so
the result always equals the reference's naive_if_lif on the same logical
tensor.  Per-neuron thresholds are given in logical [B,C,H,W] order (as
naive_if_lif reads them) and permuted to memory order for channels-last input.
"""
from __future__ import annotations

import math

import torch

from .. import _lib

NEURON_IF = 0
NEURON_LIF = 1
NEURON_CUBA = 2
NEURON_EIF = 3
NEURON_PLIF = 4

RESET_SOFT = 0
RESET_HARD = 1

THR_SCALAR = 0
THR_PER_CHANNEL = 1
THR_PER_NEURON = 2


def neuron_coeffs(neuron: str, tau: float = 2.0, decay=None, decay_input: bool = True):
    """(decay_factor, input_scale) exactly as neurons.py:349-356 derives them."""
    if neuron == "if":
        return (1.0 if decay is None else float(decay)), 1.0
    if neuron == "lif":
        df = (1.0 - 1.0 / tau) if decay is None else float(decay)
        sc = (1.0 / tau) if decay_input else 1.0
        return df, sc
    raise ValueError(f"unknown neuron: {neuron!r}")


def _is_channels_last_5d(x: torch.Tensor) -> bool:
    return x.ndim == 5 and x.permute(0, 1, 3, 4, 2).is_contiguous() and not x.is_contiguous()


def memory_geometry(x: torch.Tensor):
    """(C, HW, channel_last) for the per-channel index, from shape and strides."""
    if x.ndim == 5:
        C, HW = x.shape[2], x.shape[3] * x.shape[4]
    elif x.ndim == 4:
        C, HW = x.shape[2], x.shape[3]
    elif x.ndim == 3:
        C, HW = x.shape[-1], 1
    else:
        C, HW = 1, 1
    cl = _is_channels_last_5d(x)
    if not cl and not x.is_contiguous():
        raise AssertionError("x_seq must be contiguous or a channels-last 5-D view "
                             f"(shape {tuple(x.shape)}, strides {x.stride()})")
    return C, HW, cl


def _resolve_threshold(v_threshold, x: torch.Tensor, C: int, channel_last: bool):
    """(mode, scalar, tensor) following neurons.py:267-292."""
    if isinstance(v_threshold, (int, float)):
        return THR_SCALAR, float(v_threshold), None
    assert isinstance(v_threshold, torch.Tensor), type(v_threshold)
    assert v_threshold.is_cuda and v_threshold.dtype == torch.float32 and v_threshold.is_contiguous()
    NCL = math.prod(x.shape[1:])
    if v_threshold.numel() == C:
        return THR_PER_CHANNEL, 0.0, v_threshold
    if v_threshold.numel() == NCL:
        thr = v_threshold
        if channel_last:
            B, Cc, H, W = x.shape[1:]
            thr = thr.view(B, Cc, H, W).permute(0, 2, 3, 1).contiguous()
        return THR_PER_NEURON, 0.0, thr
    raise ValueError(f"v_threshold shape {tuple(v_threshold.shape)} matches neither C={C} "
                     f"nor NCL={NCL}")


def neuron_multistep(x_seq: torch.Tensor, *, decay_factor: float, input_scale: float,
                     soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0,
                     bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                     v_init: torch.Tensor | None = None, plif_w: torch.Tensor | None = None,
                     spikes: bool = True, spikes_dtype=None, packed: bool = False,
                     count: bool = False, v_out: bool = False):
    """One K2 launch.  Returns a dict with the requested outputs:
    'spikes' (x_seq's shape, dtype and strides unless spikes_dtype is given),
    'packed' uint32 [T, ceil(NCL/32)], 'count' float32 [B,...], 'v' float32 [B,...]."""
    assert x_seq.is_cuda
    assert x_seq.dtype in (torch.float32, torch.float16, torch.bfloat16)
    T = x_seq.shape[0]
    NCL = math.prod(x_seq.shape[1:])
    C, HW, cl = memory_geometry(x_seq)
    mode, thr_s, thr_t = _resolve_threshold(v_threshold, x_seq, C, cl)
    if bias is not None:
        assert bias.is_cuda and bias.is_contiguous() and bias.dtype == torch.float32 \
            and bias.numel() == C, f"bias shape mismatch: {tuple(bias.shape)} vs C={C}"
    if residual is not None:
        assert residual.is_cuda and residual.dtype == x_seq.dtype \
            and residual.shape == x_seq.shape and residual.stride() == x_seq.stride(), \
            f"residual {tuple(residual.shape)} must match x_seq {tuple(x_seq.shape)} in layout"
    if v_init is not None:
        assert v_init.is_cuda and v_init.dtype == torch.float32 and v_init.numel() == NCL
        v_init = v_init.contiguous() if not cl else \
            v_init.reshape(x_seq.shape[1:]).permute(0, 2, 3, 1).contiguous()
    if plif_w is not None:
        assert plif_w.is_cuda and plif_w.dtype == torch.float32 and plif_w.numel() == 1
    out = {}
    sp = None
    if spikes:
        sdt = x_seq.dtype if spikes_dtype is None else spikes_dtype
        sp = torch.empty_like(x_seq, dtype=sdt)
        out["spikes"] = sp
    pk = None
    if packed:
        pk = torch.empty((T, (NCL + 31) // 32), device=x_seq.device, dtype=torch.int32)
        out["packed"] = pk
    # state outputs live in memory order; return them in x_seq[0]'s layout
    st_shape = x_seq.shape[1:]
    if cl:
        B, Cc, H, W = st_shape
        mem_shape = (B, H, W, Cc)
    else:
        mem_shape = st_shape
    cnt = torch.empty(mem_shape, device=x_seq.device, dtype=torch.float32) if count else None
    vo = torch.empty(mem_shape, device=x_seq.device, dtype=torch.float32) if v_out else None
    L = _lib.lib()
    st = L.snnb_neuron_multistep(
        _lib.ptr(x_seq), _lib.dtype_code(x_seq.dtype), T, NCL,
        _lib.ptr(bias), _lib.ptr(residual), C, HW, int(cl),
        float(decay_factor), float(input_scale), _lib.ptr(plif_w),
        0 if soft_reset else 1, float(v_reset),
        mode, thr_s, _lib.ptr(thr_t), _lib.ptr(v_init),
        _lib.ptr(sp), _lib.dtype_code(sp.dtype) if sp is not None else 0,
        _lib.ptr(pk), _lib.ptr(cnt), _lib.ptr(vo), _lib.stream_of(x_seq))
    _lib.check(st, "snnb_neuron_multistep")
    for key, t in (("count", cnt), ("v", vo)):
        if t is not None:
            out[key] = t.permute(0, 3, 1, 2) if cl else t
    return out


def if_lif(
    x_seq: torch.Tensor,
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
    """Unified IF/LIF inference entry (reference neurons.py:311-376).

    x_seq: [T, B, ...] fp16/bf16/fp32 on CUDA.  Returns spikes with x_seq's
    dtype and layout.  ``layout`` is accepted for API compatibility; the channel
    index is derived from the tensor's actual memory format.
    """
    assert x_seq.is_cuda
    if not x_seq.is_contiguous():
        assert layout == "NHWC", f"non-contiguous x_seq requires layout='NHWC', got {layout}"
    assert x_seq.dtype in (torch.float32, torch.float16, torch.bfloat16)
    df, sc = neuron_coeffs(neuron, tau, decay, decay_input)
    return neuron_multistep(x_seq, decay_factor=df, input_scale=sc, soft_reset=soft_reset,
                            v_threshold=v_threshold, v_reset=v_reset)["spikes"]


def plif(
    x_seq: torch.Tensor,
    w: torch.Tensor,
    *,
    decay_input: bool = True,
    soft_reset: bool = False,
    v_threshold=1.0,
    v_reset: float = 0.0,
    layout: str = "NCHW",
    v_init: torch.Tensor | None = None,
    packed: bool = False,
    count: bool = False,
    v_out: bool = False,
):
    """SpikingJelly ParametricLIFNode, multi-step (snnb_neuron_plif): k = w.sigmoid() on
    w's device (as SpikingJelly evaluates it), then per step, in SpikingJelly's order,
    v = v + (x - (v - v_reset)) * k (decay_input) or v * (1 - k) + x / v - (v - v_reset) * k
    + x (not), fire at v >= v_threshold, hard or soft reset.  A hard-reset neuron starts at
    v_reset (SpikingJelly's initial state), a soft one at 0, unless v_init is given.
    Returns the spikes (x_seq's dtype and layout), or a dict with 'spikes' and the requested
    'packed' / 'count' / 'v' when any of those is asked for."""
    assert x_seq.is_cuda
    assert x_seq.dtype in (torch.float32, torch.float16, torch.bfloat16)
    assert isinstance(v_threshold, (int, float)), "PLIF takes a scalar threshold"
    if not x_seq.is_contiguous():
        assert layout == "NHWC", f"non-contiguous x_seq requires layout='NHWC', got {layout}"
    T = x_seq.shape[0]
    NCL = math.prod(x_seq.shape[1:])
    k = torch.sigmoid(w.detach().reshape(1).to(device=x_seq.device, dtype=torch.float32))
    hard = not soft_reset
    if v_init is None and hard and float(v_reset) != 0.0:
        v_init = torch.full((NCL,), float(v_reset), device=x_seq.device, dtype=torch.float32)
    elif v_init is not None:
        assert v_init.is_cuda and v_init.dtype == torch.float32 and v_init.numel() == NCL
        v_init = v_init.contiguous()
    sp = torch.empty_like(x_seq)
    pk = torch.empty((T, (NCL + 31) // 32), device=x_seq.device, dtype=torch.int32) \
        if packed else None
    cnt = torch.empty(x_seq.shape[1:], device=x_seq.device, dtype=torch.float32) \
        if count else None
    vo = torch.empty(x_seq.shape[1:], device=x_seq.device, dtype=torch.float32) \
        if v_out else None
    # elementwise: the memory order of x (NCHW or channels-last storage) is kept as is
    st = _lib.lib().snnb_neuron_plif(
        _lib.ptr(x_seq), _lib.dtype_code(x_seq.dtype), T, NCL, _lib.ptr(k), int(decay_input),
        int(hard), float(v_reset), float(v_threshold), _lib.ptr(v_init), _lib.ptr(sp),
        _lib.dtype_code(sp.dtype), _lib.ptr(pk), _lib.ptr(cnt), _lib.ptr(vo),
        _lib.stream_of(x_seq))
    _lib.check(st, "snnb_neuron_plif")
    if not (packed or count or v_out):
        return sp
    out = {"spikes": sp}
    if packed:
        out["packed"] = pk
    if count:
        out["count"] = cnt
    if v_out:
        out["v"] = vo
    return out


MODEL_CUBA = 0
MODEL_EIF = 1


def _resolve_thr_layout(v_threshold, x_seq: torch.Tensor, layout: str):
    """(mode, scalar, tensor, channel_last) as neurons.py:265-292 resolves them for
    cuba_lif / eif: x_seq is contiguous and `layout` alone says whether the per-channel
    index is n % C (NHWC) or (n // HW) % C; per-neuron thresholds are in memory order."""
    nhwc = layout == "NHWC"
    if isinstance(v_threshold, (int, float)):
        return THR_SCALAR, float(v_threshold), None, nhwc
    assert isinstance(v_threshold, torch.Tensor), type(v_threshold)
    assert v_threshold.is_cuda and v_threshold.dtype == torch.float32 and v_threshold.is_contiguous()
    if x_seq.ndim >= 4:
        C = x_seq.shape[2]
    elif x_seq.ndim == 3:
        C = x_seq.shape[-1]
    else:
        C = 1
    NCL = x_seq[0].numel()
    if v_threshold.numel() == C:
        return THR_PER_CHANNEL, 0.0, v_threshold, nhwc
    if v_threshold.numel() == NCL:
        return THR_PER_NEURON, 0.0, v_threshold, False
    raise ValueError(f"v_threshold shape {tuple(v_threshold.shape)} matches neither C={C} "
                     f"nor NCL={NCL}")


def _infer_C_HW(x_seq: torch.Tensor):
    """C and HW of the [T, B, C, ...] shape (neurons.py:295-308)."""
    if x_seq.ndim == 5:
        return x_seq.shape[2], x_seq.shape[3] * x_seq.shape[4]
    if x_seq.ndim == 4:
        return x_seq.shape[2], x_seq.shape[3]
    if x_seq.ndim == 3:
        return x_seq.shape[-1], 1
    return 1, 1


def _neuron2(x_seq, model, a, b, input_scale, delta_T, v_rh, soft_reset, v_threshold,
             v_reset, layout):
    assert x_seq.is_cuda and x_seq.is_contiguous()
    assert x_seq.dtype in (torch.float32, torch.float16, torch.bfloat16)
    T = x_seq.shape[0]
    NCL = x_seq[0].numel()
    C, HW = _infer_C_HW(x_seq)
    mode, thr_s, thr_t, cl = _resolve_thr_layout(v_threshold, x_seq, layout)
    spikes = torch.empty_like(x_seq)
    st = _lib.lib().snnb_neuron_cuba_eif(
        _lib.ptr(x_seq), _lib.dtype_code(x_seq.dtype), T, NCL, C, HW, int(cl), model,
        float(a), float(b), float(input_scale), float(delta_T), float(v_rh),
        0 if soft_reset else 1, float(v_reset), mode, thr_s, _lib.ptr(thr_t),
        _lib.ptr(spikes), _lib.stream_of(x_seq))
    _lib.check(st, "snnb_neuron_cuba_eif")
    return spikes


def cuba_lif(
    x_seq: torch.Tensor,
    *,
    tau_syn: float = 2.0,
    tau_mem: float = 4.0,
    dt: float = 1.0,
    decay_syn: float | None = None,
    decay_mem: float | None = None,
    input_scale: float = 1.0,
    soft_reset: bool = False,
    v_threshold=1.0,
    v_reset: float = 0.0,
    layout: str = "NCHW",
) -> torch.Tensor:
    """CubaLIF (reference neurons.py:379-418): synaptic current i and potential v,
    i = alpha*i + input_scale*x, v = beta*v + i, with alpha = exp(-dt/tau_syn) and
    beta = exp(-dt/tau_mem) unless decay_syn / decay_mem override them.  Spikes of
    x_seq's dtype."""
    alpha = math.exp(-dt / tau_syn) if decay_syn is None else float(decay_syn)
    beta = math.exp(-dt / tau_mem) if decay_mem is None else float(decay_mem)
    return _neuron2(x_seq, MODEL_CUBA, alpha, beta, input_scale, 1.0, 0.0, soft_reset,
                    v_threshold, v_reset, layout)


def eif(
    x_seq: torch.Tensor,
    *,
    tau: float = 2.0,
    decay: float | None = None,
    delta_T: float = 1.0,
    v_rh: float = 0.5,
    input_scale: float = 1.0,
    soft_reset: bool = False,
    v_threshold=1.0,
    v_reset: float = 0.0,
    layout: str = "NCHW",
) -> torch.Tensor:
    """Exponential IF (reference neurons.py:421-457):
    v = decay*v + delta_T*exp(min((v - v_rh)/delta_T, 16)) + input_scale*x with
    decay = 1 - 1/tau unless given.  Spikes of x_seq's dtype."""
    df = (1.0 - 1.0 / tau) if decay is None else float(decay)
    return _neuron2(x_seq, MODEL_EIF, df, 0.0, input_scale, delta_T, v_rh, soft_reset,
                    v_threshold, v_reset, layout)
