"""Multi-step IF/LIF/PLIF oracle (test infrastructure; see oracle/__init__.py).

Python side of oracle/lif.c.  Parameter derivation follows the reference:
  IF : df = decay (default 1.0), sc = 1.0            snn_compiler/kernels/neurons.py:349-351, :470-472
  LIF: df = 1 - 1/tau (or decay), sc = 1/tau if decay_input else 1.0
                                                      snn_compiler/kernels/neurons.py:352-354, :473-475
  PLIF (SpikingJelly ParametricLIFNode, no snn_compiler counterpart):
       neuron_params("plif"): the reference's charge form with k = sigmoid(w) evaluated in
       double and rounded to float32, df = 1 - k (float32 subtraction), sc = k;
       plif_sj_multistep: SpikingJelly's own charge order (what PLIFNode computes)
All arrays are flat in MEMORY order: x is [T, N] where N = numel of one step.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

THR_SCALAR, THR_PER_CHANNEL, THR_PER_NEURON = 0, 1, 2


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            subprocess.run(["make", "-s", "-C", _HERE], check=True)
        lib = ctypes.CDLL(path)
        f = lib.oracle_lif
        P = ctypes.c_void_p
        i64 = ctypes.c_int64
        f.argtypes = [P, i64, i64, P, P, i64, i64, ctypes.c_int,
                      ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                      ctypes.c_int, ctypes.c_float, P, P, P, P, P, P, ctypes.c_int]
        f.restype = ctypes.c_int
        lib.oracle_max_threads.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def max_threads() -> int:
    return int(_lib().oracle_max_threads())


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def f32(x) -> np.float32:
    """Round a Python float to float32 the way torch converts a scalar operand."""
    return np.float32(x)


def neuron_params(neuron="if", *, tau=2.0, decay=None, decay_input=True, plif_w=None):
    """(df, sc) as float32, following the reference's derivation (see module doc)."""
    if neuron == "if":
        df = 1.0 if decay is None else float(decay)
        return f32(df), f32(1.0)
    if neuron == "lif":
        df = (1.0 - 1.0 / tau) if decay is None else float(decay)
        sc = (1.0 / tau) if decay_input else 1.0
        return f32(df), f32(sc)
    if neuron == "plif":
        w = np.float64(np.float32(0.0 if plif_w is None else plif_w))
        k = np.float32(1.0 / (1.0 + np.exp(-w)))
        return np.float32(np.float32(1.0) - k), np.float32(k)
    raise ValueError(f"unknown neuron: {neuron!r}")


def plif_sj_multistep(x, *, k, decay_input=True, hard_reset=True, v_reset=0.0, thr=1.0,
                      v_init=None):
    """SpikingJelly ParametricLIFNode over x [T, N] float32 (un-vendored third-party code:
    spikingjelly.activation_based.neuron.ParametricLIFNode, as the reference's
    examples/snn_triton_pipeline/*/scripts/_common/sj_compat.py:39-44 instantiates it).
    Restates its published single-step loop, each operation rounded to float32 in its order:
      neuronal_charge  decay_input:              v = v + (x - (v - v_reset)) * k
                       else, v_reset None or 0:  v = v * (1 - k) + x
                       else:                     v = v - (v - v_reset) * k + x
      neuronal_fire    s = heaviside(v - v_threshold)  (== v >= v_threshold)
      neuronal_reset   hard: v = (1 - s) * v + s * v_reset;  soft (v_reset None): v - s * thr
    with k = w.sigmoid() given as a float32 (the caller's value), v starting at v_reset (hard)
    or 0 (soft) unless v_init is given.  Returns dict(spikes [T, N] float32, v [N])."""
    x = np.asarray(x, dtype=np.float32)
    T, N = x.shape
    k = np.float32(k)
    vr = np.float32(v_reset if hard_reset else 0.0)
    th = np.float32(thr)
    one = np.float32(1.0)
    v = np.full(N, vr, np.float32) if v_init is None else np.asarray(v_init, np.float32).copy()
    out = np.zeros((T, N), np.float32)
    for t in range(T):
        xt = x[t]
        if decay_input:
            v = v + (xt - (v - vr)) * k
        elif vr == 0:
            v = v * (one - k) + xt
        else:
            v = v - (v - vr) * k + xt
        v = v.astype(np.float32)
        s = v >= th
        out[t] = s
        if hard_reset:
            v = np.where(s, vr, v).astype(np.float32)
        else:
            v = np.where(s, v - th, v).astype(np.float32)
    return {"spikes": out, "v": v}


def lif_multistep(x, *, df, sc, hard_reset=True, v_reset=0.0, thr=1.0,
                  bias=None, residual=None, C=1, HW=1, channel_last=False,
                  v_init=None, want_spikes=True, want_count=False, want_v=False,
                  want_vpre=False, nthreads=0):
    """Run the multi-step neuron over x [T, N] (float32, memory order).

    thr: float (scalar), array of C (per channel) or of N (per neuron).
    Returns dict with 'spikes' [T,N] f32, 'count' [N] f32, 'v' [N] f32 (state after
    the last step) and 'vpre' [T,N] f32 (charged potential before each threshold
    test) as requested.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.ndim == 2
    T, N = x.shape
    if isinstance(thr, (int, float, np.floating)):
        thr_mode, thr_s, thr_a = THR_SCALAR, float(thr), None
    else:
        thr_a = np.ascontiguousarray(thr, dtype=np.float32).reshape(-1)
        if thr_a.size == C and C != N:
            thr_mode = THR_PER_CHANNEL
        elif thr_a.size == N:
            thr_mode = THR_PER_NEURON
        else:
            raise ValueError(f"threshold of size {thr_a.size} matches neither C={C} nor N={N}")
        thr_s = 0.0
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
        assert bias.size == C
    if residual is not None:
        residual = np.ascontiguousarray(residual, dtype=np.float32).reshape(T, N)
    if v_init is not None:
        v_init = np.ascontiguousarray(v_init, dtype=np.float32).reshape(-1)
        assert v_init.size == N
    out = {}
    spikes = np.empty((T, N), np.float32) if want_spikes else None
    count = np.empty((N,), np.float32) if want_count else None
    v_out = np.empty((N,), np.float32) if want_v else None
    v_pre = np.empty((T, N), np.float32) if want_vpre else None
    rc = _lib().oracle_lif(_ptr(x), T, N, _ptr(bias), _ptr(residual), int(C), int(HW),
                           int(bool(channel_last)), float(df), float(sc), int(bool(hard_reset)),
                           float(v_reset), thr_mode, thr_s, _ptr(thr_a), _ptr(v_init),
                           _ptr(spikes), _ptr(count), _ptr(v_out), _ptr(v_pre), int(nthreads))
    if rc != 0:
        raise ValueError("oracle_lif rejected its arguments")
    if want_spikes:
        out["spikes"] = spikes
    if want_count:
        out["count"] = count
    if want_v:
        out["v"] = v_out
    if want_vpre:
        out["vpre"] = v_pre
    return out


def infer_C_HW(shape):
    """C and HW of a [T, B, C, ...] shape, snn_compiler/kernels/neurons.py:295-308."""
    nd = len(shape)
    if nd == 5:
        return shape[2], shape[3] * shape[4]
    if nd == 4:
        return shape[2], shape[3]
    if nd == 3:
        return shape[-1], 1
    return 1, 1


def naive_if_lif(x_seq, *, neuron="if", tau=2.0, decay=None, decay_input=True,
                 soft_reset=False, v_threshold=1.0, v_reset=0.0, layout="NCHW", plif_w=None):
    """Oracle counterpart of neurons.py:467-502 on a torch CPU tensor [T, B, ...].

    Works in memory order: a channels-last 5-D tensor (layout='NHWC') is handed
    to the C core in its NHWC memory order with channel index n % C.  Returns a
    tensor with x_seq's shape, dtype and memory format.
    """
    import torch
    T = x_seq.shape[0]
    C, HW = infer_C_HW(tuple(x_seq.shape))
    nhwc = layout == "NHWC" and x_seq.ndim == 5
    if nhwc:
        mem = x_seq.permute(0, 1, 3, 4, 2).contiguous()
    else:
        mem = x_seq.contiguous()
    x = mem.to(torch.float32).reshape(T, -1).numpy()
    df, sc = neuron_params(neuron, tau=tau, decay=decay, decay_input=decay_input, plif_w=plif_w)
    if isinstance(v_threshold, torch.Tensor):
        thr = v_threshold.detach().to(torch.float32).reshape(-1)
        if thr.numel() == x.shape[1] and nhwc:
            # per-neuron thresholds are indexed like x_seq[0] (logical NCHW order)
            thr = thr.reshape(x_seq.shape[1:]).permute(0, 2, 3, 1).reshape(-1)
        thr = thr.contiguous().numpy()
    else:
        thr = float(v_threshold)
    r = lif_multistep(x, df=df, sc=sc, hard_reset=not soft_reset, v_reset=v_reset, thr=thr,
                      C=C, HW=HW, channel_last=nhwc)
    s = torch.from_numpy(r["spikes"]).reshape(mem.shape)
    if nhwc:
        s = s.permute(0, 1, 4, 2, 3)
    return s.to(x_seq.dtype)


# ---- CubaLIF / EIF ------------------------------------------------------------------------
# Restatement of the reference's eager naive_cuba_lif / naive_eif
# (snn_compiler/kernels/neurons.py:505-534 and :537-557) in numpy float32: every product,
# sum, difference and quotient is one IEEE float32 operation, evaluated in the reference's
# order.  exp is numpy's float32 exp, which may differ from torch's or CUDA's in the last
# bit; the tests allow spike flips only where the charged potential is that close to the
# threshold.

def _thr_per_neuron(thr, T, N, C, HW, channel_last):
    if isinstance(thr, (int, float, np.floating)):
        return np.full((N,), np.float32(thr), np.float32)
    a = np.ascontiguousarray(thr, dtype=np.float32).reshape(-1)
    if a.size == C and C != N:
        n = np.arange(N, dtype=np.int64)
        c = n % C if channel_last else (n // HW) % C
        return a[c]
    if a.size == N:
        return a
    raise ValueError(f"threshold of size {a.size} matches neither C={C} nor N={N}")


def cuba_lif_multistep(x, *, alpha, beta, input_scale=1.0, hard_reset=True, v_reset=0.0,
                       thr=1.0, C=1, HW=1, channel_last=False, want_vpre=False):
    """x [T, N] float32 (memory order) -> {'spikes' [T, N] f32, 'vpre' [T, N] f32}:
    i = alpha*i + input_scale*x; v = beta*v + i; s = v >= thr; reset."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, N = x.shape
    a, b, sc = np.float32(alpha), np.float32(beta), np.float32(input_scale)
    th = _thr_per_neuron(thr, T, N, C, HW, channel_last)
    vr = np.float32(v_reset)
    i = np.zeros((N,), np.float32)
    v = np.zeros((N,), np.float32)
    spikes = np.empty((T, N), np.float32)
    vpre = np.empty((T, N), np.float32) if want_vpre else None
    for t in range(T):
        i = a * i + sc * x[t]
        v = b * v + i
        s = v >= th
        spikes[t] = s
        if want_vpre:
            vpre[t] = v
        v = np.where(s, vr, v) if hard_reset else np.where(s, v - th, v)
    out = {"spikes": spikes}
    if want_vpre:
        out["vpre"] = vpre
    return out


def eif_multistep(x, *, decay, delta_T=1.0, v_rh=0.5, input_scale=1.0, hard_reset=True,
                  v_reset=0.0, thr=1.0, C=1, HW=1, channel_last=False, want_vpre=False):
    """x [T, N] float32 -> {'spikes', 'vpre'}:
    v = (decay*v + delta_T*exp(min((v - v_rh)/delta_T, 16))) + input_scale*x."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, N = x.shape
    df, dT, rh, sc = (np.float32(decay), np.float32(delta_T), np.float32(v_rh),
                      np.float32(input_scale))
    th = _thr_per_neuron(thr, T, N, C, HW, channel_last)
    vr = np.float32(v_reset)
    v = np.zeros((N,), np.float32)
    spikes = np.empty((T, N), np.float32)
    vpre = np.empty((T, N), np.float32) if want_vpre else None
    with np.errstate(over="ignore"):
        for t in range(T):
            e = np.exp(np.minimum((v - rh) / dT, np.float32(16.0)))
            v = (df * v + dT * e) + sc * x[t]
            s = v >= th
            spikes[t] = s
            if want_vpre:
                vpre[t] = v
            v = np.where(s, vr, v) if hard_reset else np.where(s, v - th, v)
    out = {"spikes": spikes}
    if want_vpre:
        out["vpre"] = vpre
    return out


def cuba_eif_params(model, **kw):
    """(a, b) of the reference's derivation: CubaLIF alpha = exp(-dt/tau_syn),
    beta = exp(-dt/tau_mem) (neurons.py:511-512); EIF decay = 1 - 1/tau (:541)."""
    import math
    if model == "cuba":
        dt = kw.get("dt", 1.0)
        a = math.exp(-dt / kw.get("tau_syn", 2.0)) if kw.get("decay_syn") is None \
            else float(kw["decay_syn"])
        b = math.exp(-dt / kw.get("tau_mem", 4.0)) if kw.get("decay_mem") is None \
            else float(kw["decay_mem"])
        return a, b
    tau = kw.get("tau", 2.0)
    return ((1.0 - 1.0 / tau) if kw.get("decay") is None else float(kw["decay"])), 0.0


def naive_cuba_eif(model, x_seq, *, want_vpre=False, layout="NCHW", **kw):
    """Oracle counterpart of naive_cuba_lif / naive_eif (neurons.py:505-557) on a torch CPU
    tensor [T, B, ...] in memory order; kw are the reference's keyword arguments.
    Returns the oracle dict ('spikes' / 'vpre' as [T, N] float32)."""
    import torch
    x = x_seq.detach().to(torch.float32).contiguous()
    T = x.shape[0]
    C, HW = infer_C_HW(tuple(x.shape))
    thr = kw.get("v_threshold", 1.0)
    if isinstance(thr, torch.Tensor):
        thr = thr.detach().to(torch.float32).reshape(-1).numpy()
    elif isinstance(thr, np.ndarray) and thr.ndim > 0:
        thr = thr.astype(np.float32).reshape(-1)
    else:
        thr = float(thr)
    common = dict(input_scale=kw.get("input_scale", 1.0),
                  hard_reset=not kw.get("soft_reset", False), v_reset=kw.get("v_reset", 0.0),
                  thr=thr, C=C, HW=HW, channel_last=layout == "NHWC", want_vpre=want_vpre)
    xf = x.reshape(T, -1).numpy()
    a, b = cuba_eif_params(model, **kw)
    if model == "cuba":
        return cuba_lif_multistep(xf, alpha=a, beta=b, **common)
    return eif_multistep(xf, decay=a, delta_T=kw.get("delta_T", 1.0), v_rh=kw.get("v_rh", 0.5),
                         **common)
