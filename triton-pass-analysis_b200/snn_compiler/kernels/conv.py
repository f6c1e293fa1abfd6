"""Fused conv / linear + bias + multi-step LIF (+ max-pool) entry points (K1).

Low-level entries work on channels-last frames, the layout the kernels stream:
  conv3x3_lif(x [T, B, H, W, Cin] bf16, w [Cout, 3, 3, Cin] bf16, bias f32) -> spikes
  linear_lif(x [T, B, K] bf16, w [N, K] bf16, bias)                        -> spikes
  linear_mean(x [T, B, K] bf16, w [N, K] bf16, bias)                       -> f32 [B, N]
  first_conv_lif(img f32 [Ti, B, Cin, H, W], w f32 [Cout, Cin, 3, 3], bias) -> spikes
The reference-API entries conv_neuron / linear_neuron / conv_bn_neuron
(snn_compiler/kernels/fused.py:513-611) sit on top of them.

Each call is one launch of libsnnb200.so; the conv runs on tcgen05 tensor cores
(bf16 operands, f32 accumulation in TMEM) with the neuron in the epilogue.
"""
from __future__ import annotations

import torch

from .. import _lib
from .fused import fold_conv_bn
from .neurons import neuron_coeffs


def _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold, v_reset):
    if not isinstance(v_threshold, (int, float)):
        raise NotImplementedError("the fused conv / linear kernels take a scalar v_threshold")
    df, sc = neuron_coeffs(neuron, tau, decay, decay_input)
    return float(df), float(sc), float(v_threshold), float(v_reset), 0 if soft_reset else 1


def conv3x3_lif(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, *, neuron: str = "lif",
                tau: float = 2.0, decay=None, decay_input: bool = True, soft_reset: bool = False,
                v_threshold=1.0, v_reset: float = 0.0, pool: bool = False,
                out: torch.Tensor | None = None, variant: int = 0, block_n: int = 0,
                splits: int = 1, workspace: torch.Tensor | None = None,
                residual: torch.Tensor | None = None) -> torch.Tensor:
    """x [T, B, H, W, Cin] bf16 -> spikes [T, B, Ho, Wo, Cout] bf16 (Ho = H/2 when pool).
    residual: None, or [T, B, H, W, Cout] bf16 / float32 added to conv + bias before the
    neuron (no pooling; snnb_conv3x3_lif_res).
    variant: 0 choose, 1 T-sequential CTAs, 2 T folded into M, 3 row bands with halo reuse
    and resident weights (band_block_ns), 4 = 2 with two M-tiles per CTA, 5 = 2 on CTA pairs
    (M = 256 MMAs, half the weight rows staged per CTA), 6 = 2 with the K range split across
    a thread-block cluster of `splits` CTAs that reduce through distributed shared memory
    (no workspace), 7 = 3 with the column taps shifted in the epilogue (one operand copy
    per stage, W <= 32, band_xs_block_ns); block_n: 0 or 32/64/128/256;
    splits > 1: split-K with float32 partials in `workspace` (allocated here if None)
    except with variant 6."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 5
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.shape[1:3] == (3, 3)
    T, B, H, W, Cin = x.shape
    Cout = w.shape[0]
    assert w.shape[3] == Cin, (tuple(w.shape), Cin)
    assert bias.dtype == torch.float32 and bias.is_contiguous() and bias.numel() == Cout
    df, sc, thr, vr, hard = _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold,
                                      v_reset)
    Ho, Wo = (H // 2, W // 2) if pool else (H, W)
    if out is None:
        out = torch.empty(T, B, Ho, Wo, Cout, device=x.device, dtype=torch.bfloat16)
    ws, ws_bytes = _workspace(workspace, 1 if variant == 6 else splits, T, B, H, W, Cout,
                              x.device)
    if residual is not None:
        assert not pool, "residual input with pooling is not supported"
        assert residual.is_cuda and residual.is_contiguous() and \
            residual.dtype in (torch.bfloat16, torch.float32) and \
            tuple(residual.shape) == (T, B, H, W, Cout), tuple(residual.shape)
        st = _lib.lib().snnb_conv3x3_lif_res(
            _lib.ptr(x), T, B, H, W, Cin, _lib.ptr(w), _lib.ptr(bias), Cout, df, sc, thr, vr,
            hard, _lib.ptr(residual), _lib.dtype_code(residual.dtype), int(variant),
            int(block_n), int(splits), _lib.ptr(ws), ws_bytes, _lib.ptr(out),
            _lib.stream_of(x))
        _lib.check(st, "snnb_conv3x3_lif_res")
        return out
    st = _lib.lib().snnb_conv3x3_lif(_lib.ptr(x), T, B, H, W, Cin, _lib.ptr(w), _lib.ptr(bias),
                                     Cout, df, sc, thr, vr, hard, int(bool(pool)), int(variant),
                                     int(block_n), int(splits), _lib.ptr(ws), ws_bytes,
                                     _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_conv3x3_lif")
    return out


def conv_out_size(n: int, stride: int) -> int:
    """Output size of a 3x3 / padding 1 or 1x1 / padding 0 conv with this stride."""
    return (n - 1) // stride + 1


def conv_lif_strided(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, *, stride: int = 1,
                     neuron: str = "lif", tau: float = 2.0, decay=None, decay_input: bool = True,
                     soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0,
                     out: torch.Tensor | None = None, variant: int = 0, block_n: int = 0,
                     splits: int = 1, workspace: torch.Tensor | None = None,
                     residual: torch.Tensor | None = None) -> torch.Tensor:
    """x [T, B, H, W, Cin] bf16, w [Cout, k, k, Cin] bf16 (k in {1, 3, 5, 7}, padding k // 2),
    stride 1 or 2 -> spikes [T, B, Ho, Wo, Cout] bf16, Ho = (H - 1) // stride + 1
    (snnb_conv_lif_strided: the strided, 1x1 and 7x7 stem convs of a spiking ResNet).
    residual: None
    or [T, B, Ho, Wo, Cout] bf16 / float32; variant / block_n / splits as conv3x3_lif:
    variants 0, 1 and 2 (any splits), and for 3x3 / 1x1 convs of stride 1 also 4, 5, 6."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 5
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.ndim == 4
    k = w.shape[1]
    assert k in (1, 3, 5, 7) and w.shape[2] == k and stride in (1, 2), (tuple(w.shape), stride)
    T, B, H, W, Cin = x.shape
    Cout = w.shape[0]
    assert w.shape[3] == Cin, (tuple(w.shape), Cin)
    assert bias.dtype == torch.float32 and bias.is_contiguous() and bias.numel() == Cout
    df, sc, thr, vr, hard = _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold,
                                      v_reset)
    Ho, Wo = conv_out_size(H, stride), conv_out_size(W, stride)
    if out is None:
        out = torch.empty(T, B, Ho, Wo, Cout, device=x.device, dtype=torch.bfloat16)
    ws, ws_bytes = _workspace(workspace, 1 if variant == 6 else splits, T, B, Ho, Wo, Cout,
                              x.device)
    if residual is not None:
        assert residual.is_cuda and residual.is_contiguous() and \
            residual.dtype in (torch.bfloat16, torch.float32) and \
            tuple(residual.shape) == (T, B, Ho, Wo, Cout), tuple(residual.shape)
    st = _lib.lib().snnb_conv_lif_strided(
        _lib.ptr(x), T, B, H, W, Cin, _lib.ptr(w), _lib.ptr(bias), Cout, k, stride, df, sc, thr,
        vr, hard, _lib.ptr(residual), _lib.dtype_code(residual.dtype) if residual is not None
        else 0, int(variant), int(block_n), int(splits), _lib.ptr(ws), ws_bytes, _lib.ptr(out),
        _lib.stream_of(x))
    _lib.check(st, "snnb_conv_lif_strided")
    return out


def conv_f32(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, *, stride: int = 1,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """x [T, B, H, W, Cin] bf16, w [Cout, k, k, Cin] bf16 (k in {1, 3, 5, 7}) -> float32
    [T, B, Ho, Wo, Cout] = conv + bias, no neuron (snnb_conv_f32: the downsample branch of a
    spiking ResNet block, BN folded into w and bias); T in {2, 4, 8}."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 5
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.ndim == 4
    k = w.shape[1]
    assert k in (1, 3, 5, 7) and w.shape[2] == k and stride in (1, 2), (tuple(w.shape), stride)
    T, B, H, W, Cin = x.shape
    Cout = w.shape[0]
    assert w.shape[3] == Cin and bias.dtype == torch.float32 and bias.numel() == Cout
    Ho, Wo = conv_out_size(H, stride), conv_out_size(W, stride)
    if out is None:
        out = torch.empty(T, B, Ho, Wo, Cout, device=x.device, dtype=torch.float32)
    st = _lib.lib().snnb_conv_f32(_lib.ptr(x), T, B, H, W, Cin, _lib.ptr(w),
                                  _lib.ptr(bias.contiguous()), Cout, k, stride, _lib.ptr(out),
                                  _lib.stream_of(x))
    _lib.check(st, "snnb_conv_f32")
    return out


def maxpool_nhwc(x: torch.Tensor, k: int = 3, stride: int = 2, pad: int = 1,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """x [..., H, W, C] bf16 NHWC frames (C % 8 == 0) -> k x k max-pool with stride and
    padding [..., Ho, Wo, C], Ho = (H + 2 pad - k) // stride + 1 (snnb_maxpool_nhwc: the
    ResNet stem's 3x3 / stride 2 pool, reference zoo/resnet.py:131)."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim >= 3
    H, W, C = x.shape[-3:]
    frames = x.numel() // (H * W * C) if x.numel() else 0
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    if out is None:
        out = torch.empty(*x.shape[:-3], Ho, Wo, C, device=x.device, dtype=x.dtype)
    st = _lib.lib().snnb_maxpool_nhwc(_lib.ptr(x), frames, H, W, C, int(k), int(stride),
                                      int(pad), _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_maxpool_nhwc")
    return out


def window_gather_nhwc(x: torch.Tensor, k: int, stride: int, pad: int,
                       Kp: int | None = None) -> torch.Tensor:
    """x [..., H, W, C] bf16 NHWC frames -> [..., Ho, Wo, Kp] bf16: each output pixel's
    k x k window in columns (dy * k + dx) * C + c, zero outside the image and past k*k*C
    (snnb_window_gather_nhwc; Kp defaults to k*k*C rounded up to a multiple of 8)."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim >= 3
    H, W, C = x.shape[-3:]
    Kp = (k * k * C + 7) // 8 * 8 if Kp is None else Kp
    frames = x.numel() // (H * W * C) if x.numel() else 0
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    out = torch.empty(*x.shape[:-3], Ho, Wo, Kp, device=x.device, dtype=x.dtype)
    st = _lib.lib().snnb_window_gather_nhwc(_lib.ptr(x), frames, H, W, C, int(k), int(stride),
                                            int(pad), int(Kp), _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_window_gather_nhwc")
    return out


def linear_lif(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, *, neuron: str = "lif",
               tau: float = 2.0, decay=None, decay_input: bool = True, soft_reset: bool = False,
               v_threshold=1.0, v_reset: float = 0.0, out: torch.Tensor | None = None,
               variant: int = 0, block_n: int = 0, splits: int = 1,
               workspace: torch.Tensor | None = None):
    """x [T, B, K] bf16 @ w[N, K]^T + bias -> LIF -> spikes [T, B, N] bf16.
    variant 8: the transposed form (features x rows, split-K over `splits` CTAs of a
    cluster; snnb_linear_lif_t) for layers with few rows."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 3
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.shape[1] == x.shape[2]
    T, B, K = x.shape
    N = w.shape[0]
    assert bias.dtype == torch.float32 and bias.numel() == N
    if variant == 8:
        return linear_lif_t(x, w, bias, neuron=neuron, tau=tau, decay=decay,
                            decay_input=decay_input, soft_reset=soft_reset,
                            v_threshold=v_threshold, v_reset=v_reset, out=out, splits=splits,
                            workspace=workspace)
    df, sc, thr, vr, hard = _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold,
                                      v_reset)
    if out is None:
        out = torch.empty(T, B, N, device=x.device, dtype=torch.bfloat16)
    ws, ws_bytes = _workspace(workspace, 1 if variant == 6 else splits, T, B, 1, 1, N,
                              x.device)
    st = _lib.lib().snnb_linear_lif(_lib.ptr(x), T, B, K, _lib.ptr(w), _lib.ptr(bias), N, df, sc,
                                    thr, vr, hard, int(variant), int(block_n), int(splits),
                                    _lib.ptr(ws), ws_bytes, _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_linear_lif")
    return out


def linear_t_workspace_bytes(T, B, N, splits) -> int:
    n = int(_lib.lib().snnb_linear_t_workspace_bytes(T, B, N, int(splits)))
    if n < 0:
        raise ValueError(f"transposed-linear workspace size invalid: {(T, B, N, splits)}")
    return n


def linear_lif_t(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, *, neuron: str = "lif",
                 tau: float = 2.0, decay=None, decay_input: bool = True, soft_reset: bool = False,
                 v_threshold=1.0, v_reset: float = 0.0, out: torch.Tensor | None = None,
                 splits: int = 1, workspace: torch.Tensor | None = None, pool4: bool = False):
    """The transposed linear + LIF (snnb_linear_lif_t): x [T, B, K] bf16, w [N, K] bf16
    (N % 128 == 0), bias [N] f32 -> spikes [T, B, N] bf16 ([T, B, N / 4] with pool4, the OR
    of 4 consecutive features).  splits in {1, 2, 4, 8}: the K range over a cluster, partial
    sums in `workspace` (linear_t_workspace_bytes; allocated here if None)."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 3
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.shape[1] == x.shape[2]
    T, B, K = x.shape
    N = w.shape[0]
    assert bias.dtype == torch.float32 and bias.is_contiguous() and bias.numel() == N
    df, sc, thr, vr, hard = _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold,
                                      v_reset)
    No = N // 4 if pool4 else N
    if out is None:
        out = torch.empty(T, B, No, device=x.device, dtype=torch.bfloat16)
    assert out.is_contiguous() and out.numel() == T * B * No and out.dtype == torch.bfloat16
    need = linear_t_workspace_bytes(T, B, N, splits)
    if need and workspace is None:
        workspace = torch.empty(need // 4, device=x.device, dtype=torch.float32)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    assert ws_bytes >= need
    st = _lib.lib().snnb_linear_lif_t(_lib.ptr(x), T, B, K, _lib.ptr(w), _lib.ptr(bias), N, df,
                                      sc, thr, vr, hard, int(bool(pool4)), int(splits),
                                      _lib.ptr(workspace), ws_bytes, _lib.ptr(out),
                                      _lib.stream_of(x))
    _lib.check(st, "snnb_linear_lif_t")
    return out


def split_workspace_bytes(T, B, H, W, Cout, splits) -> int:
    n = int(_lib.lib().snnb_split_workspace_bytes(T, B, H, W, Cout, int(splits)))
    if n < 0:
        raise ValueError(f"split-K workspace size overflows: {(splits, T, B, H, W, Cout)}")
    return n


def _workspace(ws, splits, T, B, H, W, Cout, device):
    need = split_workspace_bytes(T, B, H, W, Cout, splits)
    if need == 0:
        return None, 0
    if ws is None:
        ws = torch.empty(need // 4, device=device, dtype=torch.float32)
    assert ws.is_cuda and ws.is_contiguous() and ws.numel() * ws.element_size() >= need
    return ws, ws.numel() * ws.element_size()


def linear_f32(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """x [T, B, K] bf16 @ w[N, K]^T + bias -> float32 [T, B, N] (no neuron); T in {2,4,8}."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 3
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.shape[1] == x.shape[2]
    T, B, K = x.shape
    N = w.shape[0]
    assert bias.dtype == torch.float32 and bias.numel() == N
    if out is None:
        out = torch.empty(T, B, N, device=x.device, dtype=torch.float32)
    st = _lib.lib().snnb_linear_f32(_lib.ptr(x), T, B, K, _lib.ptr(w), _lib.ptr(bias), N,
                                    _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_linear_f32")
    return out


def linear_mean(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """mean over T of (x[t] @ w^T + bias): x [T, B, K] bf16 -> f32 [B, N] (N <= 64)."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 3
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.shape[1] == x.shape[2]
    T, B, K = x.shape
    N = w.shape[0]
    assert bias.dtype == torch.float32 and bias.numel() == N
    if out is None:
        out = torch.empty(B, N, device=x.device, dtype=torch.float32)
    st = _lib.lib().snnb_linear_mean(_lib.ptr(x), T, B, K, _lib.ptr(w), _lib.ptr(bias), N,
                                     _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_linear_mean")
    return out


def linear_out(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-step logits x[t] @ w^T + bias: x [T, B, K] bf16 -> f32 [T, B, N] (N <= 64)."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 3
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and w.shape[1] == x.shape[2]
    T, B, K = x.shape
    N = w.shape[0]
    assert bias.dtype == torch.float32 and bias.numel() == N
    if out is None:
        out = torch.empty(T, B, N, device=x.device, dtype=torch.float32)
    st = _lib.lib().snnb_linear_out(_lib.ptr(x), T, B, K, _lib.ptr(w), _lib.ptr(bias), N,
                                    _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_linear_out")
    return out


def first_conv_lif(img: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, *, T: int,
                   neuron: str = "lif", tau: float = 2.0, decay=None, decay_input: bool = True,
                   soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0,
                   pool: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """Real-valued input layer: img f32 [Ti, B, Cin, H, W] (Ti = T, or 1 for direct
    encoding) with f32 weights [Cout, Cin, 3, 3] -> spikes [T, B, Ho, Wo, Cout] bf16."""
    assert img.is_cuda and img.dtype == torch.float32 and img.is_contiguous() and img.ndim == 5
    assert w.dtype == torch.float32 and w.is_contiguous() and w.shape[2:] == (3, 3)
    Ti, B, Cin, H, W = img.shape
    Cout = w.shape[0]
    df, sc, thr, vr, hard = _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold,
                                      v_reset)
    Ho, Wo = (H // 2, W // 2) if pool else (H, W)
    if out is None:
        out = torch.empty(T, B, Ho, Wo, Cout, device=img.device, dtype=torch.bfloat16)
    st = _lib.lib().snnb_first_conv_lif(_lib.ptr(img), Ti, T, B, Cin, H, W, _lib.ptr(w),
                                        _lib.ptr(bias), Cout, df, sc, thr, vr, hard,
                                        int(bool(pool)), _lib.ptr(out), _lib.stream_of(img))
    _lib.check(st, "snnb_first_conv_lif")
    return out


def first_conv_split_weight(w: torch.Tensor) -> torch.Tensor:
    """Image-layer conv weight [Cout, Cin, 3, 3] (float32, BN folded) -> the tensor-core
    image kernel's operand [Cout, KP] bf16: six groups [hi, mid, lo, hi, mid, hi]
    (SPLIT_WGT) of the K0 = 9 * Cin terms in torch's (ci, ky, kx) order, each group G = K0
    rounded up to even entries wide (a zero after the values when K0 is odd), zero-padded to
    KP."""
    Cout, Cin = w.shape[:2]
    K0 = 9 * Cin
    G = K0 + (K0 & 1)
    KP = int(_lib.lib().snnb_first_conv_tc_weight_k(Cin))
    if KP < 0:
        raise ValueError(f"tensor-core image layer takes Cin <= 4, got {Cin}")
    h, m, l = split_terms_host(w.detach().float().reshape(Cout, K0))
    terms = {"hi": h, "mid": m, "lo": l}
    out = torch.zeros(Cout, KP, dtype=torch.bfloat16, device=w.device)
    for g, name in enumerate(SPLIT_WGT):
        out[:, g * G:g * G + K0] = terms[name]
    return out.contiguous()


def first_conv_lif_tc(img: torch.Tensor, w_split: torch.Tensor, bias: torch.Tensor, *, T: int,
                      neuron: str = "lif", tau: float = 2.0, decay=None, decay_input: bool = True,
                      soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Image layer on the tensor cores (snnb_first_conv_lif_tc): img [1, B, Cin, H, W] float32
    (direct encoding: the same image at every step), w_split from first_conv_split_weight ->
    spikes [T, B, H, W, Cout] bf16.  float32-accurate conv (split operands), computed once
    per pixel; no pooling."""
    assert img.is_cuda and img.dtype == torch.float32 and img.is_contiguous() and img.ndim == 5
    assert img.shape[0] == 1, "direct encoding: one image per sample"
    _, B, Cin, H, W = img.shape
    Cout = w_split.shape[0]
    assert w_split.dtype == torch.bfloat16 and w_split.is_contiguous()
    assert bias.dtype == torch.float32 and bias.is_contiguous() and bias.numel() == Cout
    df, sc, thr, vr, hard = _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold,
                                      v_reset)
    if out is None:
        out = torch.empty(T, B, H, W, Cout, device=img.device, dtype=torch.bfloat16)
    st = _lib.lib().snnb_first_conv_lif_tc(_lib.ptr(img), T, B, Cin, H, W, _lib.ptr(w_split),
                                           _lib.ptr(bias), Cout, df, sc, thr, vr, hard,
                                           _lib.ptr(out), _lib.stream_of(img))
    _lib.check(st, "snnb_first_conv_lif_tc")
    return out


def time_graph(fn, reps: int = 10) -> float:
    """Device milliseconds per call of fn (a launcher on the current stream): reps calls
    are captured into one CUDA graph and the replay is timed with events, so host-side
    launch overhead does not enter the figure."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    return ms


def band_block_ns(W: int, cin: int, cout: int):
    """Channel-block widths the band kernel (variant 3) accepts for a 3x3 layer: W in
    {8, 16, 32, 64} and the block's weights (9 * ceil(Cin/64) * block_n rows of 128 bytes)
    within 108 KB of shared memory."""
    if W not in (8, 16, 32, 64):
        return ()
    cb = (cin + 63) // 64
    return tuple(bn for bn in (32, 64) if cout % bn == 0 and 9 * cb * bn <= 864)


def band_xs_block_ns(W: int, cin: int, cout: int):
    """Channel-block widths of variant 7 (band kernel with the column taps shifted in the
    epilogue): W in {8, 16, 32} (an image row fits one warp) and the block's weights within
    160 KB of shared memory (its stages hold one band copy, not three)."""
    if W not in (8, 16, 32):
        return ()
    cb = (cin + 63) // 64
    return tuple(bn for bn in (32, 64) if cout % bn == 0 and 9 * cb * bn <= 1280)


def candidates(cout: int, T: int, kslabs: int, max_splits: int = 8, band=(),
               dense_pool: bool = False, band_xs=(), linear_t: bool = False):
    """(variant, block_n, splits) configurations a layer admits; `band` / `band_xs` list the
    block widths of variants 3 / 7 the layer qualifies for (band_block_ns,
    band_xs_block_ns); dense_pool: the pooled dense form (snnb_conv3x3_lif_dense), whose
    epilogue the plain T-folded kernel alone has (variant 2, no split)."""
    lt = [(8, 128, sp) for sp in (1, 2, 4, 8)
          if linear_t and cout % 128 == 0 and T in (1, 2, 4, 8) and sp <= max(1, kslabs)]
    if dense_pool:
        return [c for c in candidates(cout, T, kslabs, max_splits)
                if c[0] == 2 and c[2] == 1] + lt
    out = lt
    for v in ((1, 2) if T in (2, 4, 8) else (1,)):
        for bn in ((32, 64, 128) if v == 1 else (32, 64, 128, 256)):
            if cout % bn:
                continue
            out.append((v, bn, 1))
            if v == 2 and bn >= 128:
                s = 2
                while s <= max_splits and s <= kslabs // 2:
                    out.append((v, bn, s))
                    s *= 2
    if T in (2, 4, 8):                # T folded, two M-tiles per CTA
        for bn in (32, 64, 128):
            if cout % bn:
                continue
            out.append((4, bn, 1))
            s = 2
            while s <= max_splits and s <= kslabs // 2:
                out.append((4, bn, s))
                s *= 2
    if T in (2, 4, 8):                # T folded, CTA pairs
        for bn in (64, 128, 256):
            if cout % bn:
                continue
            out.append((5, bn, 1))
            s = 2
            while s <= max_splits and s <= kslabs // 2:
                out.append((5, bn, s))
                s *= 2
    if T in (2, 4, 8):                # T folded, K split across a cluster
        for bn, sk in ((128, 2), (128, 4), (256, 2), (256, 4), (256, 8)):
            if cout % bn == 0 and sk <= max_splits and sk <= kslabs // 2:
                out.append((6, bn, sk))
    out.extend((3, bn, 1) for bn in band)
    out.extend((7, bn, 1) for bn in band_xs)
    return out


def pick_fastest(launch, cout: int, T: int, kslabs: int, reps: int = 10, band=(),
                 dense_pool: bool = False, band_xs=(), linear_t: bool = False, variants=None):
    """Time launch(variant, block_n, splits) for every configuration the layer admits
    (on its real operands, device time via time_graph) and return the fastest.
    variants: only these kernel variants (e.g. (1, 2) for strided convs)."""
    best, best_ms = (0, 0, 1), float("inf")
    for cfg in candidates(cout, T, kslabs, band=band, dense_pool=dense_pool, band_xs=band_xs,
                          linear_t=linear_t):
        if variants is not None and cfg[0] not in variants:
            continue
        # the lower of two timings: one replay can catch another context's work
        ms = min(time_graph(lambda: launch(*cfg), reps) for _ in range(2))
        if ms < best_ms:
            best, best_ms = cfg, ms
    return best


def device_status(stream_tensor: torch.Tensor | None = None) -> int:
    """Read and clear the device status word (SNNB_ERR_TIMEOUT after a bounded wait gave up)."""
    import ctypes
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    v = ctypes.c_int(0)
    _lib.check(_lib.lib().snnb_read_device_status(s, ctypes.byref(v)), "snnb_read_device_status")
    return v.value


def raise_on_device_status(what: str) -> None:
    """Read (and clear) the device status word on the current stream -- a stream
    synchronisation -- and raise SnnbError if a kernel reported a failure since the last
    read (SNNB_ERR_TIMEOUT: a bounded wait gave up and the launch left its output
    incomplete)."""
    st = device_status()
    if st != 0:
        _lib.check(st, what + " (device status)")


# ---- reference-API entries ----------------------------------------------------------------
def pack_spikes(x: torch.Tensor) -> torch.Tensor:
    """bf16 {0,1} spikes [..., C] (C % 32 == 0) -> packed int32 words [..., C/32]: channel c
    in bit c % 32 of word c / 32 (snnb_bitpack's order)."""
    from .binary import bitpack
    assert x.shape[-1] % 32 == 0
    return bitpack(x, ldw=x.shape[-1] // 32)


def unpack_spikes(words: torch.Tensor, C: int | None = None) -> torch.Tensor:
    """Packed int32 words [..., C/32] -> bf16 {0,1} spikes [..., C] (snnb_unpack_spikes)."""
    assert words.is_cuda and words.is_contiguous() and words.dtype == torch.int32
    C = words.shape[-1] * 32 if C is None else C
    assert C == words.shape[-1] * 32
    rows = words.numel() // words.shape[-1] if words.numel() else 0
    out = torch.empty(*words.shape[:-1], C, device=words.device, dtype=torch.bfloat16)
    st = _lib.lib().snnb_unpack_spikes(_lib.ptr(words), rows, C, _lib.ptr(out),
                                       _lib.stream_of(words))
    _lib.check(st, "snnb_unpack_spikes")
    return out


def conv3x3_lif_packed(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, *,
                       x_packed: bool, out_packed: bool, neuron: str = "lif", tau: float = 2.0,
                       decay=None, decay_input: bool = True, soft_reset: bool = False,
                       v_threshold=1.0, v_reset: float = 0.0, pool: bool = False,
                       block_n: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """conv3x3_lif with packed spikes in and / or out (snnb_conv3x3_lif_packed, T-folded
    kernel): x [T, B, H, W, Cin] bf16, or int32 words [T, B, H, W, Cin/32] with x_packed;
    the result [T, B, Ho, Wo, Cout] bf16, or words [T, B, Ho, Wo, Cout/32] with out_packed.
    Same spikes as conv3x3_lif."""
    assert x.is_cuda and x.is_contiguous() and x.ndim == 5
    assert x.dtype == (torch.int32 if x_packed else torch.bfloat16)
    T, B, H, W, cx = x.shape
    Cin = cx * 32 if x_packed else cx
    assert w.dtype == torch.bfloat16 and w.is_contiguous() and tuple(w.shape[1:]) == (3, 3, Cin)
    Cout = w.shape[0]
    assert bias.dtype == torch.float32 and bias.is_contiguous() and bias.numel() == Cout
    df, sc, thr, vr, hard = _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold,
                                      v_reset)
    Ho, Wo = (H // 2, W // 2) if pool else (H, W)
    if out is None:
        out = torch.empty(T, B, Ho, Wo, Cout // 32 if out_packed else Cout, device=x.device,
                          dtype=torch.int32 if out_packed else torch.bfloat16)
    st = _lib.lib().snnb_conv3x3_lif_packed(
        _lib.ptr(x), int(bool(x_packed)), T, B, H, W, Cin, _lib.ptr(w), _lib.ptr(bias), Cout, df,
        sc, thr, vr, hard, int(bool(pool)), int(bool(out_packed)), int(block_n), _lib.ptr(out),
        _lib.stream_of(x))
    _lib.check(st, "snnb_conv3x3_lif_packed")
    return out


def dense_conv_weight(w_khwc: torch.Tensor, H: int, W: int, *,
                      pool: bool = False) -> torch.Tensor:
    """A 3x3 / stride 1 / padding 1 conv on H x W images (H, W <= 2) as one dense matrix:
    every output pixel's window covers the whole image, so the conv is a linear map from
    the image's H*W*Cin inputs (NHWC order) to its H*W*Cout outputs, and
    W'[(p, co), (q, ci)] = w[co, qh - ph + 1, qw - pw + 1, ci].  The padding taps, whose
    products are zero (5 of the 9 at 2x2, 8 of 9 at 1x1), drop out of the GEMM.
    pool: rows ordered (co, p) instead, so that the 2x2 max-pool is an OR over 4
    consecutive outputs (snnb_conv3x3_lif_dense with pool).
    w_khwc [Cout, 3, 3, Cin] -> [H*W*Cout, H*W*Cin], same dtype and device."""
    assert w_khwc.ndim == 4 and tuple(w_khwc.shape[1:3]) == (3, 3)
    assert 1 <= H <= 2 and 1 <= W <= 2, (H, W)
    assert not pool or (H, W) == (2, 2)
    Cout, Cin = w_khwc.shape[0], w_khwc.shape[3]
    out = w_khwc.new_zeros(H * W, Cout, H * W, Cin)
    for ph in range(H):
        for pw in range(W):
            for qh in range(H):
                for qw in range(W):
                    out[ph * W + pw, :, qh * W + qw, :] = w_khwc[:, qh - ph + 1, qw - pw + 1, :]
    if pool:
        out = out.transpose(0, 1)
    return out.reshape(H * W * Cout, H * W * Cin).contiguous()


def dense_conv_bias(bias: torch.Tensor, H: int, W: int, *, pool: bool = False) -> torch.Tensor:
    """The bias of dense_conv_weight's outputs: b'[co] for row (p, co), or (co, p) with
    pool."""
    b = bias.float()
    return (b.repeat_interleave(H * W) if pool else b.repeat(H * W)).contiguous()


def conv3x3_lif_dense(x: torch.Tensor, wd: torch.Tensor, bd: torch.Tensor, *,
                      neuron: str = "lif", tau: float = 2.0, decay=None,
                      decay_input: bool = True, soft_reset: bool = False, v_threshold=1.0,
                      v_reset: float = 0.0, pool: bool = False,
                      out: torch.Tensor | None = None, variant: int = 0, block_n: int = 0,
                      splits: int = 1, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """conv3x3_lif for images of at most 2x2 pixels as one dense GEMM per image
    (snnb_conv3x3_lif_dense): x [T, B, H, W, Cin] bf16, wd / bd from dense_conv_weight /
    dense_conv_bias (with the same `pool`) -> spikes [T, B, Ho, Wo, Cout] bf16."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.ndim == 5
    T, B, H, W, Cin = x.shape
    assert wd.dtype == torch.bfloat16 and wd.is_contiguous() and wd.shape[1] == H * W * Cin
    Cout = wd.shape[0] // (H * W)
    assert bd.dtype == torch.float32 and bd.is_contiguous() and bd.numel() == H * W * Cout
    df, sc, thr, vr, hard = _lif_args(neuron, tau, decay, decay_input, soft_reset, v_threshold,
                                      v_reset)
    Ho, Wo = (1, 1) if pool else (H, W)
    if out is None:
        out = torch.empty(T, B, Ho, Wo, Cout, device=x.device, dtype=torch.bfloat16)
    if variant == 8:
        # the transposed form: features (p, co) -- or (co, p) with pool -- as M
        linear_lif_t(x.view(T, B, H * W * Cin), wd, bd, neuron=neuron, tau=tau, decay=decay,
                     decay_input=decay_input, soft_reset=soft_reset, v_threshold=v_threshold,
                     v_reset=v_reset, out=out.view(T, B, -1), splits=splits,
                     workspace=workspace, pool4=pool)
        return out
    ws, ws_bytes = _workspace(workspace, 1 if variant == 6 else splits, T, B, 1, 1,
                              H * W * Cout, x.device)
    st = _lib.lib().snnb_conv3x3_lif_dense(
        _lib.ptr(x), T, B, H, W, Cin, _lib.ptr(wd), _lib.ptr(bd), Cout, df, sc, thr, vr, hard,
        int(bool(pool)), int(variant), int(block_n), int(splits), _lib.ptr(ws), ws_bytes,
        _lib.ptr(out), _lib.stream_of(x))
    _lib.check(st, "snnb_conv3x3_lif_dense")
    return out


# ---- float32 operands on the bf16 tensor cores (csrc/split.cu) ----------------------------
# A float32 value is carried as three bf16 terms (hi, mid, lo); activations are laid out as
# six channel groups [hi, hi, hi, mid, mid, lo] against weights [hi, mid, lo, hi, mid, hi], so
# one bf16 conv / GEMM over 6 * Cp channels sums the six larger products of the terms, each
# exact in float32 (the dropped three are below 2^-23 of the product).  Cp = Cin rounded up
# to a multiple of 4 (zero channels), so that 6 * Cp is a multiple of 8.
SPLIT_ACT = ("hi", "hi", "hi", "mid", "mid", "lo")
SPLIT_WGT = ("hi", "mid", "lo", "hi", "mid", "hi")


def split_width(C: int) -> int:
    return (C + 3) // 4 * 4


def split_terms_host(t: torch.Tensor):
    """float32 tensor -> (hi, mid, lo) bf16 tensors, hi + mid + lo == t to within 2^-24 |t|
    (the same rounding as the device split: each residual is exact in float32)."""
    t = t.detach().float()
    h = t.to(torch.bfloat16)
    over = torch.isinf(h.float()) & torch.isfinite(t)     # above bf16's largest finite value
    if bool(over.any()):
        big = torch.full_like(h, torch.finfo(torch.bfloat16).max)
        h = torch.where(over, torch.where(t > 0, big, -big), h)
    r1 = t - h.float()
    m = r1.to(torch.bfloat16)
    l = (r1 - m.float()).to(torch.bfloat16)
    bad = ~torch.isfinite(h.float())
    if bool(bad.any()):
        m = m.masked_fill(bad, 0)
        l = l.masked_fill(bad, 0)
    return h, m, l


def _split_groups(t_last: torch.Tensor, order) -> torch.Tensor:
    """[..., C] float32 -> [..., 6 * Cp] bf16, group g = term order[g] of t (zero padded)."""
    C = t_last.shape[-1]
    Cp = split_width(C)
    h, m, l = split_terms_host(t_last)
    terms = {"hi": h, "mid": m, "lo": l}
    out = torch.zeros(*t_last.shape[:-1], 6 * Cp, dtype=torch.bfloat16, device=t_last.device)
    for g, name in enumerate(order):
        out[..., g * Cp: g * Cp + C] = terms[name]
    return out.contiguous()


def split_weight_khwc(w: torch.Tensor) -> torch.Tensor:
    """torch conv weight [Cout, Cin, 3, 3] (float32) -> [Cout, 3, 3, 6 * Cp] bf16 weight
    groups for a float32-faithful conv3x3_lif on split_activations' output."""
    return _split_groups(w.detach().float().permute(0, 2, 3, 1), SPLIT_WGT)


def split_weight_rows(w: torch.Tensor) -> torch.Tensor:
    """linear weight [N, K] (float32) -> [N, 6 * Kp] bf16 weight groups."""
    return _split_groups(w.detach().float(), SPLIT_WGT)


def split_activations(x: torch.Tensor) -> torch.Tensor:
    """x [..., C] float32 (contiguous) -> [..., 6 * Cp] bf16 activation groups on the device
    (snnb_split_bf16_terms)."""
    assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
    C = x.shape[-1]
    Cp = split_width(C)
    rows = x.numel() // C if C else 0
    out = torch.empty(*x.shape[:-1], 6 * Cp, device=x.device, dtype=torch.bfloat16)
    st = _lib.lib().snnb_split_bf16_terms(_lib.ptr(x), rows, C, Cp, _lib.ptr(out),
                                          _lib.stream_of(x))
    _lib.check(st, "snnb_split_bf16_terms")
    return out


def _frames_f32(x_seq: torch.Tensor) -> torch.Tensor:
    """[T, B, C, H, W] (NCHW or channels-last view) float32 / float16 -> contiguous
    [T, B, H, W, C] float32 (float16 values are exact in float32)."""
    return x_seq.permute(0, 1, 3, 4, 2).to(torch.float32).contiguous()


def weight_khwc(w: torch.Tensor) -> torch.Tensor:
    """torch conv weight [Cout, Cin, 3, 3] -> the kernels' K-major [Cout, 3, 3, Cin] bf16."""
    return w.detach().permute(0, 2, 3, 1).contiguous().to(torch.bfloat16)


def _to_frames(x_seq: torch.Tensor) -> torch.Tensor:
    """[T, B, C, H, W] (NCHW or channels-last view) -> contiguous [T, B, H, W, C] bf16."""
    return x_seq.permute(0, 1, 3, 4, 2).to(torch.bfloat16).contiguous()


def _from_frames(y: torch.Tensor, dtype, layout: str) -> torch.Tensor:
    """[T, B, H, W, C] -> [T, B, C, H, W] view (channels-last storage) or contiguous."""
    v = y.permute(0, 1, 4, 2, 3)
    if layout == "NHWC":
        return v.to(dtype)
    return v.contiguous().to(dtype)


def conv_neuron(x_seq, weight, bias, *, stride=1, padding=0, dilation=1, groups=1,
                neuron: str = "if", tau: float = 2.0, decay=None, decay_input: bool = True,
                soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0,
                layout: str = "NCHW"):
    """conv + bias + neuron (reference fused.py:513-551) for x_seq [T, B, Cin, H, W].
    k x k / padding k // 2 convs (k in {1, 3, 5, 7}) of stride 1 or 2 with a scalar threshold
    run fused on the tcgen05 kernels when Cout % 32 == 0: bf16 operands for a bf16 input (Cin % 8 == 0); for a float32 /
    float16 input (Cin % 4 == 0) float32-faithful, each operand as three bf16 terms (a
    split-terms launch, then the conv over six channel groups); a float32 input with other
    Cin (the 3x3 / stride 1 image layer) takes the float32 CUDA-core kernel.  Any other geometry keeps the
    reference's two steps: torch's conv in the input's dtype, then the fused neuron kernel."""
    from .fused import fused_bias_if_lif
    Cin, Cout = weight.shape[1], weight.shape[0]
    kw = dict(neuron=neuron, tau=tau, decay=decay, decay_input=decay_input,
              soft_reset=soft_reset, v_threshold=v_threshold, v_reset=v_reset)
    b = bias.detach().float().contiguous() if bias is not None else \
        torch.zeros(Cout, device=x_seq.device)
    ks, st = tuple(weight.shape[2:]), _pair(stride)
    if ks in ((1, 1), (3, 3), (5, 5), (7, 7)) and st in ((1, 1), (2, 2)) and \
            (ks, st) != ((3, 3), (1, 1)) and _pair(padding) == (ks[0] // 2,) * 2 and \
            _pair(dilation) == (1, 1) and groups == 1 and \
            isinstance(v_threshold, (int, float)) and Cout % 32 == 0:
        # strided, 1x1 and 5x5 / 7x7 convs: the same kernels, activation boxes traversing the
        # input with the stride (snnb_conv_lif_strided); a float32 input of any Cin (the
        # 7x7 stem on the image) as split terms, zero padded to a multiple of 4 channels
        if x_seq.dtype == torch.bfloat16 and Cin % 8 == 0:
            y = conv_lif_strided(_to_frames(x_seq), weight_khwc(weight), b, stride=st[0], **kw)
            return _from_frames(y, x_seq.dtype, layout)
        if x_seq.dtype in (torch.float32, torch.float16):
            y = conv_lif_strided(split_activations(_frames_f32(x_seq)),
                                 split_weight_khwc(weight), b, stride=st[0], **kw)
            return _from_frames(y, x_seq.dtype, layout)
    if tuple(weight.shape[2:]) == (3, 3) and _pair(stride) == (1, 1) and \
            _pair(padding) == (1, 1) and _pair(dilation) == (1, 1) and groups == 1 and \
            isinstance(v_threshold, (int, float)):
        if x_seq.dtype == torch.bfloat16 and Cin % 8 == 0 and Cout % 32 == 0:
            y = conv3x3_lif(_to_frames(x_seq), weight_khwc(weight), b, **kw)
            return _from_frames(y, x_seq.dtype, layout)
        if x_seq.dtype in (torch.float32, torch.float16) and Cin % 4 == 0 and Cout % 32 == 0:
            # float32-faithful: three bf16 terms per operand, six products on the tensor cores
            y = conv3x3_lif(split_activations(_frames_f32(x_seq)), split_weight_khwc(weight),
                            b, **kw)
            return _from_frames(y, x_seq.dtype, layout)
        if x_seq.dtype == torch.float32 and Cout % 8 == 0:
            y = first_conv_lif(x_seq.contiguous(), weight.detach().float().contiguous(), b,
                               T=x_seq.shape[0], **kw)
            return _from_frames(y, x_seq.dtype, layout)
    T, B = x_seq.shape[:2]
    x4 = x_seq.reshape(T * B, *x_seq.shape[2:])
    x4 = x4.contiguous(memory_format=torch.channels_last) if layout == "NHWC" else x4.contiguous()
    y = torch.nn.functional.conv2d(x4, weight.to(x4.dtype), None, stride, padding, dilation,
                                   groups)
    if layout == "NHWC":
        y = y.contiguous(memory_format=torch.channels_last)
    return fused_bias_if_lif(y.view(T, B, *y.shape[1:]), None if bias is None else b,
                             layout=layout, **kw)


def linear_neuron(x_seq, weight, bias, *, neuron: str = "if", tau: float = 2.0, decay=None,
                  decay_input: bool = True, soft_reset: bool = False, v_threshold=1.0,
                  v_reset: float = 0.0):
    """linear + bias + neuron (reference fused.py:554-579); one fused tcgen05 launch with
    float32 accumulation, out_features % 32 == 0: bf16 operands for a bf16 input
    (in_features % 8 == 0); for a float32 / float16 input float32-faithful, each operand as
    three bf16 terms (in_features % 4 == 0)."""
    T, B = x_seq.shape[:2]
    N = weight.shape[0]
    b = bias.detach().float().contiguous() if bias is not None else \
        torch.zeros(N, device=x_seq.device)
    kw = dict(neuron=neuron, tau=tau, decay=decay, decay_input=decay_input,
              soft_reset=soft_reset, v_threshold=v_threshold, v_reset=v_reset)
    if x_seq.dtype == torch.bfloat16:
        x = x_seq.reshape(T, B, -1).contiguous()
        y = linear_lif(x, weight.detach().to(torch.bfloat16).contiguous(), b, **kw)
    else:
        x = split_activations(x_seq.reshape(T, B, -1).to(torch.float32).contiguous())
        y = linear_lif(x, split_weight_rows(weight), b, **kw)
    return y.to(x_seq.dtype)


def conv_bn_neuron(x_seq, conv_w, conv_b, bn_w, bn_b, bn_mean, bn_var, bn_eps, *, stride=1,
                   padding=0, dilation=1, groups=1, **neuron_kwargs):
    """conv + BN (folded on the host) + neuron (reference fused.py:602-611)."""
    new_w, new_b = fold_conv_bn(conv_w, conv_b, bn_w, bn_b, bn_mean, bn_var, bn_eps)
    return conv_neuron(x_seq, new_w, new_b, stride=stride, padding=padding, dilation=dilation,
                       groups=groups, **neuron_kwargs)


def _pair(v):
    return tuple(v) if isinstance(v, (tuple, list)) else (v, v)
