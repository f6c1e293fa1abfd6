"""Conv / linear + neuron modules, same constructors and forward signatures as the reference.

Mirrors snn_compiler/nn/modules.py of the reference:
  FusedConvNeuron        :160-217   conv (+ bias) + IF/LIF
  FusedLinearNeuron      :220-255   linear (+ bias) + IF/LIF
  FusedConvBNNeuron      :258-357   conv + BN (folded at construction, or kept separate) + IF/LIF
  FusedConvBNAddNeuron   :360-443   conv + BN + residual add + IF/LIF
x_seq is [T, B, C, H, W] (logical NCHW; channels-last storage when layout="NHWC") or
[T, B, features]; the result has the same layout.

Routing (every launch is libsnnb200.so).  The reference convolves in the input's dtype, so
the route depends on it:
  - 3x3 / stride 1 / padding 1 convs with Cout % 32 == 0 on a bf16 input (Cin % 8 == 0):
    one launch of the fused tcgen05 conv + bias + neuron kernel (bf16 operands, float32
    accumulation -- the reference's bf16 mode);
  - the same geometry on a float32 / float16 input (Cin % 4 == 0): float32-faithful on the
    same kernel -- input and weights each carried as three bf16 terms (snnb_split_bf16_terms,
    weights split once per module), six products per pair summed in float32;
  - a float32 input with other Cin (the image-input first layer): the float32 CUDA-core
    conv + neuron kernel;
  - linears with out_features % 32 == 0 (in_features % 8 == 0 for bf16, % 4 == 0 for
    float32 / float16, split as above): the fused linear kernel;
  - 3x3 / padding 1 convs of stride 2, 1x1 / padding 0 convs and 5x5 / 7x7 convs (padding
    k // 2) of stride 1 or 2 (a ResNet's strided, pointwise and stem convs) on the same
    kernels, the activation boxes traversing the input with the stride
    (snnb_conv_lif_strided), bf16 (channels zero padded to a multiple of 8) or split as
    above (a float32 input of any Cin);
  - the residual form (FusedConvBNAddNeuron) on these geometries: the same tcgen05 kernels
    with the residual added in the epilogue (snnb_conv3x3_lif_res, snnb_conv_lif_strided);
  - FusedConvBN (conv + folded BN, no neuron: a ResNet block's downsample branch) on a bf16
    input: the T-folded kernel with a float32 result (snnb_conv_f32);
  - fold_bn=False and any other conv geometry keep the reference's own two-step structure:
    torch's conv (+ eval BN) followed by the fused neuron kernel (snnb_neuron_multistep),
    exactly as modules.py:324-357 / :415-443 do.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..kernels import conv as KC
from ..kernels.fused import fold_conv_bn, fused_bias_if_lif


def _pair(v):
    return tuple(v) if isinstance(v, (tuple, list)) else (v, v)


def _store_threshold(mod, v_threshold):
    if isinstance(v_threshold, torch.Tensor):
        mod.register_buffer("v_threshold", v_threshold.float().contiguous())
    else:
        mod.v_threshold = float(v_threshold)


class _NeuronArgs:
    def _set_neuron(self, neuron, tau, decay, decay_input, soft_reset, v_threshold, v_reset):
        self.neuron = neuron
        self.tau = tau
        self.decay = decay
        self.decay_input = decay_input
        self.soft_reset = soft_reset
        self.v_reset = v_reset
        _store_threshold(self, v_threshold)

    def _neuron_kw(self):
        return dict(neuron=self.neuron, tau=self.tau, decay=self.decay,
                    decay_input=self.decay_input, soft_reset=self.soft_reset,
                    v_threshold=self.v_threshold, v_reset=self.v_reset)

    def _conv_kw(self):
        """The neuron arguments plus the kernel schedule tune_convs chose (if any)."""
        kw = self._neuron_kw()
        sched = getattr(self, "_sched", None)
        if sched is not None:
            kw.update(variant=sched[0], block_n=sched[1])
        return kw


def _fused_conv_ok(weight, stride, padding, dilation, groups, v_threshold):
    """k x k / padding k // 2 with k in {1, 3, 5, 7}, stride 1 or 2 (the convs of VGG and
    ResNet, its 7x7 stem included)."""
    ks = tuple(weight.shape[2:])
    return (ks in ((3, 3), (1, 1), (5, 5), (7, 7)) and _pair(stride) in ((1, 1), (2, 2))
            and _pair(padding) == (ks[0] // 2,) * 2 and _pair(dilation) == (1, 1)
            and groups == 1 and isinstance(v_threshold, (int, float)))


def _res_frames(r):
    """Residual [T, B, C, H, W] -> contiguous [T, B, H, W, C]: bf16 stays bf16 (spikes are
    exact in it), any other dtype goes to float32 so no value is rounded."""
    dt = torch.bfloat16 if r.dtype == torch.bfloat16 else torch.float32
    return r.permute(0, 1, 3, 4, 2).to(dt).contiguous()


def _conv_lif(x_seq, weight, bias, layout, kw, cache, residual=None, stride=1):
    """Fused conv + bias (+ residual) + neuron for a conv _fused_conv_ok accepts.  `cache`
    holds the kernel-layout weights so they are converted once per module, not per call."""
    T, B, Cin = x_seq.shape[:3]
    Cout = weight.shape[0]
    b = bias.detach().float().contiguous() if bias is not None else \
        torch.zeros(Cout, device=x_seq.device)
    res = None if residual is None else _res_frames(residual)
    st = _pair(stride)[0]
    plain = tuple(weight.shape[2:]) == (3, 3) and st == 1       # the 3x3 / stride 1 entry
    k = weight.shape[2]
    if not plain and k > 1 and Cin < 8 and Cout % 32 == 0 and \
            x_seq.dtype in (torch.bfloat16, torch.float32, torch.float16):
        return _stem_conv_lif(x_seq, weight, b, layout, kw, cache, res, st)
    conv = KC.conv3x3_lif if plain else \
        (lambda x, w, b, **k: KC.conv_lif_strided(x, w, b, stride=st, **k))
    if x_seq.dtype == torch.bfloat16 and (Cin % 8 == 0 or not plain) and Cout % 32 == 0:
        # (a bf16 image with Cin % 8 != 0, e.g. a ResNet stem: channels zero padded to a
        # multiple of 8 in the frames and the weights -- the padded products are zero)
        cp = (Cin + 7) // 8 * 8
        key = ("khwc", weight.data_ptr(), weight._version)
        if cache.get("key") != key:
            cache.clear()
            cache["key"], cache["w"] = key, F.pad(KC.weight_khwc(weight), (0, cp - Cin))
        xf = KC._to_frames(x_seq)
        if cp != Cin:
            xf = F.pad(xf, (0, cp - Cin))
        y = conv(xf, cache["w"], b, residual=res, **kw)
        return KC._from_frames(y, x_seq.dtype, layout)
    if x_seq.dtype in (torch.float32, torch.float16) and (Cin % 4 == 0 or not plain) and \
            Cout % 32 == 0:
        # float32-faithful on the tensor cores: both operands as three bf16 terms (a 3x3 /
        # stride 1 image layer with Cin % 4 != 0 takes the CUDA-core kernel below instead)
        key = ("split", weight.data_ptr(), weight._version)
        if cache.get("key") != key:
            cache.clear()
            cache["key"], cache["w"] = key, KC.split_weight_khwc(weight)
        y = conv(KC.split_activations(KC._frames_f32(x_seq)), cache["w"], b, residual=res,
                 **kw)
        return KC._from_frames(y, x_seq.dtype, layout)
    if residual is not None or not plain:
        return None
    if x_seq.dtype == torch.float32 and Cout % 8 == 0:
        w = weight.detach().float().contiguous()
        kw = {k_: v for k_, v in kw.items() if k_ not in ("variant", "block_n")}
        y = KC.first_conv_lif(x_seq.contiguous(), w, b, T=T, **kw)
        return KC._from_frames(y, x_seq.dtype, layout)
    return None


def _stem_conv_lif(x_seq, weight, b, layout, kw, cache, res, st):
    """A k x k conv on an image of few channels (a ResNet's 7x7 / stride 2 stem, Cin = 3):
    with Cin channels per tap a tap's 64-wide k-slab would be mostly zero padding (49 taps
    for 147 products per pixel), so the window is gathered into the channel dimension first
    -- each column one (dy, dx, c) of x[c, stride*h + dy - k/2, stride*w + dx - k/2] (zero
    outside) -- and the conv runs as a 1x1 conv with K = k*k*Cin on the same kernel (the
    same products, summed in another order).  bf16: snnb_window_gather_nhwc, K zero padded to
    a multiple of 8; float32 / float16: F.unfold, then split terms as the other float32
    convs."""
    T, B, Cin, H, W = x_seq.shape
    Cout, k = weight.shape[0], weight.shape[2]
    Ho, Wo = KC.conv_out_size(H, st), KC.conv_out_size(W, st)
    K = Cin * k * k
    if x_seq.dtype == torch.bfloat16:
        # the window gathered by snnb_window_gather_nhwc, columns (dy, dx, c)
        kp = (K + 7) // 8 * 8
        key = ("stem", weight.data_ptr(), weight._version)
        if cache.get("key") != key:
            cache.clear()
            w1 = KC.weight_khwc(weight).reshape(Cout, 1, 1, K)
            cache["key"], cache["w"] = key, F.pad(w1, (0, kp - K)).contiguous()
        xf = KC.window_gather_nhwc(KC._to_frames(x_seq), k, st, k // 2, kp)
    else:
        # float32 / float16: F.unfold's columns (c, dy, dx), then the split terms
        cols = F.unfold(x_seq.reshape(T * B, Cin, H, W).to(torch.float32), k, padding=k // 2,
                        stride=st)
        cols = cols.transpose(1, 2).reshape(T, B, Ho, Wo, K)      # [T, B, Ho, Wo, K]
        key = ("stem-split", weight.data_ptr(), weight._version)
        if cache.get("key") != key:
            cache.clear()
            cache["key"], cache["w"] = key, KC.split_weight_khwc(
                weight.detach().reshape(Cout, K, 1, 1))
        xf = KC.split_activations(cols.to(torch.float32).contiguous())
    y = KC.conv_lif_strided(xf, cache["w"], b, stride=1, residual=res, **kw)
    return KC._from_frames(y, x_seq.dtype, layout)


def _torch_conv(x_seq, weight, bias, stride, padding, dilation, groups, layout):
    """torch conv on [T*B, C, H, W] frames -> y_seq [T, B, Cout, Ho, Wo] (the reference's
    conv step, modules.py:199-206)."""
    T, B = x_seq.shape[:2]
    x4 = x_seq.reshape(T * B, *x_seq.shape[2:])
    w = weight
    if layout == "NHWC":
        x4 = x4.contiguous(memory_format=torch.channels_last)
        w = weight.to(memory_format=torch.channels_last)
    else:
        x4 = x4.contiguous()
    y = F.conv2d(x4, w.to(x4.dtype), bias=bias, stride=stride, padding=padding,
                 dilation=dilation, groups=groups)
    if layout == "NHWC":
        y = y.contiguous(memory_format=torch.channels_last)
    return y.view(T, B, *y.shape[1:])


class FusedConvNeuron(nn.Module, _NeuronArgs):
    """Conv2d + (optional) bias + IF/LIF (reference modules.py:160-217)."""

    def __init__(self, in_ch, out_ch, kernel_size, *, stride=1, padding=0, dilation=1,
                 groups=1, bias: bool = True, neuron: str = "if", tau: float = 2.0,
                 decay: float | None = None, decay_input: bool = True,
                 soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0,
                 layout: str = "NCHW"):
        super().__init__()
        conv = nn.Conv2d(in_ch, out_ch, kernel_size, stride=stride, padding=padding,
                         dilation=dilation, groups=groups, bias=bias)
        self.weight = nn.Parameter(conv.weight.detach().clone())
        self.bias = nn.Parameter(conv.bias.detach().clone()) if bias else None
        self.stride, self.padding = conv.stride, conv.padding
        self.dilation, self.groups = conv.dilation, conv.groups
        self.layout = layout
        self._set_neuron(neuron, tau, decay, decay_input, soft_reset, v_threshold, v_reset)
        self._cache = {}

    def forward(self, x_seq):
        if _fused_conv_ok(self.weight, self.stride, self.padding, self.dilation, self.groups,
                          self.v_threshold):
            y = _conv_lif(x_seq, self.weight, self.bias, self.layout, self._conv_kw(),
                          self._cache, stride=self.stride)
            if y is not None:
                return y
        y = _torch_conv(x_seq, self.weight, None, self.stride, self.padding, self.dilation,
                        self.groups, self.layout)
        b = None if self.bias is None else self.bias.detach().float().contiguous()
        return fused_bias_if_lif(y, b, layout=self.layout, **self._neuron_kw())


class FusedLinearNeuron(nn.Module, _NeuronArgs):
    """Linear + (optional) bias + IF/LIF (reference modules.py:220-255)."""

    def __init__(self, in_features, out_features, *, bias: bool = True, neuron: str = "if",
                 tau: float = 2.0, decay: float | None = None, decay_input: bool = True,
                 soft_reset: bool = False, v_threshold=1.0, v_reset: float = 0.0):
        super().__init__()
        lin = nn.Linear(in_features, out_features, bias=bias)
        self.weight = nn.Parameter(lin.weight.detach().clone())
        self.bias = nn.Parameter(lin.bias.detach().clone()) if bias else None
        self._set_neuron(neuron, tau, decay, decay_input, soft_reset, v_threshold, v_reset)

    def forward(self, x_seq):
        K, N = self.weight.shape[1], self.weight.shape[0]
        kmod = 8 if x_seq.dtype == torch.bfloat16 else 4
        if x_seq.dtype in (torch.bfloat16, torch.float32, torch.float16) and K % kmod == 0 \
                and N % 32 == 0 and isinstance(self.v_threshold, (int, float)):
            return KC.linear_neuron(x_seq, self.weight, self.bias, **self._neuron_kw())
        T, B = x_seq.shape[:2]
        y = F.linear(x_seq.reshape(T * B, -1), self.weight.to(x_seq.dtype)).view(T, B, N)
        b = None if self.bias is None else self.bias.detach().float().contiguous()
        return fused_bias_if_lif(y, b, layout="NCHW", **self._neuron_kw())


class _ConvBNBase(nn.Module, _NeuronArgs):
    def __init__(self, conv: nn.Conv2d, bn: nn.BatchNorm2d, fold_bn, neuron, tau, decay,
                 decay_input, soft_reset, v_threshold, v_reset, layout):
        super().__init__()
        assert bn.running_mean is not None
        self.fold_bn = fold_bn
        if fold_bn:
            new_w, new_b = fold_conv_bn(conv.weight.detach(),
                                        conv.bias.detach() if conv.bias is not None else None,
                                        bn.weight.detach(), bn.bias.detach(),
                                        bn.running_mean.detach(), bn.running_var.detach(),
                                        bn.eps)
            self.weight = nn.Parameter(new_w)
            self.bias = nn.Parameter(new_b)
        else:
            self.weight = nn.Parameter(conv.weight.detach().clone())
            self.register_parameter(
                "conv_bias",
                nn.Parameter(conv.bias.detach().clone()) if conv.bias is not None else None)
            self.register_buffer("bn_weight", bn.weight.detach().clone())
            self.register_buffer("bn_bias", bn.bias.detach().clone())
            self.register_buffer("bn_mean", bn.running_mean.detach().clone())
            self.register_buffer("bn_var", bn.running_var.detach().clone())
            self.bn_eps = bn.eps
            self.bias = None
        self.stride, self.padding = conv.stride, conv.padding
        self.dilation, self.groups = conv.dilation, conv.groups
        self.layout = layout
        self._set_neuron(neuron, tau, decay, decay_input, soft_reset, v_threshold, v_reset)
        self._cache = {}

    def _conv_bn(self, x_seq):
        """(y_seq, neuron bias) through torch's conv (+ eval BN) -- modules.py:324-345."""
        if self.fold_bn:
            y = _torch_conv(x_seq, self.weight, None, self.stride, self.padding, self.dilation,
                            self.groups, self.layout)
            return y, self.bias.detach().float().contiguous()
        y = _torch_conv(x_seq, self.weight, self.conv_bias, self.stride, self.padding,
                        self.dilation, self.groups, self.layout)
        T, B = y.shape[:2]
        y4 = F.batch_norm(y.reshape(T * B, *y.shape[2:]), self.bn_mean, self.bn_var,
                          self.bn_weight, self.bn_bias, training=False, eps=self.bn_eps)
        if self.layout == "NHWC":
            y4 = y4.contiguous(memory_format=torch.channels_last)
        return y4.view(T, B, *y4.shape[1:]), None


class FusedConvBNNeuron(_ConvBNBase):
    """Conv2d + BN + IF/LIF (reference modules.py:258-357).  fold_bn=True folds BN into
    the conv at construction and runs the fused kernel; fold_bn=False keeps conv and BN as
    separate ops (bit-identical pre-activation to the unfused network) and fuses only the
    neuron."""

    def __init__(self, conv: nn.Conv2d, bn: nn.BatchNorm2d, *, fold_bn: bool = True,
                 neuron: str = "if", tau: float = 2.0, decay: float | None = None,
                 decay_input: bool = True, soft_reset: bool = False, v_threshold=1.0,
                 v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__(conv, bn, fold_bn, neuron, tau, decay, decay_input, soft_reset,
                         v_threshold, v_reset, layout)

    def forward(self, x_seq):
        if self.fold_bn and _fused_conv_ok(self.weight, self.stride, self.padding,
                                           self.dilation, self.groups, self.v_threshold):
            y = _conv_lif(x_seq, self.weight, self.bias, self.layout, self._conv_kw(),
                          self._cache, stride=self.stride)
            if y is not None:
                return y
        y, b = self._conv_bn(x_seq)
        return fused_bias_if_lif(y, b, layout=self.layout, **self._neuron_kw())


class FusedConvBNAddNeuron(_ConvBNBase):
    """Conv2d + BN + residual add + IF/LIF (reference modules.py:360-443):
    spike = neuron((conv_bn(x) + bias) + residual).  With folded BN on a 3x3 / s1 / p1 conv
    the residual is read in the tensor-core kernel's epilogue (one launch); otherwise
    torch's conv + BN runs first and the residual is consumed in the neuron kernel."""

    def __init__(self, conv: nn.Conv2d, bn: nn.BatchNorm2d, *, fold_bn: bool = True,
                 neuron: str = "if", tau: float = 2.0, decay: float | None = None,
                 decay_input: bool = True, soft_reset: bool = False, v_threshold=1.0,
                 v_reset: float = 0.0, layout: str = "NCHW"):
        super().__init__(conv, bn, fold_bn, neuron, tau, decay, decay_input, soft_reset,
                         v_threshold, v_reset, layout)

    def forward(self, x_seq, residual_seq):
        if self.fold_bn and _fused_conv_ok(self.weight, self.stride, self.padding,
                                           self.dilation, self.groups, self.v_threshold) \
                and tuple(residual_seq.shape[:2]) == tuple(x_seq.shape[:2]):
            y = _conv_lif(x_seq, self.weight, self.bias, self.layout, self._conv_kw(),
                          self._cache, residual=residual_seq, stride=self.stride)
            if y is not None:
                return y
        y, b = self._conv_bn(x_seq)
        return fused_bias_if_lif(y, b, residual=residual_seq, layout=self.layout,
                                 **self._neuron_kw())


class FusedConvBN(nn.Module):
    """Conv2d + BN with no neuron, BN folded into the conv: the downsample branch of a
    spiking ResNet block, nn.Sequential(Conv2d 1x1 / stride 2, BatchNorm2d) in the
    reference (zoo/resnet.py:139-142).  The reference keeps it as torch ops; its result is
    the float32 residual of the block's second fused module.  On a bf16 input (spikes)
    with Cin % 8 == 0, Cout % 32 == 0, T in {2, 4, 8} and a 1x1 / padding 0 or 3x3 /
    padding 1 conv of stride 1 or 2 it is one launch of the T-folded kernel with a float32
    result (snnb_conv_f32); otherwise torch's conv in the input's dtype plus the folded
    bias.  Input [T, B, Cin, H, W] (layout as the other modules), output float32
    [T, B, Cout, Ho, Wo] for a bf16 input, else the input's dtype."""

    def __init__(self, conv: nn.Conv2d, bn: nn.BatchNorm2d, *, layout: str = "NCHW"):
        super().__init__()
        assert bn.running_mean is not None
        new_w, new_b = fold_conv_bn(conv.weight.detach(),
                                    conv.bias.detach() if conv.bias is not None else None,
                                    bn.weight.detach(), bn.bias.detach(),
                                    bn.running_mean.detach(), bn.running_var.detach(), bn.eps)
        self.weight = nn.Parameter(new_w)
        self.bias = nn.Parameter(new_b)
        self.stride, self.padding = conv.stride, conv.padding
        self.dilation, self.groups = conv.dilation, conv.groups
        self.layout = layout
        self._cache = {}

    def forward(self, x_seq):
        T, B, Cin = x_seq.shape[:3]
        Cout = self.weight.shape[0]
        if x_seq.dtype == torch.bfloat16 and T in (2, 4, 8) and Cin % 8 == 0 and \
                Cout % 32 == 0 and _fused_conv_ok(self.weight, self.stride, self.padding,
                                                  self.dilation, self.groups, 1.0):
            key = ("khwc", self.weight.data_ptr(), self.weight._version)
            if self._cache.get("key") != key:
                self._cache.clear()
                self._cache["key"], self._cache["w"] = key, KC.weight_khwc(self.weight)
            y = KC.conv_f32(KC._to_frames(x_seq), self._cache["w"],
                            self.bias.detach().float().contiguous(), stride=_pair(self.stride)[0])
            return KC._from_frames(y, torch.float32, self.layout)
        y = _torch_conv(x_seq, self.weight, None, self.stride, self.padding, self.dilation,
                        self.groups, self.layout)
        return y + self.bias.detach().to(y.dtype).view(1, 1, -1, 1, 1)


def tune_convs(model: nn.Module, *inputs, reps: int = 5) -> dict:
    """Opt-in per-layer schedule choice for the fused conv modules of `model` (the module
    path otherwise runs the library's default: T-sequential or T-folded by grid size).  One
    forward of `inputs` records every fused conv module's input; for each, the kernel
    schedules its geometry admits without a split-K workspace -- T-sequential / T-folded
    with each channel block width, and for 3x3 / 1x1 stride-1 convs the two-tile and
    CTA-pair forms -- are timed on that input (device time of graph-replayed calls, the
    lower of two) and the fastest is kept on the module (`module._sched`).  Returns
    {module name: (variant, block_n)}.  Call it before capturing the model in a graph."""
    kinds = (FusedConvNeuron, FusedConvBNNeuron, FusedConvBNAddNeuron)
    seen = {}
    hooks = [m.register_forward_pre_hook(lambda mod, inp: seen.setdefault(mod, inp))
             for m in model.modules() if isinstance(m, kinds)]
    try:
        with torch.no_grad():
            model(*inputs)
    finally:
        for h in hooks:
            h.remove()
    names = {m: n for n, m in model.named_modules()}
    chosen = {}
    for mod, inp in seen.items():
        if getattr(mod, "fold_bn", True) is False or not _fused_conv_ok(
                mod.weight, mod.stride, mod.padding, mod.dilation, mod.groups, mod.v_threshold):
            continue
        T = inp[0].shape[0]
        Cout, Cin, k = mod.weight.shape[0], mod.weight.shape[1], mod.weight.shape[2]
        st = _pair(mod.stride)[0]
        res = len(inp) > 1
        stem = not (k == 3 and st == 1) and k > 1 and Cin < 8      # runs as a 1x1 conv
        general = (st != 1 or k > 3) and not stem
        tfold = T in (2, 4, 8)
        cands = []
        for bn in (32, 64, 128, 256):
            if Cout % bn:
                continue
            if bn <= (64 if res else 128):
                cands.append((1, bn))
            if tfold:
                cands.append((2, bn))
                if not general and not res and bn != 256:
                    cands.append((4, bn))
                if not general and not res and bn >= 64:
                    cands.append((5, bn))
        best, best_ms = None, float("inf")
        with torch.no_grad():
            for c in cands:
                mod._sched = c
                try:
                    ms = min(KC.time_graph(lambda: mod(*inp), reps) for _ in range(2))
                except (RuntimeError, AssertionError):
                    continue
                if ms < best_ms:
                    best, best_ms = c, ms
        mod._sched = best
        if best is not None:
            chosen[names.get(mod, type(mod).__name__)] = best
    return chosen
