"""ResNet / SEW-ResNet block oracle (test infrastructure; see oracle/__init__.py).

Restates, on the CPU in float32, what the reference's fused modules compute for one
conv + BN (+ residual) + neuron step (snn_compiler/nn/modules.py:258-357 and :360-443 with
fused_bias_if_lif, kernels/fused.py:50-114):

    y = conv2d(x, W', stride, padding);  in = (y + b') (+ residual);  LIF / IF over T

W' / b' are the module's folded weights (fold_conv_bn, fused.py:585-599).  The reference
convolves in the input's dtype: on a bf16 input a tensor-core conv (k x k / padding k // 2
for k in {1, 3, 5, 7}, stride 1 or 2, Cin % 8 == 0, Cout % 32 == 0) has bf16 operands, so the
oracle rounds W' to bf16
for it (the products are then exact and only the float32 summation order differs); on a
float32 input the conv is float32 and W' is kept as is.  The block structure follows
snn_compiler/zoo/resnet.py:30-117 and zoo/sew_resnet.py:44-131.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import neurons as ON


def _pair(v):
    return tuple(v) if isinstance(v, (tuple, list)) else (v, v)


def tensor_core_conv(weight, stride, padding, dilation=1, groups=1) -> bool:
    """The geometries the library runs on its tensor-core conv kernels with bf16 operands:
    k x k / padding k // 2 (k in {1, 3, 5, 7}), stride 1 or 2, Cout % 32 == 0, Cin % 8 == 0
    (any Cin, zero padded, off the 3x3 / stride 1 form)."""
    cout, cin = weight.shape[0], weight.shape[1]
    ks = tuple(weight.shape[2:])
    general = ks != (3, 3) or _pair(stride) != (1, 1)     # channels zero padded to 8 there
    return (ks in ((3, 3), (1, 1), (5, 5), (7, 7)) and _pair(stride) in ((1, 1), (2, 2))
            and _pair(padding) == (ks[0] // 2,) * 2 and _pair(dilation) == (1, 1)
            and groups == 1 and (cin % 8 == 0 or general) and cout % 32 == 0)


def conv_bn_neuron(x_seq, weight, bias, *, stride, padding, neuron="lif", tau=2.0, decay=None,
                   decay_input=True, soft_reset=False, v_threshold=1.0, v_reset=0.0,
                   residual=None):
    """x_seq [T, B, Cin, H, W] float32 (CPU) -> (spikes, vpre), both [T, B, Cout, Ho, Wo]."""
    T, B = x_seq.shape[:2]
    w = weight.detach().float().cpu()
    if x_seq.dtype == torch.bfloat16 and tensor_core_conv(w, stride, padding):
        w = w.to(torch.bfloat16).float()
    y = F.conv2d(x_seq.reshape(T * B, *x_seq.shape[2:]).float(), w, None, stride=stride,
                 padding=padding)
    y = y.reshape(T, B, *y.shape[1:])
    C, HW = y.shape[2], y.shape[3] * y.shape[4]
    df, sc = ON.neuron_params(neuron, tau=tau, decay=decay, decay_input=decay_input)
    res = None if residual is None else residual.float().reshape(T, -1).numpy()
    b = bias.detach().float().cpu().numpy()
    r = ON.lif_multistep(y.reshape(T, -1).numpy(), df=df, sc=sc, hard_reset=not soft_reset,
                         v_reset=v_reset, thr=float(v_threshold), bias=b, residual=res, C=C,
                         HW=HW, want_vpre=True)
    shape = y.shape
    return (torch.from_numpy(r["spikes"]).reshape(shape),
            torch.from_numpy(r["vpre"]).reshape(shape))


def conv_bias(x_seq, weight, bias, *, stride, padding):
    """Conv + folded-BN bias with no neuron (a ResNet block's downsample branch,
    snn_compiler/zoo/resnet.py:139-142) in float32: x_seq [T, B, Cin, H, W] (CPU) ->
    [T, B, Cout, Ho, Wo]; bf16-rounded weights on a bf16 input, as conv_bn_neuron."""
    T, B = x_seq.shape[:2]
    w = weight.detach().float().cpu()
    if x_seq.dtype == torch.bfloat16 and tensor_core_conv(w, stride, padding):
        w = w.to(torch.bfloat16).float()
    y = F.conv2d(x_seq.reshape(T * B, *x_seq.shape[2:]).float(), w,
                 bias.detach().float().cpu(), stride=stride, padding=padding)
    return y.reshape(T, B, *y.shape[1:])


def fused_module_oracle(mod, x_seq, residual=None):
    """Oracle of one FusedConvBNNeuron / FusedConvBNAddNeuron (folded BN) on CPU inputs."""
    return conv_bn_neuron(x_seq, mod.weight, mod.bias, stride=mod.stride, padding=mod.padding,
                          neuron=mod.neuron, tau=mod.tau, decay=mod.decay,
                          decay_input=mod.decay_input, soft_reset=mod.soft_reset,
                          v_threshold=mod.v_threshold, v_reset=mod.v_reset, residual=residual)


def sew_connect(out, identity, connect_f):
    """snn_compiler/zoo/sew_resnet.py:28-35."""
    if connect_f == "ADD":
        return out + identity
    if connect_f == "AND":
        return out * identity
    return identity * (1.0 - out)
