"""SEW-ResNet (spike-element-wise residual) on the fused kernels
(reference snn_compiler/zoo/sew_resnet.py).

Same classes and factories as the reference (SEWBasicBlockSNN :44-131, SEWResNetSNN
:134-199, sew_resnet18_snn / sew_resnet34_snn :202-210).  Unlike the standard block the
residual joins AFTER the second neuron, and the downsample branch has its own neuron:

    out      = neuron2(bn2(conv2(neuron1(bn1(conv1(x))))))
    identity = neuron_d(bn_d(conv_d(x)))  or x
    y        = out + identity (ADD) | out * identity (AND) | identity * (1 - out) (IAND)

so a block fuses into two (three with downsample) FusedConvBNNeuron modules followed by
the element-wise connection -- never into FusedConvBNAddNeuron, whose residual enters
before the neuron.
"""
from __future__ import annotations

import torch.nn as nn

from ..nn.fused_layers import FusedConvBNNeuron
from .resnet import ResNetSNN, _build, _neuron, frames_op, node_kwargs


def sew_connect(out, identity, connect_f: str):
    if connect_f == "ADD":
        return out + identity
    if connect_f == "AND":
        return out * identity
    if connect_f == "IAND":
        return identity * (1.0 - out)
    raise ValueError(f"unknown connect_f: {connect_f!r} (expected ADD/AND/IAND)")


class SEWBasicBlockSNN(nn.Module):
    expansion = 1

    def __init__(self, in_ch, out_ch, stride=1, downsample=None, *, connect_f="ADD",
                 neuron="if", tau=2.0, decay_input=True, soft_reset=False, v_threshold=1.0,
                 v_reset=0.0, layout="NCHW"):
        super().__init__()
        self.connect_f = connect_f.upper()
        nk = dict(tau=tau, decay_input=decay_input, soft_reset=soft_reset,
                  v_threshold=v_threshold, v_reset=v_reset, layout=layout)
        self.conv1 = nn.Conv2d(in_ch, out_ch, 3, stride=stride, padding=1, bias=False)
        self.bn1 = nn.BatchNorm2d(out_ch)
        self.neuron1 = _neuron(neuron, **nk)
        self.conv2 = nn.Conv2d(out_ch, out_ch, 3, stride=1, padding=1, bias=False)
        self.bn2 = nn.BatchNorm2d(out_ch)
        self.neuron2 = _neuron(neuron, **nk)
        self.downsample = downsample
        self.downsample_neuron = _neuron(neuron, **nk) if downsample is not None else None
        self.layout = layout
        self._fused = False

    def fuse(self, *, fold_bn: bool = True):
        dev, dt = self.conv1.weight.device, self.conv1.weight.dtype

        def fused(conv, bn, node):
            return FusedConvBNNeuron(conv.eval(), bn.eval(), fold_bn=fold_bn, layout=self.layout,
                                     **node_kwargs(node)).to(device=dev, dtype=dt)

        self.block1 = fused(self.conv1, self.bn1, self.neuron1)
        self.block2 = fused(self.conv2, self.bn2, self.neuron2)
        self.ds_block = None
        if self.downsample is not None:
            conv = next(m for m in self.downsample.modules() if isinstance(m, nn.Conv2d))
            bn = next(m for m in self.downsample.modules() if isinstance(m, nn.BatchNorm2d))
            self.ds_block = fused(conv, bn, self.downsample_neuron)
        self.conv1 = self.bn1 = self.neuron1 = nn.Identity()
        self.conv2 = self.bn2 = self.neuron2 = nn.Identity()
        self.downsample = self.downsample_neuron = None
        self._fused = True
        return self

    def forward(self, x_seq):
        if self._fused:
            out = self.block2(self.block1(x_seq))
            idn = x_seq if self.ds_block is None else self.ds_block(x_seq)
            return sew_connect(out, idn, self.connect_f)
        if self.downsample is None:
            idn = x_seq
        else:
            idn = self.downsample_neuron(frames_op(self.downsample, x_seq, self.layout))
        out = self.neuron1(frames_op(lambda z: self.bn1(self.conv1(z)), x_seq, self.layout))
        out = self.neuron2(frames_op(lambda z: self.bn2(self.conv2(z)), out, self.layout))
        return sew_connect(out, idn, self.connect_f)


class SEWResNetSNN(ResNetSNN):
    """SEW-ResNet skeleton: ResNetSNN's stem, stages and head with SEW blocks."""

    block = SEWBasicBlockSNN

    def __init__(self, layers, num_classes=1000, *, in_ch=3, base_ch=64, connect_f="ADD",
                 neuron="if", tau=2.0, decay_input=True, soft_reset=False, v_threshold=1.0,
                 v_reset=0.0, layout="NCHW"):
        self.connect_f = connect_f.upper()
        super().__init__(layers, num_classes, in_ch=in_ch, base_ch=base_ch, neuron=neuron,
                         tau=tau, decay_input=decay_input, soft_reset=soft_reset,
                         v_threshold=v_threshold, v_reset=v_reset, layout=layout,
                         connect_f=self.connect_f)


def sew_resnet18_snn(*, fused=False, fold_bn=True, init_bn=True, **kw):
    return _build(SEWResNetSNN, [2, 2, 2, 2], fused=fused, fold_bn=fold_bn,
                  init_bn_stats=init_bn, **kw)


def sew_resnet34_snn(*, fused=False, fold_bn=True, init_bn=True, **kw):
    return _build(SEWResNetSNN, [3, 4, 6, 3], fused=fused, fold_bn=fold_bn,
                  init_bn_stats=init_bn, **kw)
