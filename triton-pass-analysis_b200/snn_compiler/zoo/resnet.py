"""Spiking ResNet (BasicBlock) on the fused kernels (reference snn_compiler/zoo/resnet.py).

Same classes, constructor arguments and factories as the reference (BasicBlockSNN :30-117,
ResNetSNN :120-213, resnet18_snn / resnet34_snn :216-229).  A block computes

    identity = downsample(x)           (1x1 conv + BN, no neuron) or x
    out      = neuron1(bn1(conv1(x)))
    out      = neuron2(bn2(conv2(out)) + identity)        residual added BEFORE the neuron

``fuse()`` swaps each block's three steps for two fused modules: conv1 -> FusedConvBNNeuron,
conv2 + residual -> FusedConvBNAddNeuron, and the downsample (1x1 / stride 2 conv + BN) for
FusedConvBN.  With BN folded, every 3x3 conv (stride 1 or 2) and 1x1 conv on spike input
(Cin % 8 == 0, Cout % 32 == 0) is one launch of the tcgen05 conv + neuron kernels, the
second one reading the residual in its epilogue, and the downsample one launch of the
T-folded kernel with a float32 result; the 7x7 / stride 2 stem on the real-valued image
runs on the same kernels with both operands as split bf16 terms (float32-faithful).
Unfused (``fused=False``) the network runs torch conv + BN and the K2 neuron modules.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..kernels import conv as KC
from ..nn.fused_layers import FusedConvBN, FusedConvBNAddNeuron, FusedConvBNNeuron
from ..nn.modules import IFNode, LIFNode


def _neuron(neuron, *, tau, decay_input, soft_reset, v_threshold, v_reset, layout):
    if neuron == "if":
        return IFNode(soft_reset=soft_reset, v_threshold=v_threshold, v_reset=v_reset,
                      layout=layout)
    return LIFNode(tau=tau, decay_input=decay_input, soft_reset=soft_reset,
                   v_threshold=v_threshold, v_reset=v_reset, layout=layout)


def node_kwargs(node) -> dict:
    """Constructor arguments of a fused module that reproduce neuron module `node`."""
    kw = dict(soft_reset=node.soft_reset, v_threshold=node.v_threshold,
              v_reset=node.v_reset)
    if isinstance(node, LIFNode):
        kw.update(neuron="lif", tau=node.tau, decay=node.decay, decay_input=node.decay_input)
    else:
        kw.update(neuron="if", decay=node.decay)
    return kw


def frames_op(op, x_seq, layout):
    """Apply a per-frame 2-D op (conv, BN, pool, ...) to [T, B, C, H, W]."""
    T, B = x_seq.shape[:2]
    x4 = x_seq.reshape(T * B, *x_seq.shape[2:])
    if layout == "NHWC":
        x4 = x4.contiguous(memory_format=torch.channels_last)
    y4 = op(x4)
    if layout == "NHWC":
        y4 = y4.contiguous(memory_format=torch.channels_last)
    return y4.view(T, B, *y4.shape[1:])


class BasicBlockSNN(nn.Module):
    expansion = 1

    def __init__(self, in_ch, out_ch, stride=1, downsample=None, *, neuron="lif", tau=2.0,
                 decay_input=True, soft_reset=False, v_threshold=1.0, v_reset=0.0,
                 layout="NCHW"):
        super().__init__()
        nk = dict(tau=tau, decay_input=decay_input, soft_reset=soft_reset,
                  v_threshold=v_threshold, v_reset=v_reset, layout=layout)
        self.conv1 = nn.Conv2d(in_ch, out_ch, 3, stride=stride, padding=1, bias=False)
        self.bn1 = nn.BatchNorm2d(out_ch)
        self.neuron1 = _neuron(neuron, **nk)
        self.conv2 = nn.Conv2d(out_ch, out_ch, 3, stride=1, padding=1, bias=False)
        self.bn2 = nn.BatchNorm2d(out_ch)
        self.neuron2 = _neuron(neuron, **nk)
        self.downsample = downsample          # nn.Sequential(Conv2d 1x1, BatchNorm2d) or None
        self.layout = layout
        self._fused = False

    def fuse(self, *, fold_bn: bool = True):
        """Replace conv1/bn1/neuron1 and conv2/bn2/(+identity)/neuron2 by fused modules
        (eval mode; the downsample branch stays conv + BN)."""
        dev, dt = self.conv1.weight.device, self.conv1.weight.dtype
        self.block1 = FusedConvBNNeuron(self.conv1.eval(), self.bn1.eval(), fold_bn=fold_bn,
                                        layout=self.layout, **node_kwargs(self.neuron1)
                                        ).to(device=dev, dtype=dt)
        self.block2 = FusedConvBNAddNeuron(self.conv2.eval(), self.bn2.eval(), fold_bn=fold_bn,
                                           layout=self.layout, **node_kwargs(self.neuron2)
                                           ).to(device=dev, dtype=dt)
        if self.downsample is not None and fold_bn:
            conv = next(m for m in self.downsample.modules() if isinstance(m, nn.Conv2d))
            bn = next(m for m in self.downsample.modules() if isinstance(m, nn.BatchNorm2d))
            self.downsample = FusedConvBN(conv.eval(), bn.eval(), layout=self.layout
                                          ).to(device=dev, dtype=dt)
        self.conv1 = self.bn1 = self.neuron1 = nn.Identity()
        self.conv2 = self.bn2 = self.neuron2 = nn.Identity()
        self._fused = True
        return self

    def identity(self, x_seq):
        if self.downsample is None:
            return x_seq
        if isinstance(self.downsample, FusedConvBN):
            return self.downsample(x_seq)
        return frames_op(self.downsample, x_seq, self.layout)

    def forward(self, x_seq):
        idn = self.identity(x_seq)
        if self._fused:
            return self.block2(self.block1(x_seq), idn)
        out = self.neuron1(frames_op(lambda z: self.bn1(self.conv1(z)), x_seq, self.layout))
        out = frames_op(lambda z: self.bn2(self.conv2(z)), out, self.layout)
        return self.neuron2(out + idn)


class ResNetSNN(nn.Module):
    """BasicBlock ResNet: 7x7/2 stem conv + BN + neuron, 3x3/2 max-pool, four stages,
    global average pool, linear head (no neuron).  Input [T, B, in_ch, H, W], output
    [T, B, num_classes]."""

    block = BasicBlockSNN

    def __init__(self, layers, num_classes=1000, *, in_ch=3, base_ch=64, neuron="lif", tau=2.0,
                 decay_input=True, soft_reset=False, v_threshold=1.0, v_reset=0.0,
                 layout="NCHW", **block_kw):
        super().__init__()
        self.layout = layout
        self.neuron_kwargs = dict(neuron=neuron, tau=tau, decay_input=decay_input,
                                  soft_reset=soft_reset, v_threshold=v_threshold,
                                  v_reset=v_reset, layout=layout)
        self.block_kw = dict(self.neuron_kwargs, **block_kw)
        self.stem_conv = nn.Conv2d(in_ch, base_ch, 7, stride=2, padding=3, bias=False)
        self.stem_bn = nn.BatchNorm2d(base_ch)
        self.stem_neuron = _neuron(neuron, tau=tau, decay_input=decay_input,
                                   soft_reset=soft_reset, v_threshold=v_threshold,
                                   v_reset=v_reset, layout=layout)
        self.stem_pool = nn.MaxPool2d(3, stride=2, padding=1)
        self.in_ch = base_ch
        self.layer1 = self._make_layer(base_ch, layers[0], 1)
        self.layer2 = self._make_layer(base_ch * 2, layers[1], 2)
        self.layer3 = self._make_layer(base_ch * 4, layers[2], 2)
        self.layer4 = self._make_layer(base_ch * 8, layers[3], 2)
        self.gap = nn.AdaptiveAvgPool2d(1)
        self.fc = nn.Linear(base_ch * 8, num_classes)
        self._fused = False

    def _make_layer(self, out_ch, n_blocks, stride):
        exp = self.block.expansion
        down = None
        if stride != 1 or self.in_ch != out_ch * exp:
            down = nn.Sequential(nn.Conv2d(self.in_ch, out_ch * exp, 1, stride=stride,
                                           bias=False),
                                 nn.BatchNorm2d(out_ch * exp))
        blocks = [self.block(self.in_ch, out_ch, stride=stride, downsample=down,
                             **self.block_kw)]
        self.in_ch = out_ch * exp
        blocks += [self.block(self.in_ch, out_ch, **self.block_kw) for _ in range(1, n_blocks)]
        return nn.Sequential(*blocks)

    def blocks(self):
        return [b for st in (self.layer1, self.layer2, self.layer3, self.layer4) for b in st]

    def fuse(self, *, fold_bn: bool = True):
        for b in self.blocks():
            b.fuse(fold_bn=fold_bn)
        dev, dt = self.stem_conv.weight.device, self.stem_conv.weight.dtype
        self.stem_fused = FusedConvBNNeuron(self.stem_conv.eval(), self.stem_bn.eval(),
                                            fold_bn=fold_bn, layout=self.layout,
                                            **node_kwargs(self.stem_neuron)
                                            ).to(device=dev, dtype=dt)
        self.stem_conv = self.stem_bn = self.stem_neuron = nn.Identity()
        self._fused = True
        return self

    def stem(self, x_seq):
        if self._fused:
            x = self.stem_fused(x_seq)
            xf = x.permute(0, 1, 3, 4, 2)
            pk = _square_pool(self.stem_pool)
            if pk is not None and x.is_cuda and x.dtype == torch.bfloat16 and \
                    xf.is_contiguous() and x.shape[2] % 8 == 0:
                # NHWC bf16 spikes: the pool (an OR of each window) on snnb_maxpool_nhwc
                return KC.maxpool_nhwc(xf, *pk).permute(0, 1, 4, 2, 3)
        else:
            x = self.stem_neuron(frames_op(lambda z: self.stem_bn(self.stem_conv(z)), x_seq,
                                           self.layout))
        return frames_op(self.stem_pool, x, self.layout)

    def head(self, x_seq):
        T, B = x_seq.shape[:2]
        f = frames_op(self.gap, x_seq, "NCHW").reshape(T * B, -1)
        return self.fc(f.to(self.fc.weight.dtype)).view(T, B, -1)

    def forward(self, x_seq):
        x = self.stem(x_seq)
        for b in self.blocks():
            x = b(x)
        return self.head(x)


def _square_pool(p: nn.MaxPool2d):
    """(k, stride, padding) of a square, undilated, floor-mode max-pool, else None."""
    def one(v):
        v = tuple(v) if isinstance(v, (tuple, list)) else (v, v)
        return v[0] if v[0] == v[1] else None
    k, st, pad, dil = one(p.kernel_size), one(p.stride), one(p.padding), one(p.dilation)
    if None in (k, st, pad) or dil != 1 or p.ceil_mode or pad >= k:
        return None
    return k, st, pad


def init_bn(model: nn.Module):
    """Non-trivial eval-mode BN statistics (the reference's _init_bn, resnet.py:200-206)."""
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, nn.BatchNorm2d):
                m.running_mean.copy_(torch.randn_like(m.running_mean) * 0.1)
                m.running_var.copy_(torch.rand_like(m.running_var) + 0.5)
                m.weight.copy_(torch.rand_like(m.weight) + 0.5)
                m.bias.copy_(torch.randn_like(m.bias) * 0.1)


def _build(cls, layers, *, fused=False, fold_bn=True, init_bn_stats=True, **kw):
    m = cls(layers, **kw)
    if init_bn_stats:
        init_bn(m)
    if fused:
        m.eval().fuse(fold_bn=fold_bn)
    return m


def resnet18_snn(*, fused=False, fold_bn=True, init_bn=True, **kw):
    return _build(ResNetSNN, [2, 2, 2, 2], fused=fused, fold_bn=fold_bn, init_bn_stats=init_bn,
                  **kw)


def resnet34_snn(*, fused=False, fold_bn=True, init_bn=True, **kw):
    return _build(ResNetSNN, [3, 4, 6, 3], fused=fused, fold_bn=fold_bn, init_bn_stats=init_bn,
                  **kw)
