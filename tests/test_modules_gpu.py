"""The reference's fused conv / linear nn modules (snn_compiler/nn/modules.py:160-443) on the
B200 kernels vs the oracle: same constructors, same forward signatures, same layouts."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import neurons as ON
from oracle import params as OP
from oracle import vgg as OV
from test_conv_gpu import flip_check

pytestmark = pytest.mark.gpu
DEV = "cuda"
LIF = dict(neuron="lif", tau=2.0, v_threshold=1.0)


def _conv_bn(Cin, Cout, seed, stride=1, bias=True):
    g = OP.gen(seed)
    conv = nn.Conv2d(Cin, Cout, 3, stride=stride, padding=1, bias=bias)
    bn = nn.BatchNorm2d(Cout)
    with torch.no_grad():
        conv.weight.copy_(torch.randn(conv.weight.shape, generator=g) * (2.0 / (9 * Cin)) ** 0.5)
        if bias:
            conv.bias.copy_(torch.randn(Cout, generator=g) * 0.1)
        bn.weight.copy_(torch.rand(Cout, generator=g) * 0.4 + 0.8)
        bn.bias.copy_(torch.rand(Cout, generator=g) * 0.6 + 0.4)
        bn.running_mean.copy_(torch.randn(Cout, generator=g) * 0.1)
        bn.running_var.copy_(torch.rand(Cout, generator=g) + 0.5)
    return conv.eval(), bn.eval()


def _oracle_lif(y, bias, residual=None):
    """LIF over y [T, B, C, H, W] (NCHW memory order) with per-channel bias."""
    T = y.shape[0]
    C, HW = y.shape[2], int(np.prod(y.shape[3:]))
    df, sc = ON.neuron_params("lif", tau=2.0)
    r = ON.lif_multistep(y.reshape(T, -1).contiguous().numpy(), df=df, sc=sc, thr=1.0,
                         bias=None if bias is None else bias.numpy(), C=C, HW=HW,
                         residual=None if residual is None else
                         residual.reshape(T, -1).contiguous().numpy(), want_vpre=True)
    return (torch.from_numpy(r["spikes"]).reshape(y.shape),
            torch.from_numpy(r["vpre"]).reshape(y.shape))


@pytest.mark.parametrize("layout", ["NCHW", "NHWC"])
def test_fused_conv_bn_neuron_folded_runs_the_fused_kernel(layout):
    from snn_compiler.nn import FusedConvBNNeuron
    T, B, Cin, Cout, H = 4, 2, 64, 64, 16
    conv, bn = _conv_bn(Cin, Cout, 1)
    m = FusedConvBNNeuron(conv, bn, layout=layout, **LIF).to(DEV)
    x = (torch.rand(T, B, Cin, H, H, generator=OP.gen(2)) < 0.2).float()
    xd = x.to(DEV)
    if layout == "NHWC":
        xd = xd.reshape(T * B, Cin, H, H).contiguous(memory_format=torch.channels_last) \
               .view(T, B, Cin, H, H)
    y = m(xd)
    assert y.shape == (T, B, Cout, H, H) and y.dtype == torch.float32
    w, b = OV.fold_conv_bn(conv.weight.detach(), conv.bias.detach(), bn.weight.detach(),
                           bn.bias.detach(), bn.running_mean, bn.running_var, bn.eps)
    s, _, vpre = OV.conv_bn_lif_pool(x, OV.bf16_round(w), b, pool=False, want_vpre=True)
    assert y.cpu().sum() > 0
    flip_check(y.cpu(), s, vpre)


def test_fused_conv_bn_neuron_unfolded_keeps_conv_and_bn_separate():
    from snn_compiler.nn import FusedConvBNNeuron
    T, B, Cin, Cout, H = 3, 2, 16, 24, 8
    conv, bn = _conv_bn(Cin, Cout, 3)
    m = FusedConvBNNeuron(conv, bn, fold_bn=False, **LIF).to(DEV)
    assert m.bias is None and m.bn_mean.shape == (Cout,)
    x = (torch.rand(T, B, Cin, H, H, generator=OP.gen(4)) < 0.3).float()
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        y = m(x.to(DEV)).cpu()
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    with torch.no_grad():
        z = bn(conv(x.reshape(T * B, Cin, H, H))).reshape(T, B, Cout, H, H)
    s, vpre = _oracle_lif(z, None)
    flip_check(y, s, vpre)


def test_fused_conv_bn_neuron_image_layer_uses_f32_kernel():
    from snn_compiler.nn import FusedConvBNNeuron
    T, B, H = 4, 2, 32
    conv, bn = _conv_bn(3, 64, 5)
    m = FusedConvBNNeuron(conv, bn, **LIF).to(DEV)
    img = torch.rand(T, B, 3, H, H, generator=OP.gen(6))
    y = m(img.to(DEV)).cpu()
    w, b = OV.fold_conv_bn(conv.weight.detach(), conv.bias.detach(), bn.weight.detach(),
                           bn.bias.detach(), bn.running_mean, bn.running_var, bn.eps)
    s, _, vpre = OV.conv_bn_lif_pool(img, w, b, pool=False, want_vpre=True)
    flip_check(y, s, vpre)


def test_fused_conv_neuron_other_geometry_and_residual_form():
    from snn_compiler.nn import FusedConvBNAddNeuron, FusedConvNeuron
    T, B, Cin, Cout, H = 2, 2, 16, 32, 8
    torch.manual_seed(0)
    m = FusedConvNeuron(Cin, Cout, 3, stride=2, padding=1, **LIF).to(DEV)
    x = (torch.rand(T, B, Cin, H, H, generator=OP.gen(7)) < 0.3).float()
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        y = m(x.to(DEV)).cpu()
        conv, bn = _conv_bn(Cin, Cout, 8)
        ma = FusedConvBNAddNeuron(conv, bn, **LIF).to(DEV)
        r = torch.rand(T, B, Cout, H, H, generator=OP.gen(9))
        ya = ma(x.to(DEV), r.to(DEV)).cpu()
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    with torch.no_grad():
        z = torch.nn.functional.conv2d(x.reshape(T * B, Cin, H, H), m.weight.detach().cpu(),
                                       None, 2, 1).reshape(T, B, Cout, H // 2, H // 2)
    s, vpre = _oracle_lif(z, m.bias.detach().cpu())
    flip_check(y, s, vpre)
    w, b = OV.fold_conv_bn(conv.weight.detach(), conv.bias.detach(), bn.weight.detach(),
                           bn.bias.detach(), bn.running_mean, bn.running_var, bn.eps)
    # the residual form of a 3x3 / s1 / p1 conv runs on the tensor cores: bf16 weights
    w = w.to(torch.bfloat16).float()
    with torch.no_grad():
        za = torch.nn.functional.conv2d(x.reshape(T * B, Cin, H, H), w, None, 1, 1) \
                  .reshape(T, B, Cout, H, H)
    sa, va = _oracle_lif(za, b, residual=r)
    flip_check(ya, sa, va)


def test_fused_linear_neuron_against_oracle():
    from snn_compiler.nn import FusedLinearNeuron
    T, B, K, N = 4, 16, 512, 256
    torch.manual_seed(1)
    m = FusedLinearNeuron(K, N, **LIF)
    with torch.no_grad():
        m.weight.mul_(4.0)
        m.bias.add_(0.5)
    m = m.to(DEV)
    x = (torch.rand(T, B, K, generator=OP.gen(10)) < 0.2).float()
    y = m(x.to(DEV)).cpu()
    w = OV.bf16_round(m.weight.detach().cpu())
    z = torch.nn.functional.linear(x.reshape(T * B, K), w).reshape(T, B, N)
    s, vpre = OV.lif_seq(z, m.bias.detach().cpu(), want_vpre=True)
    assert y.sum() > 0
    flip_check(y, s, vpre)
