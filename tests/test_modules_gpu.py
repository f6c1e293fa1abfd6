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
    # a float32 input convolves in float32 (both operands as three bf16 terms on the
    # tensor cores): the oracle keeps the float32 folded weights
    s, _, vpre = OV.conv_bn_lif_pool(x, w, b, pool=False, want_vpre=True)
    assert y.cpu().sum() > 0
    flip_check(y.cpu(), s, vpre)
    # a bf16 input runs the bf16 kernel: bf16 weights, as the reference's bf16 mode
    yb = m(xd.to(torch.bfloat16))
    assert yb.dtype == torch.bfloat16
    sb, _, vb = OV.conv_bn_lif_pool(x, OV.bf16_round(w), b, pool=False, want_vpre=True)
    flip_check(yb.float().cpu(), sb, vb)


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
    # the residual form of a 3x3 / s1 / p1 conv runs on the tensor cores; a float32 input
    # convolves float32-faithfully (split terms), so the oracle keeps float32 weights
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
    w = m.weight.detach().cpu()                    # float32 input: float32 linear
    z = torch.nn.functional.linear(x.reshape(T * B, K), w).reshape(T, B, N)
    s, vpre = OV.lif_seq(z, m.bias.detach().cpu(), want_vpre=True)
    assert y.sum() > 0
    flip_check(y, s, vpre)
    # bf16 input: the bf16 kernel, against bf16-rounded weights (the reference's bf16 mode)
    yb = m(x.to(torch.bfloat16).to(DEV)).float().cpu()
    zb = torch.nn.functional.linear(x.reshape(T * B, K), OV.bf16_round(w)).reshape(T, B, N)
    sb, vb = OV.lif_seq(zb, m.bias.detach().cpu(), want_vpre=True)
    flip_check(yb, sb, vb)


def test_real_valued_float32_input_is_convolved_in_float32():
    """A float32 module on a real-valued float32 input (Cin = 64, e.g. a second encoder
    layer or a membrane-shortcut block) convolves in float32 as the reference's F.conv2d
    does: the fused tcgen05 kernel carries both operands as three bf16 terms.  Membrane
    potentials agree with the float32 oracle to float32 summation order (1e-5 here, against
    ~1e-3 for bf16-rounded operands), and spikes flip only within 1e-4 of the threshold."""
    from snn_compiler.kernels import conv as KC
    from snn_compiler.nn import FusedConvBNNeuron, FusedLinearNeuron
    T, B, Cin, Cout, H = 4, 2, 64, 64, 16
    conv, bn = _conv_bn(Cin, Cout, 11)
    m = FusedConvBNNeuron(conv, bn, **LIF).to(DEV)
    x = torch.randn(T, B, Cin, H, H, generator=OP.gen(12)) * 0.7 + 0.3
    y = m(x.to(DEV)).cpu()
    assert "w" in m._cache and m._cache["key"][0] == "split"
    w, b = OV.fold_conv_bn(conv.weight.detach(), conv.bias.detach(), bn.weight.detach(),
                           bn.bias.detach(), bn.running_mean, bn.running_var, bn.eps)
    s, _, vpre = OV.conv_bn_lif_pool(x, w, b, pool=False, want_vpre=True)
    assert y.sum() > 0
    flip_check(y, s, vpre)
    # the pre-activation itself, through the GEMM form with a float32 output: the split
    # operands' six products summed on the tensor cores against the exact (float64) sum,
    # beside the bf16-rounded operands' error
    xl0 = torch.randn(T, 32, 384, generator=OP.gen(15))
    wl0 = torch.randn(96, 384, generator=OP.gen(16)) * 0.05
    bl0 = torch.zeros(96)
    ysplit = KC.linear_f32(KC.split_activations(xl0.to(DEV)), KC.split_weight_rows(wl0).to(DEV),
                           bl0.to(DEV)).cpu().double()
    exact = (xl0.double().reshape(-1, 384) @ wl0.double().t()).reshape(T, 32, 96)
    ybf = (xl0.bfloat16().double().reshape(-1, 384) @ wl0.bfloat16().double().t()).reshape(T, 32, 96)
    err = (ysplit - exact).abs().max().item()
    assert err <= 1e-5 * exact.abs().max().item(), err
    assert err * 20 < (ybf - exact).abs().max().item()
    # float16 input: exact in float32, same float32-faithful path
    y16 = m(x.to(torch.float16).to(DEV))
    assert y16.dtype == torch.float16
    s16, _, v16 = OV.conv_bn_lif_pool(x.half().float(), w, b, pool=False, want_vpre=True)
    flip_check(y16.float().cpu(), s16, v16)
    # linear on a real-valued float32 input
    K, N = 384, 256
    torch.manual_seed(2)
    ml = FusedLinearNeuron(K, N, **LIF)
    with torch.no_grad():
        ml.weight.mul_(3.0)
    ml = ml.to(DEV)
    xl = torch.randn(T, 8, K, generator=OP.gen(13))
    yl = ml(xl.to(DEV)).cpu()
    zl = torch.nn.functional.linear(xl.reshape(T * 8, K), ml.weight.detach().cpu()).reshape(T, 8, N)
    sl, vl = OV.lif_seq(zl, ml.bias.detach().cpu(), want_vpre=True)
    assert yl.sum() > 0
    flip_check(yl, sl, vl)


def test_split_terms_device_matches_host_and_sums_to_the_value():
    from snn_compiler.kernels import conv as KC
    g = OP.gen(14)
    x = torch.randn(1000, 20, generator=g) * torch.exp(torch.randn(1000, 20, generator=g) * 8)
    x[0, :5] = torch.tensor([0.0, -0.0, 1e-40, 3.4e38, -1.5])
    d = KC.split_activations(x.to(DEV)).cpu()
    Cp = KC.split_width(20)
    h, mi, lo = KC.split_terms_host(x)
    for gi, name in enumerate(KC.SPLIT_ACT):
        ref = {"hi": h, "mid": mi, "lo": lo}[name]
        assert torch.equal(d[:, gi * Cp: gi * Cp + 20].view(torch.int16), ref.view(torch.int16))
        assert (d[:, gi * Cp + 20: (gi + 1) * Cp] == 0).all()
    # within 2^-24 of the value, or of the bf16 subnormal spacing 2^-133 for values so small
    # that the terms fall below bf16's normal range
    tot = h.double() + mi.double() + lo.double()
    fin = torch.isfinite(x)
    assert ((tot - x.double()).abs()[fin] <=
            2.0 ** -24 * x.double().abs()[fin] + 2.0 ** -133).all()
