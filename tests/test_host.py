"""Host-side checks that need no GPU."""
import torch

from oracle import params as OP


def test_product_synthetic_weights_match_oracle_draws():
    """The engine's seeded VGG16 weights are bit-identical to the oracle's."""
    from snn_compiler.zoo.vgg import random_vgg_params
    a = random_vgg_params(1)
    b = OP.vgg16_params(1)
    assert len(a["convs"]) == len(b["convs"]) == 13
    for x, y in zip(a["convs"], b["convs"]):
        for k in ("w", "b", "gamma", "beta", "mean", "var"):
            assert torch.equal(x[k], y[k]), k
        assert x["pool"] == y["pool"]
    for x, y in zip(a["fcs"], b["fcs"]):
        assert torch.equal(x["w"], y["w"]) and torch.equal(x["b"], y["b"])


def test_fold_matches_oracle_fold():
    from snn_compiler.kernels.fused import fold_conv_bn
    from oracle import vgg as OV
    c = OP.vgg16_params(1)["convs"][3]
    w1, b1 = fold_conv_bn(c["w"], c["b"], c["gamma"], c["beta"], c["mean"], c["var"], c["eps"])
    w2, b2 = OV.fold_conv_bn(c["w"], c["b"], c["gamma"], c["beta"], c["mean"], c["var"], c["eps"])
    assert torch.equal(w1, w2) and torch.equal(b1, b2)


def test_vggsnn_module_structure_and_params():
    from snn_compiler.zoo.vgg import vgg16_snn
    m = vgg16_snn(num_classes=10, fc_in=512)
    P = m.params_dict()
    assert len(P["convs"]) == 13 and sum(c["pool"] for c in P["convs"]) == 5
    assert [tuple(f["w"].shape) for f in P["fcs"]] == [(4096, 512), (4096, 4096), (10, 4096)]


def test_fused_modules_construct_like_reference():
    """FusedConv(BN)(Add)Neuron / FusedLinearNeuron keep the reference's constructor
    arguments and parameter layout (snn_compiler/nn/modules.py:160-443); construction
    needs no GPU."""
    import torch.nn as nn
    from oracle import vgg as OV
    from snn_compiler.nn import (FusedConvBNAddNeuron, FusedConvBNNeuron, FusedConvNeuron,
                                 FusedLinearNeuron)
    conv, bn = nn.Conv2d(8, 16, 3, padding=1), nn.BatchNorm2d(16).eval()
    with torch.no_grad():
        bn.running_mean.uniform_(-0.1, 0.1)
        bn.running_var.uniform_(0.5, 1.5)
    m = FusedConvBNNeuron(conv, bn, neuron="lif", tau=2.0, v_threshold=0.7)
    w, b = OV.fold_conv_bn(conv.weight.detach(), conv.bias.detach(), bn.weight.detach(),
                           bn.bias.detach(), bn.running_mean, bn.running_var, bn.eps)
    assert torch.equal(m.weight.detach(), w) and torch.equal(m.bias.detach(), b)
    assert m.v_threshold == 0.7 and m.fold_bn and m.layout == "NCHW"
    u = FusedConvBNNeuron(conv, bn, fold_bn=False)
    assert u.bias is None and torch.equal(u.bn_var, bn.running_var)
    assert set(dict(u.named_parameters())) == {"weight", "conv_bias"}
    a = FusedConvBNAddNeuron(conv, bn, v_threshold=torch.ones(16))
    assert a.v_threshold.shape == (16,)
    c = FusedConvNeuron(8, 16, 3, stride=2, padding=1, bias=False)
    assert c.bias is None and c.stride == (2, 2)
    lin = FusedLinearNeuron(32, 64)
    assert lin.weight.shape == (64, 32) and lin.bias.shape == (64,)


def test_chunked_driver_passes_state_and_concatenates():
    """run_chunked / ChunkedForward (reference snn_compiler/nn/chunked.py:33-79): chunks of
    chunk_t steps, the state of one chunk handed to the next, outputs concatenated."""
    import torch.nn as nn
    from snn_compiler.nn import ChunkedForward, run_chunked

    class Acc(nn.Module):                  # y_t = running sum over all steps so far
        def forward(self, x):
            return torch.cumsum(x, 0)

        def forward_chunked(self, x, state):
            s0 = torch.zeros_like(x[0]) if state is None else state["s"]
            y = torch.cumsum(x, 0) + s0
            return y, {"s": y[-1]}

    x = torch.randn(11, 3, 5)
    full = torch.cumsum(x, 0)
    for chunk in (1, 4, 5, 11, 16):
        assert torch.allclose(ChunkedForward(Acc(), chunk_t=chunk)(x), full, atol=1e-5)
    calls = []
    run_chunked(lambda xc, st: (calls.append(xc.shape[0]) or xc, st), x, chunk_t=4)
    assert calls == [4, 4, 3]
    plain = nn.Identity()
    assert torch.equal(ChunkedForward(plain, chunk_t=2)(x), x)     # no forward_chunked


def test_cuba_eif_modules_construct_like_reference():
    """CubaLIFNode / EIFNode keep the reference's constructor arguments
    (snn_compiler/nn/modules.py:88-154)."""
    from snn_compiler.nn import CubaLIFNode, EIFNode
    c = CubaLIFNode(tau_syn=3.0, decay_mem=0.8, v_threshold=torch.ones(4))
    assert c.tau_syn == 3.0 and c.decay_mem == 0.8 and c.v_threshold.shape == (4,)
    e = EIFNode(delta_T=0.5, v_rh=0.2, soft_reset=True)
    assert e.delta_T == 0.5 and e.v_rh == 0.2 and e.soft_reset and e.v_threshold == 1.0


def test_resnet_zoo_builds_and_fuses_on_cpu():
    """ResNetSNN / SEWResNetSNN keep the reference's structure (zoo/resnet.py:120-213,
    zoo/sew_resnet.py:134-199): fuse() swaps every block for fused modules -- standard
    blocks end in FusedConvBNAddNeuron (residual before the neuron), SEW blocks in
    FusedConvBNNeuron plus the element-wise connection (after the neuron)."""
    from snn_compiler.nn import FusedConvBNAddNeuron, FusedConvBNNeuron
    from snn_compiler.zoo import resnet18_snn, resnet34_snn, sew_resnet18_snn
    m = resnet18_snn(num_classes=10, base_ch=32, fused=True)
    assert len(m.blocks()) == 8 and isinstance(m.stem_fused, FusedConvBNNeuron)
    assert all(isinstance(b.block2, FusedConvBNAddNeuron) for b in m.blocks())
    assert m.layer2[0].downsample is not None and m.layer1[0].downsample is None
    assert len(resnet34_snn(num_classes=10, base_ch=32).blocks()) == 16
    s = sew_resnet18_snn(num_classes=10, base_ch=32, connect_f="and", fused=True)
    blk = s.layer3[0]
    assert blk.connect_f == "AND" and isinstance(blk.block2, FusedConvBNNeuron)
    assert isinstance(blk.ds_block, FusedConvBNNeuron) and s.layer1[1].ds_block is None
    from snn_compiler.zoo.sew_resnet import sew_connect
    o, i = torch.tensor([0., 1., 1.]), torch.tensor([1., 1., 0.])
    assert sew_connect(o, i, "IAND").tolist() == [1.0, 0.0, 0.0]


def test_dense_conv_weight_equals_padded_conv():
    """A 3x3 / padding-1 conv on 1x1, 1x2, 2x1 and 2x2 images equals the GEMM with
    dense_conv_weight (NHWC flattening on both sides), bias repeated per pixel."""
    import torch.nn.functional as F
    from snn_compiler.kernels import conv as KC
    g = torch.Generator().manual_seed(5)
    for H, W in ((1, 1), (1, 2), (2, 1), (2, 2)):
        Cin, Cout, N = 8, 12, 3
        w = torch.randn(Cout, Cin, 3, 3, generator=g, dtype=torch.float64)
        b = torch.randn(Cout, generator=g, dtype=torch.float64)
        x = torch.randn(N, Cin, H, W, generator=g, dtype=torch.float64)
        ref = F.conv2d(x, w, b, padding=1).permute(0, 2, 3, 1).reshape(N, -1)
        wd = KC.dense_conv_weight(w.permute(0, 2, 3, 1).contiguous(), H, W)
        assert wd.shape == (H * W * Cout, H * W * Cin)
        got = x.permute(0, 2, 3, 1).reshape(N, -1) @ wd.t() + KC.dense_conv_bias(b, H, W).double()
        assert torch.allclose(got, ref, atol=1e-10), (H, W)


def test_split_terms_represent_float32_and_six_products_are_float32_accurate():
    """Host side of the float32-faithful tensor-core path: three bf16 terms reproduce a
    float32 value to 2^-24, and the six kept products of activation and weight terms give
    each x * w to within 2^-22 relative (the dropped three are below 2^-23)."""
    import torch
    from snn_compiler.kernels import conv as KC
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, generator=g) * torch.exp(torch.randn(4096, generator=g) * 5)
    w = torch.randn(4096, generator=g) * torch.exp(torch.randn(4096, generator=g) * 5)
    xh, xm, xl = (t.double() for t in KC.split_terms_host(x))
    wh, wm, wl = (t.double() for t in KC.split_terms_host(w))
    assert ((xh + xm + xl - x.double()).abs() <= 2.0 ** -24 * x.double().abs()).all()
    terms = {"hi": (xh, wh), "mid": (xm, wm), "lo": (xl, wl)}
    prod = sum(terms[a][0] * terms[b][1] for a, b in zip(KC.SPLIT_ACT, KC.SPLIT_WGT))
    exact = x.double() * w.double()
    assert ((prod - exact).abs() <= 2.0 ** -22 * exact.abs()).all()
    # the weight groups line up with the activation groups channel by channel
    wk = KC.split_weight_khwc(torch.randn(8, 6, 3, 3, generator=g))
    assert wk.shape == (8, 3, 3, 6 * KC.split_width(6)) and wk.dtype == torch.bfloat16
    assert (wk[..., 6:8] == 0).all()
