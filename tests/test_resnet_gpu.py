"""ResNet / SEW-ResNet on the fused kernels: every fused conv + BN (+ residual) + neuron
module checked against the CPU oracle on the same (teacher-forced) inputs -- the
tensor-core residual epilogue included -- and the full network run end to end."""
import pytest
import torch

from oracle import resnet as OR

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _build(kind, connect="ADD", neuron="lif"):
    from snn_compiler.zoo import resnet18_snn, sew_resnet18_snn
    torch.manual_seed(7)
    if kind == "resnet":
        m = resnet18_snn(num_classes=10, base_ch=32, neuron=neuron)
        scale, shift = 3.0, 0.5
    else:
        m = sew_resnet18_snn(num_classes=10, base_ch=32, connect_f=connect, neuron=neuron)
        scale, shift = 2.5, 0.0
    with torch.no_grad():      # livelier than the default init: every layer spikes
        for mod in m.modules():
            if isinstance(mod, torch.nn.Conv2d):
                mod.weight.mul_(scale)
            if isinstance(mod, torch.nn.BatchNorm2d):
                mod.bias.add_(shift)
    return m.eval().fuse().to(DEV)


def _check_modules(m, img):
    from snn_compiler.nn import FusedConvBNAddNeuron, FusedConvBNNeuron
    rec = []
    hooks = [mod.register_forward_hook(
        lambda mod, inp, out: rec.append((mod, [i.detach().cpu() for i in inp],
                                          out.detach().float().cpu())))
        for mod in m.modules() if isinstance(mod, (FusedConvBNNeuron, FusedConvBNAddNeuron))]
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False          # fp32 torch convs on the fallback path
    try:
        with torch.no_grad():
            y = m(img)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
        for h in hooks:
            h.remove()
    assert y.shape == (img.shape[0], img.shape[1], 10) and torch.isfinite(y).all()
    n_tc = n_res = 0
    for mod, inp, out in rec:
        res = inp[1] if len(inp) > 1 else None
        ref, vpre = OR.fused_module_oracle(mod, inp[0], residual=res)
        bad = out != ref
        near = (vpre - float(mod.v_threshold)).abs() < 1e-4
        assert not (bad & ~near).any(), (type(mod).__name__, int((bad & ~near).sum()))
        assert bad.float().mean() <= 1e-3
        assert ref.sum() > 0, "no spikes: degenerate case"
        if OR.tensor_core_conv(mod.weight, mod.stride, mod.padding):
            assert "w" in mod._cache          # ran on the tcgen05 kernel
            n_tc += 1
            n_res += res is not None
    return n_tc, n_res


def test_resnet18_fused_modules_match_oracle():
    m = _build("resnet")
    g = torch.Generator().manual_seed(3)
    img = torch.rand(2, 3, 32, 32, generator=g).unsqueeze(0).expand(4, 2, 3, 32, 32)
    n_tc, n_res = _check_modules(m, img.contiguous().to(DEV))
    assert n_tc >= 6 and n_res >= 4          # residual epilogue with spike and float identity


@pytest.mark.parametrize("connect", ["ADD", "IAND"])
def test_sew_resnet18_fused_modules_match_oracle(connect):
    m = _build("sew", connect, neuron="if")
    g = torch.Generator().manual_seed(4)
    img = torch.rand(2, 3, 32, 32, generator=g).unsqueeze(0).expand(4, 2, 3, 32, 32)
    n_tc, n_res = _check_modules(m, img.contiguous().to(DEV))
    assert n_tc >= 6 and n_res == 0


@pytest.mark.parametrize("res_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("variant,block_n,splits", [(0, 0, 1), (1, 64, 1), (1, 32, 1),
                                                    (2, 128, 1), (2, 64, 1), (2, 64, 2),
                                                    (2, 128, 3), (6, 128, 2), (6, 128, 4)])
def test_conv3x3_residual_epilogue_against_oracle(variant, block_n, splits, res_dtype):
    """The residual input in every kernel variant that takes one (T-sequential, T-folded,
    split-K finish, cluster split-K) against the oracle."""
    from snn_compiler.kernels import conv as C
    T, B, Cin, Cout, H = 4, 8, 64, 128, 8
    g = torch.Generator().manual_seed(variant * 10 + block_n + splits)
    x = (torch.rand(T, B, Cin, H, H, generator=g) < 0.2).float()
    w = (torch.randn(Cout, Cin, 3, 3, generator=g) * (2.0 / (9 * Cin)) ** 0.5)
    b = torch.rand(Cout, generator=g) * 0.3
    res = (torch.rand(T, B, Cout, H, H, generator=g) < 0.3).float() if res_dtype == torch.bfloat16 \
        else torch.randn(T, B, Cout, H, H, generator=g) * 0.5
    xd = x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV)
    rd = res.permute(0, 1, 3, 4, 2).contiguous().to(res_dtype).to(DEV)
    y = C.conv3x3_lif(xd, C.weight_khwc(w).to(DEV), b.to(DEV), tau=2.0, v_threshold=1.0,
                      variant=variant, block_n=block_n, splits=splits, residual=rd)
    assert C.device_status() == 0
    # the kernel ran on bf16 spikes: the oracle's bf16 mode (bf16-rounded weights)
    ref, vpre = OR.conv_bn_neuron(x.to(torch.bfloat16), w, b, stride=1, padding=1, residual=res)
    got = y.float().cpu().permute(0, 1, 4, 2, 3)
    assert ref.sum() > 0
    bad = got != ref
    near = (vpre - 1.0).abs() < 1e-4
    assert not (bad & ~near).any() and bad.float().mean() <= 1e-3


def test_residual_rejected_by_variants_without_it_and_with_pool():
    """Band (3), two-tile (4) and CTA-pair (5) kernels take no residual input."""
    from snn_compiler.kernels import conv as C
    x = torch.zeros(4, 2, 16, 16, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(128, 3, 3, 64, device=DEV, dtype=torch.bfloat16)
    r = torch.zeros(4, 2, 16, 16, 128, device=DEV, dtype=torch.bfloat16)
    b = torch.zeros(128, device=DEV)
    for variant, bn in ((3, 64), (4, 64), (5, 64), (1, 128)):
        with pytest.raises(RuntimeError):
            C.conv3x3_lif(x, w, b, variant=variant, block_n=bn, residual=r)
    C.conv3x3_lif(x, w, b, variant=1, block_n=64, residual=r)        # accepted
    with pytest.raises(AssertionError):
        C.conv3x3_lif(x, w, b, pool=True, residual=r)
