"""Strided, 1x1 and 7x7 convs on the tensor-core kernels (snnb_conv_lif_strided,
snnb_conv_f32): the convs of a spiking ResNet that are not 3x3 / stride 1 -- the first conv
of a downsampling BasicBlock (3x3 / stride 2), pointwise convs, the downsample branch
(1x1 / stride 2 + folded BN, float32 result) and the 7x7 / stride 2 stem on the float32
image -- against the CPU oracle
(oracle/resnet.py, restating snn_compiler/nn/modules.py:258-443 and
snn_compiler/zoo/resnet.py:30-142)."""
import pytest
import torch

from oracle import resnet as OR

pytestmark = pytest.mark.gpu
DEV = "cuda"
THR = 1.0


def _spikes(shape, p, g):
    return (torch.rand(*shape, generator=g) < p).float()


def _weights(cout, cin, k, g, gain=1.0):
    return torch.randn(cout, cin, k, k, generator=g) * gain * (2.0 / (k * k * cin)) ** 0.5


def _flip_ok(got, ref, vpre):
    """BASELINE's criterion: at most 0.1% of the elements disagree, and each neuron's FIRST
    disagreement sits within 1e-4 of the threshold (after a flip the two membranes follow
    different resets, so a neuron's later steps may differ anywhere)."""
    T = got.shape[0]
    bad = (got != ref).reshape(T, -1)
    if bad.float().mean().item() > 1e-3:
        return False
    if not bad.any():
        return True
    cols = bad.any(0).nonzero().squeeze(1)
    first = torch.argmax(bad.int(), dim=0)[cols]
    v = vpre.reshape(T, -1)[first, cols]
    return bool(((v - THR).abs() < 1e-4).all())


GEOMS = [  # (k, stride, H, W, Cin, Cout)
    (3, 2, 16, 16, 64, 128),
    (3, 2, 15, 13, 64, 64),       # odd sizes: the last output row / column reads padding
    (3, 2, 8, 8, 128, 256),
    (1, 2, 16, 16, 64, 128),
    (1, 2, 7, 9, 64, 64),
    (1, 1, 8, 8, 128, 64),
    (3, 1, 8, 8, 64, 64),         # the stride-1 3x3 conv through the same entry
    (7, 2, 16, 16, 64, 64),       # a 7x7 / stride 2 conv (the ResNet stem's geometry)
    (5, 1, 9, 9, 64, 64),
]
SCHEDS = [(0, 0, 1), (1, 64, 1), (1, 32, 1), (2, 128, 1), (2, 64, 2), (4, 64, 1), (5, 128, 1),
          (6, 128, 2)]


@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("sched", SCHEDS)
@pytest.mark.parametrize("geom", GEOMS)
def test_strided_conv_lif_against_oracle(geom, sched, residual):
    from snn_compiler.kernels import conv as C
    k, stride, H, W, Cin, Cout = geom
    variant, block_n, splits = sched
    kslabs = k * k * ((Cin + 63) // 64)
    if block_n and Cout % block_n or splits > kslabs // 2 and splits > 1:
        pytest.skip("schedule does not apply to this geometry")
    if residual and variant in (4, 5):
        pytest.skip("no residual input in this variant")
    T, B = 4, 4
    if (stride != 1 or k > 3) and variant in (4, 5, 6):
        # general tap coordinates: the T-sequential and single-CTA T-folded kernels only
        x = torch.zeros(T, B, H, W, Cin, device=DEV, dtype=torch.bfloat16)
        with pytest.raises(RuntimeError):
            C.conv_lif_strided(x, torch.zeros(Cout, k, k, Cin, device=DEV, dtype=torch.bfloat16),
                               torch.zeros(Cout, device=DEV), stride=stride, variant=variant,
                               block_n=block_n, splits=splits)
        return
    g = torch.Generator().manual_seed(hash(geom) % 1000 + 7 * variant + block_n + splits)
    x = _spikes((T, B, Cin, H, W), 0.2, g)
    w = _weights(Cout, Cin, k, g, gain=1.5)
    b = torch.rand(Cout, generator=g) * 0.4
    Ho, Wo = (H - 1) // stride + 1, (W - 1) // stride + 1
    res = torch.randn(T, B, Cout, Ho, Wo, generator=g) * 0.5 if residual else None
    xd = x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV)
    rd = None if res is None else res.permute(0, 1, 3, 4, 2).contiguous().to(DEV)
    y = C.conv_lif_strided(xd, C.weight_khwc(w).to(DEV), b.to(DEV), stride=stride, tau=2.0,
                           v_threshold=THR, variant=variant, block_n=block_n, splits=splits,
                           residual=rd)
    assert C.device_status() == 0
    assert tuple(y.shape) == (T, B, Ho, Wo, Cout)
    ref, vpre = OR.conv_bn_neuron(x.to(torch.bfloat16), w, b, stride=stride, padding=k // 2,
                                  residual=res)
    got = y.float().cpu().permute(0, 1, 4, 2, 3)
    assert ref.sum() > 0 and ref.mean() < 0.9, "degenerate case"
    assert _flip_ok(got, ref, vpre)


@pytest.mark.parametrize("geom", [(1, 2, 16, 16, 64, 128), (1, 2, 7, 9, 64, 64),
                                  (3, 2, 8, 8, 64, 128), (1, 1, 8, 8, 128, 64)])
@pytest.mark.parametrize("T", [2, 4])
def test_conv_f32_against_oracle(geom, T):
    """The float32 conv + bias (no neuron) against the oracle's float32 conv: the products of
    spikes and bf16 weights are exact, so only the summation order differs."""
    from snn_compiler.kernels import conv as C
    k, stride, H, W, Cin, Cout = geom
    B = 3
    g = torch.Generator().manual_seed(sum(geom) + T)
    x = _spikes((T, B, Cin, H, W), 0.3, g)
    w = _weights(Cout, Cin, k, g)
    b = torch.randn(Cout, generator=g) * 0.1
    y = C.conv_f32(x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV),
                   C.weight_khwc(w).to(DEV), b.to(DEV), stride=stride)
    ref = OR.conv_bias(x.to(torch.bfloat16), w, b, stride=stride, padding=k // 2)
    got = y.cpu().permute(0, 1, 4, 2, 3)
    assert got.shape == ref.shape
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)


def test_strided_entry_rejects_band_variants_and_bad_strides():
    from snn_compiler.kernels import conv as C
    x = torch.zeros(4, 2, 16, 16, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(64, 3, 3, 64, device=DEV, dtype=torch.bfloat16)
    b = torch.zeros(64, device=DEV)
    for variant in (3, 7):          # the band kernels take stride-1 3x3 convs only
        with pytest.raises(RuntimeError):
            C.conv_lif_strided(x, w, b, stride=2, variant=variant, block_n=64)
    with pytest.raises(AssertionError):
        C.conv_lif_strided(x, w, b, stride=3)


@pytest.mark.parametrize("tune", [False, True])
def test_resnet_block_with_downsample_bf16_on_the_kernels(tune):
    """A downsampling BasicBlock (3x3 / stride 2 conv, 1x1 / stride 2 downsample + BN, 3x3
    conv + residual) fused and run in bf16: each fused module against the oracle on its own
    inputs, every one of them on this library's kernels -- with the default schedules, and
    with the per-layer schedules tune_convs picks."""
    from snn_compiler.nn import FusedConvBN, FusedConvBNAddNeuron, FusedConvBNNeuron, tune_convs
    from snn_compiler.zoo.resnet import BasicBlockSNN
    torch.manual_seed(11)
    down = torch.nn.Sequential(torch.nn.Conv2d(64, 128, 1, stride=2, bias=False),
                               torch.nn.BatchNorm2d(128))
    blk = BasicBlockSNN(64, 128, stride=2, downsample=down, neuron="lif")
    with torch.no_grad():
        for mod in blk.modules():
            if isinstance(mod, torch.nn.Conv2d):
                mod.weight.mul_(3.0)
            if isinstance(mod, torch.nn.BatchNorm2d):
                mod.bias.add_(0.5)
                mod.running_mean.normal_(0, 0.1)
                mod.running_var.uniform_(0.5, 1.5)
    blk = blk.eval().fuse().to(DEV).to(torch.bfloat16)
    assert isinstance(blk.downsample, FusedConvBN)
    g = torch.Generator().manual_seed(5)
    x = _spikes((4, 2, 64, 16, 16), 0.25, g).to(torch.bfloat16).to(DEV)
    if tune:                        # (before the recording hooks: tuning captures graphs)
        chosen = tune_convs(blk, x, reps=2)
        assert set(chosen) == {"block1", "block2"}, chosen
        assert all(v[0] in (1, 2, 4, 5) for v in chosen.values())
    rec = []
    hooks = [m.register_forward_hook(
        lambda m, inp, out: rec.append((m, [i.detach().cpu() for i in inp], out.detach().cpu())))
        for m in blk.modules() if isinstance(m, (FusedConvBN, FusedConvBNNeuron,
                                                  FusedConvBNAddNeuron))]
    try:
        with torch.no_grad():
            y = blk(x)
    finally:
        for h in hooks:
            h.remove()
    assert y.shape == (4, 2, 128, 8, 8)
    kinds = set()
    for mod, inp, out in rec:
        assert "w" in mod._cache, type(mod).__name__       # ran on the tensor-core kernels
        kinds.add(type(mod).__name__)
        if isinstance(mod, FusedConvBN):
            assert out.dtype == torch.float32
            ref = OR.conv_bias(inp[0], mod.weight, mod.bias, stride=mod.stride,
                               padding=mod.padding)
            torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
            continue
        res = inp[1] if len(inp) > 1 else None
        ref, vpre = OR.fused_module_oracle(mod, inp[0], residual=res)
        assert ref.sum() > 0, type(mod).__name__
        assert _flip_ok(out.float(), ref, vpre), type(mod).__name__
    assert kinds == {"FusedConvBN", "FusedConvBNNeuron", "FusedConvBNAddNeuron"}


def test_resnet_stem_on_the_float32_image():
    """The 7x7 / stride 2 / padding 3 stem conv + BN + LIF of ResNetSNN on a float32 image
    (Cin = 3): the 7x7 x 3 window gathered into K = 147 channels, then float32-faithful on
    the tensor cores (image and weights as three bf16 terms), against the float32 oracle."""
    from snn_compiler.nn import FusedConvBNNeuron
    torch.manual_seed(3)
    conv = torch.nn.Conv2d(3, 64, 7, stride=2, padding=3, bias=False)
    bn = torch.nn.BatchNorm2d(64)
    with torch.no_grad():
        conv.weight.mul_(2.0)
        bn.bias.add_(0.3)
        bn.running_mean.normal_(0, 0.1)
        bn.running_var.uniform_(0.5, 1.5)
    mod = FusedConvBNNeuron(conv.eval(), bn.eval(), neuron="lif", tau=2.0).to(DEV)
    g = torch.Generator().manual_seed(9)
    img = torch.rand(1, 4, 3, 32, 32, generator=g).expand(4, 4, 3, 32, 32).contiguous()
    with torch.no_grad():
        y = mod(img.to(DEV))
    assert "w" in mod._cache                    # ran on the tensor-core kernel
    assert y.shape == (4, 4, 64, 16, 16) and y.dtype == torch.float32
    ref, vpre = OR.fused_module_oracle(mod, img)
    assert ref.sum() > 0 and ref.mean() < 0.9
    assert _flip_ok(y.cpu(), ref, vpre)


def test_resnet_stem_on_a_bf16_image_channel_padded():
    """The same stem module in bf16 (the reference's bf16 mode): the 7x7 x 3 window gathered
    into K = 147 channels (zero padded to 152) and run as a 1x1 conv on the bf16 kernel,
    against the oracle with bf16 weights."""
    from snn_compiler.nn import FusedConvBNNeuron
    torch.manual_seed(4)
    conv = torch.nn.Conv2d(3, 64, 7, stride=2, padding=3, bias=False)
    bn = torch.nn.BatchNorm2d(64)
    with torch.no_grad():
        conv.weight.mul_(2.0)
        bn.bias.add_(0.3)
    mod = FusedConvBNNeuron(conv.eval(), bn.eval(), neuron="lif", tau=2.0, layout="NHWC")
    mod = mod.to(DEV).to(torch.bfloat16)
    g = torch.Generator().manual_seed(10)
    img = torch.rand(1, 2, 3, 40, 40, generator=g).expand(4, 2, 3, 40, 40).to(torch.bfloat16)
    xd = img.reshape(8, 3, 40, 40).contiguous(memory_format=torch.channels_last).view(4, 2, 3, 40, 40)
    with torch.no_grad():
        y = mod(xd.to(DEV))
    assert "w" in mod._cache and tuple(mod._cache["w"].shape) == (64, 1, 1, 152)
    assert y.shape == (4, 2, 64, 20, 20) and y.dtype == torch.bfloat16
    ref, vpre = OR.fused_module_oracle(mod, img)
    assert ref.sum() > 0 and ref.mean() < 0.9
    assert _flip_ok(y.float().cpu(), ref, vpre)


@pytest.mark.parametrize("shape", [(8, 112, 112, 64), (3, 15, 13, 32), (2, 7, 9, 8)])
@pytest.mark.parametrize("kind", ["spikes", "values"])
def test_maxpool_nhwc_equals_torch(shape, kind):
    """snnb_maxpool_nhwc (3x3 / stride 2 / padding 1, the ResNet stem's pool) against torch's
    max_pool2d on the same bf16 frames: identical (a max picks one of its inputs)."""
    from snn_compiler.kernels import conv as C
    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.rand(*shape, generator=g) < 0.3).float() if kind == "spikes" \
        else torch.randn(*shape, generator=g)
    xd = x.to(torch.bfloat16).to(DEV)
    y = C.maxpool_nhwc(xd, 3, 2, 1)
    ref = torch.nn.functional.max_pool2d(xd.permute(0, 3, 1, 2).float(), 3, 2, 1)
    assert torch.equal(y.float().permute(0, 3, 1, 2), ref)


@pytest.mark.parametrize("shape,k,stride", [((3, 20, 17, 3), 7, 2), ((2, 9, 9, 4), 3, 1),
                                            ((2, 224, 224, 3), 7, 2), ((2, 70, 45, 3), 5, 1),
                                            ((1, 12, 10, 64), 7, 2)])   # (last: global form)
def test_window_gather_equals_unfold(shape, k, stride):
    """snnb_window_gather_nhwc against F.unfold on the same bf16 frames: the same values, in
    columns (dy, dx, c), zero padded to a multiple of 8 (a copy: exact) -- through the
    shared-memory staged kernel, and through the global-memory one where the staged window
    would not fit (64 channels x 7 x 69 columns)."""
    from snn_compiler.kernels import conv as C
    g = torch.Generator().manual_seed(sum(shape) + k)
    x = torch.randn(*shape, generator=g).to(torch.bfloat16)
    N, H, W, Cin = shape
    y = C.window_gather_nhwc(x.to(DEV), k, stride, k // 2).cpu()
    Ho, Wo = (H - 1) // stride + 1, (W - 1) // stride + 1
    K = k * k * Cin
    assert tuple(y.shape) == (N, Ho, Wo, (K + 7) // 8 * 8)
    cols = torch.nn.functional.unfold(x.permute(0, 3, 1, 2).float(), k, padding=k // 2,
                                      stride=stride)                 # [N, (c, dy, dx), L]
    ref = cols.reshape(N, Cin, k, k, Ho * Wo).permute(0, 4, 2, 3, 1).reshape(N, Ho, Wo, K)
    assert torch.equal(y[..., :K].float(), ref)
    assert not y[..., K:].float().any()
