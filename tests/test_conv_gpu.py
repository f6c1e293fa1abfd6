"""K1 parity: the fused tcgen05 conv3x3 / linear + bias + multi-step LIF (+ max-pool)
kernels vs the CPU oracle (torch-CPU float32 conv of the same bf16 weights + the
oracle neuron).

The products are exact in both (spikes x bf16 weights); only the float32 summation
order differs, so the criterion is BASELINE's: spikes may differ only at neurons
whose first disagreement sits where the oracle's charged potential is within 1e-4
of the threshold, and on at most 0.1% of all spikes; pooled outputs must equal the
2x2 OR of the kernel's own unpooled spikes exactly.
"""
import itertools

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import params as OP
from oracle import vgg as OV

pytestmark = pytest.mark.gpu
DEV = "cuda"
THR = 1.0


def _C():
    from snn_compiler.kernels import conv
    return conv


def flip_check(gpu, ref, vpre, thr=THR, window=1e-4, max_frac=1e-3):
    """gpu, ref, vpre: [T, ...] float tensors.  Every neuron's first mismatching step
    must have |vpre - thr| < window; total mismatch fraction <= max_frac."""
    T = gpu.shape[0]
    g = gpu.reshape(T, -1)
    r = ref.reshape(T, -1)
    v = vpre.reshape(T, -1)
    mism = g != r
    frac = mism.float().mean().item()
    assert frac <= max_frac, f"spike mismatch fraction {frac:.2e}"
    if mism.any():
        first = torch.argmax(mism.int(), dim=0)
        cols = mism.any(0).nonzero().squeeze(1)
        vt = v[first[cols], cols]
        assert ((vt - thr).abs() < window).all(), (vt - thr).abs().max()
    return frac


def _layer_case(T, B, Cin, Cout, H, p, seed, pool):
    g = OP.gen(seed)
    x = (torch.rand(T, B, Cin, H, H, generator=g) < p).float()
    w = (torch.randn(Cout, Cin, 3, 3, generator=g) * (2.0 / (9 * Cin)) ** 0.5)
    w = w.to(torch.bfloat16).float()
    b = torch.rand(Cout, generator=g) * 0.9 + 0.3
    return x, w, b


GEOMS = [  # (T, B, Cin, Cout, H) -- every pixel-block geometry of VGG16 at 32x32 input
    (4, 1, 64, 64, 32),
    (4, 2, 64, 128, 16),
    (4, 2, 128, 256, 8),
    (4, 8, 256, 512, 4),
    (4, 32, 512, 512, 2),
    (3, 2, 64, 64, 8),
    (6, 4, 192, 96, 8),
    (4, 2, 64, 64, 56),     # config-2 spatial size: partial pixel blocks at the edges
    (4, 3, 64, 64, 14),
    (2, 5, 64, 128, 7),     # odd size: no pooling
    (4, 2, 48, 64, 8),      # partial 64-channel slab (zero-filled by the TMA)
    (4, 4, 96, 64, 4),
]


VARIANTS = [(0, 0, 1), (1, 32, 1), (1, 128, 1), (2, 32, 1), (2, 64, 1), (2, 128, 1), (2, 256, 1),
            (2, 128, 3), (2, 256, 4), (3, 32, 1), (3, 64, 1), (4, 64, 1), (4, 128, 1),
            (4, 128, 2), (5, 64, 1), (5, 128, 1), (5, 256, 1), (5, 128, 2), (5, 256, 3),
            (6, 128, 2), (6, 128, 4), (6, 256, 2), (6, 256, 8), (7, 32, 1), (7, 64, 1)]


@pytest.mark.parametrize("vb", VARIANTS)
@pytest.mark.parametrize("geom", GEOMS)
def test_conv3x3_lif_against_oracle(geom, vb):
    """Both kernel variants (T sequential in the CTA / T folded into M) and several
    channel-block widths on every VGG16 pixel-block geometry."""
    T, B, Cin, Cout, H = geom
    variant, block_n, splits = vb
    if block_n and Cout % block_n:
        pytest.skip("block_n must divide Cout")
    if variant in (2, 4, 5, 6) and T not in (2, 4, 8):
        pytest.skip("T folding needs T in {2, 4, 8}")
    C = _C()
    band_ok = C.band_block_ns if variant == 3 else C.band_xs_block_ns
    if variant in (3, 7) and block_n not in band_ok(H, Cin, Cout):
        x = torch.zeros(T, B, H, H, Cin, device=DEV, dtype=torch.bfloat16)
        with pytest.raises(RuntimeError):
            C.conv3x3_lif(x, torch.zeros(Cout, 3, 3, Cin, device=DEV, dtype=torch.bfloat16),
                          torch.zeros(Cout, device=DEV), variant=variant, block_n=block_n)
        return
    x, w, b = _layer_case(T, B, Cin, Cout, H, 0.15, sum(geom) * 31 + Cout, False)
    xd = x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV)
    wd = C.weight_khwc(w).to(DEV)
    bd = b.to(DEV)
    kw = dict(tau=2.0, v_threshold=THR, variant=variant, block_n=block_n, splits=splits)
    y = C.conv3x3_lif(xd, wd, bd, pool=False, **kw)
    yp = C.conv3x3_lif(xd, wd, bd, pool=True, **kw) if H % 2 == 0 else None
    assert C.device_status() == 0
    s, _, vpre = OV.conv_bn_lif_pool(x, w, b, pool=False, want_vpre=True)
    got = y.float().cpu().permute(0, 1, 4, 2, 3)                        # -> [T,B,C,H,W]
    assert got.sum() > 0, "degenerate case: no spikes"
    flip_check(got, s, vpre)
    if yp is not None:
        own = F.max_pool2d(got.reshape(T * B, Cout, H, H), 2, 2).reshape(T, B, Cout, H // 2, H // 2)
        assert torch.equal(yp.float().cpu().permute(0, 1, 4, 2, 3), own)


@pytest.mark.parametrize("sk", [(128, 2), (128, 4), (256, 2), (256, 4), (256, 8)])
@pytest.mark.parametrize("geom", [(4, 32, 512, 512, 2), (4, 8, 256, 512, 4), (2, 16, 128, 256, 4),
                                  (8, 4, 512, 256, 2), (4, 2, 64, 128, 16)])
def test_cluster_splitk_bit_identical_to_two_launch_form(geom, sk):
    """The cluster split-K form (variant 6) adds the partial sums in the order of the
    two-launch split-K form (variant 2 + splitsum_lif_kernel): spikes identical, pooled and
    not, and with a residual input."""
    T, B, Cin, Cout, H = geom
    block_n, splits = sk
    if Cout % block_n:
        pytest.skip("block_n must divide Cout")
    C = _C()
    x, w, b = _layer_case(T, B, Cin, Cout, H, 0.2, sum(geom) * 7 + block_n + splits, False)
    xd = x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV)
    wd = C.weight_khwc(w).to(DEV)
    bd = b.to(DEV)
    g = OP.gen(Cout + splits)
    rd = (torch.randn(T, B, H, H, Cout, generator=g) * 0.5).to(DEV)
    for kw in (dict(pool=False), dict(pool=True), dict(residual=rd)):
        ref = C.conv3x3_lif(xd, wd, bd, tau=2.0, v_threshold=THR, variant=2, block_n=block_n,
                            splits=splits, **kw)
        got = C.conv3x3_lif(xd, wd, bd, tau=2.0, v_threshold=THR, variant=6, block_n=block_n,
                            splits=splits, **kw)
        assert C.device_status() == 0
        assert ref.float().sum() > 0
        assert torch.equal(got, ref), kw.keys()


@pytest.mark.parametrize("vb", [(0, 0, 1), (2, 32, 1), (2, 128, 1), (2, 64, 2), (4, 64, 1),
                                (5, 128, 1), (6, 128, 2), (6, 256, 4)])
@pytest.mark.parametrize("case", [(4, 16, 512, 512, 2), (4, 8, 128, 256, 1), (2, 8, 64, 128, 2),
                                  (8, 4, 256, 128, 2), (4, 6, 64, 64, 2)])
def test_conv3x3_dense_small_image_against_oracle(case, vb):
    """Layers on 1x1 / 2x2 images as one dense GEMM per image (snnb_conv3x3_lif_dense), with
    and without the fused 2x2 pool (OR over 4 consecutive columns), against the oracle's
    padded conv."""
    T, B, Cin, Cout, H = case
    variant, block_n, splits = vb
    if block_n and (H * H * Cout) % block_n:
        pytest.skip("block_n must divide H*W*Cout")
    if splits > (H * H * Cin + 63) // 64:
        pytest.skip("more splits than 64-channel k-slabs")
    C = _C()
    x, w, b = _layer_case(T, B, Cin, Cout, H, 0.2, sum(case) * 13 + block_n + splits, False)
    xd = x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV)
    wk = C.weight_khwc(w).to(DEV)
    bd = b.to(DEV)
    kw = dict(tau=2.0, v_threshold=THR, variant=variant, block_n=block_n, splits=splits)
    y = C.conv3x3_lif_dense(xd, C.dense_conv_weight(wk, H, H), C.dense_conv_bias(bd, H, H), **kw)
    assert C.device_status() == 0
    s, _, vpre = OV.conv_bn_lif_pool(x, w, b, pool=False, want_vpre=True)
    got = y.float().cpu().permute(0, 1, 4, 2, 3)
    assert got.sum() > 0, "degenerate case: no spikes"
    flip_check(got, s, vpre)
    if H != 2:
        return
    wp, bp = C.dense_conv_weight(wk, 2, 2, pool=True), C.dense_conv_bias(bd, 2, 2, pool=True)
    if variant not in (0, 2) or splits > 1:       # the pooled dense form: plain T-folded only
        with pytest.raises(RuntimeError):
            C.conv3x3_lif_dense(xd, wp, bp, pool=True, **kw)
        return
    yp = C.conv3x3_lif_dense(xd, wp, bp, pool=True, **kw)
    assert C.device_status() == 0 and tuple(yp.shape) == (T, B, 1, 1, Cout)
    gp = yp.float().cpu().reshape(T, B, Cout)
    ref = s.reshape(T, B, Cout, 4).amax(-1)
    # a window may differ only where one of its neurons came within 1e-4 of the threshold
    near = ((vpre - THR).abs() < 1e-4).reshape(T, B, Cout, 4).any(-1).any(0, keepdim=True)
    assert ref.sum() > 0
    assert not ((gp != ref) & ~near).any()
    assert (gp != ref).float().mean() <= 1e-3


def test_conv3x3_soft_reset_and_if_neuron():
    C = _C()
    T, B, Cin, Cout, H = 4, 2, 64, 64, 8
    x, w, b = _layer_case(T, B, Cin, Cout, H, 0.3, 11, False)
    xd = x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV)
    for (neuron, soft), variant in itertools.product((("if", True), ("lif", True), ("if", False)),
                                                     (1, 2)):
        y = C.conv3x3_lif(xd, C.weight_khwc(w).to(DEV), b.to(DEV), neuron=neuron, tau=2.0,
                          soft_reset=soft, v_threshold=0.8, v_reset=-0.1, variant=variant)
        from oracle import neurons as ON
        yc = F.conv2d(x.reshape(T * B, Cin, H, H), w, None, padding=1).reshape(T, B, Cout, H, H)
        df, sc = ON.neuron_params(neuron, tau=2.0)
        o = ON.lif_multistep(yc.reshape(T, -1).numpy(), df=df, sc=sc, hard_reset=not soft,
                             v_reset=-0.1, thr=0.8, bias=b.numpy(), C=Cout, HW=H * H,
                             want_vpre=True)
        got = y.float().cpu().permute(0, 1, 4, 2, 3)
        flip_check(got, torch.from_numpy(o["spikes"]).reshape(got.shape),
                   torch.from_numpy(o["vpre"]).reshape(got.shape), thr=0.8)


@pytest.mark.parametrize("vb", [(0, 0, 1), (1, 64, 1), (2, 32, 1), (2, 128, 1), (2, 128, 2),
                                (4, 128, 1), (4, 64, 2), (5, 128, 1), (5, 64, 2), (5, 256, 1),
                                (6, 128, 2), (6, 256, 4)])
@pytest.mark.parametrize("TBKN", [(4, 64, 512, 4096), (4, 8, 4096, 256), (2, 130, 128, 96)])
def test_linear_lif_against_oracle(TBKN, vb):
    T, B, K, N = TBKN
    variant, block_n, splits = vb
    if block_n and N % block_n:
        pytest.skip("block_n must divide N")
    C = _C()
    g = OP.gen(K + N)
    x = (torch.rand(T, B, K, generator=g) < 0.2).float()
    w = (torch.randn(N, K, generator=g) * (2.0 / K) ** 0.5).to(torch.bfloat16).float()
    b = torch.rand(N, generator=g) * 0.9 + 0.3
    y = C.linear_lif(x.to(torch.bfloat16).to(DEV), w.to(torch.bfloat16).to(DEV), b.to(DEV),
                     tau=2.0, v_threshold=THR, variant=variant, block_n=block_n, splits=splits)
    yc = F.linear(x.reshape(T * B, K), w).reshape(T, B, N)
    s, vpre = OV.lif_seq(yc, b, want_vpre=True)
    got = y.float().cpu()
    assert got.sum() > 0
    flip_check(got, s, vpre)


@pytest.mark.parametrize("TBKN", [(4, 64, 4096, 10), (4, 8, 512, 64), (3, 5, 128, 16)])
def test_linear_mean_against_oracle(TBKN):
    T, B, K, N = TBKN
    C = _C()
    g = OP.gen(3 * K + N)
    x = (torch.rand(T, B, K, generator=g) < 0.2).float()
    w = (torch.randn(N, K, generator=g) * (2.0 / K) ** 0.5).to(torch.bfloat16).float()
    b = torch.randn(N, generator=g) * 0.1
    y = C.linear_mean(x.to(torch.bfloat16).to(DEV), w.to(torch.bfloat16).to(DEV), b.to(DEV))
    ref = (F.linear(x.reshape(T * B, K), w) + b).reshape(T, B, N).mean(0)
    assert torch.allclose(y.cpu(), ref, rtol=1e-5, atol=1e-5), (y.cpu() - ref).abs().max()


@pytest.mark.parametrize("static", [True, False])
@pytest.mark.parametrize("pool", [False, True])
def test_first_conv_lif_against_oracle(static, pool):
    C = _C()
    T, B, Cin, Cout, H = 4, 3, 3, 64, 32
    g = OP.gen(21)
    img = torch.rand(1 if static else T, B, Cin, H, H, generator=g)
    w = torch.randn(Cout, Cin, 3, 3, generator=g) * (2.0 / 27) ** 0.5
    b = torch.rand(Cout, generator=g) * 0.6 + 0.3
    y = C.first_conv_lif(img.to(DEV), w.to(DEV), b.to(DEV), T=T, tau=2.0, v_threshold=THR,
                         pool=pool)
    x = img.expand(T, B, Cin, H, H) if static else img
    s, p, vpre = OV.conv_bn_lif_pool(x.contiguous(), w, b, pool=pool, want_vpre=True)
    got = y.float().cpu().permute(0, 1, 4, 2, 3)
    if not pool:
        flip_check(got, s, vpre)
    else:
        mism = (got != p).float().mean().item()
        assert mism <= 1e-3


def test_bad_geometry_is_rejected():
    C = _C()
    x = torch.zeros(4, 1, 8, 8, 20, device=DEV, dtype=torch.bfloat16)     # Cin % 8 != 0
    w = torch.zeros(64, 3, 3, 20, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        C.conv3x3_lif(x, w, torch.zeros(64, device=DEV))


# ---- packed spikes between layers (snnb_conv3x3_lif_packed / snnb_unpack_spikes) ------------
PK_GEOMS = [(4, 1, 64, 64, 32), (4, 2, 64, 128, 16), (4, 2, 128, 256, 8), (4, 8, 256, 512, 4),
            (4, 32, 512, 512, 2), (8, 2, 128, 128, 8), (2, 5, 64, 128, 7), (4, 2, 64, 64, 56)]


@pytest.mark.parametrize("block_n", [64, 128, 256])
@pytest.mark.parametrize("mode", [(True, False), (False, True), (True, True)])
@pytest.mark.parametrize("geom", PK_GEOMS)
def test_packed_spikes_identical_to_bf16_path(geom, mode, block_n):
    """Packed input (patch expanded to the bf16 A operand in shared memory) and packed
    output (16-channel half-words) give exactly the spikes of the bf16 T-folded kernel with
    the same channel block, pooled and not."""
    T, B, Cin, Cout, H = geom
    x_packed, out_packed = mode
    if Cout % block_n:
        pytest.skip("block_n must divide Cout")
    C = _C()
    x, w, b = _layer_case(T, B, Cin, Cout, H, 0.2, sum(geom) * 5 + block_n, False)
    xd = x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV)
    wd = C.weight_khwc(w).to(DEV)
    bd = b.to(DEV)
    xin = C.pack_spikes(xd) if x_packed else xd
    for pool in ((False, True) if H % 2 == 0 else (False,)):
        ref = C.conv3x3_lif(xd, wd, bd, tau=2.0, v_threshold=THR, variant=2, block_n=block_n,
                            pool=pool)
        got = C.conv3x3_lif_packed(xin, wd, bd, x_packed=x_packed, out_packed=out_packed,
                                   tau=2.0, v_threshold=THR, pool=pool, block_n=block_n)
        assert C.device_status() == 0
        if out_packed:
            assert got.dtype == torch.int32 and got.shape[-1] == Cout // 32
            got = C.unpack_spikes(got)
        assert ref.float().sum() > 0
        assert torch.equal(got, ref), (pool, (got != ref).float().mean().item())


def test_pack_unpack_round_trip_and_packed_limits():
    C = _C()
    g = OP.gen(77)
    x = (torch.rand(3, 5, 7, 96, generator=g) < 0.3).to(torch.bfloat16).to(DEV)
    words = C.pack_spikes(x)
    assert words.shape == (3, 5, 7, 3) and words.dtype == torch.int32
    # bit c % 32 of word c / 32, LSB first
    ref = (x.cpu().reshape(-1, 3, 32).to(torch.int64) << torch.arange(32)).sum(-1)
    assert torch.equal(words.cpu().reshape(-1, 3).to(torch.int64) & 0xffffffff, ref)
    assert torch.equal(C.unpack_spikes(words), x)
    w = torch.zeros(64, 3, 3, 48, device=DEV, dtype=torch.bfloat16)
    xp = torch.zeros(4, 2, 8, 8, 2, device=DEV, dtype=torch.int32)    # Cin = 64
    with pytest.raises(AssertionError):                                # Cin mismatch
        C.conv3x3_lif_packed(xp, w, torch.zeros(64, device=DEV), x_packed=True, out_packed=False)
    # Cin = 32 (one word per pixel) is not a multiple of 64: the packed-input kernel refuses it
    with pytest.raises(RuntimeError):
        C.conv3x3_lif_packed(torch.zeros(4, 2, 8, 8, 1, dtype=torch.int32, device=DEV),
                             torch.zeros(64, 3, 3, 32, device=DEV, dtype=torch.bfloat16),
                             torch.zeros(64, device=DEV), x_packed=True, out_packed=False)


@pytest.mark.parametrize("cin,cout,B,H,W,soft", [(3, 64, 3, 32, 32, False), (3, 64, 2, 7, 9, False),
                                                 (1, 32, 2, 16, 16, True), (4, 128, 2, 12, 20, False),
                                                 (2, 64, 5, 8, 8, True), (3, 32, 1, 5, 5, False),
                                                 (3, 64, 20, 32, 32, False),
                                                 (2, 128, 37, 23, 23, True),
                                                 (1, 32, 300, 16, 16, False)])
def test_first_conv_tensor_core_against_oracle(cin, cout, B, H, W, soft):
    """Image layer on tcgen05 (snnb_first_conv_lif_tc): the float32 conv from split bf16
    terms against the float32 oracle conv -- flip criterion -- including partial 128-pixel
    tiles (B*H*W not a multiple of 128), image borders, and more tiles than SMs (the
    persistent CTAs then cycle through both stages several times)."""
    C = _C()
    T = 4
    g = OP.gen(31 + cin + cout + H)
    img = torch.rand(1, B, cin, H, W, generator=g)
    w = torch.randn(cout, cin, 3, 3, generator=g) * (2.0 / (9 * cin)) ** 0.5 * 1.5
    b = torch.rand(cout, generator=g) * 0.6 + 0.3
    ws = C.first_conv_split_weight(w).to(DEV)
    y = C.first_conv_lif_tc(img.to(DEV), ws, b.to(DEV), T=T, tau=2.0, v_threshold=THR,
                            soft_reset=soft)
    assert C.device_status() == 0
    x = img.expand(T, B, cin, H, W).contiguous()
    s, _, vpre = OV.conv_bn_lif_pool(x, w, b, pool=False, want_vpre=True, soft_reset=soft)
    got = y.float().cpu().permute(0, 1, 4, 2, 3)
    assert got.sum() > 0
    flip_check(got, s, vpre)


@pytest.mark.parametrize("T,B,K,N,splits,pool4", [(4, 64, 512, 4096, 1, False),
                                                  (4, 64, 4096, 4096, 2, False),
                                                  (4, 64, 2048, 2048, 8, False),
                                                  (4, 64, 2048, 2048, 4, True),
                                                  (2, 50, 384, 256, 2, False),
                                                  (8, 70, 1000, 384, 4, True),
                                                  (1, 300, 256, 128, 1, False)])
def test_linear_transposed_against_oracle(T, B, K, N, splits, pool4):
    """snnb_linear_lif_t (D^T = W X^T, split-K over a cluster, partial sums in split order)
    against the oracle: linear of the same bf16 values in float32 + LIF, flip criterion;
    with pool4 the OR of 4 consecutive features of the kernel's own unpooled spikes, exactly;
    partial column tiles (B not a multiple of 256 / T) included."""
    C = _C()
    g = OP.gen(T * 1000 + B + K + splits)
    x = (torch.rand(T, B, K, generator=g) < 0.2).float()
    w = (torch.randn(N, K, generator=g) * (3.0 / K) ** 0.5).to(torch.bfloat16).float()
    b = torch.rand(N, generator=g) * 0.5 + 0.2
    xd, wd, bd = x.to(torch.bfloat16).to(DEV), w.to(torch.bfloat16).to(DEV), b.to(DEV)
    y = C.linear_lif_t(xd, wd, bd, tau=2.0, v_threshold=THR, splits=splits)
    assert C.device_status() == 0
    z = F.linear(x.reshape(T * B, K), w).reshape(T, B, N)
    s, vpre = OV.lif_seq(z, b, want_vpre=True)
    got = y.float().cpu()
    assert got.sum() > 0
    flip_check(got, s, vpre)
    if pool4:
        yp = C.linear_lif_t(xd, wd, bd, tau=2.0, v_threshold=THR, splits=splits, pool4=True)
        own = got.reshape(T, B, N // 4, 4).amax(-1)
        assert torch.equal(yp.float().cpu(), own)


def test_dense_conv_transposed_form_equals_row_form():
    """The dense form of a 2x2 layer through the transposed kernel (variant 8) against the
    row-major T-folded form (variant 2): flip criterion between them via the oracle."""
    C = _C()
    T, B, Cin, Cout, H = 4, 64, 512, 512, 2
    x, w, b = _layer_case(T, B, Cin, Cout, H, 0.2, 77, False)
    xd = x.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16).to(DEV)
    wk = C.weight_khwc(w).to(DEV)
    for pool in (False, True):
        wd = C.dense_conv_weight(wk, H, H, pool=pool)
        bd = C.dense_conv_bias(b.to(DEV), H, H, pool=pool)
        y8 = C.conv3x3_lif_dense(xd, wd, bd, pool=pool, variant=8, splits=4, tau=2.0,
                                 v_threshold=THR)
        y2 = C.conv3x3_lif_dense(xd, wd, bd, pool=pool, variant=2, block_n=32, tau=2.0,
                                 v_threshold=THR)
        assert C.device_status() == 0
        s, p, vpre = OV.conv_bn_lif_pool(x, w, b, pool=pool, want_vpre=True)
        got = y8.float().cpu().permute(0, 1, 4, 2, 3)
        if not pool:
            flip_check(got, s, vpre)
        else:
            assert (got != y2.float().cpu().permute(0, 1, 4, 2, 3)).float().mean() <= 1e-3
