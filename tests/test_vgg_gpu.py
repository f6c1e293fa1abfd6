"""VGG16-SNN end to end on the fused kernels vs the oracle / reference golden logits."""
import numpy as np
import pytest
import torch

from oracle import params as OP
from oracle import vgg as OV
from test_oracle_golden import _load

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _engine(P, T=4):
    from snn_compiler.zoo.vgg import SpikingVGG
    return SpikingVGG(P, T=T, device=DEV)


def test_vgg16_active_matches_reference_golden():
    """Config 0 (B=8, T=4) with the spiking-active BN calibration: top-1 identical to
    the reference's VGGSNN.forward, logits within 1e-2, hidden spikes within 0.1%."""
    g = _load("vgg16_active.npz")
    P = OV.apply_active(OP.vgg16_params(int(g["w_seed"])), g)
    x = OP.vgg16_input(int(g["x_seed"]), T=int(g["T"]), B=int(g["B"]))
    eng = _engine(P)
    per_t = eng.forward(x.to(DEV), per_step_logits=True).cpu()
    mean = eng.forward(x[:1].to(DEV)).cpu()                    # direct encoding, Ti = 1
    ref = torch.from_numpy(g["logits"])
    assert torch.equal(per_t.mean(0).argmax(-1), ref.mean(0).argmax(-1))
    assert torch.allclose(per_t, ref, rtol=1e-2, atol=1e-2), (per_t - ref).abs().max()
    assert torch.allclose(mean, per_t.mean(0), rtol=1e-5, atol=1e-5)


def test_vgg16_layer_spikes_against_oracle_trace():
    g = _load("vgg16_active.npz")
    P = OV.apply_active(OP.vgg16_params(int(g["w_seed"])), g)
    x = OP.vgg16_input(int(g["x_seed"]), T=4, B=8)
    _, trace = OV.vgg16_forward(x, P, collect=True)
    eng = _engine(P)
    steps, out = eng.plan(x[:1].contiguous().to(DEV))
    for _, _, fn in steps:
        fn()
    bufs = eng._bufs[(8, 32, 32, False)][0]
    for i, buf in enumerate(bufs):
        got = buf.float().cpu().permute(0, 1, 4, 2, 3)
        frac = (got != trace[i]).float().mean().item()
        assert frac <= 1e-3, (i, frac)


def test_vggsnn_module_forward_matches_oracle():
    from snn_compiler.zoo.vgg import vgg16_snn
    P = OP.vgg16_params(1)
    x = OP.vgg16_input(0, T=4, B=8)
    OV.calibrate_active(P, x)
    m = vgg16_snn(num_classes=10, fc_in=512).to(DEV)
    convs = [c for c in m.features if isinstance(c, torch.nn.Conv2d)]
    bns = [c for c in m.features if isinstance(c, torch.nn.BatchNorm2d)]
    lins = [c for c in m.classifier if isinstance(c, torch.nn.Linear)]
    with torch.no_grad():
        for cv, bn, p in zip(convs, bns, P["convs"]):
            cv.weight.copy_(p["w"]); cv.bias.copy_(p["b"])
            bn.weight.copy_(p["gamma"]); bn.bias.copy_(p["beta"])
            bn.running_mean.copy_(p["mean"]); bn.running_var.copy_(p["var"])
        for l, f in zip(lins, P["fcs"]):
            l.weight.copy_(f["w"]); l.bias.copy_(f["b"])
    out = m(x.to(DEV)).cpu()
    ref = OV.vgg16_forward(x, P)
    assert out.shape == ref.shape == (4, 8, 10)
    assert torch.equal(out.mean(0).argmax(-1), ref.mean(0).argmax(-1))


def test_vgg16_graph_replay_equals_eager():
    P = OP.vgg16_params(1)
    eng = _engine(P)
    img = torch.rand(1, 64, 3, 32, 32, generator=OP.gen(3)).to(DEV)
    eager = eng.forward(img).clone()
    out = eng.capture(img, split_at=3)
    eng.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_vgg16_concurrent_chains_equal_one_chain():
    """SpikingVGG(chains=2): the captured forward runs two sub-batch chains on concurrent
    streams (separate buffers and workspaces); the logits equal the one-chain forward."""
    from snn_compiler.zoo.vgg import SpikingVGG
    P = OP.vgg16_params(1)
    img = torch.rand(1, 32, 3, 32, 32, generator=OP.gen(4)).to(DEV)
    one = SpikingVGG(P, T=4, device=DEV).forward(img, graph=True).clone()
    eng2 = SpikingVGG(P, T=4, device=DEV, chains=2)
    two = eng2.forward(img, graph=True)
    torch.cuda.synchronize()
    assert eng2.kernel_launches(32) >= 2 * 16
    # each chain's kernels are tuned for its sub-batch (the schedules, hence the float32
    # summation order, may differ): equal up to that
    assert torch.allclose(one, two, rtol=1e-5, atol=1e-5)
    assert torch.equal(one.argmax(-1), two.argmax(-1))


def test_vgg16_split_graph_forward_equals_one_graph():
    """forward(graph=True, mid_event=e): the forward captured as two graphs split before
    launch mid_at, the event recorded between them; the logits equal the one-graph forward
    (the same launches) and the event completes."""
    P = OP.vgg16_params(1)
    eng = _engine(P)
    img = torch.rand(1, 64, 3, 32, 32, generator=OP.gen(5)).to(DEV)
    one = eng.forward(img, graph=True).clone()
    ev = torch.cuda.Event()
    two = eng.forward(img, graph=True, mid_event=ev, mid_at=4).clone()
    torch.cuda.synchronize()
    assert ev.query()
    assert torch.equal(one, two)
    assert eng.graph_input(tuple(img.shape), mid_at=4) is not None
