"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own code.

Run once, in a container where the reference checkout is available:
    python tests/golden/make_golden.py --reference /path/to/Triton-Pass-Analysis

It imports the reference's ``snn_compiler`` package (pure-torch parts only, on
the CPU) and records, for seeded inputs:

  lif_cases.npz     naive_if_lif (snn_compiler/kernels/neurons.py:467-502) over the
                    test matrix of snn_compiler/tests/test_correctness.py:43-108
                    (IF/LIF x soft/hard x v_reset x decay_input x threshold
                    scalar/[C]/[NCL] x NCHW/NHWC), the dtype cases (:231-250), the
                    decay overrides (:253-292), ragged shapes, and the rate-coded
                    sums of snn_compiler/tests/test_largeT_and_rate.py:71-103.
  fold_bn.npz       fold_conv_bn (snn_compiler/kernels/fused.py:585-599).
  bitpack.npz       bitpack_N (snn_compiler/explore/attention/phase6b_bitpack.py:35-46)
                    and the K^T V product the popcount path must equal
                    (snn_compiler/tests/test_spike_attention.py:142-150).
  vgg16_active.npz  VGGSNN.forward (snn_compiler/zoo/vgg.py:88-115) of the config-0
                    VGG16 (pool='max', 10 classes, 32x32 input, BN folded with
                    fold_conv_bn, spike-input layers with bf16-valued weights) with
                    every LIFNode running naive_if_lif; plus the calibrated BN / linear
                    parameters that keep the network spiking (oracle/vgg.py
                    calibrate_active), so the fixture is self-contained.
  ssa.npz           the reference test suite's mini Spikingformer block _RefSSA
                    (snn_compiler/tests/test_spike_attention.py:55-80) on spike input.
  cuba_eif.npz      naive_cuba_lif / naive_eif (snn_compiler/kernels/neurons.py:505-557)
                    over the matrix of snn_compiler/tests/test_correctness.py:111-155
                    (soft/hard x v_reset) and the decay overrides of :294-328, plus
                    per-channel thresholds.

``--only NAME[,NAME]`` regenerates just the named fixtures (file stems).

The fixtures are small; the tests that read them never need the reference.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def lif_cases(ref):
    naive = ref.naive_if_lif
    out = {}
    idx = 0

    def add(tag, x, spikes, meta):
        nonlocal idx
        k = f"c{idx:04d}"
        out[k + "_x"] = x.to(torch.float32).numpy()
        out[k + "_y"] = spikes.to(torch.float32).numpy().astype(np.uint8)
        for mk, mv in meta.items():
            if isinstance(mv, torch.Tensor):
                out[k + "_" + mk] = mv.numpy()
            else:
                out[k + "_" + mk] = np.asarray(mv)
        out[k + "_tag"] = np.asarray(tag)
        idx += 1

    shapes = [(4, 2, 8, 4, 4), (4, 8, 128), (3, 2, 3, 5, 7), (16, 2, 4, 3, 5)]
    seed = 100
    for shape in shapes:
        for neuron in ("if", "lif"):
            for soft in (True, False):
                for v_reset in (0.0, 0.3, -0.5):
                    if soft and v_reset != 0.0:
                        continue
                    for di in ((True, False) if neuron == "lif" else (True,)):
                        modes = [("scalar", "NCHW"), ("per_c", "NCHW"), ("per_n", "NCHW")]
                        if len(shape) == 5:
                            modes.append(("per_c", "NHWC"))
                        for thr_mode, layout in modes:
                            seed += 1
                            g = _gen(seed)
                            x = torch.randn(*shape, generator=g)
                            if thr_mode == "scalar":
                                thr = 1.0
                            elif thr_mode == "per_c":
                                C = shape[2] if len(shape) == 5 else shape[-1]
                                thr = torch.rand(C, generator=g) * 0.5 + 0.5
                            else:
                                thr = (torch.rand(*shape[1:], generator=g) * 0.5 + 0.5).reshape(-1)
                            xin = x
                            if layout == "NHWC":
                                T_, B_, C_, H_, W_ = shape
                                xin = x.reshape(T_ * B_, C_, H_, W_).contiguous(
                                    memory_format=torch.channels_last).view(T_, B_, C_, H_, W_)
                            y = naive(xin, neuron=neuron, tau=2.0, decay_input=di,
                                      soft_reset=soft, v_threshold=thr, v_reset=v_reset,
                                      layout=layout)
                            add("matrix", x, y, dict(neuron=neuron, soft=soft, v_reset=v_reset,
                                                     di=di, thr=thr, thr_mode=thr_mode,
                                                     layout=layout, dtype="float32",
                                                     tau=2.0, decay=np.nan))
    # dtypes (test_correctness.py:231-250)
    for dt in ("float32", "bfloat16", "float16"):
        seed += 1
        x = torch.randn(4, 2, 8, 8, 8, generator=_gen(seed)).to(getattr(torch, dt))
        y = naive(x, neuron="lif", tau=2.0, decay_input=True, soft_reset=False,
                  v_threshold=1.0, v_reset=0.0)
        add("dtype", x, y, dict(neuron="lif", soft=False, v_reset=0.0, di=True, thr=1.0,
                                thr_mode="scalar", layout="NCHW", dtype=dt, tau=2.0,
                                decay=np.nan))
    # decay overrides (test_correctness.py:253-292)
    for d in (0.0, 0.5, 0.9, 1.0):
        seed += 1
        x = torch.randn(4, 2, 16, 4, 4, generator=_gen(seed))
        y = naive(x, neuron="if", decay=d, soft_reset=False, v_threshold=1.0, v_reset=0.0)
        add("decay", x, y, dict(neuron="if", soft=False, v_reset=0.0, di=True, thr=1.0,
                                thr_mode="scalar", layout="NCHW", dtype="float32", tau=2.0,
                                decay=d))
    for d in (0.3, 0.7, 0.99):
        for di in (True, False):
            seed += 1
            x = torch.randn(4, 2, 16, 4, 4, generator=_gen(seed))
            y = naive(x, neuron="lif", tau=2.0, decay=d, decay_input=di, soft_reset=False,
                      v_threshold=1.0, v_reset=0.0)
            add("decay", x, y, dict(neuron="lif", soft=False, v_reset=0.0, di=di, thr=1.0,
                                    thr_mode="scalar", layout="NCHW", dtype="float32",
                                    tau=2.0, decay=d))
    # non-default tau (exercises non-exact products under the no-FMA rule)
    for tau in (3.0, 1.7):
        for soft in (True, False):
            seed += 1
            x = torch.randn(8, 2, 8, 4, 4, generator=_gen(seed))
            y = naive(x, neuron="lif", tau=tau, decay_input=True, soft_reset=soft,
                      v_threshold=0.8, v_reset=0.1 if not soft else 0.0)
            add("tau", x, y, dict(neuron="lif", soft=soft, v_reset=0.1 if not soft else 0.0,
                                  di=True, thr=0.8, thr_mode="scalar", layout="NCHW",
                                  dtype="float32", tau=tau, decay=np.nan))
    out["n_cases"] = np.asarray(idx)
    # rate-coded sums (test_largeT_and_rate.py:71-103): count = sum_t naive spikes
    r = 0
    for T in (4, 16):
        for soft in (True, False):
            for neuron, decay in (("lif", None), ("if", 1.0), ("if", 0.95)):
                seed += 1
                x = torch.randn(T, 2, 8, 6, 6, generator=_gen(seed))
                y = naive(x, neuron=neuron, tau=2.0, decay=decay, decay_input=True,
                          soft_reset=soft, v_threshold=1.0, v_reset=0.0).sum(0)
                k = f"r{r:03d}"
                out[k + "_x"] = x.numpy()
                out[k + "_count"] = y.numpy()
                out[k + "_meta"] = np.asarray([neuron, str(decay), str(soft)])
                r += 1
    out["n_rate"] = np.asarray(r)
    return out


def fold_case(ref):
    g = _gen(7)
    w = torch.randn(16, 8, 3, 3, generator=g)
    b = torch.randn(16, generator=g)
    gamma = torch.rand(16, generator=g) + 0.5
    beta = torch.randn(16, generator=g) * 0.1
    mean = torch.randn(16, generator=g)
    var = torch.rand(16, generator=g) + 0.1
    nw, nb = ref.fold_conv_bn(w, b, gamma, beta, mean, var, 1e-5)
    return dict(w=w.numpy(), b=b.numpy(), gamma=gamma.numpy(), beta=beta.numpy(),
                mean=mean.numpy(), var=var.numpy(), eps=np.asarray(1e-5),
                new_w=nw.numpy(), new_b=nb.numpy())


def bitpack_case(ref_root):
    path = os.path.join(ref_root, "snn_compiler", "explore", "attention", "phase6b_bitpack.py")
    spec = importlib.util.spec_from_file_location("_ref_bitpack", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    g = _gen(11)
    x = (torch.rand(3, 70, 16, generator=g) < 0.3).float()
    packed = mod.bitpack_N(x)                     # [TBH, d, W] int32
    k = (torch.rand(4, 2, 4, 70, 16, generator=g) < 0.1).float()
    v = (torch.rand(4, 2, 4, 70, 16, generator=g) < 0.15).float()
    kv = k.transpose(-2, -1) @ v
    return dict(x=x.numpy().astype(np.uint8), packed=packed.numpy(),
                k=k.numpy().astype(np.uint8), v=v.numpy().astype(np.uint8), kv=kv.numpy())


def vgg_case(ref):
    sys.path.insert(0, REPO)
    from oracle import params as OP, vgg as OV
    import torch.nn as nn
    from snn_compiler.zoo.vgg import VGGSNN, VGG16_CFG
    from snn_compiler.nn import modules as M

    P = OP.vgg16_params(1)
    x = OP.vgg16_input(0, T=4, B=8)
    OV.calibrate_active(P, x)
    layers, fcs = OV.folded_layers(P, weights="b200")

    model = VGGSNN(VGG16_CFG, num_classes=10, with_bn=False, neuron="lif", tau=2.0,
                   decay_input=True, soft_reset=False, v_threshold=1.0, v_reset=0.0,
                   layout="NCHW", pool="max")
    model.classifier[0] = nn.Linear(512, 4096)
    convs = [m for m in model.features if isinstance(m, nn.Conv2d)]
    lins = [m for m in model.classifier if isinstance(m, nn.Linear)]
    with torch.no_grad():
        for m, l in zip(convs, layers):
            m.weight.copy_(l["w"])
            m.bias.copy_(l["b"])
        for m, f in zip(lins, fcs):
            m.weight.copy_(f["w"])
            m.bias.copy_(f["b"])

    def lif_fwd(self, x_seq):
        return ref.naive_if_lif(x_seq.contiguous(), neuron="lif", tau=self.tau,
                                decay=self.decay, decay_input=self.decay_input,
                                soft_reset=self.soft_reset, v_threshold=self.v_threshold,
                                v_reset=self.v_reset, layout=self.layout)
    M.LIFNode.forward = lif_fwd
    model.eval()
    with torch.no_grad():
        logits = model(x)
    rec = {"logits": logits.numpy(), "x_seed": np.asarray(0), "w_seed": np.asarray(1),
           "T": np.asarray(4), "B": np.asarray(8)}
    for i, c in enumerate(P["convs"]):
        for key in ("mean", "var", "beta"):
            rec[f"conv{i}_{key}"] = c[key].numpy()
    for j, f in enumerate(P["fcs"][:-1]):
        rec[f"fc{j}_sd"] = f["sd"].numpy()
        rec[f"fc{j}_b"] = f["b"].numpy()
    return rec


def ssa_case(ref_root):
    path = os.path.join(ref_root, "snn_compiler", "tests", "test_spike_attention.py")
    spec = importlib.util.spec_from_file_location("_ref_attn_test", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    torch.manual_seed(0)
    blk = mod._RefSSA(C=32, heads=4).eval()
    x = (torch.rand(4, 2, 32, 8, 8) < 0.3).float()
    with torch.no_grad():
        y = blk(x)
    rec = {"x": x.numpy().astype(np.uint8), "y": y.numpy()}
    for k, v in blk.state_dict().items():
        rec["p_" + k.replace(".", "__")] = v.numpy()
    return rec


def cuba_eif_cases(N):
    """Reference naive_cuba_lif / naive_eif on seeded inputs; kwargs kept as JSON."""
    import json
    out = {}
    idx = 0
    seed = 900

    def add(model, x, y, kw):
        nonlocal idx
        k = f"c{idx:04d}"
        out[k + "_x"] = x.numpy()
        out[k + "_y"] = y.numpy().astype(np.uint8)
        out[k + "_model"] = np.asarray(model)
        kw = dict(kw)
        thr = kw.pop("v_threshold")
        out[k + "_thr"] = thr.numpy() if isinstance(thr, torch.Tensor) else np.float32(thr)
        out[k + "_kw"] = np.asarray(json.dumps(kw))
        idx += 1

    shapes = [(4, 2, 8, 4, 4), (8, 3, 16), (6, 2, 3, 5, 7)]
    for shape in shapes:
        for soft in (True, False):
            for v_reset in (0.0, -0.3):
                if soft and v_reset != 0.0:
                    continue
                # thresholds: scalar, per neuron, per channel (the reference's naive
                # versions take a [C] threshold only for 5-D CubaLIF input)
                for thr_mode in ("scalar", "per_n", "per_c"):
                    if thr_mode == "per_c" and len(shape) != 5:
                        continue
                    seed += 1
                    g = _gen(seed)
                    x = torch.randn(*shape, generator=g)
                    C = shape[2] if len(shape) == 5 else shape[-1]
                    if thr_mode == "scalar":
                        thr = 1.0
                    elif thr_mode == "per_c":
                        thr = torch.rand(C, generator=g) * 0.5 + 0.75
                    else:
                        thr = (torch.rand(*shape[1:], generator=g) * 0.5 + 0.75).reshape(-1)
                    kw = dict(tau_syn=2.0, tau_mem=4.0, soft_reset=soft, v_threshold=thr,
                              v_reset=v_reset)
                    add("cuba", x, N.naive_cuba_lif(x, **kw), kw)
                    if thr_mode == "per_c":
                        continue
                    kw = dict(tau=2.0, delta_T=1.0, v_rh=0.5, soft_reset=soft,
                              v_threshold=thr, v_reset=v_reset)
                    add("eif", x, N.naive_eif(x, **kw), kw)
    for ds, dm in ((0.0, 0.9), (0.5, 0.5), (0.7, 0.3), (1.0, 0.8)):
        seed += 1
        x = torch.randn(4, 4, 16, 8, 8, generator=_gen(seed))
        kw = dict(tau_syn=2.0, tau_mem=4.0, decay_syn=ds, decay_mem=dm, soft_reset=False,
                  v_threshold=1.0, v_reset=0.0)
        add("cuba", x, N.naive_cuba_lif(x, **kw), kw)
    for d in (0.0, 0.5, 1.0):
        seed += 1
        x = torch.randn(4, 4, 16, 8, 8, generator=_gen(seed)) * 0.3
        kw = dict(tau=2.0, decay=d, delta_T=1.0, v_rh=0.5, soft_reset=False,
                  v_threshold=1.0, v_reset=0.0)
        add("eif", x, N.naive_eif(x, **kw), kw)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    import snn_compiler.kernels.neurons as N
    import snn_compiler.kernels.fused as Fz

    class _Ref:
        naive_if_lif = staticmethod(N.naive_if_lif)
        fold_conv_bn = staticmethod(Fz.fold_conv_bn)

    makers = {
        "lif_cases": lambda: lif_cases(_Ref),
        "fold_bn": lambda: fold_case(_Ref),
        "bitpack": lambda: bitpack_case(args.reference),
        "ssa": lambda: ssa_case(args.reference),
        "vgg16_active": lambda: vgg_case(_Ref),
        "cuba_eif": lambda: cuba_eif_cases(N),
    }
    only = [n for n in args.only.split(",") if n] or list(makers)
    for name in only:
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **makers[name]())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
