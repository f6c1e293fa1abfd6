"""Pin the CPU oracle to the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by tests/golden/make_golden.py running the
reference's Python code; these tests need neither the reference nor a GPU.
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import attention as OA
from oracle import bitops as OB
from oracle import neurons as ON
from oracle import params as OP
from oracle import vgg as OV


def _load(name):
    return dict(np.load(os.path.join(GOLDEN, name), allow_pickle=False))


LIF = _load("lif_cases.npz")
N_CASES = int(LIF["n_cases"])


def lif_case(i):
    k = f"c{i:04d}"
    meta = {m: LIF[k + "_" + m] for m in ("neuron", "soft", "v_reset", "di", "thr", "thr_mode",
                                           "layout", "dtype", "tau", "decay", "tag")}
    meta = {m: (v.item() if v.ndim == 0 else v) for m, v in meta.items()}
    return LIF[k + "_x"], LIF[k + "_y"], meta


def run_oracle_case(x, meta):
    xt = torch.from_numpy(x).to(getattr(torch, meta["dtype"]))
    decay = None if np.isnan(meta["decay"]) else float(meta["decay"])
    thr = meta["thr"]
    thr = float(thr) if np.ndim(thr) == 0 else torch.from_numpy(np.asarray(thr, np.float32))
    if meta["layout"] == "NHWC":
        T_, B_, C_, H_, W_ = xt.shape
        xt = xt.reshape(T_ * B_, C_, H_, W_).contiguous(
            memory_format=torch.channels_last).view(T_, B_, C_, H_, W_)
    y = ON.naive_if_lif(xt, neuron=meta["neuron"], tau=float(meta["tau"]), decay=decay,
                        decay_input=bool(meta["di"]), soft_reset=bool(meta["soft"]),
                        v_threshold=thr, v_reset=float(meta["v_reset"]), layout=meta["layout"])
    return y.to(torch.float32).numpy()


@pytest.mark.parametrize("i", range(N_CASES))
def test_lif_matrix_bit_exact(i):
    x, y, meta = lif_case(i)
    out = run_oracle_case(x, meta)
    assert np.array_equal(out.astype(np.uint8), y), meta


def test_lif_rate_counts_exact():
    for r in range(int(LIF["n_rate"])):
        k = f"r{r:03d}"
        neuron, decay, soft = [str(s) for s in LIF[k + "_meta"]]
        x = LIF[k + "_x"]
        T = x.shape[0]
        C, HW = ON.infer_C_HW(x.shape)
        df, sc = ON.neuron_params(neuron, tau=2.0, decay=None if decay == "None" else float(decay))
        o = ON.lif_multistep(x.reshape(T, -1), df=df, sc=sc, hard_reset=soft != "True",
                             thr=1.0, want_spikes=False, want_count=True)
        assert np.array_equal(o["count"], LIF[k + "_count"].reshape(-1)), k


def test_plif_identity_with_lif_tau2():
    """PLIF with w = 0 has k = sigmoid(0) = 0.5 exactly: identical to LIF tau=2."""
    df, sc = ON.neuron_params("plif", plif_w=0.0)
    assert df == np.float32(0.5) and sc == np.float32(0.5)
    x = OP.lif_input(3, T=8, N=4096).numpy()
    a = ON.lif_multistep(x, df=df, sc=sc, want_v=True)
    b = ON.lif_multistep(x, *[], **dict(zip(("df", "sc"), ON.neuron_params("lif", tau=2.0))),
                         want_v=True)
    assert np.array_equal(a["spikes"], b["spikes"]) and np.array_equal(a["v"], b["v"])


def test_plif_spikingjelly_order_tracks_lif_tau2_at_k_half():
    """SpikingJelly's PLIF charge at k = 0.5 (init_tau 2), v + (x - v) * 0.5, against the
    reference LIF tau=2, 0.5 v + 0.5 x: the same spikes except where v sits at the threshold
    (the two round differently in the last bit), and the three charge forms of the restated
    ParametricLIFNode agree at v_reset = 0 where they must."""
    x = OP.lif_input(3, T=8, N=1 << 16).numpy()
    sj = ON.plif_sj_multistep(x, k=np.float32(0.5))
    ref = ON.lif_multistep(x, df=np.float32(0.5), sc=np.float32(0.5), want_vpre=True)
    mism = sj["spikes"] != ref["spikes"]
    assert mism.mean() < 1e-4
    assert (np.abs(ref["vpre"][mism] - 1.0) < 1e-5).all()
    # not decay_input with v_reset 0: the (1 - k) form; with v_reset != 0 the general form
    a = ON.plif_sj_multistep(x, k=np.float32(0.25), decay_input=False, v_reset=0.0)
    b = ON.plif_sj_multistep(x, k=np.float32(0.25), decay_input=False, v_reset=-0.5)
    assert a["spikes"].sum() > 0 and b["spikes"].sum() > 0


def test_stateful_chunks_compose():
    """v_out of one chunk as v_init of the next equals one full run
    (snn_compiler/tests/test_largeT_and_rate.py:106-132)."""
    x = OP.lif_input(4, T=32, N=2 * 16 * 14 * 14).numpy()
    df, sc = ON.neuron_params("lif", tau=2.0)
    for soft in (True, False):
        full = ON.lif_multistep(x, df=df, sc=sc, hard_reset=not soft, want_v=True)
        for chunk in (4, 8, 16):
            v = None
            parts = []
            for t0 in range(0, 32, chunk):
                o = ON.lif_multistep(x[t0:t0 + chunk], df=df, sc=sc, hard_reset=not soft,
                                     v_init=v, want_v=True)
                v = o["v"]
                parts.append(o["spikes"])
            assert np.array_equal(np.concatenate(parts), full["spikes"])
            assert np.array_equal(v, full["v"])


def test_fold_conv_bn_matches_reference():
    g = _load("fold_bn.npz")
    t = {k: torch.from_numpy(v) for k, v in g.items()}
    nw, nb = OV.fold_conv_bn(t["w"], t["b"], t["gamma"], t["beta"], t["mean"], t["var"],
                             float(g["eps"]))
    assert torch.equal(nw, t["new_w"]) and torch.equal(nb, t["new_b"])


def test_bitpack_matches_reference():
    g = _load("bitpack.npz")
    x = g["x"]                                            # [TBH, N, d]
    packed = OB.pack_rows(np.swapaxes(x, 1, 2))           # pack along tokens -> [TBH, d, W]
    assert np.array_equal(packed, g["packed"].view(np.uint32))


def test_ktv_popcount_equals_reference_bmm():
    g = _load("bitpack.npz")
    k = torch.from_numpy(g["k"].astype(np.float32))
    v = torch.from_numpy(g["v"].astype(np.float32))
    assert np.array_equal(OA.ktv_popcount(k, v).numpy(), g["kv"])
    assert np.array_equal(OA.ktv(k, v).numpy(), g["kv"])


def test_bgemm_oracle_equals_int_matmul():
    A, Bb = OP.binary_gemm_operands(3, 96, 200, 40)
    A = A.numpy()
    Bpm = Bb.numpy().astype(np.int64) * 2 - 1
    Ap = OB.pack_rows(A)
    Bp = OB.pack_rows(Bb.numpy().T)
    assert np.array_equal(OB.bgemm_01_pm1(Ap, Bp), OB.int_matmul(A, Bpm))
    row, col = OB.bgemm_row_col_checksums(A, Bpm)
    C = OB.int_matmul(A, Bpm)
    assert np.array_equal(row, C.sum(1)) and np.array_equal(col, C.sum(0))


def test_ssa_block_matches_reference():
    g = _load("ssa.npz")
    sd = {k[2:].replace("__", "."): v for k, v in g.items() if k.startswith("p_")}
    C = 32
    P = OA.ssa_params_from_ref_state(sd, C)
    x = torch.from_numpy(g["x"].astype(np.float32))      # [T,B,C,H,W]
    T, B, _, H, W = x.shape
    xt = x.flatten(3).transpose(2, 3).contiguous()        # [T,B,N,C]
    out = OA.ssa_forward(xt, P, heads=4, in_vth=0.3, qkv_vth=0.3, attn_vth=0.5,
                         out_vth=None, fold=False)
    ref = torch.from_numpy(g["y"]).flatten(3).transpose(2, 3)
    assert torch.allclose(out, ref, atol=1e-5, rtol=1e-5), (out - ref).abs().max()


def test_vgg16_matches_reference_forward():
    g = _load("vgg16_active.npz")
    P = OV.apply_active(OP.vgg16_params(int(g["w_seed"])), g)
    x = OP.vgg16_input(int(g["x_seed"]), T=int(g["T"]), B=int(g["B"]))
    logits = OV.vgg16_forward(x, P, bn="folded", weights="b200")
    ref = torch.from_numpy(g["logits"])
    assert torch.equal(logits.mean(0).argmax(-1), ref.mean(0).argmax(-1))
    assert torch.allclose(logits, ref, rtol=1e-3, atol=1e-3), (logits - ref).abs().max()


CE = _load("cuba_eif.npz")
CE_CASES = sorted({k[:5] for k in CE if k.startswith("c") and k.endswith("_x")})


@pytest.mark.parametrize("k", CE_CASES)
def test_cuba_eif_oracle_matches_reference(k):
    """CubaLIF bit-exact; EIF (exp of numpy vs torch) may flip a spike only where the
    charged potential lies within 1e-5 of the threshold."""
    import json
    x = torch.from_numpy(CE[k + "_x"])
    y = CE[k + "_y"].reshape(x.shape[0], -1)
    model = CE[k + "_model"].item()
    kw = json.loads(CE[k + "_kw"].item())
    thr = CE[k + "_thr"]
    kw["v_threshold"] = float(thr) if thr.ndim == 0 else thr
    r = ON.naive_cuba_eif(model, x, want_vpre=True, **kw)
    got = r["spikes"].astype(np.uint8)
    if model == "cuba":
        assert np.array_equal(got, y), (k, kw)
    else:
        bad = got != y
        T, N = got.shape
        th = ON._thr_per_neuron(kw["v_threshold"], T, N, *ON.infer_C_HW(tuple(x.shape)), False)
        near = np.abs(r["vpre"] - th[None, :]) <= 1e-5
        assert not (bad & ~near).any(), (k, int(bad.sum()))
        assert bad.mean() <= 1e-3
