"""Tail and ragged shapes run through whichever library SNNB_LIBRARY names (the bounds tests
run it once with the release build and once with the bounds-checking debug build,
libsnnb200_check.so, in separate processes).  Saves every output and the device status
word to the path given as argv[1]."""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "triton-pass-analysis_b200"))
sys.path.insert(0, REPO)


def main(path):
    import torch
    from snn_compiler.kernels import conv as KC
    from snn_compiler.kernels import neurons as K
    dev = "cuda"
    g = torch.Generator().manual_seed(5)
    out = {}
    # K2: vector and scalar paths, ragged N, every output
    for N in (999, 1000, 4104, 33):
        x = (torch.randn(3, N, generator=g) + 0.6).to(dev)
        r = K.neuron_multistep(x.view(3, 1, N), decay_factor=0.5, input_scale=0.5, packed=True,
                               count=True, v_out=True)
        for k, v in r.items():
            out[f"lif{N}_{k}"] = v.cpu()
    # K1: partial pixel blocks and channel blocks, pooled and not, every schedule family
    cases = [((4, 3, 64, 64, 14), 2, 64, False), ((4, 3, 64, 64, 14), 1, 64, False),
             ((4, 1, 64, 64, 32), 3, 64, True), ((4, 1, 64, 64, 32), 7, 64, False),
             ((4, 3, 64, 128, 16), 7, 32, True), ((2, 5, 64, 128, 7), 1, 32, False),
             ((4, 2, 128, 256, 6), 2, 128, True), ((4, 2, 64, 128, 8), 3, 64, False)]
    for (T, B, Cin, Cout, H), v, bn, pool in cases:
        x = (torch.rand(T, B, H, H, Cin, generator=g) < 0.2).to(torch.bfloat16).to(dev)
        w = (torch.randn(Cout, 3, 3, Cin, generator=g) * 0.08).to(torch.bfloat16).to(dev)
        b = (torch.rand(Cout, generator=g) * 0.5 + 0.3).to(dev)
        y = KC.conv3x3_lif(x, w, b, pool=pool, variant=v, block_n=bn)
        out[f"conv{T}x{B}x{Cin}x{Cout}x{H}_v{v}_{bn}_{int(pool)}"] = y.cpu()
    # strided and k x k convs (general tap coordinates): ragged output sizes, residual,
    # split-K, the T-sequential and T-folded forms; the float32 conv; the stem's gather+pool
    scases = [((4, 3, 64, 128, 15, 13), 3, 2, 2, 128, 1, True),
              ((4, 2, 64, 64, 9, 7), 1, 2, 1, 32, 1, False),
              ((2, 3, 128, 64, 10, 10), 7, 2, 2, 64, 2, True),
              ((4, 2, 64, 64, 11, 11), 5, 1, 0, 0, 1, False)]
    for (T, B, Cin, Cout, H, W), k, st, v, bn, sp, res in scases:
        x = (torch.rand(T, B, H, W, Cin, generator=g) < 0.2).to(torch.bfloat16).to(dev)
        w = (torch.randn(Cout, k, k, Cin, generator=g) * 0.08).to(torch.bfloat16).to(dev)
        b = (torch.rand(Cout, generator=g) * 0.5 + 0.3).to(dev)
        Ho, Wo = (H - 1) // st + 1, (W - 1) // st + 1
        r = (torch.randn(T, B, Ho, Wo, Cout, generator=g) * 0.3).to(dev) if res else None
        y = KC.conv_lif_strided(x, w, b, stride=st, variant=v, block_n=bn, splits=sp, residual=r)
        out[f"sconv{T}x{B}x{Cin}x{Cout}x{H}x{W}_k{k}s{st}_v{v}"] = y.cpu()
        if T in (2, 4, 8):
            out[f"sconvf32{T}x{B}x{Cin}x{Cout}x{H}x{W}_k{k}s{st}"] = \
                KC.conv_f32(x, w, b, stride=st).cpu()
    img = torch.rand(2, 23, 19, 3, generator=g).to(torch.bfloat16).to(dev)
    out["gather"] = KC.window_gather_nhwc(img, 7, 2, 3).cpu()
    sp = (torch.rand(2, 13, 11, 64, generator=g) < 0.3).to(torch.bfloat16).to(dev)
    out["maxpool"] = KC.maxpool_nhwc(sp, 3, 2, 1).cpu()
    # image layer on the tensor cores: partial 128-pixel tiles
    for B, H, W in ((2, 7, 9), (3, 32, 32)):
        img = torch.rand(1, B, 3, H, W, generator=g).to(dev)
        w = torch.randn(64, 3, 3, 3, generator=g) * 0.3
        b = (torch.rand(64, generator=g) * 0.5 + 0.2).to(dev)
        y = KC.first_conv_lif_tc(img, KC.first_conv_split_weight(w).to(dev), b, T=4)
        out[f"first{B}x{H}x{W}"] = y.cpu()
    torch.cuda.synchronize()
    out["status"] = torch.tensor(KC.device_status())
    torch.save(out, path)


if __name__ == "__main__":
    main(sys.argv[1])
