"""Seeded synthetic inputs and weights (test infrastructure; see oracle/__init__.py).

Everything is drawn on the HOST with ``torch.Generator().manual_seed(seed)`` so
the oracle and the CUDA kernels see identical bits.  Distributions are the
benchmark configurations':
  VGG16-SNN : image U(0,1) repeated over T; conv / linear weights Kaiming-normal
              (fan_in, gain sqrt 2); conv / linear bias U(+-1/sqrt(fan_in)) (torch's
              default bias init, as nn.Conv2d in snn_compiler/zoo/vgg.py:61 has bias);
              BN gamma U(0.8,1.2), beta N(0,0.1), running_mean N(0,0.1),
              running_var U(0.5,1.5), eps 1e-5, eval mode.
  LIF sweep : x ~ N(0.5, 1) float32 [T, N].
  conv sweep: Bernoulli(p) spikes [T, B, Cin, H, W].
  attention : Bernoulli(0.15) spikes [T, B, N, D]; weights N(0, 0.02).
  binary GEMM: A Bernoulli(0.2) {0,1} [M, K]; B {-1,+1} with p = 0.5 [K, N].
"""
from __future__ import annotations

import math

import torch

VGG16_CFG = [64, 64, "P", 128, 128, "P", 256, 256, 256, "P",
             512, 512, 512, "P", 512, 512, 512, "P"]      # snn_compiler/zoo/vgg.py:25


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(int(seed))


def conv_bn_params(g, cin, cout, k=3):
    fan_in = cin * k * k
    return {
        "w": torch.randn(cout, cin, k, k, generator=g) * math.sqrt(2.0 / fan_in),
        "b": (torch.rand(cout, generator=g) * 2 - 1) / math.sqrt(fan_in),
        "gamma": torch.rand(cout, generator=g) * 0.4 + 0.8,
        "beta": torch.randn(cout, generator=g) * 0.1,
        "mean": torch.randn(cout, generator=g) * 0.1,
        "var": torch.rand(cout, generator=g) + 0.5,
        "eps": 1e-5,
    }


def linear_params(g, fin, fout):
    return {
        "w": torch.randn(fout, fin, generator=g) * math.sqrt(2.0 / fin),
        "b": (torch.rand(fout, generator=g) * 2 - 1) / math.sqrt(fin),
    }


def vgg16_params(seed=1, *, num_classes=10, in_ch=3, fc_hidden=4096, cfg=VGG16_CFG,
                 fc_in=None):
    """Parameters of the VGG16-SNN (config 0).  fc_in defaults to the last conv width
    (32x32 input pools down to 1x1)."""
    g = gen(seed)
    convs = []
    ch = in_ch
    for v in cfg:
        if v == "P":
            convs[-1]["pool"] = True
            continue
        p = conv_bn_params(g, ch, v)
        p["pool"] = False
        convs.append(p)
        ch = v
    fc_in = ch if fc_in is None else fc_in
    fcs = [linear_params(g, fc_in, fc_hidden), linear_params(g, fc_hidden, fc_hidden),
           linear_params(g, fc_hidden, num_classes)]
    return {"convs": convs, "fcs": fcs, "num_classes": num_classes}


def vgg16_input(seed=0, *, T=4, B=8, C=3, H=32, W=32):
    """Direct encoding: one U(0,1) image per sample, repeated over T -> [T,B,C,H,W]."""
    img = torch.rand(B, C, H, W, generator=gen(seed))
    return img.unsqueeze(0).expand(T, B, C, H, W).contiguous()


def lif_input(seed=0, *, T=4, N=1 << 20):
    return torch.randn(T, N, generator=gen(seed)) + 0.5


def spikes(seed, shape, p):
    return (torch.rand(*shape, generator=gen(seed)) < p).to(torch.float32)


def binary_gemm_operands(seed, M, K, N):
    g = gen(seed)
    A = (torch.rand(M, K, generator=g) < 0.2).to(torch.uint8)
    Bbits = (torch.rand(K, N, generator=g) < 0.5).to(torch.uint8)     # 1 <=> +1
    return A, Bbits


def attention_params(seed=1, *, D=384, heads=12):
    g = gen(seed)
    P = {"heads": heads, "D": D}
    for nm in ("q", "k", "v", "proj"):
        P[nm] = {
            "w": torch.randn(D, D, generator=g) * 0.02,
            "b": torch.zeros(D),
            "gamma": torch.rand(D, generator=g) * 0.4 + 0.8,
            "beta": torch.randn(D, generator=g) * 0.1,
            "mean": torch.randn(D, generator=g) * 0.1,
            "var": torch.rand(D, generator=g) + 0.5,
            "eps": 1e-5,
        }
    return P
