"""The no-allocation conv entry point, snnb_conv3x3_lif_static_scratch.

Some hosts cannot give this library memory: a plugin interface with no scratch buffer,
or a runtime that forbids cudaMalloc (and the device-wide synchronisation it may cause)
once it is running.  For them the split-K conv keeps its partial sums in a fixed array
inside the library instead of a caller workspace.  This test calls that entry point
through the C ABI twice in a row and compares each result with the ordinary entry point
(caller workspace) on the same inputs: the kernels and their summation order are the
same, so the spikes must be identical.  It also checks that a request larger than the
fixed array is refused.  The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(seed, T=4, B=64, H=2, Cin=512, Cout=512):
    g = torch.Generator().manual_seed(seed)
    x = (torch.rand(T, B, H, H, Cin, generator=g) < 0.15).to(torch.bfloat16).to(DEV)
    w = (torch.randn(Cout, 3, 3, Cin, generator=g) * (2.0 / (9 * Cin)) ** 0.5)
    b = (torch.rand(Cout, generator=g) * 0.9 + 0.3).to(DEV)
    return x, w.to(torch.bfloat16).contiguous().to(DEV), b


def _static_call(x, w, b, out, splits, pool):
    from snn_compiler import _lib
    T, B, H, W, Cin = x.shape
    Cout = w.shape[0]
    st = _lib.lib().snnb_conv3x3_lif_static_scratch(
        _lib.ptr(x), T, B, H, W, Cin, _lib.ptr(w), _lib.ptr(b), Cout, 0.5, 0.5, 1.0, 0.0, 1,
        int(pool), 128, splits, _lib.ptr(out), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return st


@pytest.mark.parametrize("pool", [False, True])
def test_static_scratch_matches_workspace_entry_twice(pool):
    from snn_compiler.kernels import conv as KC
    for call, seed in enumerate((1, 2)):
        x, w, b = _case(seed)
        T, B, H, W, _ = x.shape
        Ho = H // 2 if pool else H
        ref = KC.conv3x3_lif(x, w, b, pool=pool, variant=2, block_n=128, splits=4)
        out = torch.full((T, B, Ho, Ho, w.shape[0]), 7.0, device=DEV, dtype=torch.bfloat16)
        assert _static_call(x, w, b, out, 4, pool) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"call {call}: {(out != ref).sum().item()} spikes differ"
        assert ref.float().sum() > 0


def test_static_scratch_rejects_oversized_requests():
    from snn_compiler.kernels import conv as KC
    x, w, b = _case(3, B=64, H=8, Cin=64, Cout=512)          # 8 x 4 x 64 x 64 x 512 x 4 B > 16 MiB
    assert KC.split_workspace_bytes(4, 64, 8, 8, 512, 8) > (16 << 20)
    out = torch.empty(4, 64, 8, 8, 512, device=DEV, dtype=torch.bfloat16)
    assert _static_call(x, w, b, out, 8, False) == -1
