"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/snnb200.h declares, and rejects bad arguments before touching a device."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "snnb200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(snnb_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    from snn_compiler import _lib
    L = _lib.lib()
    names = declared_functions()
    assert "snnb_neuron_multistep" in names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert L.snnb_abi_version() >= 1


def test_every_declared_entry_has_a_python_signature():
    from snn_compiler import _lib
    helpers = {"snnb_abi_version", "snnb_status_string", "snnb_last_cuda_error",
               "snnb_split_workspace_bytes", "snnb_first_conv_tc_weight_k",
               "snnb_linear_t_workspace_bytes"}
    for n in declared_functions():
        if n not in helpers:
            assert n in _lib.SIGNATURES, n


def test_status_strings():
    from snn_compiler import _lib
    L = _lib.lib()
    assert L.snnb_status_string(0) == b"ok"
    assert L.snnb_status_string(-1) == b"invalid argument"
    assert L.snnb_status_string(-4) == b"device wait timed out"


def test_neuron_rejects_bad_arguments_without_a_device():
    from snn_compiler import _lib
    L = _lib.lib()
    f = L.snnb_neuron_multistep
    base = dict(x=None, xd=0, T=4, N=16, bias=None, res=None, C=1, HW=1, cl=0, df=0.5, sc=0.5,
                w=None, hard=1, vr=0.0, mode=0, ts=1.0, thr=None, vinit=None, sp=None, sd=0,
                pk=None, cnt=None, vo=None, st=None)

    def call(**kw):
        a = {**base, **kw}
        return f(*a.values())
    assert call(T=-1) == -1                      # negative T
    assert call(N=-5) == -1                      # negative N
    assert call(xd=7) == -1                      # unknown x dtype
    assert call(mode=1) == -1                    # per-channel threshold without a pointer
    assert call(mode=9) == -1                    # unknown threshold mode
    assert call(x=None) == -1                    # T > 0 with no input
    assert call(N=0) == 0                        # empty input is a no-op


def test_split_workspace_size_overflow_is_rejected():
    """A byte count that overflows int64 comes back negative (not wrapped to a small or
    negative size that would pass a capacity check), and the no-allocation entry refuses it
    before touching a device."""
    from snn_compiler import _lib
    L = _lib.lib()
    big = 0x7fffffff
    assert L.snnb_split_workspace_bytes(4, 64, 32, 32, 64, 1) == 0
    assert L.snnb_split_workspace_bytes(4, 64, 32, 32, 64, 2) == 2 * 4 * 64 * 32 * 32 * 64 * 4
    assert L.snnb_split_workspace_bytes(big, big, big, big, big, 8) < 0
    assert L.snnb_split_workspace_bytes(-4, 1, 1, 1, 64, 2) < 0
    st = L.snnb_conv3x3_lif_static_scratch(
        None, big, big, big, big, 64, None, None, big, 0.5, 0.5, 1.0, 0.0, 1, 0, 0, 8, None,
        None)
    assert st == -1


def test_strided_conv_entries_reject_bad_geometry_without_a_device():
    """Kernel sizes other than 1 / 3 / 5 / 7, strides other than 1 / 2, a missing input and
    oversized dimensions come back SNNB_ERR_ARG before any device work."""
    from snn_compiler import _lib
    L = _lib.lib()

    def strided(**kw):
        a = dict(x=None, T=4, B=2, H=8, W=8, Cin=64, w=None, b=None, Cout=64, k=3, s=2,
                 df=0.5, sc=0.5, thr=1.0, vr=0.0, hard=1, res=None, rdt=0, v=0, bn=0, sp=1,
                 ws=None, wsb=0, out=None, st=None)
        a.update(kw)
        return L.snnb_conv_lif_strided(*a.values())

    def f32(**kw):
        a = dict(x=None, T=4, B=2, H=8, W=8, Cin=64, w=None, b=None, Cout=64, k=1, s=2,
                 out=None, st=None)
        a.update(kw)
        return L.snnb_conv_f32(*a.values())
    for call in (strided, f32):
        assert call(k=4) == -1
        assert call(k=9) == -1
        assert call(k=2) == -1
        assert call(s=3) == -1
        assert call(s=0) == -1
        assert call() == -1                       # no input / weight / output pointers
        assert call(T=1 << 40) == -1
    assert strided(res=ctypes.c_void_p(16), rdt=7) == -1     # unknown residual dtype


def test_stem_data_movement_entries_reject_bad_arguments_without_a_device():
    """snnb_maxpool_nhwc and snnb_window_gather_nhwc: missing pointers, channel counts the
    16-byte layout cannot hold, windows that could lie wholly in the padding, and a padded
    width below the window all come back SNNB_ERR_ARG before any device work."""
    from snn_compiler import _lib
    L = _lib.lib()
    p16 = ctypes.c_void_p(1 << 20)          # aligned stand-ins: rejected before any access

    def pool(**kw):
        a = dict(x=p16, F=2, H=8, W=8, C=64, k=3, s=2, pad=1, out=p16, st=None)
        a.update(kw)
        return L.snnb_maxpool_nhwc(*a.values())

    def gather(**kw):
        a = dict(x=p16, F=2, H=8, W=8, C=3, k=7, s=2, pad=3, Kp=152, out=p16, st=None)
        a.update(kw)
        return L.snnb_window_gather_nhwc(*a.values())
    for call in (pool, gather):
        assert call(x=None) == -1
        assert call(out=None) == -1
        assert call(k=0) == -1
        assert call(s=0) == -1
        assert call(pad=-1) == -1
        assert call(H=0) == -1
        assert call(F=0) == 0                       # nothing to do
    assert pool(C=60) == -1                         # not a multiple of 8 channels
    assert pool(k=3, pad=3) == -1                   # pad >= k: a window in the padding
    assert pool(out=ctypes.c_void_p((1 << 20) + 8)) == -1     # misaligned output
    assert gather(Kp=144) == -1                     # below k*k*C = 147
    assert gather(Kp=150) == -1                     # not a multiple of 8
