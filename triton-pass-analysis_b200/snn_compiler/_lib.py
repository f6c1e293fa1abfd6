"""ctypes binding of libsnnb200.so (the C ABI declared in include/snnb200.h).

The library is built in-tree by ``make -C triton-pass-analysis_b200`` (or
``__graft_entry__.build()``).  There is no fallback: if the library is missing
or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes
import os

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# SNNB_LIBRARY selects another build of the same ABI, e.g. the bounds-checking debug build
# libsnnb200_check.so (`make -C triton-pass-analysis_b200 check`).
LIB_PATH = os.environ.get("SNNB_LIBRARY") or os.path.join(_PKG_DIR, "libsnnb200.so")

SNNB_OK = 0
STATUS = {-1: "invalid argument", -2: "unsupported combination", -3: "CUDA error",
          -4: "device wait timed out", -5: "device-side check failed"}

F32, F16, BF16, U8 = 0, 1, 2, 3
THR_SCALAR, THR_PER_CHANNEL, THR_PER_NEURON = 0, 1, 2

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F = ctypes.c_float

# name -> (argtypes) ; every entry returns int status
SIGNATURES = {
    "snnb_neuron_multistep": [P, I32, I64, I64, P, P, I64, I64, I32, F, F, P, I32, F, I32, F, P,
                              P, P, I32, P, P, P, P],
    "snnb_neuron_cuba_eif": [P, I32, I64, I64, I64, I64, I32, I32, F, F, F, F, F, I32, F, I32, F,
                             P, P, P],
    "snnb_bitpack": [P, I32, I64, I64, I64, I32, P, P],
    "snnb_bgemm": [P, P, P, I64, I64, I64, I64, I32, I32, P],
    "snnb_popc_peak": [I64, I32, P, P],
    "snnb_conv3x3_lif": [P, I64, I64, I64, I64, I64, P, P, I64, F, F, F, F, I32, I32, I32, I32,
                         I32, P, I64, P, P],
    "snnb_conv3x3_lif_res": [P, I64, I64, I64, I64, I64, P, P, I64, F, F, F, F, I32, P, I32, I32,
                             I32, I32, P, I64, P, P],
    "snnb_conv_lif_strided": [P, I64, I64, I64, I64, I64, P, P, I64, I32, I32, F, F, F, F, I32, P,
                              I32, I32, I32, I32, P, I64, P, P],
    "snnb_conv_f32": [P, I64, I64, I64, I64, I64, P, P, I64, I32, I32, P, P],
    "snnb_maxpool_nhwc": [P, I64, I64, I64, I64, I32, I32, I32, P, P],
    "snnb_window_gather_nhwc": [P, I64, I64, I64, I64, I32, I32, I32, I64, P, P],
    "snnb_linear_lif": [P, I64, I64, I64, P, P, I64, F, F, F, F, I32, I32, I32, I32, P, I64, P, P],
    "snnb_conv3x3_lif_packed": [P, I32, I64, I64, I64, I64, I64, P, P, I64, F, F, F, F, I32, I32,
                                I32, I32, P, P],
    "snnb_unpack_spikes": [P, I64, I64, P, P],
    "snnb_conv3x3_lif_dense": [P, I64, I64, I64, I64, I64, P, P, I64, F, F, F, F, I32, I32, I32,
                               I32, I32, P, I64, P, P],
    "snnb_linear_mean": [P, I64, I64, I64, P, P, I64, P, P],
    "snnb_linear_out": [P, I64, I64, I64, P, P, I64, P, P],
    "snnb_first_conv_lif": [P, I64, I64, I64, I64, I64, I64, P, P, I64, F, F, F, F, I32, I32, P,
                            P],
    "snnb_read_device_status": [P, P],
    "snnb_set_wait_limit": [I64],
    "snnb_linear_lif_t": [P, I64, I64, I64, P, P, I64, F, F, F, F, I32, I32, I32, P, I64, P, P],
    "snnb_first_conv_lif_tc": [P, I64, I64, I64, I64, I64, P, P, I64, F, F, F, F, I32, P, P],
    "snnb_neuron_plif": [P, I32, I64, I64, P, I32, I32, F, F, P, P, I32, P, P, P, P],
    "snnb_split_bf16_terms": [P, I64, I64, I64, P, P],
    "snnb_debug_inject_status": [I32, I32],
    "snnb_debug_inject_stall": [I32],
    "snnb_linear_f32": [P, I64, I64, I64, P, P, I64, P, P],
    "snnb_spike_attention_core": [P, P, P, I64, I64, I64, I64, P, P, P, I64, I64, I64, I64,
                                  I64, I64, I64, I64, I64, F, F, F, F, F, I32, P],
    "snnb_conv3x3_lif_static_scratch": [P, I64, I64, I64, I64, I64, P, P, I64, F, F, F, F, I32,
                                        I32, I32, I32, P, P],
}

_lib = None


class SnnbError(RuntimeError):
    pass


def lib():
    """Load libsnnb200.so once; raise if it is absent (no CPU fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libsnnb200 not built (expected at {LIB_PATH}); "
                              "run `make -C triton-pass-analysis_b200`")
        L = ctypes.CDLL(LIB_PATH)
        L.snnb_abi_version.restype = ctypes.c_int
        L.snnb_status_string.restype = ctypes.c_char_p
        L.snnb_status_string.argtypes = [ctypes.c_int]
        L.snnb_last_cuda_error.restype = ctypes.c_char_p
        L.snnb_split_workspace_bytes.restype = ctypes.c_int64
        L.snnb_split_workspace_bytes.argtypes = [I64, I64, I64, I64, I64, I32]
        L.snnb_linear_t_workspace_bytes.restype = ctypes.c_int64
        L.snnb_linear_t_workspace_bytes.argtypes = [I64, I64, I64, I32]
        L.snnb_first_conv_tc_weight_k.restype = ctypes.c_int64
        L.snnb_first_conv_tc_weight_k.argtypes = [I64]
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != SNNB_OK:
        L = lib()
        msg = L.snnb_status_string(status).decode()
        if status == -3:
            msg += ": " + L.snnb_last_cuda_error().decode()
        if status == -1:
            raise ValueError(f"{what}: {msg}")
        raise SnnbError(f"{what}: {msg} (status {status})")


def dtype_code(dt) -> int:
    import torch
    m = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.uint8: U8}
    if dt not in m:
        raise AssertionError(f"unsupported dtype {dt}")
    return m[dt]


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t):
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
