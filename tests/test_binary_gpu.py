"""K4 parity: bit packing and the popcount binary GEMM vs the integer oracle
(bit-exact), including the reference's golden bit-pack and the BASELINE shapes
through size-independent row / column checksums."""
import numpy as np
import pytest
import torch

from oracle import bitops as OB
from oracle import params as OP
from test_oracle_golden import _load

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _B():
    from snn_compiler.kernels import binary
    return binary


def test_bitpack_matches_reference_golden():
    g = _load("bitpack.npz")
    x = torch.from_numpy(np.ascontiguousarray(np.swapaxes(g["x"], 1, 2))).float().to(DEV)
    p = _B().bitpack(x, ldw=(70 + 31) // 32)
    assert np.array_equal(p.cpu().numpy().view(np.uint32), g["packed"].view(np.uint32))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.uint8])
@pytest.mark.parametrize("K", [1, 31, 32, 33, 200, 1024, 4099])
def test_bitpack_against_oracle(dtype, K):
    g = OP.gen(K)
    x = (torch.rand(37, K, generator=g) < 0.3)
    p = _B().bitpack(x.to(dtype).to(DEV))
    ref = OB.pack_rows(x.numpy())
    ldw = p.shape[1]
    assert ldw % 4 == 0
    got = p.cpu().numpy().view(np.uint32)
    assert np.array_equal(got[:, :ref.shape[1]], ref) and not got[:, ref.shape[1]:].any()


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("shape", [(1, 1, 1), (100, 333, 77), (128, 1024, 128),
                                   (257, 4100, 130), (64, 25088, 96)])
def test_bgemm_exact_against_int_matmul(mode, shape):
    M, K, N = shape
    g = OP.gen(M * 7 + K + N + mode)
    A = (torch.rand(M, K, generator=g) < 0.2)
    Bb = (torch.rand(K, N, generator=g) < 0.5)
    Ai = A.long() if mode != 2 else A.long() * 2 - 1
    Bi = Bb.long() if mode == 0 else Bb.long() * 2 - 1
    ref = OB.int_matmul(Ai.numpy(), Bi.numpy())
    Bin = _B()
    Ap = Bin.bitpack(A.to(torch.uint8).to(DEV))
    Bp = Bin.bitpack(Bb.t().contiguous().to(torch.uint8).to(DEV))
    for splits in (1, 0, 3):
        C = Bin.bgemm(Ap, Bp, K, mode=mode, splits=splits)
        assert np.array_equal(C.cpu().numpy().astype(np.int64), ref), (mode, shape, splits)


@pytest.mark.parametrize("MKN", [(4096, 4096, 4096), (16384, 8192, 8192), (256, 25088, 4096)])
def test_bgemm_baseline_shapes_checksums(MKN):
    """Full BASELINE sizes: exact row and column sums (A @ (B 1), (1^T A) @ B) and an
    exact random sample of 4096 entries."""
    M, K, N = MKN
    A, Bb = OP.binary_gemm_operands(4, M, K, N)
    Bpm = Bb.to(torch.int64) * 2 - 1
    Bin = _B()
    Ap = Bin.bitpack(A.to(DEV))
    Bp = Bin.bitpack(Bb.t().contiguous().to(DEV))
    C = Bin.bgemm(Ap, Bp, K, mode=1)
    row, col = OB.bgemm_row_col_checksums(A.numpy(), Bpm.numpy())
    assert np.array_equal(C.sum(1, dtype=torch.int64).cpu().numpy(), row)
    assert np.array_equal(C.sum(0, dtype=torch.int64).cpu().numpy(), col)
    g = OP.gen(5)
    mi = torch.randint(0, M, (4096,), generator=g)
    ni = torch.randint(0, N, (4096,), generator=g)
    ref = (A[mi].long() * Bpm[:, ni].t()).sum(1)
    assert torch.equal(C[mi.to(DEV), ni.to(DEV)].cpu().long(), ref)


def test_popc_peak_helper_runs_and_leaves_sink():
    """snnb_popc_peak (the binary GEMM's roofline denominator) launches, reports success and
    never writes its sink (the sum it guards against does not occur)."""
    from snn_compiler import _lib
    sink = torch.full((256,), 7, dtype=torch.int32, device=DEV)
    L = _lib.lib()
    _lib.check(L.snnb_popc_peak(8, 16, _lib.ptr(sink), _lib.stream_of(sink)), "snnb_popc_peak")
    torch.cuda.synchronize()
    assert torch.all(sink == 7)
    assert L.snnb_popc_peak(0, 16, _lib.ptr(sink), _lib.stream_of(sink)) == -1
