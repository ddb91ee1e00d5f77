"""GEMM with a Q8_0 B operand dequantised in shared memory (through tb2_gemm).

The weight is quantised by the oracle's Q8_0 quantiser (ggml semantics); the
GEMM reads only its int8 quants and fp16 scales. Dequantisation happens in the
kernel's converter warps, which write the same split-bf16 tiles a TMA load of
dequantised planes would deliver -- so the result must be bit-identical to the
plane-operand GEMM over the dequantised weight, and within the split-bf16
accuracy (2e-5 relative) of an fp64 product. Both B orientations are covered:
K-major (forward y = x W^T) and MN-major (backward dX = dY W), with ragged
tile edges in every dimension.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests.test_gemm_gpu import _epi, _gemm, _operand, _relerr

pytestmark = pytest.mark.gpu


def _q8_operand(W, mn_major, cuda):
    """W: f32 numpy [rows][cols], cols % 32 == 0. Returns (operand, keepalive, dequantised W)."""
    import torch
    from toy_b200._lib import Operand
    rows, cols = W.shape
    blocks = O.q8_0_quantize(W).reshape(rows, cols // 32, 34)
    scales = np.ascontiguousarray(blocks[:, :, :2]).view(np.uint16).reshape(rows, cols // 32)
    quants = np.ascontiguousarray(blocks[:, :, 2:]).view(np.int8).reshape(rows, cols)
    deq = O.q8_0_dequantize(blocks.reshape(rows, -1), cols)
    tq = torch.from_numpy(quants.copy()).to(cuda)
    ts = torch.from_numpy(scales.view(np.int16).copy()).to(cuda)
    o = Operand()
    o.hi, o.lo = None, None
    o.mn_major, o.ld, o.rows, o.cols = mn_major, cols, rows, cols
    o.batch_stride, o.nbatch = rows * cols, 1
    o.bdiv1, o.bmul1, o.bdiv2, o.bmul2 = 1, 0, 1, 0
    o.q8, o.q8_scale = tq.data_ptr(), ts.data_ptr()
    return o, (tq, ts), deq


@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("M,N,K", [(256, 960, 576), (200, 576, 1536), (64, 64, 64), (130, 192, 96),
                                   (4096, 1536, 576), (128, 128, 2048)])
def test_gemm_q8_b(cuda, b_mn, M, N, K):
    import torch
    rng = np.random.default_rng(M * 31 + N * 7 + K + b_mn)
    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda)
    # stored weight: K-major B is W [N][K]; MN-major B is W^T stored [K][N]
    W = (0.02 * rng.standard_normal((K, N) if b_mn else (N, K))).astype(np.float32)
    a, ka = _operand(A, 0, M, 1)
    b, kb, deq = _q8_operand(W, b_mn, cuda)
    out = torch.full((M, N), float("nan"), device=cuda)
    _gemm(M, N, K, 1, 1, a, b, _epi(0, out, N))
    Bd = torch.from_numpy(deq).to(cuda)
    ref = A.double() @ (Bd.double() if b_mn else Bd.double().t())
    assert _relerr(out, ref) < 2e-5
    # without K splitting (same summation order), identical bits to the plane
    # operand over the dequantised weight
    out1 = torch.full((M, N), float("nan"), device=cuda)
    _gemm(M, N, K, 1, 1, a, b, _epi(0, out1, N), ksplits=1)
    bp, kp = _operand(Bd, b_mn, K if b_mn else N, 1)
    out_p = torch.full((M, N), float("nan"), device=cuda)
    _gemm(M, N, K, 1, 1, a, bp, _epi(0, out_p, N), ksplits=1)
    assert torch.equal(out1, out_p)


def test_gemm_q8_residual_epilogue(cuda):
    import torch
    rng = np.random.default_rng(5)
    M, N, K = 512, 576, 1536
    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda)
    W = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    res = torch.randn(M, N, device=cuda)
    a, ka = _operand(A, 0, M, 1)
    b, kb, deq = _q8_operand(W, 0, cuda)
    out = torch.empty(M, N, device=cuda)
    _gemm(M, N, K, 1, 1, a, b, _epi(2, out, N, res=res))
    ref = res.double() + A.double() @ torch.from_numpy(deq).to(cuda).double().t()
    assert _relerr(out, ref) < 2e-5


def test_gemm_q8_rejects_unsupported(cuda):
    """A Q8_0 operand needs split planes for A and a non-batched GEMM."""
    import torch
    from toy_b200._lib import lib
    rng = np.random.default_rng(1)
    M, N, K = 128, 128, 64
    A = torch.randn(M, K, device=cuda)
    W = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    a, ka = _operand(A, 0, M, 1)
    b, kb, deq = _q8_operand(W, 0, cuda)
    out = torch.empty(M, N, device=cuda)
    e = _epi(0, out, N)
    assert lib().tb2_gemm(M, N, K, 1, 0, C.byref(a), C.byref(b), C.byref(e), 0, 0, None) != 0   # single pass
    assert lib().tb2_gemm(M, N, K, 2, 1, C.byref(a), C.byref(b), C.byref(e), 0, 0, None) != 0   # batched
