"""tb2_gemm_noalloc — the GEMM entry point for callers that cannot allocate
device memory (hosts that own every buffer, or loops where an allocator call
would synchronise the device) — gives the same results as tb2_gemm.

It runs split-K through a workspace compiled into the library instead of one
allocated on first use. Checked through the C ABI against tb2_gemm on the same
inputs, on two calls in a row (the shared workspace keeps the previous call's
contents, which must not leak into the next result), with the error word read
after every call; the automatic split count where the workspace is what limits
it; and the size limit applied to the splits the GEMM would actually run.
This file is collected last so a failure here leaves every other test run.
"""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


def _operand(x, mn_major, rows):
    import torch
    from toy_b200._lib import Operand
    hi = x.to(torch.bfloat16).contiguous()
    lo = (x - hi.float()).to(torch.bfloat16).contiguous()
    o = Operand()
    o.hi, o.lo, o.mn_major, o.ld, o.rows, o.cols = hi.data_ptr(), lo.data_ptr(), mn_major, x.shape[1], rows, \
        x.shape[1]
    o.batch_stride, o.nbatch, o.bdiv1, o.bmul1, o.bdiv2, o.bmul2 = rows * x.shape[1], 1, 1, 0, 1, 0
    return o, (hi, lo)


def _epi(out, ldc):
    from toy_b200._lib import Epilogue
    e = Epilogue()
    e.mode, e.alpha, e.out = 0, 1.0, out.data_ptr()
    e.bstride, e.z_div, e.z_s1, e.m_div, e.m_s1, e.m_s0, e.n_div, e.n_s1 = 0, 0, 0, 0, 0, ldc, 0, 0
    return e


def test_noalloc_gemm_matches_tb2_gemm_twice(cuda):
    import torch
    from toy_b200._lib import lib
    L = lib()
    M, N, K = 576, 576, 4096          # weight-gradient shape: small tile grid, long K -> split-K
    for call in range(2):
        g = torch.Generator(device="cuda").manual_seed(100 + call)
        A = torch.randn(K, M, device=cuda, generator=g)
        B = torch.randn(K, N, device=cuda, generator=g)
        a, ka = _operand(A, 1, K)
        b, kb = _operand(B, 1, K)
        ref = torch.zeros(M, N, device=cuda)
        got = torch.full((M, N), float("nan"), device=cuda)
        for ks in (0, 4):
            assert L.tb2_gemm(M, N, K, 1, 1, C.byref(a), C.byref(b), C.byref(_epi(ref, N)), ks, 0, None) == 0
            assert L.tb2_gemm_noalloc(M, N, K, 1, 1, C.byref(a), C.byref(b), C.byref(_epi(got, N)), ks, 0,
                                      None) == 0
            assert L.tb2_gemm_noalloc_error() == 0
            torch.cuda.synchronize()
            rel = ((got.double() - ref.double()).norm() / ref.double().norm()).item()
            assert rel < 2e-5, (call, ks, rel)
            exact = (A.double().t() @ B.double())
            assert ((got.double() - exact).norm() / exact.norm()).item() < 2e-5


def test_noalloc_gemm_rejects_oversized_split(cuda):
    import torch
    from toy_b200._lib import lib
    M, N, K = 1024, 1024, 4096
    A = torch.randn(M, K, device=cuda)
    B = torch.randn(N, K, device=cuda)
    a, ka = _operand(A, 0, M)
    b, kb = _operand(B, 0, N)
    out = torch.zeros(M, N, device=cuda)
    # 4 * 1024 * 1024 floats is twice the fixed workspace
    assert lib().tb2_gemm_noalloc(M, N, K, 1, 1, C.byref(a), C.byref(b), C.byref(_epi(out, N)), 4, 0, None) == -5


def _pair(M, N, K, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(N, K, device="cuda", generator=g)
    return A, B


def test_noalloc_auto_splits_fit_the_workspace(cuda):
    """ksplits = 0 on a large tile grid with a long K: the plan's split count is
    capped at 2^21 / (M N) = 2 partial tiles."""
    import torch
    from toy_b200._lib import lib
    L = lib()
    M, N, K = 1024, 1024, 16384
    A, B = _pair(M, N, K, 7)
    a, ka = _operand(A, 0, M)
    b, kb = _operand(B, 0, N)
    ref = torch.zeros(M, N, device=cuda)
    got = torch.full((M, N), float("nan"), device=cuda)
    assert L.tb2_gemm(M, N, K, 1, 1, C.byref(a), C.byref(b), C.byref(_epi(ref, N)), 0, 0, None) == 0
    assert L.tb2_gemm_noalloc(M, N, K, 1, 1, C.byref(a), C.byref(b), C.byref(_epi(got, N)), 0, 0, None) == 0
    assert L.tb2_gemm_noalloc_error() == 0
    torch.cuda.synchronize()
    # K = 16384: the f32 sums of the split-bf16 products drift with K (the
    # 576-wide cases above keep 2e-5); tb2_gemm may pick more K splits (its
    # workspace is larger), so the two differ by summation order only
    exact = A.double() @ B.double().t()
    assert ((got.double() - exact).norm() / exact.norm()).item() < 1e-4
    assert ((got.double() - ref.double()).norm() / ref.double().norm()).item() < 1e-4


def test_noalloc_size_check_uses_the_splits_that_run(cuda):
    """ksplits = 8 over K = 128 (two k-blocks) runs 2 splits: 2 M N = 2^21 floats
    fit, so the call is accepted; a batched product runs unsplit, so any ksplits
    is accepted there too."""
    import torch
    from toy_b200._lib import lib
    L = lib()
    M, N, K = 1024, 1024, 128
    A, B = _pair(M, N, K, 8)
    a, ka = _operand(A, 0, M)
    b, kb = _operand(B, 0, N)
    got = torch.full((M, N), float("nan"), device=cuda)
    assert L.tb2_gemm_noalloc(M, N, K, 1, 1, C.byref(a), C.byref(b), C.byref(_epi(got, N)), 8, 0, None) == 0
    assert L.tb2_gemm_noalloc_error() == 0
    torch.cuda.synchronize()
    exact = A.double() @ B.double().t()
    assert ((got.double() - exact).norm() / exact.norm()).item() < 2e-5
    # two batches of [512 x 1024] x [1024 x 128]^T: batched products never split
    Mb = 512
    Ab, Bb = _pair(2 * Mb, N, K, 9)
    ab, kab = _operand(Ab, 0, Mb)
    ab.batch_stride, ab.nbatch, ab.bmul1 = Mb * K, 2, 1
    bb, kbb = _operand(Bb, 0, N)
    bb.rows, bb.batch_stride, bb.nbatch, bb.bmul1 = N // 2, (N // 2) * K, 2, 1
    outb = torch.full((2, Mb, N // 2), float("nan"), device=cuda)
    e = _epi(outb, N // 2)
    e.bstride = Mb * (N // 2)
    assert L.tb2_gemm_noalloc(Mb, N // 2, K, 2, 1, C.byref(ab), C.byref(bb), C.byref(e), 16, 0, None) == 0
    assert L.tb2_gemm_noalloc_error() == 0
    torch.cuda.synchronize()
    for z in range(2):
        ex = Ab[z * Mb:(z + 1) * Mb].double() @ Bb[z * (N // 2):(z + 1) * (N // 2)].double().t()
        assert ((outb[z].double() - ex).norm() / ex.norm()).item() < 2e-5
