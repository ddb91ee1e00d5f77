"""Split-bf16 tcgen05 GEMM against an fp64 torch product (all operand majors,
batching with grouped-query batch maps, every epilogue mode)."""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


def _split(x):
    import torch
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return hi.contiguous(), lo.contiguous()


def _operand(store, mn_major, rows_per_batch, nbatch, bmap=(1, 1, 1, 0)):
    """store: f32 tensor [nbatch * rows_per_batch, cols] (row-major)."""
    from toy_b200._lib import Operand
    hi, lo = _split(store)
    o = Operand()
    o.hi, o.lo = hi.data_ptr(), lo.data_ptr()
    o.mn_major = mn_major
    o.ld = store.shape[1]
    o.rows = rows_per_batch
    o.cols = store.shape[1]
    o.batch_stride = rows_per_batch * store.shape[1]
    o.nbatch = nbatch
    o.bdiv1, o.bmul1, o.bdiv2, o.bmul2 = bmap
    return o, (hi, lo)


def _epi(mode, out=None, ldc=0, res=None, hi=None, lo=None, bstride=0, alpha=1.0):
    from toy_b200._lib import Epilogue
    e = Epilogue()
    e.mode, e.alpha = mode, alpha
    e.out = out.data_ptr() if out is not None else None
    e.res = res.data_ptr() if res is not None else None
    e.out_hi = hi.data_ptr() if hi is not None else None
    e.out_lo = lo.data_ptr() if lo is not None else None
    e.bstride, e.z_div, e.z_s1, e.m_div, e.m_s1, e.m_s0, e.n_div, e.n_s1 = bstride, 0, 0, 0, 0, ldc, 0, 0
    return e


def _gemm(M, N, K, batch, split, a, b, e):
    import torch
    from toy_b200._lib import lib
    L = lib()
    rc = L.tb2_gemm(M, N, K, batch, split, C.byref(a), C.byref(b), C.byref(e), None)
    assert rc == 0, rc
    torch.cuda.synchronize()
    assert L.tb2_device_error() == 0


def _relerr(x, ref):
    return ((x.double() - ref).norm() / ref.norm()).item()


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(256, 384, 320), (200, 576, 576), (128, 64, 4096), (384, 960, 64),
                                   (128, 512, 128), (256, 1536, 576), (128, 256, 64), (64, 32, 32), (128, 128, 96)])
def test_gemm_majors(cuda, a_mn, b_mn, M, N, K):
    import torch
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, device=cuda, generator=g)
    B = torch.randn(N, K, device=cuda, generator=g)
    a, ka = _operand(A.t().contiguous() if a_mn else A, a_mn, K if a_mn else M, 1)
    b, kb = _operand(B.t().contiguous() if b_mn else B, b_mn, K if b_mn else N, 1)
    out = torch.full((M, N), float("nan"), device=cuda)
    _gemm(M, N, K, 1, 1, a, b, _epi(0, out, N))
    ref = A.double() @ B.double().t()
    assert _relerr(out, ref) < 2e-5


def test_gemm_single_pass_bf16(cuda):
    import torch
    M, N, K = 256, 256, 512
    A = torch.randn(M, K, device=cuda)
    B = torch.randn(N, K, device=cuda)
    a, ka = _operand(A, 0, M, 1)
    b, kb = _operand(B, 0, N, 1)
    out = torch.zeros(M, N, device=cuda)
    _gemm(M, N, K, 1, 0, a, b, _epi(0, out, N))
    ref = A.bfloat16().double() @ B.bfloat16().double().t()
    assert _relerr(out, ref) < 1e-5


def test_gemm_batched_gqa(cuda):
    """Scores per (sequence, query head) against a shared K head: z = b*H + h reads K batch b*KV + h/G."""
    import torch
    Bsz, H, KV, T, dh = 2, 6, 2, 192, 64
    G = H // KV
    Q = torch.randn(Bsz * H * T, dh, device=cuda)
    Kt = torch.randn(Bsz * KV * T, dh, device=cuda)
    a, ka = _operand(Q, 0, T, Bsz * H)
    b, kb = _operand(Kt, 0, T, Bsz * KV, bmap=(H, KV, G, 1))
    out = torch.zeros(Bsz * H, T, T, device=cuda)
    _gemm(T, T, dh, Bsz * H, 1, a, b, _epi(0, out, T, bstride=T * T))
    Qd = Q.double().view(Bsz, H, T, dh)
    Kd = Kt.double().view(Bsz, KV, T, dh).repeat_interleave(G, dim=1)
    ref = (Qd @ Kd.transpose(-1, -2)).reshape(Bsz * H, T, T)
    assert _relerr(out, ref) < 2e-5


def test_gemm_epilogues(cuda):
    import torch
    M, N, K = 256, 192, 128
    A = torch.randn(M, K, device=cuda)
    B = torch.randn(N, K, device=cuda)
    a, ka = _operand(A, 0, M, 1)
    b, kb = _operand(B, 0, N, 1)
    ref = A.double() @ B.double().t()
    # accumulate with alpha
    acc = torch.randn(M, N, device=cuda)
    acc0 = acc.clone()
    _gemm(M, N, K, 1, 1, a, b, _epi(1, acc, N, alpha=0.5))
    assert _relerr(acc, acc0.double() + 0.5 * ref) < 2e-5
    # residual
    res = torch.randn(M, N, device=cuda)
    out = torch.zeros(M, N, device=cuda)
    _gemm(M, N, K, 1, 1, a, b, _epi(2, out, N, res=res))
    assert _relerr(out, res.double() + ref) < 2e-5
    # split store
    hi = torch.zeros(M, N, device=cuda, dtype=torch.bfloat16)
    lo = torch.zeros(M, N, device=cuda, dtype=torch.bfloat16)
    _gemm(M, N, K, 1, 1, a, b, _epi(3, None, N, hi=hi, lo=lo))
    assert _relerr(hi.double() + lo.double(), ref) < 2e-5
    # head-major scatter: out[(m // T) * H*T*64 + (n // 64) * T*64 + (m % T) * 64 + n % 64]
    T, H = 64, N // 64
    e = _epi(0, None)
    outh = torch.zeros(M * N, device=cuda)
    e.out = outh.data_ptr()
    e.m_div, e.m_s1, e.m_s0, e.n_div, e.n_s1 = T, H * T * 64, 64, 64, T * 64
    _gemm(M, N, K, 1, 1, a, b, e)
    want = ref.view(M // T, T, H, 64).permute(0, 2, 1, 3).reshape(-1)
    assert _relerr(outh, want) < 2e-5


def test_split_kernel(cuda):
    import torch
    from toy_b200._lib import lib
    x = torch.randn(1000003, device=cuda)
    hi = torch.empty(x.shape, device=cuda, dtype=torch.bfloat16)
    lo = torch.empty_like(hi)
    assert lib().tb2_split_f32(x.data_ptr(), hi.data_ptr(), lo.data_ptr(), x.numel(), None) == 0
    h2, l2 = _split(x)
    torch.cuda.synchronize()
    assert torch.equal(hi, h2) and torch.equal(lo, l2)
