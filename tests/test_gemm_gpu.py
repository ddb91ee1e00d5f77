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


def _gemm(M, N, K, batch, split, a, b, e, ksplits=0, causal=0):
    import torch
    from toy_b200._lib import lib
    L = lib()
    rc = L.tb2_gemm(M, N, K, batch, split, C.byref(a), C.byref(b), C.byref(e), ksplits, causal, None)
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


def _operand16(store, mn_major, rows):
    """store: f32 tensor [rows_total, cols]; its fp16 copy as a single-plane operand."""
    from toy_b200._lib import Operand
    h = store.half().contiguous()
    o = Operand()
    o.hi, o.lo = h.data_ptr(), None
    o.mn_major = mn_major
    o.ld = store.shape[1]
    o.rows = rows
    o.cols = store.shape[1]
    o.batch_stride = rows * store.shape[1]
    o.nbatch = 1
    o.bdiv1, o.bmul1, o.bdiv2, o.bmul2 = 1, 0, 1, 0
    return o, h


@pytest.mark.parametrize("a_mn,b_mn,ksplits", [(1, 1, 0), (1, 1, 4), (0, 0, 0), (1, 0, 2)])
def test_gemm_single_pass_f16(cuda, a_mn, b_mn, ksplits):
    """split = 2: one kind::f16 pass on fp16 operands (the weight-gradient layout: both
    operands MN-major, K = tokens), against fp64 of the fp16-rounded inputs; alpha applied."""
    import torch
    M, N, K = 576, 1536, 4096
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(M, K, device=cuda, generator=g) * 3.0
    B = torch.randn(N, K, device=cuda, generator=g)
    a, ka = _operand16(A.t().contiguous() if a_mn else A, a_mn, K if a_mn else M)
    b, kb = _operand16(B.t().contiguous() if b_mn else B, b_mn, K if b_mn else N)
    out = torch.full((M, N), float("nan"), device=cuda)
    _gemm(M, N, K, 1, 2, a, b, _epi(0, out, N, alpha=0.25), ksplits=ksplits)
    ref = 0.25 * (A.half().double() @ B.half().double().t())
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


@pytest.mark.parametrize("ksplits", [2, 5, 16])
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_gemm_split_k_deterministic(cuda, ksplits, mode):
    """Split-K partials reduced in split order: exact vs fp64 and bit-identical across runs."""
    import torch
    M, N, K = 576, 576, 4096
    A = torch.randn(K, M, device=cuda)     # stored K x M (MN-major), as the dW GEMMs read activations
    B = torch.randn(K, N, device=cuda)
    a, ka = _operand(A, 1, K, 1)
    b, kb = _operand(B, 1, K, 1)
    ref = A.double().t() @ B.double()
    outs = []
    for _ in range(2):
        base = torch.randn(M, N, device=cuda, generator=torch.Generator(device="cuda").manual_seed(1))
        out = base.clone()
        hi = torch.zeros(M, N, device=cuda, dtype=torch.bfloat16)
        lo = torch.zeros_like(hi)
        e = _epi(mode, out, N, res=base if mode == 2 else None, hi=hi if mode == 3 else None,
                 lo=lo if mode == 3 else None)
        _gemm(M, N, K, 1, 1, a, b, e, ksplits=ksplits)
        got = (hi.double() + lo.double()) if mode == 3 else out.double() - (base.double() if mode in (1, 2) else 0)
        outs.append(got)
        assert _relerr(got, ref) < 2e-5
    assert torch.equal(outs[0], outs[1])


def test_gemm_auto_split_and_causal(cuda):
    import torch
    # auto split-K on a tiny tile grid
    M, N, K = 128, 192, 8192
    A = torch.randn(M, K, device=cuda)
    B = torch.randn(N, K, device=cuda)
    a, ka = _operand(A, 0, M, 1)
    b, kb = _operand(B, 0, N, 1)
    out = torch.zeros(M, N, device=cuda)
    _gemm(M, N, K, 1, 1, a, b, _epi(0, out, N))
    assert _relerr(out, A.double() @ B.double().t()) < 2e-5
    # causal 2: K clamped to each row tile's end (columns of A beyond it are zero in a causal P)
    T, dh, Z = 512, 64, 3
    P = torch.tril(torch.rand(Z * T, T, device=cuda).view(Z, T, T)).reshape(Z * T, T)
    V = torch.randn(Z * T, dh, device=cuda)
    a, ka = _operand(P, 0, T, Z)
    b, kb = _operand(V, 1, T, Z)
    out = torch.zeros(Z, T, dh, device=cuda)
    _gemm(T, dh, T, Z, 1, a, b, _epi(0, out, dh, bstride=T * dh), causal=2)
    assert _relerr(out, P.double().view(Z, T, T) @ V.double().view(Z, T, dh)) < 2e-5
    # causal 1: tiles strictly above the diagonal are skipped, the rest exact
    Q = torch.randn(Z * T, dh, device=cuda)
    Kt = torch.randn(Z * T, dh, device=cuda)
    a, ka = _operand(Q, 0, T, Z)
    b, kb = _operand(Kt, 0, T, Z)
    out = torch.full((Z, T, T), 7.0, device=cuda)
    _gemm(T, T, dh, Z, 1, a, b, _epi(0, out, T, bstride=T * T), causal=1)
    ref = Q.double().view(Z, T, dh) @ Kt.double().view(Z, T, dh).transpose(1, 2)
    mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device=cuda))
    assert _relerr(out[:, mask], ref[:, mask]) < 2e-5


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
