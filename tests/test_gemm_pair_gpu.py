"""GEMMs on CTA pairs (tcgen05 cta_group::2).

Two CTAs on neighbouring SMs share one 256-row tensor-core tile: each holds
128 rows of A and half of the B tile in its own shared memory and its 128
accumulator lanes in its own TMEM; one of them issues the MMAs. Every output
element is the same sum in the same order as on a single CTA, so pair mode 1
must give the bits of pair mode 0 -- across operand majors, ragged edges,
epilogues, K splits, batch maps and Q8_0 B operands (dequantised by both CTAs'
converter warps) -- and stay within split-bf16 accuracy of fp64. The training
steps (fused RoPE / SwiGLU / LoRA epilogues included) must match too.
"""
import numpy as np
import pytest

from tests.test_gemm_gpu import _epi, _gemm, _operand, _relerr
from tests.test_gemm_q8_gpu import _q8_operand

pytestmark = pytest.mark.gpu


@pytest.fixture
def lib(cuda):
    from toy_b200._lib import lib as _l
    L = _l()
    yield L
    L.tb2_gemm_set_pair_mode(-1)


def both(L, fn):
    """fn() -> tensor, run on single CTAs and on CTA pairs."""
    L.tb2_gemm_set_pair_mode(0)
    r0 = fn()
    L.tb2_gemm_set_pair_mode(1)
    r1 = fn()
    L.tb2_gemm_set_pair_mode(-1)
    return r0, r1


def test_mode_setter(lib):
    assert lib.tb2_gemm_set_pair_mode(2) == -1
    for m in (-1, 1, 0):
        assert lib.tb2_gemm_set_pair_mode(m) == 0


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(256, 512, 576), (296, 200, 96), (128, 64, 64), (520, 1000, 1536),
                                   (4096, 3072, 576), (384, 960, 64)])
def test_pair_majors(lib, a_mn, b_mn, M, N, K):
    import torch
    cuda = torch.device("cuda:0")
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, device=cuda, generator=g)
    B = torch.randn(N, K, device=cuda, generator=g)
    a, ka = _operand(A.t().contiguous() if a_mn else A, a_mn, K if a_mn else M, 1)
    b, kb = _operand(B.t().contiguous() if b_mn else B, b_mn, K if b_mn else N, 1)

    def run():
        out = torch.full((M, N), float("nan"), device=cuda)
        _gemm(M, N, K, 1, 1, a, b, _epi(0, out, N), ksplits=1)
        return out

    o0, o1 = both(lib, run)
    ref = A.double() @ B.double().t()
    assert _relerr(o1, ref) < 2e-5
    assert torch.equal(o0, o1)


def test_pair_epilogues(lib):
    import torch
    cuda = torch.device("cuda:0")
    M, N, K = 384, 320, 256
    A = torch.randn(M, K, device=cuda)
    B = torch.randn(N, K, device=cuda)
    a, ka = _operand(A, 0, M, 1)
    b, kb = _operand(B, 0, N, 1)
    acc0 = torch.randn(M, N, device=cuda)
    res = torch.randn(M, N, device=cuda)

    def run():
        acc = acc0.clone()
        _gemm(M, N, K, 1, 1, a, b, _epi(1, acc, N, alpha=0.5), ksplits=1)
        out = torch.zeros(M, N, device=cuda)
        _gemm(M, N, K, 1, 1, a, b, _epi(2, out, N, res=res), ksplits=1)
        hi = torch.zeros(M, N, device=cuda, dtype=torch.bfloat16)
        lo = torch.zeros_like(hi)
        _gemm(M, N, K, 1, 1, a, b, _epi(3, None, N, hi=hi, lo=lo), ksplits=1)
        return torch.cat([acc.reshape(-1), out.reshape(-1), hi.float().reshape(-1), lo.float().reshape(-1)])

    r0, r1 = both(lib, run)
    assert torch.equal(r0, r1)
    ref = A.double() @ B.double().t()
    assert _relerr(r1[M * N:2 * M * N].view(M, N), res.double() + ref) < 2e-5


@pytest.mark.parametrize("ksplits", [2, 5])
def test_pair_split_k(lib, ksplits):
    """K splits on pairs: partial slabs summed in split order, same bits as single CTAs."""
    import torch
    cuda = torch.device("cuda:0")
    M, N, K = 576, 576, 4096
    A = torch.randn(K, M, device=cuda)
    B = torch.randn(K, N, device=cuda)
    a, ka = _operand(A, 1, K, 1)
    b, kb = _operand(B, 1, K, 1)

    def run():
        out = torch.zeros(M, N, device=cuda)
        _gemm(M, N, K, 1, 1, a, b, _epi(0, out, N), ksplits=ksplits)
        return out

    o0, o1 = both(lib, run)
    assert _relerr(o1, A.double().t() @ B.double()) < 2e-5
    assert torch.equal(o0, o1)


def test_pair_batched_group_map(lib):
    """Batch z of B reads A batch z // 3 (grouped-query sharing)."""
    import torch
    cuda = torch.device("cuda:0")
    Z, G, M, N, K = 6, 3, 300, 192, 64
    A = torch.randn(Z // G * M, K, device=cuda)
    B = torch.randn(Z * N, K, device=cuda)
    a, ka = _operand(A, 0, M, Z // G, bmap=(G, 1, 1, 0))
    b, kb = _operand(B, 0, N, Z)

    def run():
        out = torch.full((Z, M, N), float("nan"), device=cuda)
        _gemm(M, N, K, Z, 1, a, b, _epi(0, out, N, bstride=M * N), ksplits=1)
        return out

    o0, o1 = both(lib, run)
    ref = torch.stack([A.view(Z // G, M, K)[z // G].double() @ B.view(Z, N, K)[z].double().t() for z in range(Z)])
    assert _relerr(o1, ref) < 2e-5
    assert torch.equal(o0, o1)


@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("M,N,K", [(256, 960, 576), (130, 192, 96), (4096, 1536, 576), (600, 576, 1536)])
def test_pair_q8(lib, b_mn, M, N, K):
    import torch
    cuda = torch.device("cuda:0")
    rng = np.random.default_rng(M * 31 + N * 7 + K + b_mn)
    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda)
    W = (0.02 * rng.standard_normal((K, N) if b_mn else (N, K))).astype(np.float32)
    a, ka = _operand(A, 0, M, 1)
    b, kb, deq = _q8_operand(W, b_mn, cuda)

    def run():
        out = torch.full((M, N), float("nan"), device=cuda)
        _gemm(M, N, K, 1, 1, a, b, _epi(0, out, N), ksplits=1)
        return out

    o0, o1 = both(lib, run)
    Bd = torch.from_numpy(deq).to(cuda)
    ref = A.double() @ (Bd.double() if b_mn else Bd.double().t())
    assert _relerr(o1, ref) < 2e-5
    assert torch.equal(o0, o1)


def _dh64_cfg():
    from oracle import oracle as O
    from toy_b200 import LlamaConfig
    oc = O.LlamaCfg(vocab=512, d_model=256, n_heads=4, n_kv=2, d_head=64, d_ff=512, n_layers=2, rope_base=1e4)
    gc = LlamaConfig(512, 256, 4, 2, 64, 512, 2, 1e4, 1e-5)
    return oc, gc


def _step_pair(lib, make, T=128, B=2):
    """One recipe step from the same init, single CTAs then pairs."""
    from oracle import oracle as O
    oc, gc = _dh64_cfg()
    ids = O.token_ids(5, T * B, oc.vocab)
    pos, lab = O.positions(T, B), O.next_token_labels(ids, T, B, oc.vocab)
    out = []
    for mode in (0, 1):
        lib.tb2_gemm_set_pair_mode(mode)
        rec, eng, names = make(gc, T, B)
        loss = rec.step(ids, pos, lab, O.hp_lora(1e-4, 1, wd=0.01), True)
        out.append((loss, {k: eng.grad(k).copy() for k in names}))
    lib.tb2_gemm_set_pair_mode(-1)
    return out


def test_pair_full_ft_step(lib):
    from toy_b200 import FromScratch, RecipeOptions

    def make(gc, T, B):
        rec = FromScratch()
        rec.realize(gc, RecipeOptions(t_seq=T, t_batch=B, seed=3, init_scale=1.0))
        eng = rec.fs_cache
        return rec, eng, [n for n in eng.param_names() if eng.trainable(n)]

    (l0, g0), (l1, g1) = _step_pair(lib, make)
    assert l0 == l1
    for k in g0:
        assert np.array_equal(g0[k], g1[k]), k


def test_pair_qlora_step(lib):
    from toy_b200 import LoRA, LoraOptions, RecipeOptions

    def make(gc, T, B):
        rec = LoRA()
        lo = LoraOptions(rank=8, alpha=16.0, targets=("q", "k", "v", "o", "gate", "up", "down"), a_std=0.125,
                         b_std=0.01, base_std=0.02)
        rec.realize(gc, 8, RecipeOptions(t_seq=T, t_batch=B, seed=11), lo)
        eng = rec.lora_cache
        return rec, eng, [n for n in eng.param_names() if eng.trainable(n)]

    (l0, g0), (l1, g1) = _step_pair(lib, make)
    assert l0 == l1
    for k in g0:
        assert np.array_equal(g0[k], g1[k]), k
