"""Data-parallel host logic on CPU (gloo ranks, world size 2): the rendezvous
that hands rank 0's NCCL id to every rank; the gradient identity the all-reduce
relies on (mean of per-rank mean gradients == gradient of the joined batch);
the gradient bucket plan the backward issues (the library's own rule, a pure
host function) and a bucket-by-bucket reduction with the 1/world scale against
the joined-batch gradient; and rank failure detected on the host (a rank that
exits between steps, a rank that stops answering) as a RankFailure within the
process group's time limit."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from toy_b200.parallel import DataParallel
    dp = DataParallel(rank, world, rank, timeout_s=60)
    uid = bytes(range(128)) if rank == 0 else None
    got = dp.exchange_uid(uid)
    mx = dp.max_scalar(1.5 + rank)
    mean = dp.mean_scalar(float(rank))
    dp.barrier()
    out.put((rank, got == bytes(range(128)), mx, mean))
    dp.close()


def test_gloo_rendezvous_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[1] for r in res)
    assert all(abs(r[2] - 2.5) < 1e-12 for r in res)
    assert all(abs(r[3] - 0.5) < 1e-12 for r in res)


def test_dp_gradient_identity():
    cfg = O.LlamaCfg(vocab=96, d_model=64, n_heads=4, n_kv=2, d_head=16, d_ff=96, n_layers=1, rope_base=1e4)
    T = 8
    mdl = O.full_ft_model(cfg, seed=3)
    ids = O.token_ids(7, 2 * T, cfg.vocab)
    lab = O.next_token_labels(ids, T, 2, cfg.vocab)
    pos = O.positions(T, 2)
    _, g_all, _ = O.forward_backward(mdl, ids, pos, lab, T, 2)
    _, g0, _ = O.forward_backward(mdl, ids[:T], pos[:T], lab[:T], T, 1)
    _, g1, _ = O.forward_backward(mdl, ids[T:], pos[T:], lab[T:], T, 1)
    for k in mdl.trainable:
        assert np.allclose(0.5 * (g0[k] + g1[k]), g_all[k], rtol=1e-10, atol=1e-14), k


# --------------------------------------------------------------------------- gradient buckets
def _plan(layer_lo, n_train, bucket):
    import ctypes as C
    from toy_b200._lib import lib
    L = lib()
    lo = (C.c_longlong * max(1, len(layer_lo)))(*layer_lo)
    n = L.tb2_dp_bucket_plan(lo, len(layer_lo), n_train, bucket, None, 0)
    assert n >= 0
    out = (C.c_longlong * (2 * n + 2))()
    assert L.tb2_dp_bucket_plan(lo, len(layer_lo), n_train, bucket, out, 2 * n + 2) == n
    return [(out[2 * i], out[2 * i + 1]) for i in range(n)]


def _plan_restated(layer_lo, n_train, bucket):
    """The backward's rule: layers finish from the last down; the pending range
    becomes a bucket once it holds `bucket` floats; the rest after the backward."""
    pend_lo = pend_hi = n_train
    out = []
    for lo in list(layer_lo)[::-1] + [0]:
        pend_lo = min(pend_lo, lo)
        if pend_hi > pend_lo and pend_hi - pend_lo >= bucket:
            out.append((pend_lo, pend_hi))
            pend_hi = pend_lo
    if pend_hi > 0:
        out.append((0, pend_hi))
    return out


def test_bucket_plan_covers_the_arena_once():
    # full fine-tune layout: embedding + final norm first, then layers ascending
    assert _plan([100, 300, 500, 700, 900], 1000, 250) == [(700, 1000), (300, 700), (0, 300)]
    assert _plan([100, 300, 500, 700, 900], 1000, 1 << 20) == [(0, 1000)]
    assert _plan([100, 300, 500, 700, 900], 1000, 1) == [(900, 1000), (700, 900), (500, 700), (300, 500),
                                                        (100, 300), (0, 100)]
    assert _plan([], 64, 8) == [(0, 64)]
    rng = np.random.default_rng(0)
    for _ in range(200):
        L = int(rng.integers(1, 40))
        sizes = rng.integers(0, 5000, L + 1)
        lo = np.cumsum(sizes)[:-1].tolist()
        n_train = int(np.sum(sizes))
        bucket = int(rng.integers(1, 20000))
        p = _plan(lo, n_train, bucket)
        assert p == _plan_restated(lo, n_train, bucket)
        # issue order is top-down, ranges are disjoint and cover [0, n_train)
        covered = sorted(p)
        assert covered[0][0] == 0 and covered[-1][1] == n_train
        assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))
        assert all(p[i][0] >= p[i + 1][1] for i in range(len(p) - 1))
        assert all(hi - lo >= bucket for lo, hi in p[:-1])


def test_bucket_plan_rejects_bad_layouts():
    import ctypes as C
    from toy_b200._lib import lib
    lo = (C.c_longlong * 3)(5, 3, 9)   # not non-decreasing
    assert lib().tb2_dp_bucket_plan(lo, 3, 10, 4, None, 0) == -1
    lo = (C.c_longlong * 1)(11)        # beyond the arena
    assert lib().tb2_dp_bucket_plan(lo, 1, 10, 4, None, 0) == -1
    assert lib().tb2_dp_bucket_plan(lo, 1, 10, 0, None, 0) == -1


def _dp_reduce_worker(rank, world, port, out):
    """Each rank: gradients of its half batch in the arena layout, reduced bucket
    by bucket (gloo sum, the plan's order), times 1 / world."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    from toy_b200.parallel import DataParallel
    dp = DataParallel(rank, world, rank, timeout_s=60)
    cfg = O.LlamaCfg(vocab=96, d_model=64, n_heads=4, n_kv=2, d_head=16, d_ff=96, n_layers=3, rope_base=1e4)
    T = 8
    mdl = O.full_ft_model(cfg, seed=3)
    ids = O.token_ids(7, world * T, cfg.vocab)
    lab = O.next_token_labels(ids, T, world, cfg.vocab)
    sl = slice(rank * T, (rank + 1) * T)
    _, g, _ = O.forward_backward(mdl, ids[sl], O.positions(T, 1), lab[sl], T, 1)
    # arena layout of the step program: embedding, final norm, then every layer's tensors
    names = ["token_embd.weight", "output_norm.weight"]
    layer_lo = []
    for l in range(cfg.n_layers):
        layer_lo.append(sum(mdl.params[k].size for k in names))
        names += sorted(k for k in mdl.params if k.startswith(f"blk.{l}."))
    arena = np.concatenate([g[k].reshape(-1) for k in names]).astype(np.float64)
    plan = _plan(layer_lo, arena.size, 5000)
    for lo, hi in plan:
        t = torch.from_numpy(arena[lo:hi].copy())
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        arena[lo:hi] = t.numpy()
    arena *= 1.0 / world
    plans = [None] * world
    dist.all_gather_object(plans, plan)
    out.put((rank, arena, plans, names))
    dp.close()


def test_bucketed_reduction_equals_the_joined_batch_gradient():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_dp_reduce_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((q.get(timeout=120) for _ in range(2)), key=lambda r: r[0])
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][2][0] == res[0][2][1] and len(res[0][2][0]) > 2   # every rank issues the same buckets
    assert np.array_equal(res[0][1], res[1][1])                     # replicas get identical gradients
    cfg = O.LlamaCfg(vocab=96, d_model=64, n_heads=4, n_kv=2, d_head=16, d_ff=96, n_layers=3, rope_base=1e4)
    T = 8
    mdl = O.full_ft_model(cfg, seed=3)
    ids = O.token_ids(7, 2 * T, cfg.vocab)
    _, g_all, _ = O.forward_backward(mdl, ids, O.positions(T, 2), O.next_token_labels(ids, T, 2, cfg.vocab), T, 2)
    ref = np.concatenate([g_all[k].reshape(-1) for k in res[0][3]])
    assert np.allclose(res[0][1], ref, rtol=1e-10, atol=1e-14)


# --------------------------------------------------------------------------- rank failure (host side)
def _leaver(rank, world, port, out, mode, done):
    """Rank 1 leaves after the first step check ('exit') or stops answering
    ('silent'); rank 0 must get a RankFailure, not a hang."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import time
    from toy_b200.parallel import DataParallel, RankFailure
    dp = DataParallel(rank, world, rank, timeout_s=5)
    dp.check_peers()                       # step 1: everyone is there
    if rank == 1:
        if mode == "silent":
            done.wait(60)                  # alive, but never joins the next check
        os._exit(0)                        # leaves without another collective
    t0 = time.time()
    try:
        dp.check_peers()                   # step 2
        out.put(("no failure", time.time() - t0))
    except RankFailure:
        out.put(("RankFailure", time.time() - t0))
    out.close()
    out.join_thread()   # flush the queue before the hard exit
    done.set()
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "silent"])
def test_rank_failure_is_reported_on_the_host(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    port = _free_port()
    ps = [ctx.Process(target=_leaver, args=(r, 2, port, q, mode, done)) for r in range(2)]
    for p in ps:
        p.start()
    kind, secs = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert kind == "RankFailure"
    assert secs < 30
