"""Data-parallel host logic on CPU: the gloo rendezvous that hands rank 0's
NCCL id to every rank (world size 2), and the gradient identity the all-reduce
relies on (mean of per-rank mean gradients == gradient of the joined batch)."""
import os
import socket

import numpy as np
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
