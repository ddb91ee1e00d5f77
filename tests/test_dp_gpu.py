"""Data-parallel step on 2 GPUs (NCCL all-reduce inside the library) equals the
single-GPU step on the joined batch, with the gradients reduced in one bucket
after the backward and in per-layer buckets overlapped with it. Needs two
B200s; skipped on one."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfgs():
    from toy_b200 import LlamaConfig
    oc = O.LlamaCfg(vocab=512, d_model=128, n_heads=4, n_kv=2, d_head=32, d_ff=256, n_layers=2, rope_base=1e4)
    return oc, LlamaConfig(512, 128, 4, 2, 32, 256, 2, 1e4, 1e-5)


def _rank(rank, world, port, q, bucket):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from toy_b200 import FromScratch, RecipeOptions
    from toy_b200.parallel import DataParallel
    oc, gc = _cfgs()
    T = 64
    dp = DataParallel(rank, world, rank, timeout_s=120)
    rec = FromScratch(device=rank)
    rec.realize(gc, RecipeOptions(t_seq=T, t_batch=1, seed=3))
    dp.attach(rec.fs_cache, bucket_floats=bucket)
    ids = O.token_ids(5, 2 * T, oc.vocab)
    lab = O.next_token_labels(ids, T, 2, oc.vocab)
    sl = slice(rank * T, (rank + 1) * T)
    losses = [rec.step(ids[sl], O.positions(T, 1), lab[sl], O.hp_lora(1e-3, s + 1, wd=0.01), s == 0)
              for s in range(2)]
    q.put((rank, losses, rec.fs_cache.param("blk.1.ffn_up.weight"), rec.fs_cache.param("token_embd.weight")))
    dp.close()
    rec.fs_cache.close()


@pytest.mark.parametrize("bucket", [None, 4096])
def test_dp2_matches_joined_batch(cuda, bucket):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q, bucket)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(2)), key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    from toy_b200 import FromScratch, RecipeOptions
    oc, gc = _cfgs()
    T = 64
    rec = FromScratch(device=0)
    rec.realize(gc, RecipeOptions(t_seq=T, t_batch=2, seed=3))
    ids = O.token_ids(5, 2 * T, oc.vocab)
    lab = O.next_token_labels(ids, T, 2, oc.vocab)
    for s in range(2):
        loss = rec.step(ids, O.positions(T, 2), lab, O.hp_lora(1e-3, s + 1, wd=0.01), s == 0)
    for name, i in (("blk.1.ffn_up.weight", 2), ("token_embd.weight", 3)):
        ref = rec.fs_cache.param(name)
        for r in res:
            assert np.linalg.norm(r[i] - ref) / np.linalg.norm(ref) < 1e-5, (name, r[0])
        assert np.array_equal(res[0][i], res[1][i])   # replicas stay identical
    # the rank losses average to the joined-batch loss of the last step's forward
    assert abs(0.5 * (res[0][1][1] + res[1][1][1]) - loss) < 1e-4 * abs(loss)
