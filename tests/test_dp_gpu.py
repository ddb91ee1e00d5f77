"""Data-parallel step on 2 GPUs (NCCL all-reduce inside the library) equals the
single-GPU step on the joined batch, with the gradients reduced in one bucket
after the backward and in per-layer buckets overlapped with it; sessions on
two devices in one process; a rank that leaves between steps or never joins a
step ends the other rank's step with an error, not a hang. Needs two
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


def _cfgs(dh=32):
    """d_head 32: the materialised attention and three-pass weight gradients; d_head 64:
    the fused attention and the one-pass fp16 weight gradients (each rank scaling its own)."""
    from toy_b200 import LlamaConfig
    d = 4 * dh
    oc = O.LlamaCfg(vocab=512, d_model=d, n_heads=4, n_kv=2, d_head=dh, d_ff=256, n_layers=2, rope_base=1e4)
    return oc, LlamaConfig(512, d, 4, 2, dh, 256, 2, 1e4, 1e-5)


def _rank(rank, world, port, q, bucket, dh=32):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from toy_b200 import FromScratch, RecipeOptions
    from toy_b200.parallel import DataParallel
    oc, gc = _cfgs(dh)
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


@pytest.mark.parametrize("bucket,dh", [(None, 32), (4096, 32), (4096, 64)])
def test_dp2_matches_joined_batch(cuda, bucket, dh):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q, bucket, dh)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(2)), key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    from toy_b200 import FromScratch, RecipeOptions
    oc, gc = _cfgs(dh)
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


def test_sessions_on_two_devices_in_one_process(cuda):
    """Kernel set-up (shared-memory limits, CTA-pair occupancy) is per device: one
    process realises the same step on GPU 0 and GPU 1 and gets identical results."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from toy_b200 import FromScratch, LoRA, LoraOptions, RecipeOptions
    oc, gc = _cfgs()
    T = 64
    ids = O.token_ids(5, 2 * T, oc.vocab)
    lab = O.next_token_labels(ids, T, 2, oc.vocab)
    res = []
    for dev in (0, 1):
        fs = FromScratch(device=dev)
        fs.realize(gc, RecipeOptions(t_seq=T, t_batch=2, seed=3))
        ql = LoRA(device=dev)
        ql.realize(gc, 8, RecipeOptions(t_seq=T, t_batch=2, seed=3),
                   LoraOptions(rank=8, targets=("q", "k", "v", "o", "gate", "up", "down")))
        out = []
        for rec, eng in ((fs, fs.fs_cache), (ql, ql.lora_cache)):
            losses = [rec.step(ids, O.positions(T, 2), lab, O.hp_lora(1e-3, s + 1, wd=0.01), s == 0) for s in range(2)]
            name = "blk.1.ffn_up.weight" if eng is fs.fs_cache else "blk.1.ffn_up.lora_b"
            out.append((losses, eng.param(name)))
        res.append(out)
    for a, b in zip(res[0], res[1]):
        assert a[0] == b[0]
        assert np.array_equal(a[1], b[1])


def _fail_rank(rank, world, port, q, mode, go):
    """Two ranks take one data-parallel step. Then, mode 'leave': rank 1 exits
    between steps (nothing in flight, no further NCCL call) and rank 0 learns it
    on the host before its next launch; mode 'stall': rank 1 stays but never
    joins step 2, and rank 0's step ends at the communicator's time limit with
    the communicator aborted. Either way rank 0's GPU stays usable."""
    import sys
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from toy_b200 import FromScratch, RecipeOptions
    from toy_b200.parallel import DataParallel, RankFailure

    def say(msg):
        print(f"[rank {rank} {mode}] {msg}", file=sys.stderr, flush=True)

    def report(item):
        q.put(item)
        q.close()
        q.join_thread()

    oc, gc = _cfgs()
    T = 64
    dp = DataParallel(rank, world, rank, timeout_s=10)
    rec = FromScratch(device=rank)
    rec.realize(gc, RecipeOptions(t_seq=T, t_batch=1, seed=3))
    dp.attach(rec.fs_cache, bucket_floats=4096, timeout_ms=3000)
    say("attached")
    ids = O.token_ids(5 + rank, T, oc.vocab)
    lab = O.next_token_labels(ids, T, 1, oc.vocab)
    dp.check_peers()
    rec.step(ids, O.positions(T, 1), lab, O.hp_lora(1e-3, 1, wd=0.01), True)
    say("step 1 done")
    if rank == 1:
        if mode == "stall":
            go.wait(60)         # alive, never joins step 2
            dp.abort()          # a rank leaving alone aborts (local), it does not finalize
            say("aborted")
        report((1, "left"))
        os._exit(0)
    outcome, code = "stepped", 0
    try:
        if mode == "leave":
            say("checking peers")
            dp.check_peers()    # the host learns of the departure before the launch
        say("step 2")
        rec.step(ids, O.positions(T, 1), lab, O.hp_lora(1e-3, 2, wd=0.01), False)
    except RankFailure:
        outcome = "RankFailure"
        say("RankFailure; aborting")
        dp.abort()
    except RuntimeError:
        outcome, code = "step error", dp.status()
    say(f"step 2: {outcome} {code}")
    # the GPU context stays usable: a fresh single-GPU session steps normally
    solo = FromScratch(device=rank)
    solo.realize(gc, RecipeOptions(t_seq=T, t_batch=1, seed=3))
    ok = bool(np.isfinite(solo.step(ids, O.positions(T, 1), lab, O.hp_lora(1e-3, 1, wd=0.01), True)))
    say(f"solo step ok={ok}")
    report((0, outcome, code, ok))
    go.set()
    os._exit(0)


@pytest.mark.parametrize("mode", ["leave", "stall"])
def test_dp_rank_failure_ends_with_an_error(cuda, mode):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    go = ctx.Event()
    port = _free_port()
    ps = [ctx.Process(target=_fail_rank, args=(r, 2, port, q, mode, go)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r = q.get(timeout=120)
            res[r[0]] = r
            go.set()
        for p in ps:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in ps:
            if p.is_alive():
                p.kill()
    if mode == "leave":
        assert res[0][1] == "RankFailure"
    else:
        assert res[0][1] == "step error" and res[0][2] == -4   # the time limit ended the step
    assert res[0][3]
