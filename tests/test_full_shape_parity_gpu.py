"""Whole-step parity at the benchmark configurations' full sizes.

The CUDA step (through the C ABI, default launch plans: fused flash attention,
CTA-pair LM head, cost-model K splits, the Q8_0 plane ring with extension
columns) against the oracle on the same seeded inputs, with the training-step
contract's tolerances: loss within 1e-4 relative; every gradient, post-AdamW
weight and Adam moment within 1e-3 relative L2; Q8_0 bytes and the seeded init
streams bit-exact.

  * SmolLM2-135M QLoRA (q, v; rank 8, alpha 16), 30 layers, V = 49152, B=1 T=64,
    seed 42, lr 1e-4, wd 0.01, two steps;
  * SmolLM2-135M full f32 fine-tune, every weight N(0, 0.02), B=8 T=512, two steps
    (the default throughput workload; the second step runs the weight gradients
    as one fp16 pass, scaled from the first step's gradient magnitudes);
  * SmolLM2-135M QLoRA (q, v) at B=8 T=512, one step (the QLoRA throughput workload).

Each test prints its three worst relative-L2 values (gradients, weights, moments).
The oracle needs ~20 GB of host memory and about a minute per step at B=8 T=512.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOSS_TOL = 1e-4
REL_L2 = 1e-3


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (nb if nb > 0 else 1.0)


def compare(eng, mdl, loss_gpu, loss_ref, grads_ref):
    """Every check of the contract; returns (loss rel error, worst 3 per kind)."""
    lerr = abs(loss_gpu - loss_ref) / abs(loss_ref)
    worst = {"grad": [], "param": [], "m": [], "v": []}
    for k in mdl.trainable:
        g = eng.grad(k)
        worst["grad"].append((rel(g, grads_ref[k].reshape(g.shape)), k))
        p = eng.param(k)
        worst["param"].append((rel(p, mdl.params[k].reshape(p.shape)), k))
        for w, nm, ref in ((0, "m", mdl.m[k]), (1, "v", mdl.v[k])):
            mo = eng.moment(k, w)
            worst[nm].append((rel(mo, ref.reshape(mo.shape)), k))
    for kind in worst:
        worst[kind] = sorted(worst[kind])[-3:][::-1]
    return lerr, worst


def report(capsys, name, step, lerr, worst):
    with capsys.disabled():
        print(f"\n[{name} step {step}] loss rel err {lerr:.2e}")
        for kind, rows in worst.items():
            print(f"  worst {kind:5s}: " + ", ".join(f"{r:.2e} {k}" for r, k in rows))


def check(lerr, worst):
    assert lerr <= LOSS_TOL, ("loss", lerr)
    for kind, rows in worst.items():
        for r, k in rows:
            assert r < REL_L2, (kind, k, r)


def smollm2():
    from toy_b200 import LlamaConfig
    return O.smollm2_135m(), LlamaConfig.smollm2_135m()


def batch(cfg, T, B, seed):
    ids = O.token_ids(seed, T * B, cfg.vocab)
    return ids, O.positions(T, B), O.next_token_labels(ids, T, B, cfg.vocab)


def test_smollm2_qlora_b1_t64_two_steps(cuda, capsys):
    """The CPU-runnable configuration: SmolLM2-135M QLoRA on q, v, B=1 T=64, seed 42."""
    from toy_b200 import LoRA, LoraOptions, RecipeOptions
    oc, gc = smollm2()
    T, B = 64, 1
    lo = LoraOptions(rank=8, alpha=16.0, targets=("q", "v"), a_std=0.125, b_std=0.01, base_std=0.02)
    rec = LoRA()
    rec.realize(gc, 8, RecipeOptions(t_seq=T, t_batch=B, seed=42), lo)
    mdl = O.qlora_model(oc, O.LoraCfg(rank=8, alpha=16.0, targets=("q", "v"), a_std=0.125, b_std=0.01), seed=42,
                        base_std=0.02)
    eng = rec.lora_cache
    for k in ("blk.0.attn_q.weight", "blk.17.ffn_down.weight", "blk.29.attn_output.weight"):
        assert np.array_equal(eng.q8_0_blocks(k).reshape(-1), mdl.q8[k].reshape(-1)), k
    for k in mdl.trainable:
        got = eng.param(k).astype(np.float32).reshape(mdl.params[k].shape)
        assert np.array_equal(got, mdl.params[k]), k
    for step, seed in ((1, 42), (2, 43)):
        ids, pos, lab = batch(oc, T, B, seed)
        hp = O.hp_lora(1e-4, step, wd=0.01)
        loss_g = rec.step(ids, pos, lab, hp, step == 1)
        loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, step == 1)
        lerr, worst = compare(eng, mdl, loss_g, loss_r, grads)
        report(capsys, "smollm2 qlora B1 T64", step, lerr, worst)
        check(lerr, worst)


def test_smollm2_full_ft_b8_t512(cuda, capsys):
    """The default throughput workload, two steps: full f32 fine-tune, B=8 T=512."""
    from toy_b200 import FromScratch, RecipeOptions
    oc, gc = smollm2()
    T, B = 512, 8
    rec = FromScratch()
    rec.realize(gc, RecipeOptions(t_seq=T, t_batch=B, seed=42, init_std=0.02))
    mdl = O.full_ft_model(oc, seed=42, std_all=0.02)
    eng = rec.fs_cache
    for k in ("token_embd.weight", "blk.0.attn_q.weight", "blk.29.ffn_down.weight"):
        got = eng.param(k).astype(np.float32).reshape(mdl.params[k].shape)
        assert np.array_equal(got.view(np.uint32), mdl.params[k].view(np.uint32)), k
    for step, seed in ((1, 7), (2, 8)):
        ids, pos, lab = batch(oc, T, B, seed)
        hp = O.hp_lora(1e-4, step, wd=0.01)
        loss_g = rec.step(ids, pos, lab, hp, step == 1)
        loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, step == 1)
        lerr, worst = compare(eng, mdl, loss_g, loss_r, grads)
        report(capsys, "smollm2 full FT B8 T512", step, lerr, worst)
        check(lerr, worst)


def test_smollm2_qlora_b8_t512(cuda, capsys):
    """The QLoRA throughput workload, one step: q, v adapters over the Q8_0 base, B=8 T=512."""
    from toy_b200 import LoRA, LoraOptions, RecipeOptions
    oc, gc = smollm2()
    T, B = 512, 8
    lo = LoraOptions(rank=8, alpha=16.0, targets=("q", "v"), a_std=0.125, b_std=0.01, base_std=0.02)
    rec = LoRA()
    rec.realize(gc, 8, RecipeOptions(t_seq=T, t_batch=B, seed=42), lo)
    mdl = O.qlora_model(oc, O.LoraCfg(rank=8, alpha=16.0, targets=("q", "v"), a_std=0.125, b_std=0.01), seed=42,
                        base_std=0.02)
    eng = rec.lora_cache
    ids, pos, lab = batch(oc, T, B, 7)
    hp = O.hp_lora(1e-4, 1, wd=0.01)
    loss_g = rec.step(ids, pos, lab, hp, True)
    loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, True)
    lerr, worst = compare(eng, mdl, loss_g, loss_r, grads)
    report(capsys, "smollm2 qlora B8 T512", 1, lerr, worst)
    check(lerr, worst)
