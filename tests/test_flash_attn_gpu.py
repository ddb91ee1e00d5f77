"""Fused flash attention (head widths 64 and 128) inside the training step, through the C ABI.

The step with the fused attention kernels is checked against the oracle with
the training-step tolerances (loss 1e-4 relative; gradients, post-AdamW
weights and moments 1e-3 relative L2), and against the materialised-score path
of the same library on identical inputs, where both compute the same products
in split-bf16 and differ only by f32 summation order: loss 1e-6 relative and
gradients 1e-4 relative L2 after one step.

AdamW's first update is close to lr * sign(g), so elements whose gradient is
near zero can move either way under 1e-5-level gradient differences; a second
step on the same batch then amplifies that. Multi-step checks therefore use
lr 1e-4 (the LoRA recipe's rate) and a fresh batch for step 2.
Sequence lengths cover whole 128-row tiles, a ragged last tile and a sequence
shorter than one tile. At head width 128 the kernels tile by 64 keys (forward)
and 64 queries (backward), so the lengths also cover a ragged 64-wide tile;
that configuration has grouped-query attention with two query heads per
key/value head.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.test_step_parity_gpu import compare_step, inputs, rel

pytestmark = pytest.mark.gpu


def cfgs64(n_layers=2, dh=64):
    """Two-layer model: 4 query heads of width 64 over d 256, or of width 128 over d 512; 2 KV heads."""
    from toy_b200 import LlamaConfig
    d = 4 * dh
    oc = O.LlamaCfg(vocab=512, d_model=d, n_heads=4, n_kv=2, d_head=dh, d_ff=512, n_layers=n_layers,
                    rope_base=1e4)
    gc = LlamaConfig(512, d, 4, 2, dh, 512, n_layers, 1e4, 1e-5)
    return oc, gc


@pytest.mark.parametrize("dh,T,B", [(64, 128, 2), (64, 96, 2), (64, 200, 1),
                                    (128, 128, 2), (128, 96, 2), (128, 200, 1), (128, 40, 2)])
def test_flash_step_matches_oracle(cuda, dh, T, B):
    from toy_b200 import FromScratch, RecipeOptions
    oc, gc = cfgs64(dh=dh)
    rec = FromScratch()
    rec.realize(gc, RecipeOptions(t_seq=T, t_batch=B, seed=3, init_scale=1.0, attention="flash"))
    mdl = O.full_ft_model(oc, seed=3, init_scale=1.0)
    for step in (1, 2):
        ids, pos, lab = inputs(oc, T, B, seed=5 if step == 1 else 9)
        hp = O.hp_lora(1e-4, step, wd=0.01)
        loss_g = rec.step(ids, pos, lab, hp, step == 1)
        loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, step == 1)
        compare_step(rec.fs_cache, mdl, loss_g, loss_r, grads)


@pytest.mark.parametrize("dh", [64, 128])
def test_flash_qlora_step_matches_oracle(cuda, dh):
    from toy_b200 import LoRA, LoraOptions, RecipeOptions
    oc, gc = cfgs64(dh=dh)
    T, B = 128, 2
    targets = ("q", "k", "v", "o")
    rec = LoRA()
    lo = LoraOptions(rank=8, alpha=16.0, targets=targets, a_std=0.125, b_std=0.01, base_std=0.02)
    rec.realize(gc, 8, RecipeOptions(t_seq=T, t_batch=B, seed=11, attention="flash"), lo)
    mdl = O.qlora_model(oc, O.LoraCfg(rank=8, alpha=16.0, targets=targets, a_std=0.125, b_std=0.01), seed=11,
                        base_std=0.02)
    ids, pos, lab = inputs(oc, T, B)
    hp = O.hp_lora(1e-4, 1, wd=0.01)
    loss_g = rec.step(ids, pos, lab, hp, True)
    loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, True)
    compare_step(rec.lora_cache, mdl, loss_g, loss_r, grads)


def _run(gc, T, B, attention, steps=1):
    from toy_b200 import FromScratch, RecipeOptions
    oc, _ = cfgs64(gc.n_layers, gc.d_head)
    rec = FromScratch()
    rec.realize(gc, RecipeOptions(t_seq=T, t_batch=B, seed=7, init_scale=1.0, attention=attention))
    ids, pos, lab = inputs(oc, T, B, seed=9)
    losses = []
    for s in range(steps):
        losses.append(rec.step(ids, pos, lab, O.hp_lora(1e-3, s + 1, wd=0.01), s == 0))
    eng = rec.fs_cache
    names = [n for n in eng.param_names() if eng.trainable(n)]
    return losses, {n: eng.grad(n) for n in names}, {n: eng.param(n) for n in names}


@pytest.mark.parametrize("dh,T,B", [(64, 512, 2), (64, 384, 1), (64, 192, 2), (128, 512, 2), (128, 192, 2)])
def test_flash_matches_materialized(cuda, dh, T, B):
    _, gc = cfgs64(dh=dh)
    lf, gf, pf = _run(gc, T, B, "flash")
    lm, gm, pm = _run(gc, T, B, "materialized")
    for a, b in zip(lf, lm):
        assert abs(a - b) <= 1e-6 * abs(b), (a, b)
    for n in gm:
        assert rel(gf[n], gm[n]) < 1e-4, ("grad", n, rel(gf[n], gm[n]))
        assert rel(pf[n], pm[n]) < 1e-3, ("param", n, rel(pf[n], pm[n]))


@pytest.mark.parametrize("dh", [64, 128])
def test_flash_deterministic(cuda, dh):
    _, gc = cfgs64(dh=dh)
    a = _run(gc, 256, 2, "flash", steps=2)
    b = _run(gc, 256, 2, "flash", steps=2)
    assert a[0] == b[0]
    for n in a[1]:
        assert np.array_equal(a[1][n], b[1][n]), n
