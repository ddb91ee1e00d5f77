"""toy's own LoRA recipe on the fused step: per-head LoRA-Q.

Toy::LLM::Recipes::LoRA#realize! enables one adapter pair per query head
(A_h [r x d], B_h [d_head x r], no alpha / r scale; transformer_block.rb:522-579,
861-871) and initialises it with upload_lora_q_init!(seed, init_scale): the raw
seed drives the LCG, A = init_scale * N(0, 1) from the cos branch, B = 0
(llama_seq_engine.rb:2545-2575). Checked through the C ABI against the oracle
with the training-step tolerances (loss 1e-4 relative; gradients, weights and
moments 1e-3 relative L2; A's init bit-exact, B zero) over two steps, the
second on a fresh batch (on step one B = 0 makes dA exactly zero).

A tensor that starts at zero (every B_h) leaves the first AdamW step as
-lr * g / (|g| + eps), i.e. +-lr per element: its post-step weights compare
the gradients' signs. An element whose oracle gradient is below 1e-3 of the
tensor's RMS gradient has a sign the gradient tolerance does not determine, so
those elements (at most 1 % of the tensor) are left out of that tensor's
weight comparison, its gradient and moments are compared in full, and the
oracle then takes the device's values of those elements, so that the next
step compares arithmetic rather than that sign choice.
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


def run(oc, gc, T, B, rank, init_scale, seed, lr, capsys=None, tag=""):
    from toy_b200 import LoRA, RecipeOptions
    rec = LoRA()
    rec.realize(gc, rank, RecipeOptions(t_seq=T, t_batch=B, seed=seed, init_scale=init_scale))
    mdl = O.qlora_model(oc, O.LoraCfg(rank=rank, per_head_q=True, targets=("q",), a_std=init_scale), seed=seed,
                        base_std=0.02)
    eng = rec.lora_cache
    assert sorted(k for k in eng.param_names() if eng.trainable(k)) == sorted(mdl.trainable)
    for k in mdl.trainable:
        got = eng.param(k).astype(np.float32).reshape(mdl.params[k].shape)
        assert np.array_equal(got.view(np.uint32), mdl.params[k].view(np.uint32)), k
    sign_free = {}   # zero-initialised tensors: elements whose first update sign is undetermined
    for step, bseed in ((1, 5), (2, 6)):
        ids = O.token_ids(bseed, T * B, oc.vocab)
        pos, lab = O.positions(T, B), O.next_token_labels(ids, T, B, oc.vocab)
        hp = O.hp_lora(lr, step, wd=0.01)
        before = {k: mdl.params[k].copy() for k in mdl.trainable}
        loss_g = rec.step(ids, pos, lab, hp, step == 1)
        loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, step == 1)
        assert abs(loss_g - loss_r) <= LOSS_TOL * abs(loss_r), (step, loss_g, loss_r)
        worst = []
        for k in mdl.trainable:
            g = eng.grad(k)
            gr = grads[k].reshape(g.shape)
            worst.append((rel(g, gr), "grad " + k))
            if not np.any(before[k]):
                tiny = np.abs(gr) < 1e-3 * np.sqrt(np.mean(gr * gr))
                sign_free[k] = tiny | sign_free.get(k, False)
                assert sign_free[k].mean() <= 1e-2, (k, sign_free[k].mean())
            keep = ~sign_free[k] if k in sign_free else np.ones(g.shape, bool)
            p = eng.param(k)
            worst.append((rel(p[keep], mdl.params[k].reshape(p.shape)[keep]), "param " + k))
            for w, ref in ((0, mdl.m[k]), (1, mdl.v[k])):
                mo = eng.moment(k, w)
                worst.append((rel(mo, ref.reshape(mo.shape)), ("m " if w == 0 else "v ") + k))
        worst.sort()
        if capsys is not None:
            with capsys.disabled():
                print(f"\n[{tag} step {step}] loss rel err {abs(loss_g - loss_r) / abs(loss_r):.2e}; worst "
                      + ", ".join(f"{r:.2e} {k}" for r, k in worst[-3:][::-1]))
        for r, k in worst:
            assert r < REL_L2, (step, k, r)
        if step == 1:   # B = 0 on the first step: no gradient reaches A
            for k in mdl.trainable:
                if k.endswith("lora_a"):
                    assert not np.any(eng.grad(k)), k
        # the undetermined signs are the device's choice from here on: the
        # oracle continues from the device's value of those elements (and their
        # moments), so later steps compare the arithmetic, not that choice
        for k, mask in sign_free.items():
            if step == 1 and mask.any():
                shp = mdl.params[k].shape
                for dst, src in ((mdl.params, eng.param(k)), (mdl.m, eng.moment(k, 0)), (mdl.v, eng.moment(k, 1))):
                    arr = dst[k].reshape(-1).copy()
                    arr[mask.reshape(-1)] = np.asarray(src, arr.dtype).reshape(-1)[mask.reshape(-1)]
                    dst[k] = arr.reshape(shp)
        sign_free = {k: np.zeros_like(v) for k, v in sign_free.items()}


@pytest.mark.parametrize("init_scale", [1.0, 0.125])
def test_lora_q_tiny(cuda, init_scale):
    from toy_b200 import LlamaConfig
    oc = O.LlamaCfg(vocab=512, d_model=128, n_heads=4, n_kv=2, d_head=32, d_ff=256, n_layers=3, rope_base=1e4)
    gc = LlamaConfig(512, 128, 4, 2, 32, 256, 3, 1e4, 1e-5)
    run(oc, gc, 64, 2, 8, init_scale, 7, 1e-3)


def test_lora_q_smollm2_b1_t64(cuda, capsys):
    """The reference recipe at its own model size: SmolLM2-135M, 9 query heads of
    rank 8 per layer (72 extension columns on the q|k|v GEMMs), init_scale 1.0."""
    from toy_b200 import LlamaConfig
    run(O.smollm2_135m(), LlamaConfig.smollm2_135m(), 64, 1, 8, 1.0, 42, 1e-4, capsys, "smollm2 LoRA-Q")


def test_lora_q_needs_ring_and_q_only(cuda):
    from toy_b200 import LlamaConfig, LoRA, LoraOptions, RecipeOptions
    from toy_b200._lib import lib
    gc = LlamaConfig(512, 128, 4, 2, 32, 256, 1, 1e4, 1e-5)
    with pytest.raises(ValueError):
        LoRA().realize(gc, 8, RecipeOptions(t_seq=64), LoraOptions(rank=8, targets=("q", "v"), per_head_q=True))
    prev = lib().tb2_set_q8_base_mode(0)
    try:
        with pytest.raises(RuntimeError):
            LoRA().realize(gc, 8, RecipeOptions(t_seq=64))
    finally:
        lib().tb2_set_q8_base_mode(prev)
