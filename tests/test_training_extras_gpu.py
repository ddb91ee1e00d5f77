"""Training-step features beyond the benchmark configurations, through the C ABI
against the oracle with the step contract's tolerances (loss 1e-4 relative;
gradients, weights and Adam moments 1e-3 relative L2):

  * true gradient accumulation: two micro-batches of one sequence each give the
    step on the joined two-sequence batch (the reference only approximates it by
    running AdamW every micro-batch at lr / N,
    examples/legacy/06_train_from_scratch.rb:64-78); weights do not move on the
    accumulating call;
  * untied LM head (RecipeOptions.untied; output.weight drawn after the
    embedding, llama_seq_engine.rb:1161-1340), full fine-tune and QLoRA;
  * embedding training at the large vocabularies of the other configurations
    (Llama-3.2: 128256, Qwen2.5: 151936 padded to 152064), tied and untied: the
    deterministic scatter-add of get_rows_back and the CE over ~150k columns.
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


def tiny(tied=True):
    from toy_b200 import LlamaConfig
    oc = O.LlamaCfg(vocab=512, d_model=128, n_heads=4, n_kv=2, d_head=32, d_ff=256, n_layers=2, rope_base=1e4,
                    tied=tied)
    gc = LlamaConfig(512, 128, 4, 2, 32, 256, 2, 1e4, 1e-5, tied=tied)
    return oc, gc


def check_state(eng, mdl, grads=None):
    for k in mdl.trainable:
        if grads is not None:
            g = eng.grad(k)
            assert rel(g, grads[k].reshape(g.shape)) < REL_L2, ("grad", k)
        p = eng.param(k)
        assert rel(p, mdl.params[k].reshape(p.shape)) < REL_L2, ("param", k)
        for w, ref in ((0, mdl.m[k]), (1, mdl.v[k])):
            mo = eng.moment(k, w)
            assert rel(mo, ref.reshape(mo.shape)) < REL_L2, ("moment", w, k)


def make(mode, gc, T, B, seed):
    from toy_b200 import FromScratch, LoRA, LoraOptions, RecipeOptions
    if mode == "full":
        rec = FromScratch()
        rec.realize(gc, RecipeOptions(t_seq=T, t_batch=B, seed=seed))
        return rec, rec.fs_cache
    rec = LoRA()
    rec.realize(gc, 8, RecipeOptions(t_seq=T, t_batch=B, seed=seed),
                LoraOptions(rank=8, targets=("q", "v", "down")))
    return rec, rec.lora_cache


def oracle_model(mode, oc, seed):
    if mode == "full":
        return O.full_ft_model(oc, seed=seed)
    return O.qlora_model(oc, O.LoraCfg(rank=8, alpha=16.0, targets=("q", "v", "down")), seed=seed)


@pytest.mark.parametrize("mode", ["full", "qlora"])
def test_grad_accumulation_equals_joined_batch(cuda, mode):
    oc, gc = tiny()
    T = 64
    rec, eng = make(mode, gc, T, 1, 3)
    eng.set_grad_accumulation(2)
    mdl = oracle_model(mode, oc, 3)
    for window in range(2):
        ids = O.token_ids(20 + window, 2 * T, oc.vocab)
        lab = O.next_token_labels(ids, T, 2, oc.vocab)
        hp = O.hp_lora(1e-3, window + 1, wd=0.01)
        before = {k: eng.param(k) for k in mdl.trainable}
        for micro in range(2):
            sl = slice(micro * T, (micro + 1) * T)
            loss = rec.step(ids[sl], O.positions(T, 1), lab[sl], hp, window == 0 and micro == 0)
            ref, _, _ = O.forward_backward(mdl, ids[sl], O.positions(T, 1), lab[sl], T, 1, want_grads=False)
            assert abs(loss - ref) <= LOSS_TOL * abs(ref), (window, micro, loss, ref)
            if micro == 0:   # accumulating call: no optimiser step
                for k in mdl.trainable:
                    assert np.array_equal(eng.param(k), before[k]), k
        O.train_step(mdl, ids, O.positions(T, 2), lab, T, 2, hp, window == 0)
        check_state(eng, mdl)


@pytest.mark.parametrize("mode", ["full", "qlora"])
def test_untied_head(cuda, mode):
    oc, gc = tiny(tied=False)
    T, B = 64, 2
    from toy_b200 import FromScratch, LoRA, LoraOptions, RecipeOptions
    rec, eng = make(mode, gc, T, B, 5)
    mdl = oracle_model(mode, oc, 5)
    assert "output.weight" in eng.param_names()
    got = eng.param("output.weight").astype(np.float32)
    assert np.array_equal(got, mdl.params["output.weight"])
    for step in (1, 2):
        ids = O.token_ids(30 + step, T * B, oc.vocab)
        pos, lab = O.positions(T, B), O.next_token_labels(ids, T, B, oc.vocab)
        hp = O.hp_lora(1e-3, step, wd=0.01)
        loss = rec.step(ids, pos, lab, hp, step == 1)
        ref, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, step == 1)
        assert abs(loss - ref) <= LOSS_TOL * abs(ref)
        check_state(eng, mdl, grads)


@pytest.mark.parametrize("vocab", [128256, 152064])
@pytest.mark.parametrize("tied", [True, False])
def test_large_vocab_embedding_training(cuda, vocab, tied):
    from toy_b200 import FromScratch, LlamaConfig, RecipeOptions
    oc = O.LlamaCfg(vocab=vocab, d_model=64, n_heads=1, n_kv=1, d_head=64, d_ff=128, n_layers=1, rope_base=5e5,
                    tied=tied)
    gc = LlamaConfig(vocab, 64, 1, 1, 64, 128, 1, 5e5, 1e-5, tied=tied)
    T, B = 64, 2
    rec = FromScratch()
    rec.realize(gc, RecipeOptions(t_seq=T, t_batch=B, seed=9))
    mdl = O.full_ft_model(oc, seed=9)
    ids = O.token_ids(4, T * B, vocab)
    ids[5] = ids[70] = ids[100]   # a repeated id: the scatter-add sums its rows
    pos, lab = O.positions(T, B), O.next_token_labels(ids, T, B, vocab)
    hp = O.hp_lora(1e-3, 1, wd=0.01)
    loss = rec.step(ids, pos, lab, hp, True)
    ref, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, True)
    assert abs(loss - ref) <= LOSS_TOL * abs(ref)
    check_state(rec.fs_cache, mdl, grads)
    # rows of ids that never occur get no embedding gradient unless the head is tied
    g = rec.fs_cache.grad("token_embd.weight")
    unseen = np.setdiff1d(np.arange(vocab), ids)[:50]
    assert (np.count_nonzero(g[unseen]) == 0) == (not tied)
