"""GGUF weights into the step engine, and checkpoints out of it, through the
C ABI (tb2_llama_load_gguf / tb2_llama_save_gguf):

  * the gguf-py fixture (Q8_0 projections, F32 embedding and norms) loads into
    a QLoRA engine with the Q8_0 blocks bit-identical to the file and the f32
    tensors exact; a training step from it matches the oracle built from the
    same tensors (loss 1e-4 relative, gradients / weights 1e-3 relative L2);
  * a full fine-tune loads the same file with the projections dequantised;
    toy's legacy transposed layout loads to the same values;
  * a checkpoint (trainable tensors + Adam moments) written after two steps and
    loaded into a fresh engine continues bit-identically; toy's per-head LoRA-Q
    tensors are written under their per-head names and read back.
"""
import os
import sys

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLD)
import make_gguf as MG  # noqa: E402

NATIVE = os.path.join(GOLD, "tiny_llama_q8.gguf")
LEGACY = os.path.join(GOLD, "tiny_llama_q8_legacy.gguf")


def cfgs():
    from toy_b200 import LlamaConfig
    oc = O.LlamaCfg(vocab=MG.V, d_model=MG.D, n_heads=MG.H, n_kv=MG.KV, d_head=MG.DH, d_ff=MG.FF, n_layers=MG.L,
                    rope_base=1e4)
    return oc, LlamaConfig(MG.V, MG.D, MG.H, MG.KV, MG.DH, MG.FF, MG.L, 1e4, 1e-5)


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300)


def qlora(T=64, B=2, targets=("q", "v")):
    from toy_b200 import LoRA, LoraOptions, RecipeOptions
    oc, gc = cfgs()
    rec = LoRA()
    rec.realize(gc, 8, RecipeOptions(t_seq=T, t_batch=B, seed=4), LoraOptions(rank=8, targets=targets))
    return rec, rec.lora_cache


def test_load_fixture_into_qlora_and_step(cuda):
    oc, gc = cfgs()
    T, B = 64, 2
    rec, eng = qlora(T, B)
    n = eng.load_gguf(NATIVE)
    want = MG.tensors()
    assert n == len(want)
    mdl = O.qlora_model(oc, O.LoraCfg(rank=8, alpha=16.0, targets=("q", "v")), seed=4)
    for name, x in want.items():
        if name in mdl.q8:
            blocks = O.q8_0_quantize(x)
            assert np.array_equal(eng.q8_0_blocks(name).reshape(-1), blocks.reshape(-1)), name
            mdl.q8[name] = blocks
            mdl.params[name] = O.q8_0_dequantize(blocks, x.shape[1])
        else:
            assert np.array_equal(eng.param(name).astype(np.float32).reshape(x.shape), x), name
            mdl.params[name] = x.copy()
    for k in mdl.trainable:   # adapters keep their seeded init
        assert np.array_equal(eng.param(k).astype(np.float32), mdl.params[k]), k
    ids = O.token_ids(3, T * B, oc.vocab)
    pos, lab = O.positions(T, B), O.next_token_labels(ids, T, B, oc.vocab)
    hp = O.hp_lora(1e-3, 1, wd=0.01)
    loss = rec.step(ids, pos, lab, hp, True)
    ref, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, True)
    assert abs(loss - ref) <= 1e-4 * abs(ref)
    for k in mdl.trainable:
        assert rel(eng.grad(k), grads[k]) < 1e-3, k
        assert rel(eng.param(k), mdl.params[k]) < 1e-3, k


@pytest.mark.parametrize("path", [NATIVE, LEGACY])
def test_full_ft_loads_dequantised_or_legacy(cuda, path):
    from toy_b200 import FromScratch, RecipeOptions
    oc, gc = cfgs()
    rec = FromScratch()
    rec.realize(gc, RecipeOptions(t_seq=64, t_batch=1, seed=4))
    rec.fs_cache.load_gguf(path)
    for name, x in MG.tensors().items():
        quant = x.ndim == 2 and name.startswith("blk.")
        want = O.q8_0_dequantize(O.q8_0_quantize(x), x.shape[1]) if (quant and path == NATIVE) else x
        assert np.array_equal(rec.fs_cache.param(name).astype(np.float32).reshape(x.shape), want), name


def test_checkpoint_continues_bit_identically(cuda, tmp_path):
    """Two steps, checkpoint, then one more step in the original session and in a
    fresh one restored from the base file and the checkpoint."""
    from toy_b200._lib import lib
    oc, gc = cfgs()
    T, B = 64, 2
    targets = ("q", "v", "down")
    rec, eng = qlora(T, B, targets)
    eng.load_gguf(NATIVE)
    batches = []
    for s in range(3):
        ids = O.token_ids(50 + s, T * B, oc.vocab)
        batches.append((ids, O.positions(T, B), O.next_token_labels(ids, T, B, oc.vocab), O.hp_lora(1e-3, s + 1)))
    for s in range(2):
        rec.step(*batches[s], s == 0)
    ck = str(tmp_path / "ck.gguf")
    eng.save_gguf(ck, moments=True)
    rec2, eng2 = qlora(T, B, targets)
    eng2.load_gguf(NATIVE)
    eng2.load_gguf(ck, moments=True, partial=True)   # resume: the next step is not a first step, so the moments stay
    names = [k for k in eng.param_names() if eng.trainable(k)]
    for k in names:
        assert np.array_equal(eng2.param(k), eng.param(k)), k
        assert np.array_equal(eng2.moment(k, 0), eng.moment(k, 0)), k
    l1 = rec.step(*batches[2], False)
    l2 = rec2.step(*batches[2], False)
    assert l1 == l2
    for k in names:
        assert np.array_equal(eng2.param(k), eng.param(k)), k


def test_lora_q_checkpoint_uses_per_head_names(cuda, tmp_path):
    from toy_b200 import LoRA, RecipeOptions
    from toy_b200._lib import lib
    oc, gc = cfgs()
    rec = LoRA()
    rec.realize(gc, 8, RecipeOptions(t_seq=64, t_batch=1, seed=4, init_scale=0.5))
    eng = rec.lora_cache
    ids = O.token_ids(3, 64, oc.vocab)
    rec.step(ids, O.positions(64, 1), O.next_token_labels(ids, 64, 1, oc.vocab), O.hp_lora(1e-3, 1), True)
    ck = str(tmp_path / "lq.gguf")
    eng.save_gguf(ck)
    L = lib()
    h = L.tnn_gguf_load(ck.encode())
    try:
        for l in range(MG.L):
            for hd in range(MG.H):
                for ab, shape in (("a", (8, MG.D)), ("b", (MG.DH, 8))):
                    i = L.tnn_gguf_find_index(h, f"blk.{l}.attn_q.head_{hd}.lora_{ab}.weight".encode())
                    assert i >= 0
                    assert (L.tnn_gguf_tensor_ne(h, i, 1), L.tnn_gguf_tensor_ne(h, i, 0)) == shape
        assert L.tnn_gguf_find_index(h, b"blk.0.attn_q.lora_a") == -1
    finally:
        L.tnn_gguf_free(h)
    rec2 = LoRA()
    rec2.realize(gc, 8, RecipeOptions(t_seq=64, t_batch=1, seed=99, init_scale=0.5))
    rec2.lora_cache.load_gguf(ck, partial=True)
    for k in ("blk.0.attn_q.lora_a", "blk.1.attn_q.lora_b"):
        assert np.array_equal(rec2.lora_cache.param(k), eng.param(k)), k
