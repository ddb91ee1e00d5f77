"""Decode with a KV cache (tb2_kv_*, through the C ABI) against the oracle's
full-sequence forward: the logits after each teacher-forced token equal the
oracle's logits row for that position (f32 cache: 1e-4 relative L2 per row;
Q8_0 cache: the oracle with the same Q8_0 round trip of K and V, median row
1e-3, every row 1e-2), for
several sequences in lockstep, over the Q8_0 base with its LoRA adapters
(plain adapters on q and v, on all seven projections, and toy's per-head
LoRA-Q, each with nonzero B so that the adapters change the logits) and over
f32 weights, at SmolLM2-135M's full shape, plus a greedy continuation and
argument checks."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / np.linalg.norm(b)


def tiny():
    from toy_b200 import LlamaConfig
    oc = O.LlamaCfg(vocab=512, d_model=128, n_heads=4, n_kv=2, d_head=32, d_ff=256, n_layers=2, rope_base=1e4)
    return oc, LlamaConfig(512, 128, 4, 2, 32, 256, 2, 1e4, 1e-5)


def set_adapters_b(eng, mdl, seed):
    """B starts at zero; give every adapter B seeded N(0, 0.05) values on both sides."""
    rng = np.random.default_rng(seed)
    for k in mdl.trainable:
        if k.endswith(".lora_b"):
            v = (rng.standard_normal(mdl.params[k].shape) * 0.05).astype(np.float32)
            mdl.params[k] = v
            eng.set_param(k, v)


def base_model(mode, oc, gc, seed, targets=("q", "v")):
    """A realised step engine (its weights feed the decoder) and the oracle model
    of the same weights, adapters included ("q8": plain adapters on `targets`;
    "lora_q": toy's per-head LoRA-Q)."""
    from toy_b200 import FromScratch, LoRA, LoraOptions, RecipeOptions
    if mode == "q8":
        rec = LoRA()
        rec.realize(gc, 8, RecipeOptions(t_seq=64, t_batch=1, seed=seed), LoraOptions(rank=8, targets=targets))
        mdl = O.qlora_model(oc, O.LoraCfg(rank=8, alpha=16.0, targets=targets), seed=seed)
        set_adapters_b(rec.lora_cache, mdl, seed + 100)
        return rec.lora_cache, mdl
    if mode == "lora_q":
        rec = LoRA()
        rec.realize(gc, 4, RecipeOptions(t_seq=64, t_batch=1, seed=seed, init_scale=0.05))
        mdl = O.qlora_model(oc, O.LoraCfg(rank=4, per_head_q=True, targets=("q",), a_std=0.05), seed=seed,
                            base_std=0.02)
        set_adapters_b(rec.lora_cache, mdl, seed + 100)
        return rec.lora_cache, mdl
    rec = FromScratch()
    rec.realize(gc, RecipeOptions(t_seq=64, t_batch=1, seed=seed))
    return rec.fs_cache, O.full_ft_model(oc, seed=seed)


def check_decode(eng, mdl, oc, T, nseq, kv_q8, tol):
    from toy_b200.decode import KVDecoder
    dec = KVDecoder(eng, max_T=max(T, 300), n_seq=nseq, kv_q8=kv_q8)
    ids = O.token_ids(11, T * nseq, oc.vocab)
    got = dec.decode_batch(ids.reshape(nseq, T))                      # [T, nseq, V]
    _, _, ref = O.forward_backward(mdl, ids, O.positions(T, nseq), O.next_token_labels(ids, T, nseq, oc.vocab),
                                   T, nseq, want_grads=False, kv_q8=kv_q8)
    ref = ref.reshape(nseq, T, -1)
    errs = np.array([rel(got[t, b], ref[b, t]) for t in range(T) for b in range(nseq)])
    worst = float(errs.max())
    if kv_q8:
        # a K / V value on a rounding boundary of the Q8_0 grid can land on either
        # side between the f32 device and the f64 oracle, moving that element by
        # one quantum (1/127 of its block's largest value): the typical position
        # stays at the bound, a few may exceed it by an order of magnitude
        assert float(np.median(errs)) < tol and worst < 10 * tol, (float(np.median(errs)), worst)
    else:
        assert worst < tol, worst
    dec.reset()   # a fresh set of sequences reproduces the first step exactly
    again = dec.decode_step(ids.reshape(nseq, T)[:, 0], np.zeros(nseq, np.int64))
    assert np.array_equal(again, got[0])
    dec.close()
    return worst


@pytest.mark.parametrize("mode", ["q8", "f32"])
@pytest.mark.parametrize("kv_q8", [False, True])
def test_decode_tiny(cuda, mode, kv_q8):
    oc, gc = tiny()
    eng, mdl = base_model(mode, oc, gc, 3)
    check_decode(eng, mdl, oc, 40, 3, kv_q8, 1e-3 if kv_q8 else 1e-4)


@pytest.mark.parametrize("mode", ["lora_q", "all7"])
def test_decode_adapters(cuda, mode):
    """toy's per-head LoRA-Q (its KV engine adds B_h A_h h to each query head
    before the bias, llama_kv_engine.rb:2157-2167) and plain adapters on all
    seven projections."""
    oc, gc = tiny()
    if mode == "lora_q":
        eng, mdl = base_model("lora_q", oc, gc, 4)
    else:
        eng, mdl = base_model("q8", oc, gc, 4, targets=("q", "k", "v", "o", "gate", "up", "down"))
    check_decode(eng, mdl, oc, 24, 2, False, 1e-4)


def test_decode_history_longer_than_a_chunk(cuda):
    """Positions past 256 keys: the attention splits the history into chunks."""
    oc, gc = tiny()
    eng, mdl = base_model("q8", oc, gc, 5)
    check_decode(eng, mdl, oc, 290, 1, False, 1e-4)


@pytest.mark.parametrize("kv_q8", [False, True])
def test_decode_smollm2(cuda, kv_q8, capsys):
    from toy_b200 import LlamaConfig
    oc, gc = O.smollm2_135m(), LlamaConfig.smollm2_135m()
    eng, mdl = base_model("q8", oc, gc, 42)
    w = check_decode(eng, mdl, oc, 48, 2, kv_q8, 1e-3 if kv_q8 else 1e-4)
    with capsys.disabled():
        print(f"\n[smollm2 decode kv_q8={kv_q8}] worst logits rel L2 {w:.2e}")


def test_generate_and_bad_arguments(cuda):
    from toy_b200._lib import lib
    from toy_b200.decode import KVDecoder
    oc, gc = tiny()
    eng, mdl = base_model("q8", oc, gc, 3)
    dec = KVDecoder(eng, max_T=64, n_seq=2)
    prompt = O.token_ids(2, 16, oc.vocab).reshape(2, 8)
    out = dec.generate(prompt, 6)
    assert out.shape == (2, 6) and out.min() >= 0 and out.max() < oc.vocab
    # the greedy tokens are the oracle's argmax over the growing sequence
    seq = np.concatenate([prompt, out], axis=1)
    for b in range(2):
        _, _, ref = O.forward_backward(mdl, seq[b], O.positions(14, 1), O.next_token_labels(seq[b], 14, 1, oc.vocab),
                                       14, 1, want_grads=False)
        assert np.array_equal(np.argmax(ref[7:13], axis=-1), out[b, :6])
    with pytest.raises(RuntimeError):
        dec.decode_step([1, 2], [64, 0])            # past max_T
    with pytest.raises(RuntimeError):
        dec.decode_step([oc.vocab, 2], [0, 0])      # token out of range
    dec.close()
    assert lib().tb2_kv_realize(eng.sess, 64, 9, 0) == -1   # 9 sequences: not a supported width
    assert lib().tb2_kv_realize(eng.sess, 64, 1, 4) == -1   # unknown cache type
