"""Step parity for the model families of the other benchmark configurations,
at reduced width / depth so the float64 oracle finishes in seconds:

* Llama-3.2-1B family: grouped-query attention (4:1), RoPE base 5e5 with
  llama3 frequency factors (factor 32, low / high 1 / 4, original context 8192),
  QLoRA rank 16 on all seven projections;
* Qwen2.5-7B family: d_head 128 (the materialised attention path), q/k/v bias,
  RoPE base 1e6, RMSNorm eps 1e-6, QLoRA rank 16 on all seven projections, and
  the same shape fully fine-tuned (bias gradients included);
* both at their full layer width (one layer, small vocabulary), where the
  adapters' down passes run over column chunks.

Same contract as the SmolLM2 tests: loss 1e-4 relative; gradients, post-AdamW
parameters and moments 1e-3 relative L2; Q8_0 blocks bit-exact.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.test_step_parity_gpu import compare_step, inputs

pytestmark = pytest.mark.gpu


def llama3_family():
    from toy_b200 import LlamaConfig
    ff = O.llama3_freq_factors(64, 5.0e5, 8192, 32.0, 1.0, 4.0)
    oc = O.LlamaCfg(vocab=640, d_model=256, n_heads=8, n_kv=2, d_head=64, d_ff=512, n_layers=2, rope_base=5.0e5,
                    rope_freq_factors=ff)
    gc = LlamaConfig(640, 256, 8, 2, 64, 512, 2, 5.0e5, 1e-5, rope_freq_factors=list(ff))
    return oc, gc


def qwen_family():
    from toy_b200 import LlamaConfig
    oc = O.LlamaCfg(vocab=512, d_model=256, n_heads=4, n_kv=2, d_head=128, d_ff=640, n_layers=2, rope_base=1.0e6,
                    rms_eps=1e-6, qkv_bias=True)
    gc = LlamaConfig(512, 256, 4, 2, 128, 640, 2, 1.0e6, 1e-6, qkv_bias=True)
    return oc, gc


def llama3_full_width():
    """Llama-3.2-1B's full layer width (d 2048, 32 / 8 heads, d_ff 8192), one layer, a small vocabulary."""
    from toy_b200 import LlamaConfig
    ff = O.llama3_freq_factors(64, 5.0e5, 8192, 32.0, 1.0, 4.0)
    oc = O.LlamaCfg(vocab=1024, d_model=2048, n_heads=32, n_kv=8, d_head=64, d_ff=8192, n_layers=1,
                    rope_base=5.0e5, rope_freq_factors=ff)
    gc = LlamaConfig(1024, 2048, 32, 8, 64, 8192, 1, 5.0e5, 1e-5, rope_freq_factors=list(ff))
    return oc, gc


def qwen_full_width():
    """Qwen2.5-7B's full layer width (d 3584, 28 / 4 heads of 128, d_ff 18944), one layer, a small vocabulary."""
    from toy_b200 import LlamaConfig
    oc = O.LlamaCfg(vocab=1024, d_model=3584, n_heads=28, n_kv=4, d_head=128, d_ff=18944, n_layers=1,
                    rope_base=1.0e6, rms_eps=1e-6, qkv_bias=True)
    gc = LlamaConfig(1024, 3584, 28, 4, 128, 18944, 1, 1.0e6, 1e-6, qkv_bias=True)
    return oc, gc


ALL = ("q", "k", "v", "o", "gate", "up", "down")


@pytest.mark.parametrize("family", [llama3_family, qwen_family])
def test_qlora_rank16_all_targets(cuda, family):
    from toy_b200 import LoRA, LoraOptions, RecipeOptions
    oc, gc = family()
    T, B = 128, 2
    rec = LoRA()
    lo = LoraOptions(rank=16, alpha=32.0, targets=ALL, a_std=0.125, b_std=0.01, base_std=0.02)
    rec.realize(gc, 16, RecipeOptions(t_seq=T, t_batch=B, seed=21), lo)
    mdl = O.qlora_model(oc, O.LoraCfg(rank=16, alpha=32.0, targets=ALL, a_std=0.125, b_std=0.01), seed=21,
                        base_std=0.02)
    eng = rec.lora_cache
    for k in mdl.trainable:   # the adapters' init is bit-exact
        got = eng.param(k).astype(np.float32).reshape(mdl.params[k].shape)
        assert np.array_equal(got, mdl.params[k]), k
    for k, blocks in mdl.q8.items():
        assert np.array_equal(eng.q8_0_blocks(k).reshape(-1), blocks.reshape(-1)), k
    ids, pos, lab = inputs(oc, T, B, seed=8)
    for step in (1, 2):
        hp = O.hp_lora(1e-4, step, wd=0.01)
        loss_g = rec.step(ids, pos, lab, hp, step == 1)
        loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, step == 1)
        compare_step(eng, mdl, loss_g, loss_r, grads)


@pytest.mark.parametrize("family", [llama3_full_width, qwen_full_width])
def test_qlora_rank16_full_width(cuda, family):
    """At the real layer widths the adapters' A (rank 16 x d_in, up to three per
    group) no longer fit in shared memory: the adapter down passes run over
    column chunks, summed in order. One layer, T = 64, one sequence."""
    from toy_b200 import LoRA, LoraOptions, RecipeOptions
    oc, gc = family()
    T, B = 64, 1
    rec = LoRA()
    lo = LoraOptions(rank=16, alpha=32.0, targets=ALL, a_std=0.125, b_std=0.01, base_std=0.02)
    rec.realize(gc, 16, RecipeOptions(t_seq=T, t_batch=B, seed=23), lo)
    mdl = O.qlora_model(oc, O.LoraCfg(rank=16, alpha=32.0, targets=ALL, a_std=0.125, b_std=0.01), seed=23,
                        base_std=0.02)
    eng = rec.lora_cache
    ids, pos, lab = inputs(oc, T, B, seed=9)
    for step in (1, 2):
        hp = O.hp_lora(1e-4, step, wd=0.01)
        loss_g = rec.step(ids, pos, lab, hp, step == 1)
        loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, step == 1)
        compare_step(eng, mdl, loss_g, loss_r, grads)


def test_qwen_family_full_ft(cuda):
    from toy_b200 import FromScratch, RecipeOptions
    oc, gc = qwen_family()
    T, B = 128, 2
    rec = FromScratch()
    rec.realize(gc, RecipeOptions(t_seq=T, t_batch=B, seed=5, init_scale=1.0))
    mdl = O.full_ft_model(oc, seed=5, init_scale=1.0)
    eng = rec.fs_cache
    ids, pos, lab = inputs(oc, T, B, seed=4)
    hp = O.hp_lora(1e-4, 1, wd=0.01)
    loss_g = rec.step(ids, pos, lab, hp, True)
    loss_r, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, True)
    compare_step(eng, mdl, loss_g, loss_r, grads)
