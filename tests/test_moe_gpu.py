"""Mixture-of-experts blocks (the OLMoE configuration's FFN) in the fused
training step, through the C ABI against the oracle's restatement (the
reference has no backward for mul_mat_id, so the oracle's hand-written MoE
backward -- itself checked against torch autograd on CPU -- is the reference
here). QLoRA over frozen Q8_0 experts and an f32 router, adapters on q, k, v, o,
whole-vector QK-RMSNorm; loss within 1e-4 relative, gradients, weights and
moments within 1e-3 relative L2, over two steps; the Q8_0 expert blocks
bit-exact."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (nb if nb > 0 else 1.0)


def run(d, H, dh, E, K, norm_topk, qk_norm, attention="flash", T=64, B=2, capsys=None, tag=""):
    from toy_b200 import LlamaConfig, LoRA, LoraOptions, RecipeOptions
    targets = ("q", "k", "v", "o")
    oc = O.LlamaCfg(vocab=512, d_model=d, n_heads=H, n_kv=H, d_head=dh, d_ff=64, n_layers=2, rope_base=1e4,
                    n_experts=E, n_experts_used=K, norm_topk=norm_topk, qk_norm=qk_norm)
    gc = LlamaConfig(512, d, H, H, dh, 64, 2, 1e4, 1e-5, n_experts=E, n_experts_used=K, norm_topk=norm_topk,
                     qk_norm=qk_norm)
    rec = LoRA()
    rec.realize(gc, 8, RecipeOptions(t_seq=T, t_batch=B, seed=21, attention=attention),
                LoraOptions(rank=8, alpha=16.0, targets=targets))
    mdl = O.qlora_model(oc, O.LoraCfg(rank=8, alpha=16.0, targets=targets), seed=21)
    eng = rec.lora_cache
    for k in ("blk.0.ffn_gate_exps.weight", "blk.1.ffn_down_exps.weight"):
        assert np.array_equal(eng.q8_0_blocks(k).reshape(-1), mdl.q8[k].reshape(-1)), k
    assert np.array_equal(eng.param("blk.1.ffn_gate_inp.weight").astype(np.float32),
                          mdl.params["blk.1.ffn_gate_inp.weight"])
    worst = []
    for step, seed in ((1, 3), (2, 4)):
        ids = O.token_ids(seed, T * B, oc.vocab)
        pos, lab = O.positions(T, B), O.next_token_labels(ids, T, B, oc.vocab)
        hp = O.hp_lora(1e-3, step, wd=0.01)
        loss = rec.step(ids, pos, lab, hp, step == 1)
        ref, grads = O.train_step(mdl, ids, pos, lab, T, B, hp, step == 1)
        assert abs(loss - ref) <= 1e-4 * abs(ref), (step, loss, ref)
        for k in mdl.trainable:
            g = eng.grad(k)
            worst.append((rel(g, grads[k].reshape(g.shape)), f"step {step} grad {k}"))
            p = eng.param(k)
            worst.append((rel(p, mdl.params[k].reshape(p.shape)), f"step {step} param {k}"))
            for w, refm in ((0, mdl.m[k]), (1, mdl.v[k])):
                mo = eng.moment(k, w)
                worst.append((rel(mo, refm.reshape(mo.shape)), f"step {step} moment{w} {k}"))
    worst.sort()
    if capsys is not None:
        with capsys.disabled():
            print(f"\n[{tag}] worst " + ", ".join(f"{r:.2e} {k}" for r, k in worst[-3:][::-1]))
    for r, k in worst:
        assert r < 1e-3, (k, r)


@pytest.mark.parametrize("norm_topk", [False, True])
def test_moe_flash_qknorm(cuda, norm_topk, capsys):
    """d_head 64 (fused flash attention), 8 experts, top 2, QK-RMSNorm."""
    run(128, 2, 64, 8, 2, norm_topk, 2, capsys=capsys, tag=f"moe dh64 norm_topk={norm_topk}")


def test_moe_dh128_materialised(cuda, capsys):
    """d_head 128 as in OLMoE (materialised attention), 16 experts, top 4."""
    run(256, 2, 128, 16, 4, False, 2, attention="materialized", capsys=capsys, tag="moe dh128")


def test_moe_without_qk_norm(cuda):
    run(128, 2, 64, 8, 3, False, 0)
