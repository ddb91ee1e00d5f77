"""The oracle against the reference's golden vectors, and its hand-written
backward against torch autograd (float64) on small configs. CPU only."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _gold(name):
    with open(os.path.join(GOLD, name)) as f:
        return json.load(f)


def test_adamw_smoke():
    g = _gold("op_smokes.json")["adamw"]
    p, m, v = O.adamw(np.array(g["param"]), np.array(g["grad"]), np.array(g["m"]), np.array(g["v"]),
                      np.array(g["hp"]))
    assert np.max(np.abs(p - g["want_param"])) < g["tol_param"]
    assert np.max(np.abs(m - g["want_m"])) < g["tol_mv"]
    assert np.max(np.abs(v - g["want_v"])) < g["tol_mv"]


def test_ce_grad_smoke():
    g = _gold("op_smokes.json")["ce_grad"]
    d = O.cross_entropy_loss_back(np.array(g["logits"]), np.array(g["targets"]))
    assert np.max(np.abs(d - np.array(g["want"]))) < g["tol"]


def test_silu_back_smoke():
    g = _gold("op_smokes.json")["silu_back"]
    d = O.silu_back(np.array(g["x"]), np.array(g["dy"]))
    assert np.max(np.abs(d - np.array(g["want"]))) < g["tol"]


def test_rms_norm_smoke():
    g = _gold("op_smokes.json")["rms_norm"]
    y, _ = O.rms_norm(np.array(g["x"]), np.array(g["gamma"]), g["eps"])
    assert np.max(np.abs(y - np.array(g["want"]))) < g["tol"]


def test_softmax_and_back_smokes():
    g = _gold("op_smokes.json")
    s = O.softmax(np.array(g["softmax"]["x"]))
    assert np.max(np.abs(s - np.array(g["softmax"]["want"]))) < g["softmax"]["tol"]
    gb = g["softmax_back"]
    a = O.softmax(np.array(gb["x"]))
    dy = np.array(gb["dy"])
    d = a * (dy - np.sum(a * dy, axis=-1, keepdims=True))
    assert np.max(np.abs(d - np.array(gb["want"]))) < gb["tol"]


def test_rms_norm_back_known_answer():
    g = _gold("op_smokes.json")["rms_norm_back_known"]
    d = O.rms_norm_back(np.array([g["x"]]), np.array([g["dz"]]), g["eps"])[0]
    assert np.max(np.abs(d - np.array(g["want"]))) < g["tol"]


def test_q8_0_bit_exact_vs_gguf():
    z = np.load(os.path.join(GOLD, "q8_0.npz"))
    for name in "abcde":
        x = z[name + "_x"]
        q = O.q8_0_quantize(x)
        assert np.array_equal(q, z[name + "_q"]), name
        dq = O.q8_0_dequantize(q, x.shape[-1])
        assert np.array_equal(dq.view(np.uint32), z[name + "_dq"].view(np.uint32)), name


def test_q8_0_error_bound():
    """tinynn/ab_smoke_q8_kv.rb:12-14,64-73: its integer-hash input pattern
    (64 x 64 values in [-0.5, 0.5]) -> max abs < 0.02, RMS < 0.005."""
    i = np.arange(64 * 64, dtype=np.int64)
    bit = (i * 2654435761) & 0xFFFF
    x = ((bit.astype(np.float64) / 32768.0 - 1.0) * 0.5).astype(np.float32).reshape(64, 64)
    dq = O.q8_0_dequantize(O.q8_0_quantize(x), 64)
    err = dq - x
    assert np.max(np.abs(err)) < 0.02 and np.sqrt(np.mean(err ** 2)) < 0.005


def test_lcg_streams_match_bigint_restatement():
    g = _gold("lcg.json")
    for sd, st in g["seed_state"].items():
        assert O.lcg_seed_state(int(sd)) == st
    gg = g["gaussian_seed42"]
    st = O.lcg_seed_state(42)
    v1, st = O.gaussian_fill(st, gg["n1"], gg["std1"])
    v2, st = O.gaussian_fill(st, gg["n2"], gg["std2"])
    assert np.array_equal(v1, np.array(gg["values1"], np.float32))
    assert np.array_equal(v2, np.array(gg["values2"], np.float32))
    assert st == gg["state_after"]
    la = g["lora_a_seed42"]
    v, st = O.lora_a_fill(42, la["n"], la["init_scale"])
    assert np.array_equal(v, np.array(la["values"], np.float32)) and st == la["state_after"]


def test_labels_and_positions():
    ids = np.array([5, 6, 7, 8, 1, 2, 3, 4])
    lab = O.next_token_labels(ids, 4, 2, 10)
    assert lab.tolist() == [6, 7, 8, 8, 2, 3, 4, 4]
    assert O.next_token_labels(np.array([1, 99]), 2, 1, 10).tolist() == [-1, -1]
    assert O.positions(3, 2).tolist() == [0, 1, 2, 0, 1, 2]


def _torch_reference_grads(mdl, ids, pos, labels, T, B):
    """Same graph in torch float64 with autograd (independent of the hand-written backward)."""
    import math

    import torch
    cfg = mdl.cfg
    N, H, KV, dh, G = T * B, cfg.n_heads, cfg.n_kv, cfg.d_head, cfg.group
    P = {k: torch.tensor(v.astype(np.float64), requires_grad=k in mdl.trainable) for k, v in mdl.params.items()}
    cos, sin = O.rope_cache(pos, dh, cfg.rope_base, 1.0, cfg.rope_freq_factors)
    cos, sin = torch.tensor(cos), torch.tensor(sin)

    def rms(x, g):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + cfg.rms_eps) * g

    def rope(x):
        h = x.shape[-1] // 2
        c, s = cos[:, None], sin[:, None]
        return torch.cat([x[..., :h] * c - x[..., h:] * s, x[..., :h] * s + x[..., h:] * c], -1)

    def proj(l, p, x):
        y = x @ P[f"blk.{l}.{O.PNAME[p]}.weight"].T
        ka = f"blk.{l}.{O.PNAME[p]}.lora_a"
        if ka in P:
            A, Bm = P[ka], P[f"blk.{l}.{O.PNAME[p]}.lora_b"]
            if mdl.lora.per_head_q:
                r = mdl.lora.rank
                u = x @ A.T
                y = y + torch.cat([u[:, h * r:(h + 1) * r] @ Bm[h * dh:(h + 1) * dh].T for h in range(H)], -1)
            else:
                y = y + mdl.lora.scale * ((x @ A.T) @ Bm.T)
        return y

    x = P["token_embd.weight"][torch.tensor(ids)]
    mask = torch.triu(torch.full((T, T), float("-inf"), dtype=torch.float64), 1)
    for l in range(cfg.n_layers):
        h1 = rms(x, P[f"blk.{l}.attn_norm.weight"])
        qf, kf = proj(l, "q", h1), proj(l, "k", h1)
        if cfg.qk_norm:
            qf, kf = rms(qf, P[f"blk.{l}.attn_q_norm.weight"]), rms(kf, P[f"blk.{l}.attn_k_norm.weight"])
        q = rope(qf.view(N, H, dh))
        k = rope(kf.view(N, KV, dh))
        v = proj(l, "v", h1).view(N, KV, dh)
        outs = []
        for b in range(B):
            sl = slice(b * T, (b + 1) * T)
            heads = []
            for h in range(H):
                j = h // G
                s = q[sl, h] @ k[sl, j].T / math.sqrt(dh) + mask
                heads.append(torch.softmax(s, -1) @ v[sl, j])
            outs.append(torch.cat(heads, -1))
        o = torch.cat(outs, 0)
        x = x + proj(l, "o", o)
        h2 = rms(x, P[f"blk.{l}.ffn_norm.weight"])
        if cfg.n_experts:
            pr = torch.softmax(h2 @ P[f"blk.{l}.ffn_gate_inp.weight"].T, -1)
            idx = torch.argsort(-pr.detach(), dim=1, stable=True)[:, :cfg.n_experts_used]
            w = torch.gather(pr, 1, idx)
            if cfg.norm_topk:
                w = w / w.sum(1, keepdim=True)
            y = torch.zeros_like(h2)
            for e in range(cfg.n_experts):
                for kk in range(cfg.n_experts_used):
                    sel = idx[:, kk] == e
                    if sel.any():
                        X = h2[sel]
                        a = torch.nn.functional.silu(X @ P[f"blk.{l}.ffn_gate_exps.weight"][e].T) * \
                            (X @ P[f"blk.{l}.ffn_up_exps.weight"][e].T)
                        ye = a @ P[f"blk.{l}.ffn_down_exps.weight"][e].T
                        y = y.index_add(0, torch.nonzero(sel)[:, 0], w[sel, kk:kk + 1] * ye)
            x = x + y
            continue
        a = torch.nn.functional.silu(proj(l, "gate", h2)) * proj(l, "up", h2)
        x = x + proj(l, "down", a)
    xf = rms(x, P["output_norm.weight"])
    logits = xf @ P["token_embd.weight"].T
    lab = torch.tensor(labels)
    lp = torch.log_softmax(logits, -1)
    ok = lab >= 0
    loss = -(lp[torch.arange(N)[ok], lab[ok]]).sum() / N
    # ggml's CROSS_ENTROPY_LOSS_BACK is (softmax - y) / N for every row, so a row
    # with no target (all-zero labels) still receives softmax / N: the gradient
    # of logsumexp(z) / N. Add that surrogate term for the backward only.
    surrogate = loss + torch.logsumexp(logits[~ok], -1).sum() / N
    surrogate.backward()
    return loss.item(), {k: P[k].grad.numpy() for k in mdl.trainable}


@pytest.mark.parametrize("mode", ["full", "qlora", "qlora_all7", "qlora_per_head", "qlora_moe", "qlora_moe_norm"])
def test_backward_matches_torch_autograd(mode):
    cfg = O.LlamaCfg(vocab=96, d_model=64, n_heads=4, n_kv=2, d_head=16, d_ff=96, n_layers=2, rope_base=1e4)
    T, B = 8, 2
    if mode.startswith("qlora_moe"):   # OLMoE-style block: QK-RMSNorm, 6 experts, top 3
        cfg = O.LlamaCfg(vocab=96, d_model=64, n_heads=4, n_kv=4, d_head=16, d_ff=32, n_layers=2, rope_base=1e4,
                         n_experts=6, n_experts_used=3, norm_topk=mode.endswith("norm"), qk_norm=2)
        mdl = O.qlora_model(cfg, O.LoraCfg(rank=4, alpha=8, targets=("q", "k", "v", "o")), seed=3)
    elif mode == "full":
        mdl = O.full_ft_model(cfg, seed=3, init_scale=1.0)
    elif mode == "qlora":
        mdl = O.qlora_model(cfg, O.LoraCfg(rank=4, alpha=8, targets=("q", "v")), seed=3)
    elif mode == "qlora_all7":
        mdl = O.qlora_model(cfg, O.LoraCfg(rank=4, alpha=8, targets=O.PROJ), seed=3)
    else:
        mdl = O.qlora_model(cfg, O.LoraCfg(rank=4, per_head_q=True, targets=("q",)), seed=3)
        for k in mdl.trainable:   # non-zero B so the adapter contributes
            if k.endswith("lora_b"):
                mdl.params[k] = (np.random.default_rng(1).standard_normal(mdl.params[k].shape) * 0.1).astype(np.float32)
    ids = O.token_ids(5, T * B, cfg.vocab)
    lab = O.next_token_labels(ids, T, B, cfg.vocab)
    lab[3] = -1
    pos = O.positions(T, B)
    loss, grads, _ = O.forward_backward(mdl, ids, pos, lab, T, B)
    tl, tg = _torch_reference_grads(mdl, ids, pos, lab, T, B)
    assert abs(loss - tl) < 1e-12 * abs(tl)
    for k in mdl.trainable:
        rel = np.linalg.norm(grads[k] - tg[k]) / max(np.linalg.norm(tg[k]), 1e-300)
        assert rel < 1e-10, (k, rel)


def test_llama3_freq_factors_shape():
    ff = O.llama3_freq_factors(64, 5e5, 8192, 32.0, 1.0, 4.0)
    assert ff.shape == (32,) and ff[0] == 1.0 and ff[-1] == 32.0
