"""Oracle — TEST INFRASTRUCTURE ONLY.

A CPU restatement (numpy, float64 arithmetic on the float32 parameter values)
of the training step toy's recipes run: forward, cross-entropy, backward and
AdamW of the Llama decoder built by

  lib/toy/llm/archs/llama_arch.rb:395-507          (embed -> blocks -> norm -> tied head)
  lib/toy/llm/blocks/transformer_block.rb:153-268  (one block, per-head attention)
  lib/toy/llm/blocks/transformer_block.rb:861-893  (Q head with the LoRA splice)
  lib/toy/llm/primitives/gqa.rb:196-206            (scores, scale, causal mask, softmax, V)
  lib/toy/llm/engine/llama_seq_engine.rb:1786-1958 (CE loss, autograd, opt_step_adamw)

with ggml's op semantics as the shim documents them (tinynn/tinynn_ggml.h). The
backward is written out by hand (the reference gets it from ggml autograd);
the tests cross-check it against torch autograd in float64.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this module, and only as the checker / the timed CPU baseline. The product
(toy_b200/) never calls it.

Parity status: the per-op formulas are pinned by the reference's own A/B smoke
inputs and its one recorded known answer (tests/golden/, built by
tests/golden/make_golden.py); Q8_0 is pinned bit-exactly against gguf-py's
quantizer (the one the reference converter uses). Whole-step loss curves of the
reference cannot be reproduced here: their inputs (data/smollm2-135m-native.gguf,
data/ts_seqs.*) are not part of the reference tree.
"""
from __future__ import annotations

import ctypes as C
import math
import os
import subprocess
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_CLIB = None


# --------------------------------------------------------------------------- C part
def build_clib() -> str:
    out_dir = os.path.join(HERE, "_build")
    os.makedirs(out_dir, exist_ok=True)
    so = os.path.join(out_dir, "liboracle.so")
    src = os.path.join(HERE, "oracle_c.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", src, "-o", so,
                        "-lm"], check=True)
    return so


def clib() -> C.CDLL:
    global _CLIB
    if _CLIB is None:
        L = C.CDLL(build_clib())
        L.toy_lcg_next.restype = C.c_int64
        L.toy_lcg_next.argtypes = [C.c_int64]
        L.toy_lcg_seed_state.restype = C.c_int64
        L.toy_lcg_seed_state.argtypes = [C.c_int64]
        L.toy_gaussian_fill.restype = C.c_int64
        L.toy_gaussian_fill.argtypes = [C.c_int64, C.c_void_p, C.c_int64, C.c_double]
        L.toy_lora_a_fill.restype = C.c_int64
        L.toy_lora_a_fill.argtypes = [C.c_int64, C.c_void_p, C.c_int64, C.c_double]
        L.toy_q8_0_quantize.restype = None
        L.toy_q8_0_quantize.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.toy_q8_0_dequantize.restype = None
        L.toy_q8_0_dequantize.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.toy_fp32_to_fp16.restype = C.c_uint16
        L.toy_fp32_to_fp16.argtypes = [C.c_float]
        L.toy_lcg_skip.restype = C.c_int64
        L.toy_lcg_skip.argtypes = [C.c_int64, C.c_int64]
        _CLIB = L
    return _CLIB


def lcg_seed_state(seed: int) -> int:
    return clib().toy_lcg_seed_state(seed)


def gaussian_fill(state: int, n: int, std: float):
    """(values float32[n], new_state) — llama_seq_engine.rb:1383-1407."""
    out = np.empty(n, dtype=np.float32)
    st = clib().toy_gaussian_fill(state, out.ctypes.data, n, std)
    return out, st


def lora_a_fill(state: int, n: int, init_scale: float):
    out = np.empty(n, dtype=np.float32)
    st = clib().toy_lora_a_fill(state, out.ctypes.data, n, init_scale)
    return out, st


def q8_0_quantize(x: np.ndarray) -> np.ndarray:
    """float32 [..., K] (K % 32 == 0) -> uint8 [..., K/32*34] Q8_0 blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.shape[-1] % 32 == 0
    out = np.empty(x.shape[:-1] + (x.shape[-1] // 32 * 34,), dtype=np.uint8)
    clib().toy_q8_0_quantize(x.ctypes.data, x.size, out.ctypes.data)
    return out


def q8_0_dequantize(b: np.ndarray, k: int) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    n = b.size // 34 * 32
    out = np.empty(n, dtype=np.float32)
    clib().toy_q8_0_dequantize(b.ctypes.data, n, out.ctypes.data)
    return out.reshape(b.shape[:-1] + (k,))


# --------------------------------------------------------------------------- config
@dataclass
class LlamaCfg:
    vocab: int
    d_model: int
    n_heads: int
    n_kv: int
    d_head: int
    d_ff: int
    n_layers: int
    rope_base: float = 1.0e5
    rms_eps: float = 1.0e-5
    tied: bool = True
    qkv_bias: bool = False
    rope_freq_factors: Optional[np.ndarray] = None   # llama3-style per-dim factors (d_head/2)
    # mixture of experts in every block's FFN (n_experts > 0): router softmax over
    # the experts, the top n_experts_used by probability, their SwiGLU outputs
    # (expert FFN width d_ff) weighted by the probabilities (renormalised to sum
    # 1 with norm_topk) -- llama_kv_engine.rb build_moe_ffn :2073
    n_experts: int = 0
    n_experts_used: int = 0
    norm_topk: bool = False
    # 2: RMSNorm over the whole q and k vectors before the head split and RoPE
    # (OLMoE / Granite, llama_kv_engine.rb build_block_step :1687)
    qk_norm: int = 0

    @property
    def group(self) -> int:
        return self.n_heads // self.n_kv


@dataclass
class LoraCfg:
    rank: int = 8
    alpha: float = 16.0
    targets: tuple = ("q", "v")
    a_std: float = 0.125
    b_std: float = 0.01
    per_head_q: bool = False   # the reference's LoRA-Q: one (A_h, B_h) pair per Q head, no scale, B = 0

    @property
    def scale(self) -> float:
        return 1.0 if self.per_head_q else self.alpha / self.rank


PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def proj_shape(cfg: LlamaCfg, p: str):
    d, H, KV, dh, ff = cfg.d_model, cfg.n_heads, cfg.n_kv, cfg.d_head, cfg.d_ff
    return {"q": (H * dh, d), "k": (KV * dh, d), "v": (KV * dh, d), "o": (d, H * dh),
            "gate": (ff, d), "up": (ff, d), "down": (d, ff)}[p]


# --------------------------------------------------------------------------- init
def random_init(cfg: LlamaCfg, seed: int, init_scale: float, std_all: Optional[float] = None) -> Dict[str, np.ndarray]:
    """Weights in the draw order of realize_for_random_init/upload_random_init!
    (llama_seq_engine.rb:1161-1340): token embed N(0,0.02); [untied output
    N(0,0.02)]; per layer: each Q head, then (K head, V head) per KV head, O,
    gate, up, down; projections N(0, init_scale/sqrt(fan_in)); gammas 1.
    std_all overrides every std (the synthetic N(0, std) base of the QLoRA configs)."""
    d, ff, H, KV, dh, V = cfg.d_model, cfg.d_ff, cfg.n_heads, cfg.n_kv, cfg.d_head, cfg.vocab
    st = lcg_seed_state(seed)
    P: Dict[str, np.ndarray] = {}
    s_emb = 0.02 if std_all is None else std_all
    s_d = init_scale / math.sqrt(d) if std_all is None else std_all
    s_ff = init_scale / math.sqrt(ff) if std_all is None else std_all
    w, st = gaussian_fill(st, V * d, s_emb)
    P["token_embd.weight"] = w.reshape(V, d)
    P["output_norm.weight"] = np.ones(d, np.float32)
    if not cfg.tied:
        w, st = gaussian_fill(st, V * d, s_emb)
        P["output.weight"] = w.reshape(V, d)
    for l in range(cfg.n_layers):
        P[f"blk.{l}.attn_norm.weight"] = np.ones(d, np.float32)
        P[f"blk.{l}.ffn_norm.weight"] = np.ones(d, np.float32)
        wq = np.empty((H * dh, d), np.float32)
        for h in range(H):
            w, st = gaussian_fill(st, dh * d, s_d)
            wq[h * dh:(h + 1) * dh] = w.reshape(dh, d)
        wk = np.empty((KV * dh, d), np.float32)
        wv = np.empty((KV * dh, d), np.float32)
        for j in range(KV):
            w, st = gaussian_fill(st, dh * d, s_d)
            wk[j * dh:(j + 1) * dh] = w.reshape(dh, d)
            w, st = gaussian_fill(st, dh * d, s_d)
            wv[j * dh:(j + 1) * dh] = w.reshape(dh, d)
        P[f"blk.{l}.attn_q.weight"], P[f"blk.{l}.attn_k.weight"], P[f"blk.{l}.attn_v.weight"] = wq, wk, wv
        w, st = gaussian_fill(st, d * H * dh, s_d)
        P[f"blk.{l}.attn_output.weight"] = w.reshape(d, H * dh)
        if cfg.n_experts:
            E = cfg.n_experts
            w, st = gaussian_fill(st, E * d, s_emb)
            P[f"blk.{l}.ffn_gate_inp.weight"] = w.reshape(E, d)
            w, st = gaussian_fill(st, E * ff * d, s_d)
            P[f"blk.{l}.ffn_gate_exps.weight"] = w.reshape(E, ff, d)
            w, st = gaussian_fill(st, E * ff * d, s_d)
            P[f"blk.{l}.ffn_up_exps.weight"] = w.reshape(E, ff, d)
            w, st = gaussian_fill(st, E * d * ff, s_ff)
            P[f"blk.{l}.ffn_down_exps.weight"] = w.reshape(E, d, ff)
        else:
            w, st = gaussian_fill(st, ff * d, s_d)
            P[f"blk.{l}.ffn_gate.weight"] = w.reshape(ff, d)
            w, st = gaussian_fill(st, ff * d, s_d)
            P[f"blk.{l}.ffn_up.weight"] = w.reshape(ff, d)
            w, st = gaussian_fill(st, d * ff, s_ff)
            P[f"blk.{l}.ffn_down.weight"] = w.reshape(d, ff)
        if cfg.qk_norm:
            P[f"blk.{l}.attn_q_norm.weight"] = np.ones(H * dh, np.float32)
            P[f"blk.{l}.attn_k_norm.weight"] = np.ones(KV * dh, np.float32)
        if cfg.qkv_bias:
            for nm, rows in (("q", H * dh), ("k", KV * dh), ("v", KV * dh)):
                w, st = gaussian_fill(st, rows, 0.02 if std_all is None else std_all)
                P[f"blk.{l}.attn_{nm}.bias"] = w
    P["_state"] = np.array([st], dtype=np.int64)
    return P


PNAME = {"q": "attn_q", "k": "attn_k", "v": "attn_v", "o": "attn_output", "gate": "ffn_gate", "up": "ffn_up",
         "down": "ffn_down"}


def lora_init(cfg: LlamaCfg, lcfg: LoraCfg, state: int, seed: int, init_scale: float = 0.01) -> Dict[str, np.ndarray]:
    """Config-style LoRA (A [r, d_in] ~ N(0, a_std), B [d_out, r] ~ N(0, b_std)),
    drawn after the base from the same stream, per layer in target order, A then B.
    per_head_q reproduces upload_lora_q_init! (llama_seq_engine.rb:2545-2575):
    raw-seed stream, cos branch only, B = 0, one pair per Q head."""
    L: Dict[str, np.ndarray] = {}
    r = lcfg.rank
    if lcfg.per_head_q:
        s = seed
        H, dh, d = cfg.n_heads, cfg.d_head, cfg.d_model
        for l in range(cfg.n_layers):
            A = np.empty((H * r, d), np.float32)
            for h in range(H):
                a, s = lora_a_fill(s, r * d, init_scale)
                A[h * r:(h + 1) * r] = a.reshape(r, d)
            L[f"blk.{l}.attn_q.lora_a"] = A
            L[f"blk.{l}.attn_q.lora_b"] = np.zeros((H * dh, r), np.float32)   # packed per head: rows h*dh.. use cols 0..r
        return L
    st = state
    for l in range(cfg.n_layers):
        for p in lcfg.targets:
            dout, din = proj_shape(cfg, p)
            a, st = gaussian_fill(st, r * din, lcfg.a_std)
            b, st = gaussian_fill(st, dout * r, lcfg.b_std)
            L[f"blk.{l}.{PNAME[p]}.lora_a"] = a.reshape(r, din)
            L[f"blk.{l}.{PNAME[p]}.lora_b"] = b.reshape(dout, r)
    return L


def token_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    """Synthetic uniform ids in [0, vocab): floor(u * vocab) over the LCG stream
    seeded with seed + 1 (u from lcg_uniform!, llama_seq_engine.rb:1409-1414)."""
    L = clib()
    s = L.toy_lcg_seed_state(seed + 1)
    out = np.empty(n, np.int64)
    for i in range(n):
        s = L.toy_lcg_next(s)
        u = (s + 1.0) / 2147483648.0
        out[i] = min(int(u * vocab), vocab - 1)
    return out


def next_token_labels(ids: np.ndarray, T: int, B: int, vocab: int) -> np.ndarray:
    """Labels.next_token_guarded_batched (lib/toy/llm/labels.rb:180-204) as ids:
    window-local shift by one, last position targets itself, -1 = no target."""
    lab = np.empty(T * B, np.int64)
    for w in range(B):
        for k in range(T):
            t = ids[w * T + k + 1] if k + 1 < T else ids[w * T + k]
            lab[w * T + k] = t if 0 <= t < vocab else -1
    return lab


def positions(T: int, B: int) -> np.ndarray:
    """0..T-1 per sequence (lib/toy/llm/training_batch.rb:64-71)."""
    return np.tile(np.arange(T, dtype=np.int64), B)


# --------------------------------------------------------------------------- ops
def rms_norm(x, g, eps):
    """ggml rms_norm + mul(gamma) (tnn_rms_norm, tinynn_ggml.c:1104-1115)."""
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * r * g, r


def rms_norm_back(x, dz, eps):
    """ggml rms_norm_back (tinynn/rms_norm_back_probe.c:4-20):
    dx = (dz - x * sum(x*dz) / (sum(x^2) + n*eps)) * rrms."""
    n = x.shape[-1]
    sxx = np.sum(x * x, axis=-1, keepdims=True)
    sxdz = np.sum(x * dz, axis=-1, keepdims=True)
    rrms = 1.0 / np.sqrt(sxx / n + eps)
    return (dz - x * (sxdz / (sxx + n * eps))) * rrms


def rope_cache(pos: np.ndarray, n_dims: int, base: float, freq_scale: float = 1.0, ff=None):
    """cos/sin per (position, pair) as ggml's rope cache builds them: theta starts
    at float(pos) and is multiplied by theta_scale = powf(base, -2/n_dims) in f32
    per pair; theta/ff[i] * freq_scale; ext_factor 0, attn_factor 1
    (tnn_rope_ext, tinynn_ggml.c:1482-1508, NEOX mode)."""
    ts = np.float32(np.power(np.float32(base), np.float32(-2.0) / np.float32(n_dims)))
    half = n_dims // 2
    cos = np.empty((len(pos), half), np.float64)
    sin = np.empty((len(pos), half), np.float64)
    for pi, p in enumerate(pos):
        theta = np.float32(p)
        for i in range(half):
            f = np.float32(1.0) if ff is None else np.float32(ff[i])
            th = np.float32(np.float32(freq_scale) * np.float32(theta / f))
            cos[pi, i] = math.cos(float(th))
            sin[pi, i] = math.sin(float(th))
            theta = np.float32(theta * ts)
    return cos, sin


def rope(x, cos, sin):
    """NEOX rotation of pairs (i, i + d/2); x [N, nh, dh]."""
    h = x.shape[-1] // 2
    x0, x1 = x[..., :h], x[..., h:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)


def rope_back(dy, cos, sin):
    """ggml rope_back: rotation by -theta."""
    h = dy.shape[-1] // 2
    d0, d1 = dy[..., :h], dy[..., h:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([d0 * c + d1 * s, -d0 * s + d1 * c], axis=-1)


def softmax(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def silu(x):
    return x / (1.0 + np.exp(-x))


def silu_back(x, dy):
    """tinynn/ab_smoke_silu_back.rb:3-7: dx = dy * s * (1 + x * (1 - s))."""
    s = 1.0 / (1.0 + np.exp(-x))
    return dy * s * (1.0 + x * (1.0 - s))


def cross_entropy_loss(logits, labels):
    """ggml cross_entropy_loss over rows (tnn_cross_entropy_loss,
    tinynn_ggml.c:1806-1819): -(1/N) sum_n sum_v y log softmax(z). labels: int ids
    (-1 = all-zero row) or a dense [N, V] distribution."""
    m = np.max(logits, axis=-1, keepdims=True)
    lse = m[:, 0] + np.log(np.sum(np.exp(logits - m), axis=-1))
    N = logits.shape[0]
    if labels.ndim == 1:
        ok = labels >= 0
        picked = np.where(ok, logits[np.arange(N), np.where(ok, labels, 0)] - lse, 0.0)
        return -np.sum(picked) / N
    return -np.sum(labels * (logits - lse[:, None])) / N


def cross_entropy_loss_back(logits, labels, dloss=1.0):
    """tinynn/ab_smoke_cegrad.rb:1-3: dz = (softmax(z) - y) * dloss / N, for every
    row: a row with no target (label -1, an all-zero one-hot row) still gets
    softmax(z) / N, exactly as ggml's CROSS_ENTROPY_LOSS_BACK computes it."""
    N = logits.shape[0]
    p = softmax(logits)
    if labels.ndim == 1:
        ok = labels >= 0
        p[np.arange(N)[ok], labels[ok]] -= 1.0
    else:
        p = p - labels
    return p * (dloss / N)


def adamw(p, g, m, v, hp):
    """opt_step_adamw (tinynn_ggml.h:457-465):
    m = m*b1 + g*(1-b1); v = v*b2 + g*g*(1-b2);
    p = p*(1 - alpha*wd) - alpha * (m*beta1h) / (sqrt(v*beta2h) + eps)."""
    alpha, b1, b2, eps, wd, b1h, b2h = [float(x) for x in hp]
    m2 = m * b1 + g * (1.0 - b1)
    v2 = v * b2 + g * g * (1.0 - b2)
    p2 = p * (1.0 - alpha * wd) - alpha * (m2 * b1h) / (np.sqrt(v2 * b2h) + eps)
    return p2, m2, v2


def hp_lora(lr, step_1based, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.0):
    """Toy::AdamW.for_lora hp row (lib/toy/llm/adamw.rb:112-146)."""
    return np.array([lr, beta1, beta2, eps, wd, 1.0 / (1.0 - beta1 ** step_1based),
                     1.0 / (1.0 - beta2 ** step_1based)], np.float64)


def hp_from_scratch(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, wd=0.0):
    """Toy::AdamW.for_from_scratch: slots 5/6 carry the constant betas."""
    return np.array([lr, beta1, beta2, eps, wd, beta1, beta2], np.float64)


# --------------------------------------------------------------------------- model
@dataclass
class Model:
    cfg: LlamaCfg
    params: Dict[str, np.ndarray]                 # float32 values (Q8_0 base dequantised for the math)
    trainable: List[str]
    lora: Optional[LoraCfg] = None
    q8: Dict[str, np.ndarray] = field(default_factory=dict)   # raw Q8_0 blocks of frozen projections
    m: Dict[str, np.ndarray] = field(default_factory=dict)
    v: Dict[str, np.ndarray] = field(default_factory=dict)
    # arithmetic type of the step: float64 for parity checks; float32 times the
    # restatement at the precision toy's CPU path (ggml-cpu) computes in
    dtype: type = np.float64

    def zero_moments(self):
        self.m = {k: np.zeros(self.params[k].shape, self.dtype) for k in self.trainable}
        self.v = {k: np.zeros(self.params[k].shape, self.dtype) for k in self.trainable}


def full_ft_model(cfg: LlamaCfg, seed: int = 42, init_scale: float = 1.0, std_all: Optional[float] = None) -> Model:
    P = random_init(cfg, seed, init_scale, std_all)
    P.pop("_state")
    mdl = Model(cfg, P, [k for k in P])
    mdl.zero_moments()
    return mdl


def qlora_model(cfg: LlamaCfg, lcfg: LoraCfg, seed: int = 42, base_std: float = 0.02) -> Model:
    """Synthetic frozen base N(0, base_std), 2-D projections quantised to Q8_0
    (token embedding and norms stay F32, as the reference converter keeps them),
    plus trainable LoRA adapters."""
    P = random_init(cfg, seed, 1.0, std_all=base_std)
    st = int(P.pop("_state")[0])
    q8 = {}
    for l in range(cfg.n_layers):
        names = [f"blk.{l}.{PNAME[p]}.weight" for p in PROJ if cfg.n_experts == 0 or p in ("q", "k", "v", "o")]
        if cfg.n_experts:   # expert tensors quantised per expert row (along d_in), router kept in f32
            names += [f"blk.{l}.ffn_{t}_exps.weight" for t in ("gate", "up", "down")]
        for k in names:
            q8[k] = q8_0_quantize(P[k])
            P[k] = q8_0_dequantize(q8[k], P[k].shape[-1])
    # per-head LoRA-Q draws A with init_scale = a_std (upload_lora_q_init!'s init_scale)
    L = lora_init(cfg, lcfg, st, seed, init_scale=lcfg.a_std if lcfg.per_head_q else 0.01)
    P.update(L)
    mdl = Model(cfg, P, sorted(L.keys()), lora=lcfg, q8=q8)
    mdl.zero_moments()
    return mdl


def _lora_delta(mdl: Model, l: int, p: str, h1):
    """LoRA contribution s * B (A h) for projection p of layer l, plus the cache."""
    lc = mdl.lora
    ka, kb = f"blk.{l}.{PNAME[p]}.lora_a", f"blk.{l}.{PNAME[p]}.lora_b"
    if lc is None or ka not in mdl.params:
        return None, None
    A = mdl.params[ka].astype(mdl.dtype)
    B = mdl.params[kb].astype(mdl.dtype)
    if lc.per_head_q:
        cfg = mdl.cfg
        r, dh = lc.rank, cfg.d_head
        u = h1 @ A.T                                   # [N, H*r]
        out = np.empty((h1.shape[0], cfg.n_heads * dh), mdl.dtype)
        for h in range(cfg.n_heads):
            out[:, h * dh:(h + 1) * dh] = u[:, h * r:(h + 1) * r] @ B[h * dh:(h + 1) * dh].T
        return out, u
    u = h1 @ A.T
    return lc.scale * (u @ B.T), u


def _lora_back(mdl: Model, l: int, p: str, h1, u, dy, grads):
    lc = mdl.lora
    ka, kb = f"blk.{l}.{PNAME[p]}.lora_a", f"blk.{l}.{PNAME[p]}.lora_b"
    A = mdl.params[ka].astype(mdl.dtype)
    B = mdl.params[kb].astype(mdl.dtype)
    if lc.per_head_q:
        cfg = mdl.cfg
        r, dh = lc.rank, cfg.d_head
        dB = np.zeros_like(B)
        du = np.empty_like(u)
        for h in range(cfg.n_heads):
            dyh = dy[:, h * dh:(h + 1) * dh]
            dB[h * dh:(h + 1) * dh] = dyh.T @ u[:, h * r:(h + 1) * r]
            du[:, h * r:(h + 1) * r] = dyh @ B[h * dh:(h + 1) * dh]
    else:
        s = lc.scale
        dB = s * (dy.T @ u)
        du = s * (dy @ B)
    grads[kb] = dB
    grads[ka] = du.T @ h1
    return du @ A


def _attn_backward(mdl: Model, l: int, c: dict, dx1, cos, sin, grads, tr):
    """Backward of one block's attention half: from d(x1) to d(x), adapters and
    weight gradients into grads."""
    cfg, P = mdl.cfg, mdl.params
    N, H, KV, dh, G = c["x"].shape[0], cfg.n_heads, cfg.n_kv, cfg.d_head, cfg.group
    B = c["probs"].shape[0]
    T = N // B
    eps = cfg.rms_eps
    dt = mdl.dtype
    scale = dt(1.0 / math.sqrt(dh))
    f64 = lambda k: P[k].astype(dt)
    pre = f"blk.{l}."
    do = dx1 @ f64(pre + "attn_output.weight")
    if pre + "attn_output.weight" in tr:
        grads[pre + "attn_output.weight"] = dx1.T @ c["o"]
    if "u_o" in c:
        do = do + _lora_back(mdl, l, "o", c["o"], c["u_o"], dx1, grads)
    do = do.reshape(N, H, dh)
    q, k, v, probs = c["q"], c["k"], c["v"], c["probs"]
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for b in range(B):
        sl = slice(b * T, (b + 1) * T)
        for h in range(H):
            j = h // G
            pr = probs[b, h]
            dP = do[sl, h] @ v[sl, j].T
            dS = pr * (dP - np.sum(dP * pr, axis=-1, keepdims=True)) * scale
            dq[sl, h] = dS @ k[sl, j]
            dk[sl, j] += dS.T @ q[sl, h]
            dv[sl, j] += pr.T @ do[sl, h]
    dq = rope_back(dq, cos, sin).reshape(N, H * dh)
    dk = rope_back(dk, cos, sin).reshape(N, KV * dh)
    dv = dv.reshape(N, KV * dh)
    if cfg.qk_norm:   # through the whole-vector q / k RMSNorm
        for nm, pre_v in (("q", "q_pre"), ("k", "k_pre")):
            gk = pre + f"attn_{nm}_norm.weight"
            xv = c[pre_v]
            dpost = dq if nm == "q" else dk
            if gk in tr:
                rr = 1.0 / np.sqrt(np.mean(xv * xv, axis=-1, keepdims=True) + eps)
                grads[gk] = np.sum(dpost * xv * rr, axis=0)
            back = rms_norm_back(xv, dpost * f64(gk), eps)
            if nm == "q":
                dq = back
            else:
                dk = back
    h1 = c["h1"]
    dh1 = dq @ f64(pre + "attn_q.weight") + dk @ f64(pre + "attn_k.weight") + dv @ f64(pre + "attn_v.weight")
    for p, dy in (("q", dq), ("k", dk), ("v", dv)):
        if pre + PNAME[p] + ".weight" in tr:
            grads[pre + PNAME[p] + ".weight"] = dy.T @ h1
        if cfg.qkv_bias and pre + PNAME[p] + ".bias" in tr:
            grads[pre + PNAME[p] + ".bias"] = dy.sum(axis=0)
        if "u_" + p in c:
            dh1 = dh1 + _lora_back(mdl, l, p, h1, c["u_" + p], dy, grads)
    x0 = c["x"]
    r1 = 1.0 / np.sqrt(np.mean(x0 * x0, axis=-1, keepdims=True) + eps)
    if pre + "attn_norm.weight" in tr:
        grads[pre + "attn_norm.weight"] = np.sum(dh1 * x0 * r1, axis=0)
    return dx1 + rms_norm_back(x0, dh1 * f64(pre + "attn_norm.weight"), eps)


def moe_forward(mdl: Model, l: int, h2):
    """The FFN of an MoE block (llama_kv_engine.rb build_moe_ffn :2073) for every
    token row of h2: probs = softmax(h2 Wr^T) over the experts, the top
    n_experts_used by probability (ties to the lower index), weights = their
    probabilities (renormalised with norm_topk), and the weighted sum of the
    selected experts' SwiGLU FFNs. Returns (y, cache)."""
    cfg, P = mdl.cfg, mdl.params
    dt = mdl.dtype
    E, K = cfg.n_experts, cfg.n_experts_used
    f = lambda k: P[k].astype(dt)
    pre = f"blk.{l}."
    Wr, Wg, Wu, Wd = f(pre + "ffn_gate_inp.weight"), f(pre + "ffn_gate_exps.weight"), f(pre + "ffn_up_exps.weight"), \
        f(pre + "ffn_down_exps.weight")
    N = h2.shape[0]
    probs = softmax(h2 @ Wr.T)
    idx = np.argsort(-probs, axis=1, kind="stable")[:, :K]
    w = np.take_along_axis(probs, idx, 1)
    if cfg.norm_topk:
        w = w / np.sum(w, axis=1, keepdims=True)
    g = np.zeros((N, K, Wg.shape[1]), dt)
    u = np.zeros_like(g)
    ye = np.zeros((N, K, h2.shape[1]), dt)
    for e in range(E):
        n_i, k_i = np.nonzero(idx == e)
        if n_i.size == 0:
            continue
        X = h2[n_i]
        ge, ue = X @ Wg[e].T, X @ Wu[e].T
        g[n_i, k_i], u[n_i, k_i] = ge, ue
        ye[n_i, k_i] = (silu(ge) * ue) @ Wd[e].T
    y = np.einsum("nk,nkd->nd", w, ye)
    return y, {"probs": probs, "idx": idx, "w": w, "g": g, "u": u, "ye": ye}


def moe_backward(mdl: Model, l: int, h2, mc: dict, dy):
    """d(h2) of moe_forward for the output gradient dy, the experts and the
    router frozen: through every selected expert (weighted by its routing
    weight) and through the routing weights into the router's softmax."""
    cfg, P = mdl.cfg, mdl.params
    dt = mdl.dtype
    E, K = cfg.n_experts, cfg.n_experts_used
    f = lambda k: P[k].astype(dt)
    pre = f"blk.{l}."
    Wr, Wg, Wu, Wd = f(pre + "ffn_gate_inp.weight"), f(pre + "ffn_gate_exps.weight"), f(pre + "ffn_up_exps.weight"), \
        f(pre + "ffn_down_exps.weight")
    probs, idx, w, g, u, ye = mc["probs"], mc["idx"], mc["w"], mc["g"], mc["u"], mc["ye"]
    dh2 = np.zeros_like(h2)
    dw = np.einsum("nd,nkd->nk", dy, ye)
    for e in range(E):
        n_i, k_i = np.nonzero(idx == e)
        if n_i.size == 0:
            continue
        dye = w[n_i, k_i][:, None] * dy[n_i]
        da = dye @ Wd[e]
        ge, ue = g[n_i, k_i], u[n_i, k_i]
        dge = silu_back(ge, da * ue)
        due = da * silu(ge)
        np.add.at(dh2, n_i, dge @ Wg[e] + due @ Wu[e])
    if cfg.norm_topk:   # w = p_sel / sum(p_sel)
        ssum = np.sum(np.take_along_axis(probs, idx, 1), axis=1, keepdims=True)
        dsel = (dw - np.sum(dw * w, axis=1, keepdims=True)) / ssum
    else:
        dsel = dw
    dprobs = np.zeros_like(probs)
    np.put_along_axis(dprobs, idx, dsel, 1)
    dlogits = probs * (dprobs - np.sum(probs * dprobs, axis=1, keepdims=True))
    return dh2 + dlogits @ Wr


def q8_0_roundtrip(x: np.ndarray) -> np.ndarray:
    """The values a Q8_0 cache holds for x [..., n] (n % 32 == 0): x narrowed
    to f32, quantised (ggml's quantiser) and dequantised."""
    xf = np.ascontiguousarray(x, np.float32)
    n = xf.shape[-1]
    return q8_0_dequantize(q8_0_quantize(xf.reshape(-1, n)), n).reshape(x.shape).astype(np.float64)


def forward_backward(mdl: Model, ids: np.ndarray, pos: np.ndarray, labels: np.ndarray, T: int, B: int,
                     want_grads: bool = True, trace: Optional[dict] = None, kv_q8: bool = False):
    """Loss and gradients (float64) of one step. ids/pos/labels have T*B entries,
    token (b, t) at b*T + t; labels are ids (-1 = none) or a dense [N, V] array.
    When `trace` is a dict it receives the per-layer forward caches and logits.
    kv_q8 (forward only): K (after RoPE) and V pass through a Q8_0 round trip
    per token and head, as a Q8_0 KV cache stores them (llama_kv_engine.rb
    enable_kv_q8!)."""
    cfg, P = mdl.cfg, mdl.params
    N, d, H, KV, dh, G = T * B, cfg.d_model, cfg.n_heads, cfg.n_kv, cfg.d_head, cfg.group
    eps = cfg.rms_eps
    scale = 1.0 / math.sqrt(dh)
    dt = mdl.dtype
    f64 = lambda k: P[k].astype(dt)
    cos, sin = rope_cache(pos, dh, cfg.rope_base, 1.0, cfg.rope_freq_factors)
    cos, sin = cos.astype(dt), sin.astype(dt)
    scale = dt(scale)
    E = f64("token_embd.weight")
    x = E[ids]
    causal = np.triu(np.full((T, T), -np.inf, dt), 1)
    caches = []
    for l in range(cfg.n_layers):
        c = {"x": x}
        h1, r1 = rms_norm(x, f64(f"blk.{l}.attn_norm.weight"), eps)
        c["h1"] = h1
        qkv = {}
        for p in ("q", "k", "v"):
            y = h1 @ f64(f"blk.{l}.{PNAME[p]}.weight").T
            dlt, u = _lora_delta(mdl, l, p, h1)
            if dlt is not None:
                y = y + dlt
                c["u_" + p] = u
            if cfg.qkv_bias:
                y = y + f64(f"blk.{l}.{PNAME[p]}.bias")
            qkv[p] = y
        if cfg.qk_norm:
            c["q_pre"], c["k_pre"] = qkv["q"], qkv["k"]
            qkv["q"] = rms_norm(qkv["q"], f64(f"blk.{l}.attn_q_norm.weight"), eps)[0]
            qkv["k"] = rms_norm(qkv["k"], f64(f"blk.{l}.attn_k_norm.weight"), eps)[0]
        q = rope(qkv["q"].reshape(N, H, dh), cos, sin)
        k = rope(qkv["k"].reshape(N, KV, dh), cos, sin)
        v = qkv["v"].reshape(N, KV, dh)
        if kv_q8:
            k, v = q8_0_roundtrip(k).astype(dt), q8_0_roundtrip(v).astype(dt)
        o = np.empty((N, H, dh), dt)
        probs = np.empty((B, H, T, T), dt)
        for b in range(B):
            sl = slice(b * T, (b + 1) * T)
            for h in range(H):
                j = h // G
                s = (q[sl, h] @ k[sl, j].T) * scale + causal
                pr = softmax(s)
                probs[b, h] = pr
                o[sl, h] = pr @ v[sl, j]
        c.update(q=q, k=k, v=v, probs=probs, o=o.reshape(N, H * dh))
        x1 = x + c["o"] @ f64(f"blk.{l}.attn_output.weight").T
        dlt, u = _lora_delta(mdl, l, "o", c["o"])
        if dlt is not None:
            x1 = x1 + dlt
            c["u_o"] = u
        c["x1"] = x1
        h2, r2 = rms_norm(x1, f64(f"blk.{l}.ffn_norm.weight"), eps)
        c["h2"] = h2
        if cfg.n_experts:
            y, c["moe"] = moe_forward(mdl, l, h2)
            x2 = x1 + y
            caches.append(c)
            x = x2
            continue
        g = h2 @ f64(f"blk.{l}.ffn_gate.weight").T
        up = h2 @ f64(f"blk.{l}.ffn_up.weight").T
        for p, y in (("gate", "g"), ("up", "up")):
            dlt, u = _lora_delta(mdl, l, p, h2)
            if dlt is not None:
                if p == "gate":
                    g = g + dlt
                else:
                    up = up + dlt
                c["u_" + p] = u
        a = silu(g) * up
        c.update(g=g, up=up, a=a)
        x2 = x1 + a @ f64(f"blk.{l}.ffn_down.weight").T
        dlt, u = _lora_delta(mdl, l, "down", a)
        if dlt is not None:
            x2 = x2 + dlt
            c["u_down"] = u
        caches.append(c)
        x = x2
    xf, rf = rms_norm(x, f64("output_norm.weight"), eps)
    W_out = E if cfg.tied else f64("output.weight")
    logits = xf @ W_out.T
    loss = cross_entropy_loss(logits, labels)
    if trace is not None:
        trace.update(layers=caches, logits=logits, x_final=x)
    if not want_grads:
        return loss, {}, logits
    grads: Dict[str, np.ndarray] = {}
    tr = set(mdl.trainable)
    dlog = cross_entropy_loss_back(logits, labels)
    dxf = dlog @ W_out
    if cfg.tied and "token_embd.weight" in tr:
        grads["token_embd.weight"] = dlog.T @ xf
    if not cfg.tied and "output.weight" in tr:
        grads["output.weight"] = dlog.T @ xf
    xhat = x * rf
    if "output_norm.weight" in tr:
        grads["output_norm.weight"] = np.sum(dxf * xhat, axis=0)
    dx = rms_norm_back(x, dxf * f64("output_norm.weight"), eps)
    for l in reversed(range(cfg.n_layers)):
        c = caches[l]
        pre = f"blk.{l}."
        if cfg.n_experts:
            dh2 = moe_backward(mdl, l, c["h2"], c["moe"], dx)
            x1 = c["x1"]
            r2 = 1.0 / np.sqrt(np.mean(x1 * x1, axis=-1, keepdims=True) + eps)
            if pre + "ffn_norm.weight" in tr:
                grads[pre + "ffn_norm.weight"] = np.sum(dh2 * x1 * r2, axis=0)
            dx1 = dx + rms_norm_back(x1, dh2 * f64(pre + "ffn_norm.weight"), eps)
            dx = _attn_backward(mdl, l, c, dx1, cos, sin, grads, tr)
            continue
        # FFN
        da = dx @ f64(pre + "ffn_down.weight")
        if pre + "ffn_down.weight" in tr:
            grads[pre + "ffn_down.weight"] = dx.T @ c["a"]
        if "u_down" in c:
            da = da + _lora_back(mdl, l, "down", c["a"], c["u_down"], dx, grads)
        sg = 1.0 / (1.0 + np.exp(-c["g"]))
        dgate = silu_back(c["g"], da * c["up"])
        dup = da * (c["g"] * sg)
        dh2 = dgate @ f64(pre + "ffn_gate.weight") + dup @ f64(pre + "ffn_up.weight")
        if pre + "ffn_gate.weight" in tr:
            grads[pre + "ffn_gate.weight"] = dgate.T @ c["h2"]
            grads[pre + "ffn_up.weight"] = dup.T @ c["h2"]
        if "u_gate" in c:
            dh2 = dh2 + _lora_back(mdl, l, "gate", c["h2"], c["u_gate"], dgate, grads)
        if "u_up" in c:
            dh2 = dh2 + _lora_back(mdl, l, "up", c["h2"], c["u_up"], dup, grads)
        x1 = c["x1"]
        r2 = 1.0 / np.sqrt(np.mean(x1 * x1, axis=-1, keepdims=True) + eps)
        if pre + "ffn_norm.weight" in tr:
            grads[pre + "ffn_norm.weight"] = np.sum(dh2 * x1 * r2, axis=0)
        dx1 = dx + rms_norm_back(x1, dh2 * f64(pre + "ffn_norm.weight"), eps)
        dx = _attn_backward(mdl, l, c, dx1, cos, sin, grads, tr)
    if "token_embd.weight" in tr:
        gE = grads.get("token_embd.weight", np.zeros(E.shape, dt))
        np.add.at(gE, ids, dx)     # get_rows_back: scatter-add (tinynn_ggml.c:1683-1700)
        grads["token_embd.weight"] = gE
    return loss, grads, logits


def train_step(mdl: Model, ids, pos, labels, T, B, hp, is_first: bool):
    """One step!: (is_first zeroes the Adam moments, as tnn_graph_reset does),
    forward/backward, then AdamW on every trainable tensor. Returns (loss, grads)."""
    if is_first:
        mdl.zero_moments()
    loss, grads, _ = forward_backward(mdl, ids, pos, labels, T, B)
    for k in mdl.trainable:
        p2, m2, v2 = adamw(mdl.params[k].astype(mdl.dtype), grads[k], mdl.m[k], mdl.v[k], hp)
        mdl.params[k] = p2.astype(np.float32)
        mdl.m[k], mdl.v[k] = m2, v2
    return loss, grads


# --------------------------------------------------------------------------- configs
def smollm2_135m(**kw) -> LlamaCfg:
    """SmolLM2-135M shape (lib/toy/models/toy_smollm2.rb:206-208)."""
    return LlamaCfg(vocab=49152, d_model=576, n_heads=9, n_kv=3, d_head=64, d_ff=1536, n_layers=30,
                    rope_base=1.0e5, rms_eps=1.0e-5, **kw)


def tiny(**kw) -> LlamaCfg:
    return LlamaCfg(vocab=512, d_model=128, n_heads=4, n_kv=2, d_head=32, d_ff=256, n_layers=2,
                    rope_base=1.0e4, rms_eps=1.0e-5, **kw)


def llama3_freq_factors(d_head, base, orig_max_pos, factor, low_freq, high_freq) -> np.ndarray:
    """Toy::RopeScaling.compute_llama3_freq_factors (lib/toy/models/toy_smollm2.rb:112-142)."""
    n = d_head // 2
    low_w, high_w = orig_max_pos / low_freq, orig_max_pos / high_freq
    out = np.empty(n)
    for i in range(n):
        freq = 1.0 / (base ** ((2.0 * i) / d_head))
        wl = 2.0 * math.pi / freq
        if wl < high_w:
            out[i] = 1.0
        elif wl > low_w:
            out[i] = factor
        else:
            sm = (orig_max_pos / wl - low_freq) / (high_freq - low_freq)
            out[i] = (1.0 - sm) * factor + sm * 1.0
    return out
