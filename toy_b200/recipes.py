"""Host mirror of toy's training recipes over the toy_b200 C ABI.

  Toy::LLM::Recipes::FromScratch  (lib/toy/llm/recipes/from_scratch.rb:68-103)
  Toy::LLM::Recipes::LoRA         (lib/toy/llm/recipes/lora.rb:71-107)
  Toy::LLM::Engine::LlamaSeqEngine, the subset the recipes call
                                  (lib/toy/llm/engine/llama_seq_engine.rb)

realize() builds the training program on the GPU; step() is the reference's
step! verbatim in order: graph reset (first step) or grads-only reset, the four
uploads (token ids, positions, labels, hp), compute_backward, download loss.
Labels may be the reference's dense one-hot [T*B, vocab] matrix or, as a fast
path, one target id per token (-1 = none).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import tinynn as TinyNN
from ._lib import LlamaConfigC, check, lib

LORA_BITS = {"q": 1, "k": 2, "v": 4, "o": 8, "gate": 16, "up": 32, "down": 64}
IO_TOKEN_IDS, IO_POSITIONS, IO_LABELS, IO_HP, IO_LOSS = range(5)


@dataclass
class LlamaConfig:
    """Model dims (Toy::SmolLM2Config, lib/toy/models/toy_smollm2.rb:147-260)."""
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
    rope_freq_factors: Optional[Sequence[float]] = None
    # mixture-of-experts FFN (QLoRA): n_experts, the top n_experts_used per token,
    # expert width d_ff; qk_norm 2 = RMSNorm over the whole q and k vectors
    n_experts: int = 0
    n_experts_used: int = 0
    norm_topk: bool = False
    qk_norm: int = 0

    @staticmethod
    def olmoe_1b_7b() -> "LlamaConfig":
        """OLMoE-1B-7B shape: 64 experts, top 8, expert FFN 1024, QK-RMSNorm."""
        return LlamaConfig(50304, 2048, 16, 16, 128, 1024, 16, 1.0e4, 1.0e-5, n_experts=64, n_experts_used=8,
                           qk_norm=2)

    @staticmethod
    def smollm2_135m() -> "LlamaConfig":
        return LlamaConfig(49152, 576, 9, 3, 64, 1536, 30, 1.0e5, 1.0e-5)

    @staticmethod
    def llama32_1b() -> "LlamaConfig":
        from .rope import llama3_freq_factors
        return LlamaConfig(128256, 2048, 32, 8, 64, 8192, 16, 5.0e5, 1.0e-5,
                           rope_freq_factors=llama3_freq_factors(64, 5.0e5, 8192, 32.0, 1.0, 4.0))

    @staticmethod
    def qwen25_7b() -> "LlamaConfig":
        return LlamaConfig(152064, 3584, 28, 4, 128, 18944, 28, 1.0e6, 1.0e-6, qkv_bias=True)


@dataclass
class RecipeOptions:
    """Toy::LLM::RecipeOptions (lib/toy/llm/recipe_options.rb:57-137), the fields the GPU path consumes."""
    t_seq: int = 64
    t_batch: int = 1
    untied: bool = False
    qkv_bias: bool = False
    seed: int = 42
    init_scale: float = 1.0
    # > 0: every weight N(0, init_std) instead of the reference's fan-in scaled
    # init (the benchmark configurations' "all weights N(0, 0.02)")
    init_std: float = 0.0
    # attention core: "flash" (fused kernels, d_head 64 or 128; other widths
    # use the materialised path) or "materialized" (score GEMM + softmax + PV GEMM)
    attention: str = "flash"


@dataclass
class LoraOptions:
    """Adapter placement and synthetic init.

    Per-projection adapters (the benchmark configurations): rank r, scale
    alpha / r, A ~ N(0, a_std), B ~ N(0, b_std), drawn after the base from the
    seeded stream. per_head_q=True is toy's own LoRA-Q recipe instead
    (transformer_block.rb:522-579,861-871): one (A_h, B_h) pair per query head,
    no scale, A = a_std * N(0, 1) from upload_lora_q_init!'s raw-seed stream
    (a_std plays init_scale), B = 0; targets must be ("q",)."""
    rank: int = 8
    alpha: float = 16.0
    targets: Sequence[str] = ("q", "v")
    a_std: float = 0.125
    b_std: float = 0.01
    base_std: float = 0.02   # synthetic frozen base N(0, base_std), quantised to Q8_0
    per_head_q: bool = False

    @staticmethod
    def lora_q(rank: int, init_scale: float = 1.0, base_std: float = 0.02) -> "LoraOptions":
        """toy's LoRA recipe: enable_lora_q!(rank) + upload_lora_q_init!(seed, init_scale)."""
        return LoraOptions(rank=rank, alpha=float(rank), targets=("q",), a_std=init_scale, b_std=0.0,
                           base_std=base_std, per_head_q=True)


class LlamaSeqEngine:
    """The engine subset the recipes use: realize, the step's I/O tensors, parameter access."""

    def __init__(self, device: int = 0):
        self.sess = lib().tnn_session_new_on(1, device)
        if not self.sess:
            raise RuntimeError("toy_b200: no CUDA session (is a B200 visible?)")
        self.cfg: Optional[LlamaConfig] = None
        self.t_seq = self.t_batch = 0

    def close(self):
        if self.sess:
            lib().tnn_session_free(self.sess)
            self.sess = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # realize_for_random_init (llama_seq_engine.rb:932) / realize_for_mmap (:713) + build_training_step (:1786)
    def realize(self, cfg: LlamaConfig, opts: RecipeOptions, mode: int, lora: Optional[LoraOptions] = None):
        self.cfg = cfg
        self.t_seq, self.t_batch = opts.t_seq, opts.t_batch
        c = LlamaConfigC()
        c.vocab, c.d_model, c.n_heads, c.n_kv, c.d_head, c.d_ff, c.n_layers = (
            cfg.vocab, cfg.d_model, cfg.n_heads, cfg.n_kv, cfg.d_head, cfg.d_ff, cfg.n_layers)
        c.rope_base, c.rms_eps, c.freq_scale = cfg.rope_base, cfg.rms_eps, 1.0
        c.tied = 0 if (opts.untied or not cfg.tied) else 1
        c.qkv_bias = 1 if (opts.qkv_bias or cfg.qkv_bias) else 0
        c.t_seq, c.t_batch, c.mode = opts.t_seq, opts.t_batch, mode
        if opts.attention not in ("flash", "materialized"):
            raise ValueError(f"unknown attention implementation {opts.attention!r}")
        c.attn_impl = 0 if opts.attention == "flash" else 1
        c.n_experts, c.n_experts_used = cfg.n_experts, cfg.n_experts_used
        c.norm_topk, c.qk_norm = 1 if cfg.norm_topk else 0, cfg.qk_norm
        if lora is not None:
            c.lora_rank, c.lora_alpha = lora.rank, lora.alpha
            c.lora_targets = sum(LORA_BITS[t] for t in lora.targets)
            c.lora_per_head_q = 1 if lora.per_head_q else 0
            if lora.per_head_q and tuple(lora.targets) != ("q",):
                raise ValueError("per-head LoRA-Q adapts the query projection only: targets must be ('q',)")
        self._ff = None
        if cfg.rope_freq_factors is not None:
            self._ff = np.ascontiguousarray(np.asarray(cfg.rope_freq_factors, np.float64))
            c.rope_freq_factors = self._ff.ctypes.data_as(C.POINTER(C.c_double))
        check(lib().tb2_llama_realize(self.sess, C.byref(c)), "tb2_llama_realize")
        if lora is None:
            check(lib().tb2_llama_init_random(self.sess, opts.seed, opts.init_scale, opts.init_std, 0.0, 0.0),
                  "tb2_llama_init_random")
        else:
            check(lib().tb2_llama_init_random(self.sess, opts.seed, 1.0, lora.base_std, lora.a_std, lora.b_std),
                  "tb2_llama_init_random")

    @property
    def t_seq_token_ids(self):
        return lib().tb2_llama_io(self.sess, IO_TOKEN_IDS)

    @property
    def t_seq_positions(self):
        return lib().tb2_llama_io(self.sess, IO_POSITIONS)

    def build_training_step(self):
        """[t_loss, t_labels, t_hp], the triple build_training_step returns."""
        L = lib()
        return [L.tb2_llama_io(self.sess, IO_LOSS), L.tb2_llama_io(self.sess, IO_LABELS),
                L.tb2_llama_io(self.sess, IO_HP)]

    # ---- parameter access (by GGUF-style name)
    def param_names(self):
        L = lib()
        return [L.tb2_llama_param_name(self.sess, i).decode() for i in range(L.tb2_llama_n_params(self.sess))]

    def trainable(self, name: str) -> bool:
        return lib().tb2_llama_param_trainable(self.sess, name.encode()) == 1

    def _shape(self, name):
        t = lib().tb2_llama_param(self.sess, name.encode())
        if not t:
            raise KeyError(name)
        return t, lib().tnn_tensor_ne1(t), lib().tnn_tensor_ne0(t)

    def param(self, name: str) -> np.ndarray:
        t, r, c = self._shape(name)
        return TinyNN.download_row_major(self.sess, t, r, c).squeeze(0) if r == 1 else \
            TinyNN.download_row_major(self.sess, t, r, c)

    def set_param(self, name: str, value) -> None:
        t, r, c = self._shape(name)
        TinyNN.upload_row_major(self.sess, t, np.asarray(value).reshape(r * c))

    def grad(self, name: str) -> np.ndarray:
        t, r, c = self._shape(name)
        out = np.empty(r * c, np.float64)
        check(lib().tb2_param_grad_to_f64(self.sess, name.encode(), out.ctypes.data_as(C.POINTER(C.c_double)),
                                          out.size), "tb2_param_grad_to_f64")
        return out.reshape(r, c) if r > 1 else out

    def moment(self, name: str, which: int) -> np.ndarray:
        t, r, c = self._shape(name)
        out = np.empty(r * c, np.float64)
        check(lib().tb2_param_moment_to_f64(self.sess, name.encode(), which,
                                            out.ctypes.data_as(C.POINTER(C.c_double)), out.size),
              "tb2_param_moment_to_f64")
        return out.reshape(r, c) if r > 1 else out

    def q8_0_blocks(self, name: str) -> np.ndarray:
        t, r, c = self._shape(name)
        out = np.empty(r * (c // 32) * 34, np.uint8)
        check(lib().tb2_param_download_q8_0(self.sess, name.encode(), out.ctypes.data, out.size),
              "tb2_param_download_q8_0")
        return out.reshape(r, c // 32 * 34)

    def set_q8_0_blocks(self, name: str, blocks: np.ndarray) -> None:
        b = np.ascontiguousarray(blocks, np.uint8)
        check(lib().tb2_param_upload_q8_0(self.sess, name.encode(), b.ctypes.data, b.size), "tb2_param_upload_q8_0")

    def launches_per_step(self) -> int:
        return lib().tb2_step_launches(self.sess)

    # ---- GGUF weights and checkpoints
    def load_gguf(self, path: str, moments: bool = False, partial: bool = False) -> int:
        """Load every parameter found in a GGUF file (toy's converter layout or
        its legacy transposed one; Q8_0 blocks verbatim into the frozen base);
        with moments, also the Adam state a checkpoint carries; partial: a
        checkpoint that holds only some tensors (the rest keep their values).
        Returns the number of tensors loaded."""
        L = lib()
        h = L.tnn_gguf_load(path.encode())
        if not h:
            raise RuntimeError(f"toy_b200: cannot read GGUF {path}")
        try:
            n = L.tb2_llama_load_gguf(self.sess, h, (1 if moments else 0) | (2 if partial else 0))
        finally:
            L.tnn_gguf_free(h)
        if n < 0:
            raise RuntimeError(f"toy_b200: tb2_llama_load_gguf failed with code {n}")
        return n

    def save_gguf(self, path: str, frozen: bool = False, moments: bool = False, stacked: bool = False) -> None:
        """Checkpoint the trainable tensors (plus the frozen ones, plus Adam
        moments) as GGUF; per-head LoRA-Q goes under toy's per-head names unless
        stacked."""
        what = 1 | (2 if frozen else 0) | (4 if moments else 0) | (8 if stacked else 0)
        check(lib().tb2_llama_save_gguf(self.sess, path.encode(), what), "tb2_llama_save_gguf")

    def set_grad_accumulation(self, n_micro: int) -> None:
        """Accumulate gradients over n_micro step calls; AdamW runs on every
        n_micro-th call with the mean gradient (the joined-batch step)."""
        check(lib().tb2_llama_set_grad_accumulation(self.sess, int(n_micro)), "tb2_llama_set_grad_accumulation")


def _step(eng: LlamaSeqEngine, t_loss, t_labels, t_hp, seq_ids, positions, m_labels, m_hp, is_first) -> float:
    """from_scratch.rb:89-103 == lora.rb:94-107, in the same order."""
    L = lib()
    s = eng.sess
    if is_first:
        check(L.tnn_graph_reset(s), "tnn_graph_reset")
    else:
        check(L.tnn_graph_reset_grads_only(s), "tnn_graph_reset_grads_only")
    TinyNN.upload_int_array(s, eng.t_seq_token_ids, seq_ids)
    TinyNN.upload_int_array(s, eng.t_seq_positions, positions)
    lab = np.asarray(m_labels)
    if lab.ndim == 1 and np.issubdtype(lab.dtype, np.integer):
        TinyNN.upload_label_ids(s, t_labels, lab)
    else:
        TinyNN.upload_row_major(s, t_labels, lab)
    TinyNN.upload_row_major(s, t_hp, m_hp)
    check(L.tnn_compute_backward(s), "tnn_compute_backward")
    return float(TinyNN.download_row_major(s, t_loss, 1, 1)[0, 0])


class FromScratch:
    """Toy::LLM::Recipes::FromScratch: random-init, every weight trainable."""

    def __init__(self, device: int = 0):
        self.fs_cache = LlamaSeqEngine(device)
        self.fs_t_loss = self.fs_t_labels = self.fs_t_hp = None
        self.fs_step_index = 0

    def realize(self, cfg: LlamaConfig, opts: RecipeOptions) -> None:
        self.fs_cache.realize(cfg, opts, mode=0)
        self.fs_t_loss, self.fs_t_labels, self.fs_t_hp = self.fs_cache.build_training_step()

    def step(self, seq_ids, positions, m_labels, m_hp, is_first: bool) -> float:
        return _step(self.fs_cache, self.fs_t_loss, self.fs_t_labels, self.fs_t_hp, seq_ids, positions, m_labels,
                     m_hp, is_first)


class LoRA:
    """Toy::LLM::Recipes::LoRA over a frozen Q8_0 base (QLoRA).

    realize(cfg, rank, opts) with no LoraOptions runs the reference recipe's own
    adapters: per-head LoRA-Q of the given rank, initialised by
    upload_lora_q_init!(opts.seed, opts.init_scale) (lora.rb:71-82). A
    LoraOptions selects per-projection adapters (q, k, v, o, gate, up, down)."""

    def __init__(self, device: int = 0):
        self.lora_cache = LlamaSeqEngine(device)
        self.lora_t_loss = self.lora_t_labels = self.lora_t_hp = None
        self.lora_step_index = 0

    def realize(self, cfg: LlamaConfig, rank: int, opts: RecipeOptions, lora: Optional[LoraOptions] = None) -> None:
        lo = lora or LoraOptions.lora_q(rank, init_scale=opts.init_scale)
        lo.rank = rank
        self.lora_cache.realize(cfg, opts, mode=1, lora=lo)
        self.lora_t_loss, self.lora_t_labels, self.lora_t_hp = self.lora_cache.build_training_step()

    def step(self, seq_ids, positions, m_labels, m_hp, is_first: bool) -> float:
        return _step(self.lora_cache, self.lora_t_loss, self.lora_t_labels, self.lora_t_hp, seq_ids, positions,
                     m_labels, m_hp, is_first)
