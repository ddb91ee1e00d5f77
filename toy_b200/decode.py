"""Decode with a KV cache over the session's weights: the host side of toy's
KV engine (lib/toy/llm/engine/llama_kv_engine.rb; SmolLM2KVStepResult.decode_step
:2350 takes one token at a position and returns the next token's logits,
decode_batch :2381 runs a prompt through it; enable_kv_q8! :359 keeps K and V
as Q8_0). The weights are those of a realised LlamaSeqEngine (after training,
or after load_gguf); every step is one graph replay on the GPU."""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from ._lib import check, lib


class KVDecoder:
    def __init__(self, engine, max_T: int, n_seq: int = 1, kv_q8: bool = False):
        self.eng = engine
        self.max_T, self.n_seq = max_T, n_seq
        self.vocab = engine.cfg.vocab
        check(lib().tb2_kv_realize(engine.sess, max_T, n_seq, 8 if kv_q8 else 0), "tb2_kv_realize")
        self._logits = np.empty((n_seq, self.vocab), np.float32)

    def reset(self) -> None:
        check(lib().tb2_kv_reset(self.eng.sess), "tb2_kv_reset")

    def decode_step(self, tokens: Sequence[int], positions: Sequence[int]) -> np.ndarray:
        """One token per sequence at its position; returns logits [n_seq, vocab]."""
        t = np.ascontiguousarray(np.asarray(tokens, np.int64).reshape(self.n_seq))
        p = np.ascontiguousarray(np.asarray(positions, np.int64).reshape(self.n_seq))
        check(lib().tb2_kv_decode(self.eng.sess, t.ctypes.data_as(C.POINTER(C.c_longlong)),
                                  p.ctypes.data_as(C.POINTER(C.c_longlong)), self.n_seq,
                                  self._logits.ctypes.data_as(C.POINTER(C.c_float))), "tb2_kv_decode")
        return self._logits.copy()

    def decode_batch(self, token_ids: np.ndarray, pos0: int = 0) -> np.ndarray:
        """Run [n_seq, n] prompt tokens through the cache from position pos0;
        returns the logits after every token, [n, n_seq, vocab]."""
        ids = np.asarray(token_ids, np.int64).reshape(self.n_seq, -1)
        return np.stack([self.decode_step(ids[:, i], np.full(self.n_seq, pos0 + i)) for i in range(ids.shape[1])])

    def generate(self, prompt: np.ndarray, n_new: int) -> np.ndarray:
        """Greedy continuation of [n_seq, n] prompts by n_new tokens each."""
        ids = np.asarray(prompt, np.int64).reshape(self.n_seq, -1)
        logits = self.decode_batch(ids)[-1]
        out = []
        pos = ids.shape[1]
        for _ in range(n_new):
            nxt = np.argmax(logits, axis=-1)
            out.append(nxt)
            logits = self.decode_step(nxt, np.full(self.n_seq, pos))
            pos += 1
        return np.stack(out, axis=1)

    def close(self) -> None:
        lib().tb2_kv_free(self.eng.sess)
