"""Host-side batch helpers of toy's training loop.

  positions            Toy::LLM::TrainingBatch, 0..T-1 per sequence
                       (lib/toy/llm/training_batch.rb:64-71)
  next_token_labels    Labels.next_token_guarded_batched as target ids: shift by
                       one inside each window, the last position targets itself,
                       -1 marks an id outside the vocabulary
                       (lib/toy/llm/labels.rb:180-204)
  synthetic_token_ids  uniform ids in [0, vocab) from the reference's seeded LCG
                       (lcg_seed_state + lcg_uniform!, llama_seq_engine.rb:1409-1428),
                       floor(u * vocab) per draw, over the stream seeded with seed + 1

Token (b, t) sits at index b * T + t, as the step's inputs expect.
"""
from __future__ import annotations

import numpy as np

_MASK31 = 0x7FFFFFFF


def _lcg_next(s: int) -> int:
    return (s * 1103515245 + 12345) & _MASK31


def _lcg_seed_state(seed: int) -> int:
    s = ((seed + 104729) * 2654435761) % 2147483647
    if s <= 0:
        s = seed + 104729
    for _ in range(8):
        s = _lcg_next(s)
    return s


def synthetic_token_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    s = _lcg_seed_state(seed + 1)
    out = np.empty(n, np.int64)
    for i in range(n):
        s = _lcg_next(s)
        out[i] = min(int((s + 1.0) / 2147483648.0 * vocab), vocab - 1)
    return out


def positions(T: int, B: int) -> np.ndarray:
    return np.tile(np.arange(T, dtype=np.int64), B)


def next_token_labels(ids: np.ndarray, T: int, B: int, vocab: int) -> np.ndarray:
    ids = np.asarray(ids, np.int64).reshape(B, T)
    lab = np.empty((B, T), np.int64)
    lab[:, :-1] = ids[:, 1:]
    lab[:, -1] = ids[:, -1]
    lab[(lab < 0) | (lab >= vocab)] = -1
    return lab.reshape(-1)
