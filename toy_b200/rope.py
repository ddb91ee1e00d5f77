"""RoPE scaling helpers (Toy::RopeScaling, lib/toy/models/toy_smollm2.rb:66-142)."""
from __future__ import annotations

import math


def llama3_freq_factors(d_head: int, freq_base: float, orig_max_pos: int, factor: float, low_freq: float,
                        high_freq: float):
    """compute_llama3_freq_factors (toy_smollm2.rb:112-142): d_head/2 per-pair divisors."""
    n = d_head // 2
    low_w, high_w = orig_max_pos / low_freq, orig_max_pos / high_freq
    out = []
    for i in range(n):
        freq = 1.0 / (freq_base ** ((2.0 * i) / d_head))
        wl = 2.0 * math.pi / freq
        if wl < high_w:
            out.append(1.0)
        elif wl > low_w:
            out.append(factor)
        else:
            sm = (orig_max_pos / wl - low_freq) / (high_freq - low_freq)
            out.append((1.0 - sm) * factor + sm * 1.0)
    return out
