"""Toy::AdamW (lib/toy/llm/adamw.rb): the 7-slot hp row the training step reads.

Slots: [alpha, beta1, beta2, eps, weight_decay, beta1h, beta2h]. Slots 5/6 mean
different things per graph family and the mode must be declared:
  for_from_scratch(): slots 5/6 = the constant betas
  for_lora():         slots 5/6 = 1/(1-beta^t), beta2 = 0.999 (also full fine-tune)
"""
from __future__ import annotations

import numpy as np

MODE_UNSET, MODE_FROM_SCRATCH, MODE_LORA = 0, 1, 2


class AdamW:
    def __init__(self):
        self.lr = 0.001
        self.beta1 = 0.9
        self.beta2 = 0.95
        self.eps = 1.0e-8
        self.weight_decay = 0.0
        self.bias_correct = False
        self.mode = MODE_UNSET

    @classmethod
    def for_from_scratch(cls) -> "AdamW":
        a = cls()
        a.mode = MODE_FROM_SCRATCH
        return a

    @classmethod
    def for_lora(cls) -> "AdamW":
        a = cls()
        a.beta2 = 0.999
        a.bias_correct = True
        a.mode = MODE_LORA
        return a

    def hp(self, step: int) -> np.ndarray:
        """adamw.rb:112-146; `step` is 1-indexed for the lora convention."""
        if self.mode == MODE_UNSET:
            raise ValueError("AdamW.hp: mode unset -- use AdamW.for_from_scratch() or AdamW.for_lora()")
        if self.mode == MODE_FROM_SCRATCH and self.bias_correct:
            raise ValueError("AdamW.hp: mode=from_scratch but bias_correct=True")
        if self.mode == MODE_LORA and not self.bias_correct:
            raise ValueError("AdamW.hp: mode=lora but bias_correct=False")
        m = np.zeros(7)
        m[:5] = [self.lr, self.beta1, self.beta2, self.eps, self.weight_decay]
        if self.bias_correct:
            m[5] = 1.0 / (1.0 - self.beta1 ** float(step))
            m[6] = 1.0 / (1.0 - self.beta2 ** float(step))
        else:
            m[5], m[6] = self.beta1, self.beta2
        return m

    def hp_for_step(self, step: int) -> np.ndarray:
        """adamw.rb:148-170: 0-indexed loop step; lora adds one."""
        return self.hp(step + 1) if self.mode == MODE_LORA else self.hp(step)
