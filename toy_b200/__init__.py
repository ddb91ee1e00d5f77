"""toy_b200: a B200-native (sm_100a) backend for toy's training step.

The product is the C-ABI library libtoyb200.so (include/toy_b200.h). This
package holds its ctypes binding and the host mirror of toy's recipe surface.
"""
from .adamw import AdamW
from .recipes import FromScratch, LlamaConfig, LlamaSeqEngine, LoRA, LoraOptions, RecipeOptions

__all__ = ["AdamW", "FromScratch", "LoRA", "LlamaConfig", "LlamaSeqEngine", "LoraOptions", "RecipeOptions"]
