"""Generate tests/golden/tiny_llama_q8.gguf with gguf-py (the GGUF writer of
llama.cpp's converters; the reference's prep/convert_smollm2_to_gguf.py writes
its SmolLM2 files with it), plus tiny_llama_q8_legacy.gguf in toy's legacy
transposed layout (2-D linears stored ne=[out, in], no toy.ggml_native key).

A 2-layer Llama (vocab 512, d 128, 4 query / 2 KV heads of d_head 32, d_ff 256) in the layout toy's converter emits: token_embd, output_norm and the
norms in F32, the seven projections of every block as Q8_0 (gguf-py's
quantizer), llama.* metadata; the values are seeded N(0, 0.02) draws (norms
around 1; tensors() regenerates them with numpy alone, which the tests use as
the expected values). The GGUF tests read the files with the library's own
reader and load them into the step engine; only this script needs gguf-py.

    python tests/golden/make_gguf.py
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
V, D, H, KV, DH, FF, L = 512, 128, 4, 2, 32, 256, 2


def tensors(seed=7):
    rng = np.random.default_rng(seed)
    g = lambda *s: (rng.standard_normal(s) * 0.02).astype(np.float32)
    out = {"token_embd.weight": g(V, D), "output_norm.weight": (1.0 + g(D)).astype(np.float32)}
    for l in range(L):
        p = f"blk.{l}."
        out[p + "attn_norm.weight"] = (1.0 + g(D)).astype(np.float32)
        out[p + "ffn_norm.weight"] = (1.0 + g(D)).astype(np.float32)
        out[p + "attn_q.weight"] = g(H * DH, D)
        out[p + "attn_k.weight"] = g(KV * DH, D)
        out[p + "attn_v.weight"] = g(KV * DH, D)
        out[p + "attn_output.weight"] = g(D, H * DH)
        out[p + "ffn_gate.weight"] = g(FF, D)
        out[p + "ffn_up.weight"] = g(FF, D)
        out[p + "ffn_down.weight"] = g(D, FF)
    return out


def write(path, legacy):
    import gguf
    w = gguf.GGUFWriter(path, "llama")
    w.add_uint32("llama.vocab_size", V)
    w.add_uint32("llama.embedding_length", D)
    w.add_uint32("llama.feed_forward_length", FF)
    w.add_uint32("llama.block_count", L)
    w.add_uint32("llama.attention.head_count", H)
    w.add_uint32("llama.attention.head_count_kv", KV)
    w.add_uint32("llama.context_length", 64)
    w.add_float32("llama.attention.layer_norm_rms_epsilon", 1e-5)
    w.add_float32("llama.rope.freq_base", 1e4)
    w.add_string("general.name", "tiny-llama-q8")
    w.add_array("tokenizer.ggml.token_type", [1, 3, 3, 1])
    for name, x in tensors().items():
        if x.ndim == 2 and name.startswith("blk."):
            if legacy:
                w.add_tensor(name, np.ascontiguousarray(x.T))     # ne=[out, in], F32
            else:
                q = gguf.quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)
                w.add_tensor(name, q, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        else:
            w.add_tensor(name, x)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


if __name__ == "__main__":
    write(os.path.join(HERE, "tiny_llama_q8.gguf"), legacy=False)
    write(os.path.join(HERE, "tiny_llama_q8_legacy.gguf"), legacy=True)
    print("wrote tiny_llama_q8.gguf, tiny_llama_q8_legacy.gguf")
