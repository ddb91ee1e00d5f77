"""The library's GGUF reader and writer on the host (no GPU): the committed
fixtures written by gguf-py (tests/golden/make_gguf.py) read back tensor by
tensor -- directory, offsets, metadata, values (F32 exact; Q8_0 blocks
bit-identical to gguf-py's quantizer and dequantised as scale * quant) -- the
zero tail after the mapping (tinynn_gguf.h:89-94), the native / legacy layout
rule, writer round trips, and malformed files."""
import ctypes as C
import os
import sys

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLD)
import make_gguf as MG  # noqa: E402

Q8, F32 = 8, 0


@pytest.fixture(scope="module")
def L():
    from toy_b200._lib import lib
    return lib()


@pytest.fixture(scope="module")
def native(L):
    h = L.tnn_gguf_load(os.path.join(GOLD, "tiny_llama_q8.gguf").encode())
    assert h
    yield h
    L.tnn_gguf_free(h)


def values(L, h, i):
    n = 1
    for d in range(4):
        n *= max(1, L.tnn_gguf_tensor_ne(h, i, d))
    out = np.empty(n, np.float64)
    assert L.tnn_gguf_read_f32_to_doubles(h, i, out.ctypes.data_as(C.POINTER(C.c_double)), n) == 0
    return out


def test_directory_and_values(L, native):
    want = MG.tensors()
    assert L.tnn_gguf_n_tensors(native) == len(want)
    for name, x in want.items():
        i = L.tnn_gguf_find_index(native, name.encode())
        assert i >= 0 and L.tnn_gguf_tensor_name(native, i).decode() == name
        assert L.tnn_gguf_tensor_ne(native, i, 0) == x.shape[-1]
        assert L.tnn_gguf_tensor_ne(native, i, 1) == (x.shape[0] if x.ndim == 2 else 1)
        quant = x.ndim == 2 and name.startswith("blk.")
        assert L.tnn_gguf_tensor_type(native, i) == (Q8 if quant else F32)
        assert L.tnn_gguf_tensor_is_quantized(native, i) == (1 if quant else 0)
        got = values(L, native, i).reshape(x.shape)
        if quant:
            blocks = O.q8_0_quantize(x)
            assert L.tnn_gguf_tensor_nbytes(native, i) == blocks.size
            base = L.tnn_gguf_mmap_base(native)
            raw = C.string_at(base + L.tnn_gguf_tensor_file_offset(native, i), blocks.size)
            assert raw == blocks.tobytes(), name                      # gguf-py's blocks, verbatim
            assert np.array_equal(got, O.q8_0_dequantize(blocks, x.shape[1]))
        else:
            assert np.array_equal(got, x.astype(np.float64)), name
    assert L.tnn_gguf_find_index(native, b"no.such.tensor") == -1


def test_offsets_match_gguf_py(L, native):
    gguf = pytest.importorskip("gguf")
    r = gguf.GGUFReader(os.path.join(GOLD, "tiny_llama_q8.gguf"))
    for t in r.tensors:
        i = L.tnn_gguf_find_index(native, t.name.encode())
        assert L.tnn_gguf_tensor_file_offset(native, i) == t.data_offset
        assert L.tnn_gguf_tensor_nbytes(native, i) == t.n_bytes


def test_metadata(L, native):
    assert L.tnn_gguf_get_u32(native, b"llama.embedding_length") == MG.D
    assert L.tnn_gguf_get_u32(native, b"llama.block_count") == MG.L
    assert abs(L.tnn_gguf_get_f32(native, b"llama.attention.layer_norm_rms_epsilon") - 1e-5) < 1e-12
    assert L.tnn_gguf_get_str(native, b"general.architecture") == b"llama"
    assert L.tnn_gguf_get_str(native, b"general.name") == b"tiny-llama-q8"
    assert L.tnn_gguf_arch_prefix(native) == b"llama"
    assert L.tnn_gguf_arr_n(native, b"tokenizer.ggml.token_type") == 4
    assert [L.tnn_gguf_arr_i32(native, b"tokenizer.ggml.token_type", k) for k in range(4)] == [1, 3, 3, 1]
    assert L.tnn_gguf_get_u32(native, b"missing.key") == -1
    assert L.tnn_gguf_get_str(native, b"llama.block_count") is None    # wrong type
    assert L.tnn_gguf_get_bool(native, b"toy.ggml_native") == -1


def test_zero_tail_after_the_mapping(L, native):
    base, size = L.tnn_gguf_mmap_base(native), L.tnn_gguf_mmap_size(native)
    assert size == os.path.getsize(os.path.join(GOLD, "tiny_llama_q8.gguf"))
    assert C.string_at(base + size, 4096) == bytes(4096)


def test_layout_rule(L, native):
    assert L.tnn_gguf_is_native_layout(native) == 1
    h = L.tnn_gguf_load(os.path.join(GOLD, "tiny_llama_q8_legacy.gguf").encode())
    assert h
    try:
        assert L.tnn_gguf_is_native_layout(h) == 0
        i = L.tnn_gguf_find_index(h, b"blk.0.ffn_gate.weight")
        assert (L.tnn_gguf_tensor_ne(h, i, 0), L.tnn_gguf_tensor_ne(h, i, 1)) == (MG.FF, MG.D)
        x = MG.tensors()["blk.0.ffn_gate.weight"]
        assert np.array_equal(values(L, h, i).reshape(MG.D, MG.FF), x.T.astype(np.float64))
    finally:
        L.tnn_gguf_free(h)


def test_writer_round_trip(L, tmp_path):
    path = str(tmp_path / "w.gguf").encode()
    w = L.tnn_gguf_w_init()
    L.tnn_gguf_w_set_str(w, b"general.architecture", b"llama")
    L.tnn_gguf_w_set_u32(w, b"llama.block_count", 7)
    L.tnn_gguf_w_set_f32(w, b"llama.rope.freq_base", 1e5)
    L.tnn_gguf_w_set_bool(w, b"toy.ggml_native", 1)
    rng = np.random.default_rng(1)
    a = rng.standard_normal((3, 40)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    qx = rng.standard_normal((4, 64)).astype(np.float32)
    qb = O.q8_0_quantize(qx)
    assert L.tb2_gguf_w_add_f32(w, b"a.weight", 40, 3, a.ctypes.data_as(C.POINTER(C.c_float))) == 0
    assert L.tb2_gguf_w_add_f32(w, b"b", 5, 1, b.ctypes.data_as(C.POINTER(C.c_float))) == 0
    assert L.tb2_gguf_w_add_q8_0(w, b"q.weight", 64, 4, qb.ctypes.data) == 0
    assert L.tb2_gguf_w_add_q8_0(w, b"bad", 40, 4, qb.ctypes.data) == -1    # ne0 not a multiple of 32
    assert L.tnn_gguf_w_finalize(w, path) == 0
    L.tnn_gguf_w_free(w)
    h = L.tnn_gguf_load(path)
    assert h
    try:
        assert L.tnn_gguf_n_tensors(h) == 3
        assert L.tnn_gguf_get_u32(h, b"llama.block_count") == 7
        assert L.tnn_gguf_get_f32(h, b"llama.rope.freq_base") == 1e5
        assert L.tnn_gguf_get_bool(h, b"toy.ggml_native") == 1
        assert np.array_equal(values(L, h, L.tnn_gguf_find_index(h, b"a.weight")).reshape(3, 40), a)
        assert np.array_equal(values(L, h, L.tnn_gguf_find_index(h, b"b")), b)
        i = L.tnn_gguf_find_index(h, b"q.weight")
        raw = C.string_at(L.tnn_gguf_mmap_base(h) + L.tnn_gguf_tensor_file_offset(h, i), qb.size)
        assert raw == qb.tobytes() and L.tnn_gguf_tensor_file_offset(h, i) % 32 == 0
    finally:
        L.tnn_gguf_free(h)
    gguf = pytest.importorskip("gguf")
    r = gguf.GGUFReader(path.decode())
    assert sorted(t.name for t in r.tensors) == ["a.weight", "b", "q.weight"]
    ta = [t for t in r.tensors if t.name == "a.weight"][0]
    assert np.array_equal(np.asarray(ta.data).reshape(3, 40), a)


def test_demo_file_and_bad_files(L, tmp_path):
    p = str(tmp_path / "demo.gguf").encode()
    assert L.tnn_gguf_write_demo_file(p) == 0
    h = L.tnn_gguf_load(p)
    assert h and L.tnn_gguf_tensor_name(h, 0) == b"demo.tensor"
    assert np.array_equal(values(L, h, 0), np.arange(1, 7, dtype=np.float64))
    L.tnn_gguf_free(h)
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"not a gguf file at all")
    assert not L.tnn_gguf_load(str(bad).encode())
    data = open(os.path.join(GOLD, "tiny_llama_q8.gguf"), "rb").read()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(data[: len(data) // 2])     # tensors past the end of the file
    assert not L.tnn_gguf_load(str(cut).encode())
    assert not L.tnn_gguf_load(str(tmp_path / "missing.gguf").encode())
