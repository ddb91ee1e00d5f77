"""ctypes binding of ``libtoyb200.so`` (the C ABI declared in include/toy_b200.h).

The library is the product; this module only declares argument types. It
fails loudly when the shared library is missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtoyb200.so")


class Operand(C.Structure):
    _fields_ = [("hi", C.c_void_p), ("lo", C.c_void_p), ("mn_major", C.c_int), ("ld", C.c_longlong),
                ("rows", C.c_int), ("cols", C.c_int), ("batch_stride", C.c_longlong), ("nbatch", C.c_int),
                ("bdiv1", C.c_int), ("bmul1", C.c_int), ("bdiv2", C.c_int), ("bmul2", C.c_int),
                ("q8", C.c_void_p), ("q8_scale", C.c_void_p)]


class Epilogue(C.Structure):
    _fields_ = [("mode", C.c_int), ("alpha", C.c_float), ("out", C.c_void_p), ("res", C.c_void_p),
                ("out_hi", C.c_void_p), ("out_lo", C.c_void_p), ("bstride", C.c_longlong), ("z_div", C.c_int),
                ("z_s1", C.c_longlong), ("m_div", C.c_int),
                ("m_s1", C.c_longlong), ("m_s0", C.c_longlong), ("n_div", C.c_int), ("n_s1", C.c_longlong)]


class LlamaConfigC(C.Structure):
    _fields_ = [("vocab", C.c_int), ("d_model", C.c_int), ("n_heads", C.c_int), ("n_kv", C.c_int),
                ("d_head", C.c_int), ("d_ff", C.c_int), ("n_layers", C.c_int), ("rope_base", C.c_double),
                ("rms_eps", C.c_double), ("freq_scale", C.c_double), ("tied", C.c_int), ("qkv_bias", C.c_int),
                ("t_seq", C.c_int), ("t_batch", C.c_int), ("mode", C.c_int), ("lora_rank", C.c_int),
                ("lora_alpha", C.c_double), ("lora_targets", C.c_int),
                ("rope_freq_factors", C.POINTER(C.c_double)), ("attn_impl", C.c_int), ("lora_per_head_q", C.c_int),
                ("n_experts", C.c_int), ("n_experts_used", C.c_int), ("norm_topk", C.c_int), ("qk_norm", C.c_int)]


_lib = None
VP, D, DP, LP, SZ, I, LL = C.c_void_p, C.c_double, C.POINTER(C.c_double), C.POINTER(C.c_long), C.c_size_t, C.c_int, \
    C.c_longlong

# (name, restype, argtypes) for every exported symbol this module binds.
_SIGS = [
    ("tnn_session_new", VP, [I]),
    ("tnn_session_new_on", VP, [I, I]),
    ("tnn_cuda_get_device_count", I, []),
    ("tnn_session_free", None, [VP]),
    ("tnn_backend_name", C.c_char_p, [VP]),
    ("tnn_link_check", I, []),
    ("tb2_llama_realize", I, [VP, C.POINTER(LlamaConfigC)]),
    ("tb2_llama_init_random", I, [VP, LL, D, D, D, D]),
    ("tb2_llama_io", VP, [VP, I]),
    ("tb2_llama_param", VP, [VP, C.c_char_p]),
    ("tb2_llama_n_params", I, [VP]),
    ("tb2_llama_param_name", C.c_char_p, [VP, I]),
    ("tb2_llama_param_trainable", I, [VP, C.c_char_p]),
    ("tb2_llama_n_trainable", LL, [VP]),
    ("tb2_param_grad_to_f64", I, [VP, C.c_char_p, DP, SZ]),
    ("tb2_param_moment_to_f64", I, [VP, C.c_char_p, I, DP, SZ]),
    ("tb2_param_upload_q8_0", I, [VP, C.c_char_p, VP, SZ]),
    ("tb2_param_download_q8_0", I, [VP, C.c_char_p, VP, SZ]),
    ("tb2_upload_label_ids", I, [VP, VP, LP, SZ]),
    ("tb2_step_launches", I, [VP]),
    ("tb2_set_use_graph", I, [VP, I]),
    ("tb2_forward_only", I, [VP]),
    ("tb2_sync", I, [VP]),
    ("tb2_debug_activation", LL, [VP, I, I, C.POINTER(C.c_float), LL]),
    ("tb2_run_steps", I, [VP, I, C.POINTER(C.c_float)]),
    ("tb2_llama_set_grad_accumulation", I, [VP, I]),
    ("tb2_nccl_unique_id", I, [VP, SZ]),
    ("tb2_dp_init", I, [VP, VP, I, I]),
    ("tb2_dp_free", I, [VP]),
    ("tb2_dp_set_bucket_floats", I, [VP, LL]),
    ("tb2_dp_set_timeout_ms", I, [LL]),
    ("tb2_dp_wait", I, [VP]),
    ("tb2_dp_status", I, [VP]),
    ("tb2_dp_abort", I, [VP]),
    ("tb2_dp_bucket_plan", LL, [C.POINTER(C.c_longlong), I, LL, LL, C.POINTER(C.c_longlong), LL]),
    ("tb2_dp_session_bucket_plan", LL, [VP, C.POINTER(C.c_longlong), LL]),
    ("tb2_profile_step", I, [VP, I, C.POINTER(C.c_int), C.POINTER(C.c_float), C.POINTER(C.c_double), I]),
    ("tnn_graph_reset", I, [VP]),
    ("tnn_graph_reset_grads_only", I, [VP]),
    ("tnn_compute_backward", I, [VP]),
    ("tnn_upload_from_float_array", I, [VP, VP, DP, SZ]),
    ("tnn_upload_from_int_array", I, [VP, VP, LP, SZ]),
    ("tnn_download_to_f64_array", I, [VP, VP, DP, SZ]),
    ("tnn_tensor_ne0", I, [VP]),
    ("tnn_tensor_ne1", I, [VP]),
    ("tnn_tensor_ne2", I, [VP]),
    ("tnn_tensor_ne3", I, [VP]),
    ("tnn_tensor_nbytes", SZ, [VP]),
    ("tnn_tensor_nelements", I, [VP]),
    ("tnn_tensor_name", C.c_char_p, [VP]),
    ("tnn_tensor_set_name", None, [VP, C.c_char_p]),
    ("tnn_tensor_dtype", I, [VP]),
    ("tb2_gemm", C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(Operand), C.POINTER(Operand),
                           C.POINTER(Epilogue), C.c_int, C.c_int, C.c_void_p]),
    ("tb2_gemm_noalloc", C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(Operand),
                                   C.POINTER(Operand), C.POINTER(Epilogue), C.c_int, C.c_int, C.c_void_p]),
    ("tb2_gemm_noalloc_error", C.c_int, []),
    ("tb2_split_f32", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    ("tb2_gemm_set_pair_mode", C.c_int, [C.c_int]),
    ("tb2_gemm_set_tile_width", C.c_int, [C.c_int]),
    ("tb2_set_q8_base_mode", C.c_int, [C.c_int]),
    ("tb2_set_q8_ring_l2", C.c_int, [C.c_int]),
    ("tb2_set_side_gemm_ctas", C.c_int, [C.c_int]),
    ("tb2_set_side_gemm_tile_width", C.c_int, [C.c_int]),
    ("tb2_set_plan_alone", C.c_int, [C.c_int]),
    ("tb2_set_f16_wgrad", C.c_int, [C.c_int]),
    ("tb2_device_error", C.c_int, []),
    ("tb2_q8_0_quantize", C.c_int, [C.c_void_p, C.c_void_p, C.c_longlong, C.c_int, C.c_void_p]),
    ("tb2_q8_0_dequantize", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_longlong, C.c_int,
                                      C.c_void_p]),
    ("tb2_version", C.c_char_p, []),
    # primitive op graph
    ("tnn_input_1d_f32", VP, [VP, I]),
    ("tnn_input_2d_f32", VP, [VP, I, I]),
    ("tnn_input_2d_f32_persistent", VP, [VP, I, I]),
    ("tnn_input_1d_f32_persistent", VP, [VP, I]),
    ("tnn_input_3d_f32_persistent", VP, [VP, I, I, I]),
    ("tnn_input_4d_f32_persistent", VP, [VP, I, I, I, I]),
    ("tnn_input_2d_persistent_typed", VP, [VP, I, I, I]),
    ("tnn_input_1d_i32", VP, [VP, I]),
    ("tnn_input_1d_i32_ctx", VP, [VP, I]),
    ("tnn_rope_freq_factors_alloc", VP, [VP, I]),
    ("tnn_row_size", C.c_long, [I, I]),
    ("tnn_finalize_weights", I, [VP]),
    ("tnn_session_set_graph_capacity", I, [VP, I]),
    ("tnn_zero_tensor", I, [VP, VP]),
    ("tnn_upload_q8_0_blocks", I, [VP, VP, VP, SZ]),
    ("tnn_matmul", VP, [VP, VP, VP]),
    ("tnn_out_prod", VP, [VP, VP, VP]),
    ("tnn_add", VP, [VP, VP, VP]),
    ("tnn_sub", VP, [VP, VP, VP]),
    ("tnn_mul", VP, [VP, VP, VP]),
    ("tnn_scale", VP, [VP, VP, D]),
    ("tnn_silu", VP, [VP, VP]),
    ("tnn_silu_back", VP, [VP, VP, VP]),
    ("tnn_swiglu_split", VP, [VP, VP, VP]),
    ("tnn_rms_norm", VP, [VP, VP, VP, D]),
    ("tnn_rms_norm_back", VP, [VP, VP, VP, D]),
    ("tnn_rope_ext", VP, [VP, VP, VP, I, D, D, D, D, D, D, VP]),
    ("tnn_rope_ext_back", VP, [VP, VP, VP, I, D, D, D, D, D, D, VP]),
    ("tnn_softmax", VP, [VP, VP]),
    ("tnn_soft_max_ext", VP, [VP, VP, VP, D, D]),
    ("tnn_softmax_back", VP, [VP, VP, VP]),
    ("tnn_diag_mask_inf", VP, [VP, VP, I]),
    ("tnn_transpose", VP, [VP, VP]),
    ("tnn_permute", VP, [VP, VP, I, I, I, I]),
    ("tnn_cont", VP, [VP, VP]),
    ("tnn_cont_2d", VP, [VP, VP, I, I]),
    ("tnn_reshape_2d", VP, [VP, VP, I, I]),
    ("tnn_reshape_3d", VP, [VP, VP, I, I, I]),
    ("tnn_view_1d", VP, [VP, VP, I, C.c_long]),
    ("tnn_view_2d", VP, [VP, VP, I, I, C.c_long, C.c_long]),
    ("tnn_view_3d", VP, [VP, VP, I, I, I, C.c_long, C.c_long, C.c_long]),
    ("tnn_concat", VP, [VP, VP, VP, I]),
    ("tnn_get_rows", VP, [VP, VP, VP]),
    ("tnn_get_rows_back", VP, [VP, VP, VP, VP]),
    ("tnn_mul_mat_id", VP, [VP, VP, VP, VP]),
    ("tnn_null_ptr", VP, []),
    ("tnn_detach", VP, [VP, VP]),
    ("tnn_cpy", VP, [VP, VP, VP]),
    ("tnn_set_rows", VP, [VP, VP, VP, VP]),
    ("tnn_upload_causal_mask", C.c_int, [VP, VP, C.c_int, C.c_int, C.c_int]),
    ("tnn_upload_cell_mask", C.c_int, [VP, VP, C.c_int, C.c_int, C.POINTER(C.c_long), C.POINTER(C.c_long),
                                       C.POINTER(C.c_long), C.POINTER(C.c_long), C.POINTER(C.c_long)]),
    ("tnn_add_id", VP, [VP, VP, VP, VP]),
    ("tnn_argsort", VP, [VP, VP, C.c_int]),
    ("tnn_top_k", VP, [VP, VP, C.c_int]),
    ("tnn_cross_entropy_loss", VP, [VP, VP, VP]),
    ("tnn_sum", VP, [VP, VP]),
    ("tnn_sum_rows", VP, [VP, VP]),
    ("tnn_opt_step_adamw", VP, [VP, VP, VP, VP, VP, VP]),
    ("tnn_set_param", None, [VP]),
    ("tnn_set_loss", None, [VP]),
    ("tnn_set_output", None, [VP]),
    ("tnn_add_to_graph", I, [VP, VP]),
    ("tnn_realize", I, [VP, VP]),
    ("tnn_build_forward_only", I, [VP, VP]),
    ("tnn_build_backward", I, [VP]),
    ("tnn_extend_backward_graph", I, [VP, VP]),
    ("tnn_realize_backward", I, [VP]),
    ("tnn_tensor_grad", VP, [VP, VP]),
    ("tnn_compute", I, [VP]),
    ("tnn_reset_for_rebuild", I, [VP]),
    ("tnn_tensor_op", I, [VP]),
    ("tnn_tensor_op_name", C.c_char_p, [VP]),
    ("tnn_tensor_src", VP, [VP, I]),
    ("tnn_tensor_flags", I, [VP]),
    ("tnn_graph_n_nodes", I, [VP]),
    ("tnn_graph_node", VP, [VP, I]),
    ("tnn_input_1d_i32_persistent", VP, [VP, I]),
    ("tnn_input_3d_persistent_typed", VP, [VP, I, I, I, I]),
    ("tnn_session_attach_weight_mmap", I, [VP, VP, SZ]),
    ("tnn_input_2d_persistent_mmap", VP, [VP, I, I, I, SZ]),
    ("tnn_input_3d_persistent_mmap", VP, [VP, I, I, I, I, SZ]),
    ("tnn_input_1d_persistent_mmap", VP, [VP, I, I, SZ]),
    ("tnn_opt_step_sgd", VP, [VP, VP, VP, VP]),
    ("tnn_cast", VP, [VP, VP, I]),
    ("tnn_flash_attn_ext", VP, [VP, VP, VP, VP, VP, D, D, D]),
    ("tnn_pin_all_graph_b_nodes", I, [VP]),
    ("tnn_scratch_set", None, [VP, I, D]),
    ("tnn_scratch_get", D, [VP, I]),
    ("tnn_scratch_set_i32", None, [VP, I, I]),
    ("tnn_scratch_get_i32", I, [VP, I]),
    ("tnn_upload", I, [VP, VP]),
    ("tnn_download", I, [VP, VP]),
    ("tnn_scratch_min_f32", D, [VP, I]),
    ("tnn_scratch_max_f32", D, [VP, I]),
    ("tnn_scratch_sum_abs_f32", D, [VP, I]),
    ("tnn_scratch_nan_count_f32", I, [VP, I]),
    ("tnn_upload_transposed_f64", I, [VP, VP, DP, I, I]),
    # GGUF files
    ("tnn_gguf_load", VP, [C.c_char_p]),
    ("tnn_gguf_free", None, [VP]),
    ("tnn_gguf_n_tensors", I, [VP]),
    ("tnn_gguf_tensor_name", C.c_char_p, [VP, I]),
    ("tnn_gguf_tensor_ne", I, [VP, I, I]),
    ("tnn_gguf_tensor_type", I, [VP, I]),
    ("tnn_gguf_tensor_nbytes", SZ, [VP, I]),
    ("tnn_gguf_read_f32_to_doubles", I, [VP, I, DP, SZ]),
    ("tnn_gguf_tensor_is_quantized", I, [VP, I]),
    ("tnn_gguf_get_u32", I, [VP, C.c_char_p]),
    ("tnn_gguf_get_f32", D, [VP, C.c_char_p]),
    ("tnn_gguf_get_bool", I, [VP, C.c_char_p]),
    ("tnn_gguf_get_str", C.c_char_p, [VP, C.c_char_p]),
    ("tnn_gguf_arch_prefix", C.c_char_p, [VP]),
    ("tnn_gguf_is_native_layout", I, [VP]),
    ("tnn_gguf_arr_n", I, [VP, C.c_char_p]),
    ("tnn_gguf_arr_str", C.c_char_p, [VP, C.c_char_p, I]),
    ("tnn_gguf_arr_i32", I, [VP, C.c_char_p, I]),
    ("tnn_gguf_mmap_base", VP, [VP]),
    ("tnn_gguf_mmap_size", SZ, [VP]),
    ("tnn_gguf_tensor_file_offset", SZ, [VP, I]),
    ("tnn_gguf_find_index", I, [VP, C.c_char_p]),
    ("tnn_gguf_write_demo_file", I, [C.c_char_p]),
    ("tnn_gguf_w_init", VP, []),
    ("tnn_gguf_w_set_str", None, [VP, C.c_char_p, C.c_char_p]),
    ("tnn_gguf_w_set_u32", None, [VP, C.c_char_p, I]),
    ("tnn_gguf_w_set_f32", None, [VP, C.c_char_p, D]),
    ("tnn_gguf_w_set_bool", None, [VP, C.c_char_p, I]),
    ("tnn_gguf_w_add_tensor", None, [VP, VP]),
    ("tnn_gguf_w_finalize", I, [VP, C.c_char_p]),
    ("tnn_gguf_w_free", None, [VP]),
    ("tb2_gguf_w_add_f32", I, [VP, C.c_char_p, I, I, C.POINTER(C.c_float)]),
    ("tb2_gguf_w_add_q8_0", I, [VP, C.c_char_p, I, I, VP]),
    ("tb2_llama_load_gguf", I, [VP, VP, I]),
    ("tb2_kv_realize", I, [VP, I, I, I]),
    ("tb2_kv_reset", I, [VP]),
    ("tb2_kv_decode", I, [VP, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong), I, C.POINTER(C.c_float)]),
    ("tb2_kv_logits", I, [VP, C.POINTER(C.c_float), LL]),
    ("tb2_kv_run", I, [VP, I, C.POINTER(C.c_float)]),
    ("tb2_kv_launches", I, [VP]),
    ("tb2_kv_free", I, [VP]),
    ("tb2_llama_save_gguf", I, [VP, C.c_char_p, I]),
]


def lib() -> C.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"toy_b200: {LIB_PATH} is missing; run `python toy_b200/build.py` "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"toy_b200: {what} failed with code {rc}")
