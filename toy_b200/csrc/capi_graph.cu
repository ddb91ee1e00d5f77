// C ABI of the tnn_* primitive op surface (tinynn/tinynn_ggml.h): tensor
// creation, op nodes, realize / compute, autograd and introspection. Names,
// arguments and NULL / negative-code error behaviour follow the reference
// header; see graph.cu for the execution model.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "prims.cuh"
#include "toy_b200.h"

using tb2::Session;
using tb2::Tensor;

namespace {

Session* S(void* p) { return static_cast<Session*>(p); }
Tensor* T(void* p) { return static_cast<Tensor*>(p); }

// a session that runs the fused step program has no primitive graph
Session* graph_session(void* sess) {
  if (!sess) return nullptr;
  Session* s = S(sess);
  return s->eng ? nullptr : s;
}

bool mine(Session* s, void* t) { return t && T(t)->sess == s; }

Tensor* input(void* sess, int type, int ne0, int ne1, int ne2, int ne3, bool persistent) {
  Session* s = graph_session(sess);
  if (!s) return nullptr;
  return tb2::prim_new(s, type, ne0, ne1, ne2, ne3, tb2::kOpNone, persistent);
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- tensors (tinynn_ggml.h:97-141,303-308,394,455)
void* tnn_input_1d_f32(void* sess, int n) { return input(sess, 0, n, 1, 1, 1, false); }
void* tnn_input_2d_f32(void* sess, int rows, int cols) { return input(sess, 0, cols, rows, 1, 1, false); }
void* tnn_input_2d_f32_persistent(void* sess, int rows, int cols) { return input(sess, 0, cols, rows, 1, 1, true); }
void* tnn_input_1d_f32_persistent(void* sess, int n) { return input(sess, 0, n, 1, 1, 1, true); }
void* tnn_input_3d_f32_persistent(void* sess, int ne0, int ne1, int ne2) {
  return input(sess, 0, ne0, ne1, ne2, 1, true);
}
void* tnn_input_4d_f32_persistent(void* sess, int ne0, int ne1, int ne2, int ne3) {
  return input(sess, 0, ne0, ne1, ne2, ne3, true);
}
void* tnn_input_2d_persistent_typed(void* sess, int rows, int cols, int ggml_type) {
  if (ggml_type != 0 && ggml_type != 8) return nullptr;
  if (ggml_type == 8 && cols % 32) return nullptr;
  return input(sess, ggml_type, cols, rows, 1, 1, true);
}
void* tnn_input_1d_i32(void* sess, int n) { return input(sess, 26, n, 1, 1, 1, false); }
void* tnn_input_1d_i32_ctx(void* sess, int n) { return input(sess, 26, n, 1, 1, 1, true); }
void* tnn_rope_freq_factors_alloc(void* sess, int n_dims) {
  if (n_dims <= 0 || n_dims % 2) return nullptr;
  return input(sess, 0, n_dims / 2, 1, 1, 1, true);
}
long tnn_row_size(int ggml_type, int ne0) {
  if (ggml_type == 8) return ne0 % 32 ? -1 : (long)ne0 / 32 * 34;
  if (ggml_type == 0 || ggml_type == 26) return (long)ne0 * 4;
  return -1;
}
int tnn_finalize_weights(void* sess) { return graph_session(sess) ? 0 : -1; }
int tnn_session_set_graph_capacity(void* sess, int capacity) { return sess && capacity > 0 ? 0 : -1; }
int tnn_zero_tensor(void* sess, void* tensor) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, tensor)) return -1;
  return tb2::prim_zero(s, T(tensor));
}

// ---------------------------------------------------------------- ops (tinynn_ggml.h:157-400)
void* tnn_matmul(void* sess, void* a, void* b) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) ? tb2::prim_mul_mat(s, T(a), T(b)) : nullptr;
}
void* tnn_out_prod(void* sess, void* a, void* b) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) ? tb2::prim_out_prod(s, T(a), T(b)) : nullptr;
}
void* tnn_add(void* sess, void* a, void* b) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) ? tb2::prim_binary(s, tb2::kOpAdd, T(a), T(b)) : nullptr;
}
void* tnn_sub(void* sess, void* a, void* b) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) ? tb2::prim_binary(s, tb2::kOpSub, T(a), T(b)) : nullptr;
}
void* tnn_mul(void* sess, void* a, void* b) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) ? tb2::prim_binary(s, tb2::kOpMul, T(a), T(b)) : nullptr;
}
void* tnn_scale(void* sess, void* a, double v) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_scale(s, T(a), v) : nullptr;
}
void* tnn_silu(void* sess, void* a) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_unary(s, tb2::kOpSilu, T(a), nullptr) : nullptr;
}
void* tnn_silu_back(void* sess, void* x, void* dy) {
  Session* s = graph_session(sess);
  return s && mine(s, x) && mine(s, dy) ? tb2::prim_unary(s, tb2::kOpSiluBack, T(x), T(dy)) : nullptr;
}
void* tnn_swiglu_split(void* sess, void* gate, void* up) {
  Session* s = graph_session(sess);
  return s && mine(s, gate) && mine(s, up) ? tb2::prim_unary(s, tb2::kOpSwiglu, T(gate), T(up)) : nullptr;
}
// RMSNorm(x) * gamma_row: two nodes, as tinynn_ggml.c builds it
void* tnn_rms_norm(void* sess, void* x, void* gamma_row, double eps) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, x) || !mine(s, gamma_row)) return nullptr;
  Tensor* n = tb2::prim_rms_norm(s, T(x), eps);
  return n ? tb2::prim_binary(s, tb2::kOpMul, n, T(gamma_row)) : nullptr;
}
void* tnn_rms_norm_back(void* sess, void* x, void* dy, double eps) {
  Session* s = graph_session(sess);
  return s && mine(s, x) && mine(s, dy) ? tb2::prim_rms_norm_back(s, T(x), T(dy), eps) : nullptr;
}
void* tnn_rope_ext(void* sess, void* a, void* pos, int n_dims, double freq_base, double freq_scale, double ext_factor,
                   double attn_factor, double beta_fast, double beta_slow, void* freq_factors) {
  (void)beta_fast; (void)beta_slow;
  Session* s = graph_session(sess);
  if (!s || !mine(s, a) || !mine(s, pos) || (freq_factors && !mine(s, freq_factors))) return nullptr;
  return tb2::prim_rope(s, tb2::kOpRope, T(a), T(pos), n_dims, freq_base, freq_scale, ext_factor, attn_factor,
                        freq_factors ? T(freq_factors) : nullptr);
}
void* tnn_rope_ext_back(void* sess, void* dy, void* pos, int n_dims, double freq_base, double freq_scale,
                        double ext_factor, double attn_factor, double beta_fast, double beta_slow, void* freq_factors) {
  (void)beta_fast; (void)beta_slow;
  Session* s = graph_session(sess);
  if (!s || !mine(s, dy) || !mine(s, pos) || (freq_factors && !mine(s, freq_factors))) return nullptr;
  return tb2::prim_rope(s, tb2::kOpRopeBack, T(dy), T(pos), n_dims, freq_base, freq_scale, ext_factor, attn_factor,
                        freq_factors ? T(freq_factors) : nullptr);
}
void* tnn_softmax(void* sess, void* a) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_softmax(s, T(a), nullptr, 1.0, 0.0) : nullptr;
}
void* tnn_soft_max_ext(void* sess, void* a, void* mask, double scale, double max_bias) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, a) || (mask && !mine(s, mask))) return nullptr;
  return tb2::prim_softmax(s, T(a), mask ? T(mask) : nullptr, scale, max_bias);
}
void* tnn_softmax_back(void* sess, void* a, void* dy) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, dy) ? tb2::prim_softmax_back(s, T(a), T(dy), 1.0) : nullptr;
}
void* tnn_diag_mask_inf(void* sess, void* a, int n_past) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_diag_mask(s, tb2::kOpDiagMaskInf, T(a), n_past) : nullptr;
}
void* tnn_transpose(void* sess, void* a) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_permute(s, T(a), 1, 0, 2, 3) : nullptr;
}
void* tnn_permute(void* sess, void* a, int axis0, int axis1, int axis2, int axis3) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_permute(s, T(a), axis0, axis1, axis2, axis3) : nullptr;
}
void* tnn_cont(void* sess, void* a) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, a)) return nullptr;
  Tensor* x = T(a);
  return tb2::prim_cont(s, x, x->ne[0], x->ne[1], x->ne[2], x->ne[3]);
}
void* tnn_cont_2d(void* sess, void* a, int ne0, int ne1) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_cont(s, T(a), ne0, ne1, 1, 1) : nullptr;
}
void* tnn_reshape_2d(void* sess, void* a, int ne0, int ne1) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_reshape(s, T(a), ne0, ne1, 1, 1) : nullptr;
}
void* tnn_reshape_3d(void* sess, void* a, int ne0, int ne1, int ne2) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_reshape(s, T(a), ne0, ne1, ne2, 1) : nullptr;
}
void* tnn_view_1d(void* sess, void* a, int ne0, long offset) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, a) || offset < 0) return nullptr;
  return tb2::prim_view(s, T(a), ne0, 1, 1, 0, 0, (size_t)offset);
}
void* tnn_view_2d(void* sess, void* a, int ne0, int ne1, long nb1, long offset) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, a) || offset < 0 || nb1 < 0) return nullptr;
  return tb2::prim_view(s, T(a), ne0, ne1, 1, (size_t)nb1, 0, (size_t)offset);
}
void* tnn_view_3d(void* sess, void* a, int ne0, int ne1, int ne2, long nb1, long nb2, long offset) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, a) || offset < 0 || nb1 < 0 || nb2 < 0) return nullptr;
  return tb2::prim_view(s, T(a), ne0, ne1, ne2, (size_t)nb1, (size_t)nb2, (size_t)offset);
}
void* tnn_concat(void* sess, void* a, void* b, int dim) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) ? tb2::prim_concat(s, T(a), T(b), dim) : nullptr;
}
void* tnn_get_rows(void* sess, void* table, void* idx) {
  Session* s = graph_session(sess);
  return s && mine(s, table) && mine(s, idx) ? tb2::prim_get_rows(s, T(table), T(idx)) : nullptr;
}
void* tnn_null_ptr(void) { return nullptr; }

// tinynn_ggml.c tnn_upload_causal_mask semantics: f32 [hist][n_tok] (ne0 =
// hist), column i open (0) for keys j <= pos0 + i, -inf beyond; hist must be
// pos0 + n_tok (-2 otherwise), a tensor of another shape or type gives -3.
int tnn_upload_causal_mask(void* sess, void* tensor, int hist, int n_tok, int pos0) {
  if (!sess || !tensor) return -1;
  if (hist <= 0 || n_tok <= 0 || pos0 < 0 || hist != pos0 + n_tok) return -2;
  Session* s = graph_session(sess);
  if (!s || !mine(s, tensor)) return -1;
  Tensor* t = T(tensor);
  if (t->type != 0 || t->ne[0] != hist || t->ne[1] != n_tok || t->ne[2] != 1 || t->ne[3] != 1) return -3;
  std::vector<double> m((size_t)hist * n_tok);
  for (int i = 0; i < n_tok; ++i)
    for (int j = 0; j < hist; ++j) m[(size_t)i * hist + j] = j <= pos0 + i ? 0.0 : -INFINITY;
  return tb2::prim_upload_f64(s, t, m.data(), m.size());
}

// tinynn_ggml.c tnn_upload_cell_mask semantics: f32 [hi][n_tok], cell c open to
// token t when it holds an earlier-or-equal position of t's sequence
// (cell_owner[c] == tok_owner[t] && cell_pos[c] <= tok_pos[t]) or is a shared
// prefix cell (owner -1) below t's shared-prefix length; owner -2 is free.
int tnn_upload_cell_mask(void* sess, void* tensor, int hi, int n_tok, const long* cell_owner, const long* cell_pos,
                         const long* tok_owner, const long* tok_pos, const long* tok_shared) {
  if (!sess || !tensor || !cell_owner || !cell_pos || !tok_owner || !tok_pos || !tok_shared) return -1;
  if (hi <= 0 || n_tok <= 0) return -2;
  Session* s = graph_session(sess);
  if (!s || !mine(s, tensor)) return -1;
  Tensor* t = T(tensor);
  if (t->type != 0 || t->ne[0] != hi || t->ne[1] != n_tok || t->ne[2] != 1 || t->ne[3] != 1) return -3;
  std::vector<double> m((size_t)hi * n_tok);
  for (int k = 0; k < n_tok; ++k)
    for (int c = 0; c < hi; ++c) {
      const bool own = cell_owner[c] == tok_owner[k] && cell_pos[c] <= tok_pos[k];
      const bool shared = cell_owner[c] == -1 && cell_pos[c] < tok_shared[k];
      m[(size_t)k * hi + c] = own || shared ? 0.0 : -INFINITY;
    }
  return tb2::prim_upload_f64(s, t, m.data(), m.size());
}
void* tnn_detach(void* sess, void* a) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_detach(s, T(a)) : nullptr;
}
void* tnn_cpy(void* sess, void* a, void* b) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) ? tb2::prim_cpy(s, T(a), T(b)) : nullptr;
}
void* tnn_set_rows(void* sess, void* a, void* b, void* idx) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) && mine(s, idx) ? tb2::prim_set_rows(s, T(a), T(b), T(idx)) : nullptr;
}
void* tnn_mul_mat_id(void* sess, void* as, void* b, void* ids) {
  Session* s = graph_session(sess);
  return s && mine(s, as) && mine(s, b) && mine(s, ids) ? tb2::prim_mul_mat_id(s, T(as), T(b), T(ids)) : nullptr;
}
void* tnn_add_id(void* sess, void* a, void* b, void* ids) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) && mine(s, ids) ? tb2::prim_add_id(s, T(a), T(b), T(ids)) : nullptr;
}
void* tnn_argsort(void* sess, void* a, int descending) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_argsort(s, T(a), descending, 0) : nullptr;
}
void* tnn_top_k(void* sess, void* a, int k) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && k > 0 ? tb2::prim_argsort(s, T(a), 1, k) : nullptr;
}
void* tnn_get_rows_back(void* sess, void* d_out, void* idx, void* table_shape) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, d_out) || !mine(s, idx) || !mine(s, table_shape)) return nullptr;
  return tb2::prim_get_rows_back(s, T(d_out), T(idx), T(table_shape));
}
void* tnn_cross_entropy_loss(void* sess, void* a, void* b) {
  Session* s = graph_session(sess);
  return s && mine(s, a) && mine(s, b) ? tb2::prim_cross_entropy(s, T(a), T(b)) : nullptr;
}
void* tnn_sum(void* sess, void* a) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_sum(s, tb2::kOpSum, T(a)) : nullptr;
}
void* tnn_sum_rows(void* sess, void* a) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_sum(s, tb2::kOpSumRows, T(a)) : nullptr;
}
void* tnn_opt_step_adamw(void* sess, void* a, void* grad, void* m, void* v, void* params) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, a) || !mine(s, grad) || !mine(s, m) || !mine(s, v) || !mine(s, params)) return nullptr;
  return tb2::prim_opt_adamw(s, T(a), T(grad), T(m), T(v), T(params));
}

// ---------------------------------------------------------------- programs (tinynn_ggml.h:376-469)
void tnn_set_param(void* tensor) {
  if (tensor) T(tensor)->is_param = true;
}
void tnn_set_loss(void* tensor) {
  if (!tensor) return;
  T(tensor)->is_loss = true;
  T(tensor)->sess->loss = T(tensor);
}
void tnn_set_output(void* tensor) {
  if (!tensor) return;
  T(tensor)->is_output = true;
  T(tensor)->sess->roots.push_back(T(tensor));
}
int tnn_add_to_graph(void* sess, void* tensor) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, tensor)) return -1;
  s->roots.push_back(T(tensor));
  return 0;
}
int tnn_realize(void* sess, void* result) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, result)) return -1;
  return tb2::prim_realize(s, T(result));
}
int tnn_build_forward_only(void* sess, void* result) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, result)) return -1;
  return tb2::prim_build_forward(s, T(result));
}
int tnn_build_backward(void* sess) {
  Session* s = graph_session(sess);
  if (!s) return -1;
  return tb2::prim_build_backward(s);
}
int tnn_extend_backward_graph(void* sess, void* node) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, node) || !s->bwd_built) return -2;
  s->ext.push_back(T(node));
  s->prim_realized = false;
  return 0;
}
int tnn_realize_backward(void* sess) {
  Session* s = graph_session(sess);
  if (!s || !s->bwd_built) return -2;
  return tb2::prim_realize_backward(s);
}
void* tnn_tensor_grad(void* sess, void* tensor) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, tensor)) return nullptr;
  return T(tensor)->grad;
}
int tnn_compute(void* sess) {
  Session* s = graph_session(sess);
  if (!s) return -1;
  if (!s->prim_realized) return -2;
  return tb2::prim_compute(s);
}
int tnn_reset_for_rebuild(void* sess) {
  Session* s = graph_session(sess);
  if (!s) return -1;
  s->nodes.clear();
  s->bwd.clear();
  s->ext.clear();
  s->roots.clear();
  s->loss = nullptr;
  s->bwd_built = false;
  s->prim_realized = false;
  return 0;
}
void* tnn_input_1d_i32_persistent(void* sess, int n) { return input(sess, 26, n, 1, 1, 1, true); }
void* tnn_input_3d_persistent_typed(void* sess, int ne0, int ne1, int ne2, int ggml_type) {
  if (ggml_type != 0 && ggml_type != 8) return nullptr;
  if (ggml_type == 8 && ne0 % 32) return nullptr;
  return input(sess, ggml_type, ne0, ne1, ne2, 1, true);
}
void* tnn_cast(void* sess, void* a, int dtype) {
  Session* s = graph_session(sess);
  return s && mine(s, a) ? tb2::prim_cast(s, T(a), dtype) : nullptr;
}
void* tnn_flash_attn_ext(void* sess, void* q, void* k, void* v, void* mask, double scale, double max_bias,
                         double logit_softcap) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, q) || !mine(s, k) || !mine(s, v) || (mask && !mine(s, mask)) || logit_softcap != 0.0)
    return nullptr;
  return tb2::prim_flash_attn_ext(s, T(q), T(k), T(v), mask ? T(mask) : nullptr, scale, max_bias);
}
void* tnn_opt_step_sgd(void* sess, void* a, void* grad, void* params) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, a) || !mine(s, grad) || !mine(s, params)) return nullptr;
  return tb2::prim_opt_sgd(s, T(a), T(grad), T(params));
}
int tnn_pin_all_graph_b_nodes(void* sess) { return graph_session(sess) ? 0 : -1; }   // every node keeps its buffer

// ---------------------------------------------------------------- weights from a host region (tinynn_ggml.h:120-131)
int tnn_session_attach_weight_mmap(void* sess, void* base, size_t size) {
  Session* s = graph_session(sess);
  if (!s || !base || !size) return -1;
  s->mmap_base = static_cast<const uint8_t*>(base);
  s->mmap_size = size;
  return 0;
}

namespace {
// a persistent tensor whose bytes are copied from the attached region at buf_offset
void* mmap_input(void* sess, int type, int ne0, int ne1, int ne2, size_t off) {
  Session* s = graph_session(sess);
  if (!s || !s->mmap_base || (type != 0 && type != 8) || (type == 8 && ne0 % 32)) return nullptr;
  Tensor* t = tb2::prim_new(s, type, ne0, ne1, ne2, 1, tb2::kOpNone, true);
  if (!t) return nullptr;
  const size_t nbytes = type == 8 ? (size_t)t->nel() / 32 * 34 : (size_t)t->nel() * 4;
  if (off > s->mmap_size || nbytes > s->mmap_size - off) return nullptr;
  const uint8_t* src = s->mmap_base + off;
  int rc;
  if (type == 8) {
    rc = tb2::prim_upload_q8_0(s, t, src, nbytes);
  } else {
    std::vector<float> h((size_t)t->nel());
    std::memcpy(h.data(), src, nbytes);   // the region may be unaligned
    rc = tb2::prim_upload_f32_raw(s, t, h.data(), h.size());
  }
  return rc ? nullptr : t;
}
}  // namespace

void* tnn_input_2d_persistent_mmap(void* sess, int rows, int cols, int ggml_type, size_t buf_offset) {
  return mmap_input(sess, ggml_type, cols, rows, 1, buf_offset);
}
void* tnn_input_3d_persistent_mmap(void* sess, int ne0, int ne1, int ne2, int ggml_type, size_t buf_offset) {
  return mmap_input(sess, ggml_type, ne0, ne1, ne2, buf_offset);
}
void* tnn_input_1d_persistent_mmap(void* sess, int n, int ggml_type, size_t buf_offset) {
  return mmap_input(sess, ggml_type, n, 1, 1, buf_offset);
}

// ---------------------------------------------------------------- scratch staging (tinynn_ggml.h:471-484,563-567)
namespace {
constexpr size_t kScratchFloats = (16u << 20) / 4;   // 16 MiB
std::vector<float>* scratch_of(void* sess) {
  if (!sess) return nullptr;
  Session* s = S(sess);
  if (s->scratch.empty()) s->scratch.assign(kScratchFloats, 0.0f);
  return &s->scratch;
}
}  // namespace

void tnn_scratch_set(void* sess, int idx, double v) {
  auto* sc = scratch_of(sess);
  if (sc && idx >= 0 && (size_t)idx < sc->size()) (*sc)[idx] = (float)v;
}
double tnn_scratch_get(void* sess, int idx) {
  auto* sc = scratch_of(sess);
  return sc && idx >= 0 && (size_t)idx < sc->size() ? (double)(*sc)[idx] : 0.0;
}
void tnn_scratch_set_i32(void* sess, int idx, int value) {
  auto* sc = scratch_of(sess);
  if (sc && idx >= 0 && (size_t)idx < sc->size()) std::memcpy(&(*sc)[idx], &value, 4);
}
int tnn_scratch_get_i32(void* sess, int idx) {
  auto* sc = scratch_of(sess);
  int v = 0;
  if (sc && idx >= 0 && (size_t)idx < sc->size()) std::memcpy(&v, &(*sc)[idx], 4);
  return v;
}
int tnn_upload(void* sess, void* tensor) {
  auto* sc = scratch_of(sess);
  if (!sc || !tensor || T(tensor)->sess != S(sess)) return -1;
  Tensor* t = T(tensor);
  const size_t n = (size_t)t->nel();
  if (n > sc->size()) return -2;
  const bool ints = t->type == 26 || t->role == Tensor::kIds || t->role == Tensor::kPos;
  if (ints) {
    std::vector<long> v(n);
    for (size_t i = 0; i < n; ++i) {
      int x;
      std::memcpy(&x, &(*sc)[i], 4);
      v[i] = x;
    }
    return tnn_upload_from_int_array(sess, tensor, v.data(), n);
  }
  if (t->role == Tensor::kPrim && t->type == 0) return tb2::prim_upload_f32_raw(S(sess), t, sc->data(), n);
  std::vector<double> v(sc->begin(), sc->begin() + n);
  return tnn_upload_from_float_array(sess, tensor, v.data(), n);
}
int tnn_download(void* sess, void* tensor) {
  auto* sc = scratch_of(sess);
  if (!sc || !tensor || T(tensor)->sess != S(sess)) return -1;
  Tensor* t = T(tensor);
  const size_t n = t->role == Tensor::kLoss ? 1 : (size_t)t->nel();
  if (n > sc->size()) return -2;
  if (t->role == Tensor::kPrim) {
    if (t->type == 26) {
      std::vector<float> f(n);
      const int rc = tb2::prim_download_f32_raw(S(sess), t, f.data(), n);
      for (size_t i = 0; i < n && !rc; ++i) tnn_scratch_set_i32(sess, (int)i, (int)f[i]);
      return rc;
    }
    return tb2::prim_download_f32_raw(S(sess), t, sc->data(), n);
  }
  std::vector<double> v(n);
  const int rc = tnn_download_to_f64_array(sess, tensor, v.data(), n);
  for (size_t i = 0; i < n && !rc; ++i) (*sc)[i] = (float)v[i];
  return rc;
}
int tnn_upload_transposed_f64(void* sess, void* tensor, const double* src, int br, int bc) {
  if (!sess || !tensor || !src || br <= 0 || bc <= 0) return -1;
  Tensor* t = T(tensor);
  if ((long long)br * bc > t->nel()) return -2;
  // column j of the row-major (br x bc) matrix becomes the contiguous run t[j * br ..]
  std::vector<double> v((size_t)br * bc);
  for (int j = 0; j < bc; ++j)
    for (int i = 0; i < br; ++i) v[(size_t)j * br + i] = src[(size_t)i * bc + j];
  return tnn_upload_from_float_array(sess, tensor, v.data(), v.size());
}
double tnn_scratch_min_f32(void* sess, int n) {
  auto* sc = scratch_of(sess);
  if (!sc || n <= 0) return 0.0;
  float m = (*sc)[0];
  for (int i = 1; i < n && (size_t)i < sc->size(); ++i) m = std::min(m, (*sc)[i]);
  return m;
}
double tnn_scratch_max_f32(void* sess, int n) {
  auto* sc = scratch_of(sess);
  if (!sc || n <= 0) return 0.0;
  float m = (*sc)[0];
  for (int i = 1; i < n && (size_t)i < sc->size(); ++i) m = std::max(m, (*sc)[i]);
  return m;
}
double tnn_scratch_sum_abs_f32(void* sess, int n) {
  auto* sc = scratch_of(sess);
  double a = 0.0;
  for (int i = 0; sc && i < n && (size_t)i < sc->size(); ++i) a += std::fabs((double)(*sc)[i]);
  return a;
}
int tnn_scratch_nan_count_f32(void* sess, int n) {
  auto* sc = scratch_of(sess);
  int c = 0;
  for (int i = 0; sc && i < n && (size_t)i < sc->size(); ++i) c += std::isnan((*sc)[i]) ? 1 : 0;
  return c;
}

int tnn_upload_q8_0_blocks(void* sess, void* tensor, const void* blocks, size_t nbytes) {
  Session* s = graph_session(sess);
  if (!s || !mine(s, tensor) || !blocks) return -1;
  return tb2::prim_upload_q8_0(s, T(tensor), blocks, nbytes);
}

// ---------------------------------------------------------------- introspection (tinynn_ggml.h:516-537)
int tnn_tensor_op(void* t) { return t ? T(t)->op : -1; }
const char* tnn_tensor_op_name(void* t) { return t ? tb2::prim_op_name(T(t)->op) : ""; }
void* tnn_tensor_src(void* t, int i) { return t && i >= 0 && i < 5 ? T(t)->src[i] : nullptr; }
int tnn_tensor_flags(void* t) {
  if (!t) return 0;
  const Tensor* x = T(t);
  // INPUT 1 | OUTPUT 2 | PARAM 4 | LOSS 8 | COMPUTE 16
  return (x->op == 0 ? 1 : 16) | (x->is_output ? 2 : 0) | (x->is_param ? 4 : 0) | (x->is_loss ? 8 : 0);
}
int tnn_graph_n_nodes(void* sess) {
  Session* s = graph_session(sess);
  return s ? (int)(s->nodes.size() + s->bwd.size()) : 0;
}
void* tnn_graph_node(void* sess, int i) {
  Session* s = graph_session(sess);
  if (!s || i < 0) return nullptr;
  if ((size_t)i < s->nodes.size()) return s->nodes[i];
  i -= (int)s->nodes.size();
  return (size_t)i < s->bwd.size() ? s->bwd[i] : nullptr;
}

}  // extern "C"
