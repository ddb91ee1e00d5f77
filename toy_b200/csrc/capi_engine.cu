// C ABI: sessions, tensor handles and the training-step entry points
// (tnn_* drop-ins for tinynn/tinynn_ggml.h, tb2_* additions).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "engine.cuh"
#include "prims.cuh"
#include "session.cuh"
#include "toy_b200.h"

using tb2::LlamaEngine;
using tb2::Session;
using tb2::Tensor;

namespace {

Session* S(void* s) { return static_cast<Session*>(s); }
Tensor* Tn(void* t) { return static_cast<Tensor*>(t); }

Tensor* make_io(Session* s, int role, int ne0, int ne1, int type, const char* name) {
  auto t = std::make_unique<Tensor>();
  t->sess = s;
  t->role = role;
  t->ne[0] = ne0;
  t->ne[1] = ne1;
  t->type = type;
  t->name = name;
  s->tensors.push_back(std::move(t));
  return s->tensors.back().get();
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------ session
void* tnn_session_new_on(int backend_kind, int device) {
  if (backend_kind != 1) {
    fprintf(stderr, "[toy_b200] backend_kind %d requested: this library is the CUDA (sm_100a) backend only\n",
            backend_kind);
    return nullptr;
  }
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return nullptr;
  if (cudaSetDevice(device) != cudaSuccess) return nullptr;
  auto* s = new Session();
  s->kind = backend_kind;
  s->device = device;
  return s;
}

void* tnn_session_new(int backend_kind) { return tnn_session_new_on(backend_kind, 0); }

int tnn_cuda_get_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

void tnn_session_free(void* sess) {
  if (!sess) return;
  cudaSetDevice(S(sess)->device);
  delete S(sess);
}

const char* tnn_backend_name(void* sess) { return sess ? "CUDA-sm100a" : "none"; }

int tnn_link_check(void) { return 73; }

// ------------------------------------------------------------------ engine realize
int tb2_llama_realize(void* sess, const tb2_llama_config* cfg) {
  if (!sess || !cfg) return -1;
  Session* s = S(sess);
  if (s->eng) return -2;
  tb2::LlamaConfig c;
  c.vocab = cfg->vocab; c.d_model = cfg->d_model; c.n_heads = cfg->n_heads; c.n_kv = cfg->n_kv;
  c.d_head = cfg->d_head; c.d_ff = cfg->d_ff; c.n_layers = cfg->n_layers;
  c.rope_base = (float)cfg->rope_base; c.rms_eps = (float)cfg->rms_eps;
  c.freq_scale = cfg->freq_scale > 0 ? (float)cfg->freq_scale : 1.0f;
  c.tied = cfg->tied; c.qkv_bias = cfg->qkv_bias; c.T = cfg->t_seq; c.B = cfg->t_batch; c.mode = cfg->mode;
  c.lora_rank = cfg->lora_rank; c.lora_alpha = (float)cfg->lora_alpha; c.lora_targets = cfg->lora_targets;
  c.attn_impl = cfg->attn_impl;
  c.lora_per_head_q = cfg->lora_per_head_q;
  c.n_experts = cfg->n_experts;
  c.n_experts_used = cfg->n_experts_used;
  c.norm_topk = cfg->norm_topk;
  c.qk_norm = cfg->qk_norm;
  if (cfg->rope_freq_factors)
    for (int i = 0; i < cfg->d_head / 2; ++i) c.freq_factors.push_back((float)cfg->rope_freq_factors[i]);
  if (cudaSetDevice(s->device) != cudaSuccess) return -3;
  auto e = std::make_unique<LlamaEngine>(c, s->device);
  const int rc = e->realize();
  if (rc) return rc;
  s->eng = std::move(e);
  const int N = c.T * c.B;
  s->io[TB2_IO_TOKEN_IDS] = make_io(s, Tensor::kIds, N, 1, 26, "token_ids");
  s->io[TB2_IO_POSITIONS] = make_io(s, Tensor::kPos, N, 1, 26, "positions");
  s->io[TB2_IO_LABELS] = make_io(s, Tensor::kLabels, c.vocab, N, 0, "labels");
  s->io[TB2_IO_HP] = make_io(s, Tensor::kHp, 7, 1, 0, "adamw_params");
  s->io[TB2_IO_LOSS] = make_io(s, Tensor::kLoss, 1, 1, 0, "loss");
  for (const auto& p : s->eng->params()) {
    Tensor* t = make_io(s, Tensor::kParam, p.cols, p.rows, p.q8 ? 8 : 0, p.name.c_str());
    t->param = p.name;
  }
  return 0;
}

int tb2_llama_init_random(void* sess, long long seed, double init_scale, double std_all, double lora_a_std,
                          double lora_b_std) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->init_random(seed, init_scale, std_all, lora_a_std, lora_b_std);
}

void* tb2_llama_io(void* sess, int which) {
  if (!sess || !S(sess)->eng || which < 0 || which >= TB2_IO_COUNT) return nullptr;
  return S(sess)->io[which];
}

void* tb2_llama_param(void* sess, const char* name) {
  if (!sess || !name || !S(sess)->eng) return nullptr;
  for (auto& t : S(sess)->tensors)
    if (t->role == Tensor::kParam && t->param == name) return t.get();
  return nullptr;
}

int tb2_llama_n_params(void* sess) {
  if (!sess || !S(sess)->eng) return -2;
  return (int)S(sess)->eng->params().size();
}

const char* tb2_llama_param_name(void* sess, int i) {
  if (!sess || !S(sess)->eng || i < 0 || i >= (int)S(sess)->eng->params().size()) return nullptr;
  return S(sess)->eng->params()[i].name.c_str();
}

int tb2_llama_param_trainable(void* sess, const char* name) {
  if (!sess || !name || !S(sess)->eng) return -1;
  const tb2::Param* p = S(sess)->eng->find(name);
  return p ? (p->trainable ? 1 : 0) : -1;
}

long long tb2_llama_n_trainable(void* sess) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->n_trainable();
}

static int param_to_f64(void* sess, const char* name, double* dst, size_t n, int what) {
  if (!sess || !name || !dst) return -1;
  LlamaEngine* e = S(sess)->eng.get();
  if (!e) return -2;
  const tb2::Param* p = e->find(name);
  if (!p || (long long)n != p->numel()) return -1;
  std::vector<float> h(n);
  int rc = what == 0 ? e->get_param(name, h.data(), n)
         : what == 1 ? e->get_grad(name, h.data(), n)
                     : e->get_moment(name, what - 2, h.data(), n);
  if (rc) return rc;
  for (size_t i = 0; i < n; ++i) dst[i] = h[i];
  return 0;
}

int tb2_param_grad_to_f64(void* sess, const char* name, double* dst, size_t n) {
  return param_to_f64(sess, name, dst, n, 1);
}

int tb2_param_moment_to_f64(void* sess, const char* name, int which, double* dst, size_t n) {
  if (which != 0 && which != 1) return -1;
  return param_to_f64(sess, name, dst, n, 2 + which);
}

int tb2_param_upload_q8_0(void* sess, const char* name, const void* blocks, size_t nbytes) {
  if (!sess || !name || !blocks) return -1;
  if (!S(sess)->eng) return -2;
  return S(sess)->eng->set_param_q8(name, static_cast<const uint8_t*>(blocks), (long long)nbytes);
}

int tb2_param_download_q8_0(void* sess, const char* name, void* blocks, size_t nbytes) {
  if (!sess || !name || !blocks) return -1;
  if (!S(sess)->eng) return -2;
  return S(sess)->eng->get_param_q8(name, static_cast<uint8_t*>(blocks), (long long)nbytes);
}

int tb2_upload_label_ids(void* sess, void* labels_tensor, const long* ids, size_t n) {
  if (!sess || !labels_tensor || !ids) return -1;
  if (!S(sess)->eng || Tn(labels_tensor)->role != Tensor::kLabels) return -2;
  std::vector<long long> v(ids, ids + n);
  return S(sess)->eng->set_label_ids(v.data(), (int)n);
}

int tb2_step_launches(void* sess) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->launches_per_step();
}

int tb2_set_use_graph(void* sess, int on) {
  if (!sess || !S(sess)->eng) return -2;
  S(sess)->eng->set_use_graph(on != 0);
  return 0;
}

int tb2_forward_only(void* sess) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->forward_only();
}

int tb2_llama_set_grad_accumulation(void* sess, int n_micro) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->set_grad_accumulation(n_micro);
}

int tb2_run_steps(void* sess, int n, float* ms) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->run_steps(n, ms);
}

int tb2_profile_step(void* sess, int is_first, int* kinds, float* ms, double* flops, int cap) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->profile_step(is_first != 0, kinds, ms, flops, cap);
}

int tb2_sync(void* sess) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->sync();
}

// ------------------------------------------------------------------ step (tnn_* drop-ins)
int tnn_graph_reset(void* sess) {
  if (!sess) return -1;
  if (!S(sess)->eng) {   // primitive graph: zero the optimizer moments at the next backward
    S(sess)->reset_pending = true;
    return 0;
  }
  S(sess)->first_pending = true;
  return 0;
}

int tnn_graph_reset_grads_only(void* sess) {
  if (!sess) return -1;
  return 0;  // every gradient element is overwritten by the next backward (both programs)
}

int tnn_compute_backward(void* sess) {
  if (!sess) return -1;
  Session* s = S(sess);
  if (!s->eng) return s->bwd_built ? tb2::prim_compute_backward(s) : -2;
  if (s->dp && tb2::dp_status(s)) return -2;   // its communicator was aborted: no more steps
  const bool first = s->first_pending;
  s->first_pending = false;
  const int rc = s->eng->step(first, true);
  // a data-parallel step waits for its collectives with a time limit, so a
  // rank that never joins ends the step with an error instead of a hang
  return rc ? rc : (s->dp ? tb2::dp_wait_step(s) : 0);
}

// ------------------------------------------------------------------ tensor I/O
int tnn_upload_from_float_array(void* sess, void* tensor, const double* data, size_t n) {
  if (!sess || !tensor || !data) return -1;
  Session* s = S(sess);
  Tensor* t = Tn(tensor);
  if (t->sess != s) return -1;
  if (t->role == Tensor::kPrim) return tb2::prim_upload_f64(s, t, data, n);
  if (!s->eng) return -2;
  switch (t->role) {
    case Tensor::kLabels: return s->eng->set_labels_dense(data, (long long)n);
    case Tensor::kHp: return s->eng->set_hp(data, (int)n);
    case Tensor::kParam: {
      const tb2::Param* p = s->eng->find(t->param);
      if (!p || (long long)n != p->numel()) return -1;
      std::vector<float> h(n);
      for (size_t i = 0; i < n; ++i) h[i] = (float)data[i];
      return s->eng->set_param(t->param, h.data(), (long long)n);
    }
    default: return -1;
  }
}

int tnn_upload_from_int_array(void* sess, void* tensor, const long* data, size_t n) {
  if (!sess || !tensor || !data) return -1;
  Session* s = S(sess);
  Tensor* t = Tn(tensor);
  if (t->sess != s) return -1;
  if (t->role == Tensor::kPrim) return tb2::prim_upload_i64(s, t, data, n);
  if (!s->eng) return -2;
  std::vector<long long> v(data, data + n);
  if (t->role == Tensor::kIds) return s->eng->set_tokens(v.data(), (int)n);
  if (t->role == Tensor::kPos) return s->eng->set_positions(v.data(), (int)n);
  if (t->role == Tensor::kLabels) return s->eng->set_label_ids(v.data(), (int)n);
  return -1;
}

int tnn_download_to_f64_array(void* sess, void* tensor, double* dst, size_t n) {
  if (!sess || !tensor || !dst) return -1;
  Session* s = S(sess);
  Tensor* t = Tn(tensor);
  if (t->sess != s) return -1;
  if (t->role == Tensor::kPrim) return tb2::prim_download_f64(s, t, dst, n);
  if (!s->eng) return -2;
  if (t->role == Tensor::kLoss) {
    if (n < 1) return -2;
    dst[0] = (double)s->eng->last_loss();
    return 0;
  }
  if (t->role == Tensor::kParam) return param_to_f64(sess, t->param.c_str(), dst, n, 0);
  return -1;
}

int tnn_tensor_ne0(void* t) { return t ? Tn(t)->ne[0] : 0; }
int tnn_tensor_ne1(void* t) { return t ? Tn(t)->ne[1] : 0; }
int tnn_tensor_ne2(void* t) { return t ? Tn(t)->ne[2] : 0; }
int tnn_tensor_ne3(void* t) { return t ? Tn(t)->ne[3] : 0; }
int tnn_tensor_nelements(void* t) {
  return t ? Tn(t)->ne[0] * Tn(t)->ne[1] * Tn(t)->ne[2] * Tn(t)->ne[3] : 0;
}
size_t tnn_tensor_nbytes(void* t) {
  if (!t) return 0;
  const size_t n = (size_t)tnn_tensor_nelements(t);
  if (Tn(t)->type == 8) return n / 32 * 34;
  return n * 4;
}
const char* tnn_tensor_name(void* t) { return t ? Tn(t)->name.c_str() : ""; }
void tnn_tensor_set_name(void* t, const char* name) {
  if (t && name) Tn(t)->name = name;
}
int tnn_tensor_dtype(void* t) { return t ? Tn(t)->type : -1; }

}  // extern "C"

extern "C" long long tb2_debug_activation(void* sess, int which, int layer, float* dst, long long cap) {
  if (!sess || !S(sess)->eng) return -2;
  return S(sess)->eng->debug_activation(which, layer, dst, cap);
}
