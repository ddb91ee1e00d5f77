// LlamaEngine: allocation, parameter I/O, seeded init and the step program.
#include "engine.cuh"

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>

#include "flash_attn.cuh"
#include "lora.cuh"
#include "runtime.cuh"

namespace tb2 {

#define CK(x)                  \
  do {                         \
    const int rc_ = (x);       \
    if (rc_ != 0) return rc_;  \
  } while (0)
#define CU(x)                                 \
  do {                                        \
    if ((x) != cudaSuccess) return -3;        \
  } while (0)

int g_q8_base_mode = 1;
int g_ring_l2 = 1;
// 0: 100 CTAs for the one-pass fp16 weight gradients of a full fine-tune
// (measured in the step: 231.3k-233.7k tokens/s at 88-112 CTAs against 227.5k
// uncapped; 225.2k at 124, 223.0k at 40), one per SM otherwise
int g_side_gemm_ctas = 0;
int g_plan_alone = 0;   // measured neutral for QLoRA (270.4k alone vs 270.8k shared, two runs each)
int engine_set_plan_alone(int on) {
  if (on < 0 || on > 1) return -1;
  const int prev = g_plan_alone;
  g_plan_alone = on;
  return prev;
}
int g_side_gemm_bn = 128;   // measured in the step: 223.2k vs 222.1k (plan's choice), 216.1k (256), 210.0k (64)
int g_f16_wgrad = 1;

int engine_set_f16_wgrad(int on) {
  if (on < 0 || on > 1) return -1;
  const int prev = g_f16_wgrad;
  g_f16_wgrad = on;
  return prev;
}

int engine_set_side_gemm_tile_width(int bn) {
  if (bn != 0 && bn != 64 && bn != 128 && bn != 192 && bn != 256) return -1;
  const int prev = g_side_gemm_bn;
  g_side_gemm_bn = bn;
  return prev;
}

int engine_set_side_gemm_ctas(int n) {
  if (n < 0 || n > 148) return -1;
  const int prev = g_side_gemm_ctas;
  g_side_gemm_ctas = n;
  return prev;
}

int engine_set_q8_ring_l2(int on) {
  if (on < 0 || on > 1) return -1;
  const int prev = g_ring_l2;
  g_ring_l2 = on;
  return prev;
}

int engine_set_q8_base_mode(int mode) {
  if (mode < 0 || mode > 1) return -1;
  const int prev = g_q8_base_mode;
  g_q8_base_mode = mode;
  return prev;
}

namespace {

Operand op(Planes p, int rows, int cols, long long ld, int mn) {
  Operand o;
  o.hi = p.hi; o.lo = p.lo; o.mn_major = mn; o.ld = ld; o.rows = rows; o.cols = cols;
  o.batch_stride = (long long)rows * ld; o.nbatch = 1; o.bdiv1 = 1; o.bmul1 = 0; o.bdiv2 = 1; o.bmul2 = 0;
  return o;
}

// an fp16 array as a single-plane operand (GemmDesc::f16)
Operand op16(const __half* p, int rows, int cols, long long ld, int mn) {
  return op(Planes{reinterpret_cast<bf16*>(const_cast<__half*>(p)), nullptr}, rows, cols, ld, mn);
}

Operand bop(Planes p, int rows, int cols, long long ld, int nbatch, int mn, int d1 = 1, int m1 = 1, int d2 = 1,
            int m2 = 0) {
  Operand o = op(p, rows, cols, ld, mn);
  o.nbatch = nbatch; o.bdiv1 = d1; o.bmul1 = m1; o.bdiv2 = d2; o.bmul2 = m2;
  return o;
}

Planes offset(Planes p, long long off) { return Planes{p.hi + off, p.lo + off}; }

// ---- the reference's host init streams (llama_seq_engine.rb:1383-1428) ----
constexpr uint64_t kA = 1103515245ULL, kC = 12345ULL, kMask = 0x7FFFFFFFULL;

struct Affine {
  uint64_t a, c;
};
Affine compose(Affine f, Affine g) {  // g after f
  return Affine{(g.a * f.a) & kMask, (g.a * f.c + g.c) & kMask};
}
uint64_t lcg_skip(uint64_t s, unsigned long long k) {
  Affine acc{1, 0}, step{kA, kC};
  while (k) {
    if (k & 1) acc = compose(acc, step);
    step = compose(step, step);
    k >>= 1;
  }
  return (acc.a * s + acc.c) & kMask;
}
uint64_t lcg_next(uint64_t s) { return (s * kA + kC) & kMask; }

uint64_t lcg_seed_state(long long seed) {
  __int128 v = ((__int128)seed + 104729) * (__int128)2654435761LL;
  __int128 m = v % 2147483647;
  if (m < 0) m += 2147483647;
  long long s = (long long)m;
  if (s <= 0) s = seed + 104729;
  uint64_t st = (uint64_t)s;
  for (int w = 0; w < 8; ++w) st = lcg_next(st);
  return st;
}

// upload_gaussian: pairs of uniforms -> Box-Muller (cos, then sin); returns the new state.
uint64_t gaussian_fill(uint64_t state, float* out, long long n, double stdv) {
  const long long pairs = (n + 1) / 2;
  const int nth = (int)std::min<long long>(16, std::max<long long>(1, pairs / 200000));
  auto work = [&](long long p0, long long p1) {
    uint64_t s = lcg_skip(state, 2ULL * (unsigned long long)p0);
    for (long long p = p0; p < p1; ++p) {
      s = lcg_next(s);
      double u1 = ((double)s + 1.0) / 2147483648.0;
      s = lcg_next(s);
      const double u2 = ((double)s + 1.0) / 2147483648.0;
      if (u1 < 1.0e-300) u1 = 1.0e-300;
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double th = 2.0 * M_PI * u2;
      out[2 * p] = (float)(r * std::cos(th) * stdv);
      if (2 * p + 1 < n) out[2 * p + 1] = (float)(r * std::sin(th) * stdv);
    }
  };
  if (nth <= 1) {
    work(0, pairs);
  } else {
    std::vector<std::thread> ts;
    for (int t = 0; t < nth; ++t) ts.emplace_back(work, pairs * t / nth, pairs * (t + 1) / nth);
    for (auto& t : ts) t.join();
  }
  return lcg_skip(state, 2ULL * (unsigned long long)pairs);
}

const char* kProjName[kLoraCount] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};

}  // namespace

LlamaEngine::LlamaEngine(const LlamaConfig& cfg, int device) : cfg_(cfg), device_(device) {}

LlamaEngine::~LlamaEngine() {
  cudaSetDevice(device_);
  if (ring_keep_) l2_keep_release((size_t)q8pl_.bytes);
  if (graph_) cudaGraphExecDestroy(graph_);
  if (graph_acc_) cudaGraphExecDestroy(graph_acc_);
  for (DeviceBuf* b : {&p32_, &phi_, &plo_, &g_, &m_, &v_, &q8_, &q8v_, &q8s_, &q8pl_, &wsc_ws_, &acc_})
    if (b->p) cudaFree(b->p);
  for (auto& b : bufs_)
    if (b.p) cudaFree(b.p);
  if (stage_) cudaFreeHost(stage_);
  for (cudaEvent_t e : bucket_ev_) cudaEventDestroy(e);
  if (comm_stream_) cudaStreamDestroy(comm_stream_);
  for (cudaEvent_t e : sev_) cudaEventDestroy(e);
  if (wst_) cudaStreamDestroy(wst_);
  if (stream_) cudaStreamDestroy(stream_);
}

// ---------------------------------------------------------------- gradient buckets
int LlamaEngine::bucket_begin() {
  bucket_next_ = 0;
  pend_lo_ = pend_hi_ = n_train_;
  comm_used_ = false;
  if (!allreduce_fn_ || profiling_) return 0;
  if (!comm_stream_) {   // gradient buckets: high priority, so a reduction is not held behind weight gradients
    int prio_lo = 0, prio_hi = 0;
    CU(cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi));
    CU(cudaStreamCreateWithPriority(&comm_stream_, cudaStreamNonBlocking, prio_hi));
  }
  return 0;
}

// Trainable gradients at arena offsets >= lo are final. With flush (or once the
// pending range reaches bucket_floats_) the pending range is all-reduced: on
// comm_stream_ after an event on the step stream, or, in a profiled step, on
// the step stream itself. Every rank runs the same bucket sequence.
int LlamaEngine::bucket_ready(long long lo, bool flush) {
  if (!allreduce_fn_) return 0;
  long long b_lo = 0, b_hi = 0;
  if (!bucket_take(pend_lo_, pend_hi_, lo, flush, bucket_floats_, b_lo, b_hi)) return 0;
  float* buf = grad_arena() + b_lo;
  const long long n = b_hi - b_lo;
  if (profiling_) {
    prof_begin(kKAllreduce, 0.0);
    const int rc = allreduce_fn_(allreduce_ctx_, buf, n, stream_);
    prof_end();
    return rc;
  }
  if (bucket_next_ == bucket_ev_.size()) {
    cudaEvent_t e;
    CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    bucket_ev_.push_back(e);
  }
  cudaEvent_t e = bucket_ev_[bucket_next_++];
  // the range is final once both streams are past it: the side stream waits
  // for the step stream, then marks the point
  CK(fork_side());
  CU(cudaEventRecord(e, side_ ? wst_ : stream_));
  CU(cudaStreamWaitEvent(comm_stream_, e, 0));
  comm_used_ = true;
  return allreduce_fn_(allreduce_ctx_, buf, n, comm_stream_);
}

// The step stream waits for every bucket before the optimiser.
int LlamaEngine::bucket_join() {
  if (!comm_used_) return 0;
  if (bucket_next_ == bucket_ev_.size()) {
    cudaEvent_t e;
    CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    bucket_ev_.push_back(e);
  }
  cudaEvent_t e = bucket_ev_[bucket_next_++];
  CU(cudaEventRecord(e, comm_stream_));
  CU(cudaStreamWaitEvent(stream_, e, 0));
  comm_used_ = false;
  return 0;
}

int LlamaEngine::alloc(DeviceBuf& b, size_t bytes) {
  bytes = (bytes + 255) / 256 * 256;
  if (bytes == 0) bytes = 256;
  if (cudaMalloc(&b.p, bytes) != cudaSuccess) return -3;
  b.bytes = bytes;
  if (cudaMemsetAsync(b.p, 0, bytes, stream_) != cudaSuccess) return -3;
  return 0;
}

int LlamaEngine::add_param(const std::string& name, int rows, int cols, bool trainable, bool q8) {
  Param p;
  p.name = name; p.rows = rows; p.cols = cols; p.trainable = trainable; p.q8 = q8;
  pidx_[name] = (int)params_.size();
  params_.push_back(p);
  return 0;
}

const Param* LlamaEngine::find(const std::string& name) const {
  auto it = pidx_.find(name);
  return it == pidx_.end() ? nullptr : &params_[it->second];
}

const Param& LlamaEngine::P(const std::string& n) const { return params_[pidx_.at(n)]; }

int LlamaEngine::realize() {
  if (realized_) return -2;
  const LlamaConfig& c = cfg_;
  if (c.vocab <= 0 || c.d_model <= 0 || c.n_heads <= 0 || c.n_kv <= 0 || c.d_head <= 0 || c.d_ff <= 0 ||
      c.n_layers <= 0 || c.T <= 0 || c.B <= 0)
    return -1;
  if (c.n_heads % c.n_kv || c.d_model % 64 || c.d_ff % 64 || c.d_head % 32 || c.vocab % 8) return -1;
  // the materialised score path tiles T x T matrices in 64-wide blocks; the
  // fused attention masks ragged tiles and takes any T
  if (c.T % 64 && !(c.attn_impl == 0 && flash_supported(c.d_head))) return -1;
  if (c.mode == 1 && (c.lora_rank <= 0 || c.lora_rank > kLoraMaxRank || c.lora_targets == 0)) return -1;
  per_head_ = c.mode == 1 && c.lora_per_head_q;
  if (per_head_ && (c.lora_targets != (1 << kLoraQ) || g_q8_base_mode != 1)) return -1;
  moe_ = c.n_experts > 0;
  if (moe_) {
    // QLoRA over frozen experts; adapters on the attention projections only
    const int ffn_bits = (1 << kLoraGate) | (1 << kLoraUp) | (1 << kLoraDown);
    if (c.mode != 1 || per_head_ || c.n_experts > 256 || c.n_experts % 8 || c.n_experts_used < 1 ||
        c.n_experts_used > 16 || c.n_experts_used > c.n_experts || (c.lora_targets & ffn_bits))
      return -1;
  }
  if (c.qk_norm && (c.qk_norm != 2 || c.mode != 1 || c.qkv_bias)) return -1;
  CU(cudaSetDevice(device_));
  // Adapter steps: the activation / activation-gradient chain is the critical
  // path and the second stream carries light work (adapter weight gradients,
  // ring fills), so the chain's stream gets the highest priority and SMs freed
  // by a finishing kernel go to its next kernel first (kernel nodes captured
  // into the step graph keep these). Measured on one B200, SmolLM2 B=8 T=512:
  // QLoRA q,v 267.9k -> 271.1k tokens/s. Full fine-tunes keep equal
  // priorities: their second stream holds the weight-gradient GEMMs, and
  // favouring either stream lengthened the step (222.6k -> 218.6k with the
  // chain first, 221.3k -> 218.5k with the weight gradients first).
  int prio_lo = 0, prio_hi = 0;
  CU(cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi));
  CU(cudaStreamCreateWithPriority(&stream_, cudaStreamNonBlocking, c.mode == 1 ? prio_hi : prio_lo));
  CU(cudaStreamCreateWithPriority(&wst_, cudaStreamNonBlocking, prio_lo));
  err_ = device_error_word();
  if (!err_) return -3;
  const bool full = c.mode == 0;
  const int d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff, V = c.vocab, r = c.lora_rank;
  // Trainable parameters first so the optimiser walks one contiguous range.
  if (full) {
    add_param("token_embd.weight", V, d, true, false);
    if (!c.tied) add_param("output.weight", V, d, true, false);
    add_param("output_norm.weight", 1, d, true, false);
  } else {
    for (int l = 0; l < c.n_layers; ++l)
      for (int t = 0; t < kLoraCount; ++t) {
        if (!(c.lora_targets & (1 << t))) continue;
        const int rows_out = t == kLoraQ ? H * dh : (t == kLoraK || t == kLoraV) ? KV * dh
                             : (t == kLoraO || t == kLoraDown) ? d : ff;
        const int cols_in = t == kLoraO ? H * dh : t == kLoraDown ? ff : d;
        const std::string pre = "blk." + std::to_string(l) + "." + kProjName[t];
        add_param(pre + ".lora_a", (per_head_ && t == kLoraQ) ? H * r : r, cols_in, true, false);
        add_param(pre + ".lora_b", rows_out, r, true, false);
      }
  }
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string pre = "blk." + std::to_string(l) + ".";
    const bool q8 = !full;
    add_param(pre + "attn_norm.weight", 1, d, full, false);
    add_param(pre + "attn_q.weight", H * dh, d, full, q8);   // q | k | v contiguous: one fused GEMM operand
    add_param(pre + "attn_k.weight", KV * dh, d, full, q8);
    add_param(pre + "attn_v.weight", KV * dh, d, full, q8);
    if (c.qkv_bias) {
      add_param(pre + "attn_q.bias", 1, H * dh, full, false);
      add_param(pre + "attn_k.bias", 1, KV * dh, full, false);
      add_param(pre + "attn_v.bias", 1, KV * dh, full, false);
    }
    add_param(pre + "attn_output.weight", d, H * dh, full, q8);
    if (c.qk_norm) {
      add_param(pre + "attn_q_norm.weight", 1, H * dh, false, false);
      add_param(pre + "attn_k_norm.weight", 1, KV * dh, false, false);
    }
    add_param(pre + "ffn_norm.weight", 1, d, full, false);
    if (moe_) {   // router (f32) and the experts stacked, [expert][rows][cols] (GGUF ne = [cols, rows, experts])
      const int E = c.n_experts;
      add_param(pre + "ffn_gate_inp.weight", E, d, false, false);
      add_param(pre + "ffn_gate_exps.weight", E * ff, d, false, true);
      add_param(pre + "ffn_up_exps.weight", E * ff, d, false, true);
      add_param(pre + "ffn_down_exps.weight", E * d, ff, false, true);
      continue;
    }
    add_param(pre + "ffn_gate.weight", ff, d, full, q8);      // gate | up contiguous
    add_param(pre + "ffn_up.weight", ff, d, full, q8);
    add_param(pre + "ffn_down.weight", d, ff, full, q8);
  }
  if (!full) {
    add_param("token_embd.weight", V, d, false, false);
    if (!c.tied) add_param("output.weight", V, d, false, false);
    add_param("output_norm.weight", 1, d, false, false);
  }
  long long off = 0, qoff = 0, qvoff = 0, qsoff = 0;
  for (auto& p : params_) {
    if (p.trainable && off != n_train_) return -1;
    if (p.q8) {
      // frozen Q8_0 projection: only the blocks and their quant / scale split
      p.offset = -1;
      p.q8_offset = qoff;
      qoff += p.numel() / 32 * 34;
      p.q8v_offset = qvoff;
      qvoff += p.numel();
      p.q8s_offset = qsoff;
      qsoff += p.numel() / 32;
      continue;
    }
    p.offset = off;
    off += (p.numel() + 63) / 64 * 64;
    if (p.trainable) n_train_ = off;
  }
  n_total_ = off;
  q8_bytes_ = qoff;
  // Q8_0 base as ring planes: the four group operands of a block, each with
  // 64 extra reduction columns / rows when its adapters are folded in
  q8_planes_ = q8_bytes_ && g_q8_base_mode == 1 && !moe_;   // expert blocks dequantise inside their GEMMs
  for (auto& p : params_) {
    if (!p.q8) continue;
    p.layer = std::atoi(p.name.c_str() + 4);
    if (p.name.compare(0, 4, "blk.") != 0 || p.layer < 0 || p.layer >= c.n_layers) return -1;
    static const char* kFirst[4] = {"attn_q.weight", "attn_output.weight", "ffn_gate.weight", "ffn_down.weight"};
    const size_t dot = p.name.find('.', 4);
    for (int g = 0; g < 4; ++g)
      if (dot != std::string::npos && p.name.compare(dot + 1, std::string::npos, kFirst[g]) == 0) p.ring_group = g;
  }
  if (q8_planes_) {
    const int dims[4][2] = {{(H + 2 * KV) * dh, d}, {d, H * dh}, {2 * ff, d}, {d, ff}};
    long long slot = 0;
    for (int g = 0; g < 4; ++g) {
      RingGroup& rg = ring_[g];
      rg.d_out = dims[g][0];
      rg.d_in = dims[g][1];
      if (rg.d_in % 16) return -1;
      const LoraGroup G = lora_group(g);
      const bool fold = G.n && lora_grouped(rg.d_in);
      rg.ext = fold ? 64 : 0;
      if (per_head_ && g == kGroupQKV) rg.ext = (H * r + 63) / 64 * 64;   // the H r columns of u
      ext_[g] = rg.ext;
      rg.off = slot;
      slot += ((long long)(rg.d_out + rg.ext) * (rg.d_in + rg.ext) + 127) / 128 * 128;
      ring_chunks_ += (long long)(rg.d_out + rg.ext) * (rg.d_in + rg.ext) / 16;
    }
    q8_slot_elems_ = slot;
  }
  o_ld_ = (long long)H * dh + ext_[kGroupO];
  a_ld_ = (long long)ff + ext_[kGroupDown];
  dxp_ld_ = (long long)d + std::max(ext_[kGroupO], ext_[kGroupDown]);
  layer_grad_lo_.assign(c.n_layers, n_train_);
  for (const auto& p : params_) {
    if (!p.trainable || p.name.compare(0, 4, "blk.") != 0) continue;
    const int l = std::atoi(p.name.c_str() + 4);
    if (l >= 0 && l < c.n_layers) layer_grad_lo_[l] = std::min(layer_grad_lo_[l], p.offset);
  }
  // fused operands must be contiguous
  auto follows = [](const Param& a, const Param& b) {   // b stored right after a
    return a.q8 ? (b.q8v_offset == a.q8v_offset + a.numel() && b.q8s_offset == a.q8s_offset + a.numel() / 32)
                : b.offset == a.offset + a.numel();
  };
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string pre = "blk." + std::to_string(l) + ".";
    if (!follows(P(pre + "attn_q.weight"), P(pre + "attn_k.weight"))) return -1;
    if (!follows(P(pre + "attn_k.weight"), P(pre + "attn_v.weight"))) return -1;
    if (!moe_ && !follows(P(pre + "ffn_gate.weight"), P(pre + "ffn_up.weight"))) return -1;
  }
  CK(alloc(p32_, n_total_ * 4));
  CK(alloc(phi_, n_total_ * 2));
  CK(alloc(plo_, n_total_ * 2));
  CK(alloc(g_, std::max<long long>(n_train_, 64) * 4));
  CK(alloc(m_, std::max<long long>(n_train_, 64) * 4));
  CK(alloc(v_, std::max<long long>(n_train_, 64) * 4));
  if (q8_bytes_) {
    CK(alloc(q8_, q8_bytes_));
    CK(alloc(q8v_, qvoff));
    CK(alloc(q8s_, qsoff * 2));
    if (q8_planes_) {
      CK(alloc(q8pl_, q8_slot_elems_ * 2 * 2 * 2));   // 2 slots x (hi, lo) x bf16
      CK(build_ring(qvoff));
      // keep the ring in the L2's persisting set-aside: its planes are written
      // and read with the evict-last policy, so they stay on chip between the
      // fill and the GEMMs that read them instead of being written back to HBM
      if (g_ring_l2 && l2_keep_acquire((size_t)q8pl_.bytes)) {
        ring_keep_ = true;
        for (RingLayer& L : ring_desc_) L.keep = 1;
      }
    }
  }

  const int N = this->N(), T = c.T, B = c.B, W = (H + 2 * KV) * dh;
  // adapter weight gradients on tensor cores for the wide layers of 1B+ models
  wg_tc_ = !full && !per_head_ && r <= 16 && std::max(std::max(d, H * dh), ff) >= kWgTcMinWidth;
  if (full || per_head_ || wg_tc_) {   // split-K workspace of the weight-gradient GEMMs on wst_
    wsc_.ws_floats = gemm_scratch().ws_floats;
    CK(alloc(wsc_ws_, (size_t)wsc_.ws_floats * sizeof(float)));
    wsc_.ws = static_cast<float*>(wsc_ws_.p);
  }
  auto f32 = [&](long long n) -> float* {
    bufs_.emplace_back();
    if (alloc(bufs_.back(), n * 4)) return nullptr;
    return static_cast<float*>(bufs_.back().p);
  };
  auto pl = [&](long long n) -> Planes {   // hi and lo planes, each padded to 128 elements
    const long long np = (n + 127) / 128 * 128;
    bufs_.emplace_back();
    if (alloc(bufs_.back(), np * 4)) return Planes{};
    bf16* base = static_cast<bf16*>(bufs_.back().p);
    return Planes{base, base + np};
  };
  const long long att = (long long)B * H * T * T;
  flash_ = c.attn_impl == 0 && flash_supported(dh);
  for (int l = 0; l <= c.n_layers; ++l) x_.push_back(f32((long long)N * d));
  lora_u_.resize(c.n_layers);
  lora_bt_.resize(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    x1_.push_back(f32((long long)N * d));
    gu_.push_back(moe_ ? nullptr : f32((long long)N * 2 * ff));
    h1_.push_back(pl((long long)N * (d + ext_[kGroupQKV])));   // + the q|k|v adapters' u columns
    h2_.push_back(pl((long long)N * (d + ext_[kGroupGU])));    // + the gate|up adapters' u columns
    a_.push_back(moe_ ? Planes{} : pl((long long)N * a_ld_));   // + the down adapters' u columns
    Qh_.push_back(pl((long long)N * H * dh));
    Kh_.push_back(pl((long long)N * KV * dh));
    Vh_.push_back(pl((long long)N * KV * dh));
    Pm_.push_back(flash_ ? Planes{} : pl(att));
    lse2_.push_back(flash_ ? f32((long long)B * H * T) : nullptr);
    O_.push_back(pl((long long)N * o_ld_));   // + the o adapters' u columns
    lora_u_[l].assign(kLoraCount, nullptr);
    lora_bt_[l].assign(kLoraCount, nullptr);
    for (int t = 0; t < kLoraCount; ++t)
      if (!full && (c.lora_targets & (1 << t))) {
        lora_u_[l][t] = f32((long long)N * r);
        lora_bt_[l][t] = f32((long long)r * std::max(std::max(d, ff), H * dh));
      }
  }
  qkv_ = f32((long long)N * W);
  if (c.qk_norm)
    for (int l = 0; l < c.n_layers; ++l) qkpre_.push_back(f32((long long)N * (H + KV) * dh));
  if (moe_) {
    const int E = c.n_experts, K = c.n_experts_used;
    const long long NK = (long long)N * K;
    moe_l_.resize(c.n_layers);
    for (auto& M : moe_l_) {
      M.probs = f32((long long)N * E);
      M.w = f32(NK);
      M.idx = reinterpret_cast<int*>(f32(NK));
      M.perm = reinterpret_cast<int*>(f32(NK));
      M.pos = reinterpret_cast<int*>(f32(NK));
      M.gu = f32(NK * 2 * ff);
      M.a = pl(NK * ff);
      M.ye = f32(NK * d);
      M.gtab = reinterpret_cast<int*>(f32(3 * (NK / 128 + E + 1)));
    }
    moe_logits_ = f32((long long)N * E);
    moe_xs_ = pl(NK * d);
    moe_dye_ = pl(NK * d);
    moe_das_ = f32(NK * ff);
    moe_dgu_ = pl(NK * 2 * ff);
    moe_dxs_ = f32(NK * d);
    moe_dw_ = f32(NK);
    moe_dlog_ = pl((long long)N * E);
    moe_hidx_.resize(NK);
    moe_hperm_.resize(NK);
    moe_hpos_.resize(NK);
    use_graph_ = false;   // host round trip per block: eager steps
  }
  if (!flash_) S_ = f32(att);
  logits_ = f32((long long)N * V);
  loss_rows_ = f32(N);
  loss_ = f32(64);
  dx_ = f32((long long)N * d);
  dh_ = f32((long long)N * d);
  da_ = f32((long long)N * ff);
  dO32_ = f32((long long)N * H * dh);
  if (!flash_) {
    dQ_ = f32((long long)N * H * dh);
    dK_ = f32((long long)N * KV * dh);
    dV_ = f32((long long)N * KV * dh);
  } else {
    dvec_ = f32((long long)B * H * T);
    fws_ = f32(flash_bwd_ws_floats(B, T, H, KV, dh));
  }
  for (int k = 0; k < 2; ++k) gpart2_[k] = f32((long long)rmsnorm_bwd_blocks() * d);
  gpart_ = gpart2_[0];
  xf_ = pl((long long)N * d);
  dlog_ = pl((long long)N * V);
  lse_part_ = reinterpret_cast<float2*>(f32(2LL * ((V + 63) / 64) * N));
  lse_ms_ = reinterpret_cast<float2*>(f32(2LL * N));
  for (int k = 0; k < 2; ++k) {   // two copies of each transient the weight-gradient stream reads
    dxp2_[k] = pl((long long)N * dxp_ld_);   // + du of the o / down adapters
    dgu2_[k] = pl((long long)N * (2 * ff + ext_[kGroupGU]));
    dqkv2_[k] = pl((long long)N * (W + ext_[kGroupQKV]));
  }
  dxp_ = dxp2_[0];
  dgu_ = dgu2_[0];
  dqkv_ = dqkv2_[0];
  // fp16 copies of the weight-gradient operands (full fine-tune on the fused
  // attention, dense FFN): every activation operand in place, the gradients
  // scaled per tensor (slots: 4 per layer + the logits' gradient)
  f16w_ = full && flash_ && !moe_ && g_f16_wgrad;
  f16w_ready_ = false;
  if (f16w_) {
    auto h16 = [&](long long n) -> __half* {
      bufs_.emplace_back();
      if (alloc(bufs_.back(), ((n + 127) / 128 * 128) * 2)) return nullptr;
      return static_cast<__half*>(bufs_.back().p);
    };
    for (int l = 0; l < c.n_layers; ++l) {
      h1_[l].f16 = h16((long long)N * d);
      h2_[l].f16 = h16((long long)N * d);
      a_[l].f16 = h16((long long)N * a_ld_);
      O_[l].f16 = h16((long long)N * o_ld_);
    }
    xf_.f16 = h16((long long)N * d);
    dlog_.f16 = h16((long long)N * V);
    for (int k = 0; k < 2; ++k) {
      dxp2_[k].f16 = h16((long long)N * dxp_ld_);
      dgu2_[k].f16 = h16((long long)N * (2 * ff + ext_[kGroupGU]));
      dqkv2_[k].f16 = h16((long long)N * (W + ext_[kGroupQKV]));
    }
    n16_ = 4 * c.n_layers;
    amax16_ = reinterpret_cast<unsigned*>(f32(n16_ + 1));
    scale16_ = f32(n16_ + 1);
    inv16_ = f32(n16_ + 1);
    // |dlogits| <= 1 / N: a static scale 2^(14 + floor(log2 N)) keeps them <= 2^14
    const int e = 14 + (int)std::floor(std::log2((double)N));
    std::vector<float> sc(n16_ + 1, 1.0f), iv(n16_ + 1, 1.0f);
    sc[n16_] = std::ldexp(1.0f, e);
    iv[n16_] = std::ldexp(1.0f, -e);
    CU(cudaMemcpy(scale16_, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(inv16_, iv.data(), iv.size() * 4, cudaMemcpyHostToDevice));
    CU(cudaMemset(amax16_, 0, (n16_ + 1) * 4));
    dlog_.f16_scale = scale16_ + n16_;
  }
  dO_ = pl((long long)N * H * dh);
  if (!flash_) dS_ = pl(att);
  if (!full) {
    for (int k = 0; k < 2; ++k) du2_[k] = f32((long long)kLoraMaxSegs * N * r);   // du of each adapter of a group
    du32_ = du2_[0];
    long long part = std::max(lora_wgrad_partial_floats(N, std::max(std::max(d, ff), H * dh), r),
                              lora_bwd_partial_floats(N, std::max(ff, H * dh), d, r));
    if (r <= 16) {
      part = std::max(part, lora_group_partial_floats(N, r, d, W, 3));             // q|k|v
      part = std::max(part, lora_group_partial_floats(N, r, d, 2 * ff, 2));        // gate|up
      part = std::max(part, lora_group_partial_floats(N, r, H * dh, d, 1));        // o
      part = std::max(part, lora_group_partial_floats(N, r, ff, d, 1));            // down
    }
    lora_part_ = f32(part);
    lora_part2_ = f32(part);
  }
  if (per_head_) bd_dense_ = f32((long long)H * dh * H * r);
  if (wg_tc_) {
    wg_ubp_ = pl((long long)N * kWgTcCols);
    wg_dubp_ = pl((long long)N * kWgTcCols);
    wg_da_ = f32((long long)std::max(std::max(d, H * dh), ff) * kWgTcCols);
    wg_db_ = f32((long long)std::max(std::max(W, 2 * ff), d) * kWgTcCols);
    wg_u_ = f32((long long)N * kWgTcCols);
    wg_wp_ = pl((long long)kWgTcCols * std::max(std::max(std::max(d, H * dh), ff), std::max(std::max(W, 2 * ff), d)));
  }
  hp_ = f32(8);
  bufs_.emplace_back();
  CK(alloc(bufs_.back(), (size_t)N * 4 * 5 + 64));
  int* ib = static_cast<int*>(bufs_.back().p);
  ids_ = ib; pos_ = ib + N; labels_ = ib + 2 * N; ord_ = ib + 3 * N; seg_id_ = ib + 4 * N;
  bufs_.emplace_back();
  CK(alloc(bufs_.back(), (size_t)(N + 2) * 4));
  seg_start_ = static_cast<int*>(bufs_.back().p);
  nseg_dev_ = seg_start_ + N + 1;
  for (const auto& b : bufs_)
    if (!b.p) return -3;
  // RoPE cos/sin table, ggml's rope cache: theta starts at float(pos), times
  // theta_scale = powf(base, -2/n_dims) per pair, divided by the freq factor.
  cs_rows_ = std::max(T, 4096);
  const int half = dh / 2;
  std::vector<float> tab((size_t)cs_rows_ * half * 2);
  const float ts = powf(c.rope_base, -2.0f / (float)dh);
  for (int p = 0; p < cs_rows_; ++p) {
    float theta = (float)p;
    for (int i = 0; i < half; ++i) {
      const float f = c.freq_factors.empty() ? 1.0f : c.freq_factors[i];
      const float th = c.freq_scale * (theta / f);
      tab[((size_t)p * half + i) * 2] = (float)std::cos((double)th);
      tab[((size_t)p * half + i) * 2 + 1] = (float)std::sin((double)th);
      theta = theta * ts;
    }
  }
  cs_ = f32((long long)cs_rows_ * half * 2);
  if (!cs_) return -3;
  CU(cudaMemcpyAsync(cs_, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, stream_));
  // default ids/positions: 0 and 0..T-1
  std::vector<long long> pos0(N);
  for (int i = 0; i < N; ++i) pos0[i] = i % T;
  realized_ = true;
  CK(set_positions(pos0.data(), N));
  std::vector<long long> z(N, 0);
  CK(set_tokens(z.data(), N));
  CK(set_label_ids(z.data(), N));
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

int LlamaEngine::staged(size_t bytes) {
  if (bytes <= stage_bytes_) return 0;
  if (stage_) {
    cudaStreamSynchronize(stream_);
    cudaFreeHost(stage_);
  }
  stage_bytes_ = std::max(bytes, (size_t)1 << 20);
  if (cudaMallocHost(&stage_, stage_bytes_) != cudaSuccess) {
    stage_ = nullptr;
    stage_bytes_ = 0;
    return -3;
  }
  return 0;
}

int LlamaEngine::refresh_planes(const Param& p) {
  return launch_split_f32(P32(p), PP(p).hi, PP(p).lo, p.numel(), stream_);
}

int LlamaEngine::set_param(const std::string& name, const float* host, long long n) {
  const Param* p = find(name);
  if (!p || !host) return -1;
  if (n != p->numel()) return -1;
  // Stream-ordered copy: a plain cudaMemcpy from pageable memory may return
  // before its DMA lands, and stream_ does not order against the legacy stream.
  CU(cudaStreamSynchronize(stream_));
  if (p->q8) {
    // quantise through a temporary f32 copy; only the Q8_0 data is kept
    float* tmp = nullptr;
    CU(cudaMalloc(&tmp, n * 4));
    int rc = cudaMemcpyAsync(tmp, host, n * 4, cudaMemcpyHostToDevice, stream_) == cudaSuccess ? 0 : -3;
    if (!rc) rc = launch_q8_0_quantize(tmp, static_cast<uint8_t*>(q8_.p) + p->q8_offset, p->rows, p->cols, stream_);
    if (!rc) rc = split_q8(*p);
    if (cudaStreamSynchronize(stream_) != cudaSuccess && !rc) rc = -3;
    cudaFree(tmp);
    return rc;
  }
  CU(cudaMemcpyAsync(P32(*p), host, n * 4, cudaMemcpyHostToDevice, stream_));
  CK(refresh_planes(*p));
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

int LlamaEngine::split_q8(const Param& p) {
  return launch_q8_0_split(static_cast<const uint8_t*>(q8_.p) + p.q8_offset,
                           static_cast<int8_t*>(q8v_.p) + p.q8v_offset,
                           static_cast<uint16_t*>(q8s_.p) + p.q8s_offset, p.numel() / 32, stream_);
}

Operand LlamaEngine::wop(const Param& p, int rows, int cols, long long ld, int mn) {
  if (!p.q8) return op(PP(p), rows, cols, ld, mn);
  if (q8_planes_) {
    // the ring slot dequant_layer filled for this block (a null operand, which
    // the GEMM rejects, if the step program did not fill it first); the
    // group's extra reduction width extends K: columns of the rows (forward)
    // or rows of the MN-major read (dX)
    const int slot = p.layer & 1;
    if (p.ring_group < 0 || ring_layer_[slot] != p.layer) return op(Planes{}, rows, cols, ld, mn);
    const RingGroup& rg = ring_[p.ring_group];
    bf16* base = static_cast<bf16*>(q8pl_.p) + (long long)slot * 2 * q8_slot_elems_ + rg.off;
    const Planes pl{base, base + q8_slot_elems_};
    const int e = rg.ext;
    Operand o = mn ? op(pl, rows + e, cols, rg.d_in + e, 1) : op(pl, rows, cols + e, rg.d_in + e, 0);
    o.l2_keep = ring_keep_;
    return o;
  }
  Operand o = op(Planes{}, rows, cols, ld, mn);
  o.q8 = static_cast<const int8_t*>(q8v_.p) + p.q8v_offset;
  o.q8_scale = static_cast<const uint16_t*>(q8s_.p) + p.q8s_offset;
  return o;
}

Planes LlamaEngine::ring_ext_b(int l) const {
  const int slot = l & 1;
  if (!q8_planes_ || ring_layer_[slot] != l) return Planes{};
  const RingGroup& rg = ring_[kGroupQKV];
  bf16* base = static_cast<bf16*>(q8pl_.p) + (long long)slot * 2 * q8_slot_elems_ + rg.off + rg.d_in;
  return Planes{base, base + q8_slot_elems_};
}

int LlamaEngine::set_param_q8(const std::string& name, const uint8_t* blocks, long long nbytes) {
  const Param* p = find(name);
  if (!p || !p->q8 || !blocks || nbytes != p->numel() / 32 * 34) return -1;
  CU(cudaStreamSynchronize(stream_));
  uint8_t* dst = static_cast<uint8_t*>(q8_.p) + p->q8_offset;
  CU(cudaMemcpyAsync(dst, blocks, nbytes, cudaMemcpyHostToDevice, stream_));
  CK(split_q8(*p));
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

int LlamaEngine::get_param_q8(const std::string& name, uint8_t* blocks, long long nbytes) {
  const Param* p = find(name);
  if (!p || !p->q8 || !blocks || nbytes != p->numel() / 32 * 34) return -1;
  CU(cudaStreamSynchronize(stream_));
  CU(cudaMemcpy(blocks, static_cast<uint8_t*>(q8_.p) + p->q8_offset, nbytes, cudaMemcpyDeviceToHost));
  return 0;
}

int LlamaEngine::get_param(const std::string& name, float* host, long long n) {
  const Param* p = find(name);
  if (!p || !host || n != p->numel()) return -1;
  CU(cudaStreamSynchronize(stream_));
  if (p->q8) {   // dequantise the blocks on the host: value = fp16 scale * int8 quant
    std::vector<uint8_t> blk((size_t)(n / 32 * 34));
    CU(cudaMemcpy(blk.data(), static_cast<uint8_t*>(q8_.p) + p->q8_offset, blk.size(), cudaMemcpyDeviceToHost));
    for (long long b = 0; b < n / 32; ++b) {
      const uint8_t* q = blk.data() + b * 34;
      __half_raw hr;
      hr.x = (unsigned short)(q[0] | (q[1] << 8));
      const float dsc = __half2float(__half(hr));
      for (int j = 0; j < 32; ++j) host[b * 32 + j] = dsc * (float)(int8_t)q[2 + j];
    }
    return 0;
  }
  CU(cudaMemcpy(host, P32(*p), n * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int LlamaEngine::get_grad(const std::string& name, float* host, long long n) {
  const Param* p = find(name);
  if (!p || !host || n != p->numel() || !p->trainable) return -1;
  CU(cudaStreamSynchronize(stream_));
  CU(cudaMemcpy(host, G32(*p), n * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int LlamaEngine::get_moment(const std::string& name, int which, float* host, long long n) {
  const Param* p = find(name);
  if (!p || !host || n != p->numel() || !p->trainable) return -1;
  CU(cudaStreamSynchronize(stream_));
  const float* src = static_cast<float*>(which == 0 ? m_.p : v_.p) + p->offset;
  CU(cudaMemcpy(host, src, n * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int LlamaEngine::set_moment(const std::string& name, int which, const float* host, long long n) {
  const Param* p = find(name);
  if (!p || !host || n != p->numel() || !p->trainable || which < 0 || which > 1) return -1;
  CU(cudaStreamSynchronize(stream_));
  float* dst = static_cast<float*>(which == 0 ? m_.p : v_.p) + p->offset;
  CU(cudaMemcpyAsync(dst, host, n * 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

// Seeded init in the reference's draw order (upload_random_init!,
// llama_seq_engine.rb:1161-1340); std_all > 0 replaces every std (the synthetic
// N(0, std) frozen base of the QLoRA configs, then quantised to Q8_0); LoRA
// adapters follow from the same stream, per layer and target, A then B.
int LlamaEngine::init_random(long long seed, double init_scale, double std_all, double lora_a_std,
                             double lora_b_std) {
  if (!realized_) return -2;
  const LlamaConfig& c = cfg_;
  const int d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff, V = c.vocab;
  const bool all = std_all > 0.0;
  const double s_emb = all ? std_all : 0.02;
  const double s_d = all ? std_all : init_scale / std::sqrt((double)d);
  const double s_ff = all ? std_all : init_scale / std::sqrt((double)ff);
  uint64_t st = lcg_seed_state(seed);
  std::vector<float> buf;
  auto fill = [&](const std::string& name, double stdv) -> int {
    const Param& p = P(name);
    buf.resize(p.numel());
    st = gaussian_fill(st, buf.data(), p.numel(), stdv);
    return set_param(name, buf.data(), p.numel());
  };
  auto ones = [&](const std::string& name) -> int {
    const Param& p = P(name);
    buf.assign(p.numel(), 1.0f);
    return set_param(name, buf.data(), p.numel());
  };
  CK(fill("token_embd.weight", s_emb));
  CK(ones("output_norm.weight"));
  if (!c.tied) CK(fill("output.weight", s_emb));
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string pre = "blk." + std::to_string(l) + ".";
    CK(ones(pre + "attn_norm.weight"));
    CK(ones(pre + "ffn_norm.weight"));
    // per-head draws, stored into the fused row blocks
    std::vector<float> wq((size_t)H * dh * d), wk((size_t)KV * dh * d), wv((size_t)KV * dh * d);
    for (int h = 0; h < H; ++h) st = gaussian_fill(st, wq.data() + (size_t)h * dh * d, (long long)dh * d, s_d);
    for (int j = 0; j < KV; ++j) {
      st = gaussian_fill(st, wk.data() + (size_t)j * dh * d, (long long)dh * d, s_d);
      st = gaussian_fill(st, wv.data() + (size_t)j * dh * d, (long long)dh * d, s_d);
    }
    CK(set_param(pre + "attn_q.weight", wq.data(), (long long)wq.size()));
    CK(set_param(pre + "attn_k.weight", wk.data(), (long long)wk.size()));
    CK(set_param(pre + "attn_v.weight", wv.data(), (long long)wv.size()));
    CK(fill(pre + "attn_output.weight", s_d));
    if (moe_) {   // router, then the stacked experts' gate, up and down
      CK(fill(pre + "ffn_gate_inp.weight", s_emb));
      CK(fill(pre + "ffn_gate_exps.weight", s_d));
      CK(fill(pre + "ffn_up_exps.weight", s_d));
      CK(fill(pre + "ffn_down_exps.weight", s_ff));
    } else {
      CK(fill(pre + "ffn_gate.weight", s_d));
      CK(fill(pre + "ffn_up.weight", s_d));
      CK(fill(pre + "ffn_down.weight", s_ff));
    }
    if (c.qk_norm) {
      CK(ones(pre + "attn_q_norm.weight"));
      CK(ones(pre + "attn_k_norm.weight"));
    }
    if (c.qkv_bias) {
      const double sb = all ? std_all : 0.02;
      CK(fill(pre + "attn_q.bias", sb));
      CK(fill(pre + "attn_k.bias", sb));
      CK(fill(pre + "attn_v.bias", sb));
    }
  }
  if (per_head_) {
    // upload_lora_q_init! (llama_seq_engine.rb:2545-2575): the raw seed drives
    // the LCG (no fold, no warm-up), two draws per A element, cos branch only,
    // A = init_scale N(0, 1) (init_scale arrives as lora_a_std), every B_h = 0
    const int r = c.lora_rank;
    uint64_t s = (uint64_t)seed & kMask;
    for (int l = 0; l < c.n_layers; ++l) {
      const std::string pre = "blk." + std::to_string(l) + ".attn_q";
      std::vector<float> A((size_t)H * r * d), Bz((size_t)H * dh * r, 0.0f);
      for (size_t i = 0; i < A.size(); ++i) {
        s = lcg_next(s);
        const double u1 = ((double)s + 1.0) / 2147483648.0;
        s = lcg_next(s);
        const double u2 = ((double)s + 1.0) / 2147483648.0;
        A[i] = (float)(lora_a_std * std::sqrt(-2.0 * std::log(u1)) * std::cos(2.0 * M_PI * u2));
      }
      CK(set_param(pre + ".lora_a", A.data(), (long long)A.size()));
      CK(set_param(pre + ".lora_b", Bz.data(), (long long)Bz.size()));
    }
  } else if (c.mode == 1) {
    for (int l = 0; l < c.n_layers; ++l)
      for (int t = 0; t < kLoraCount; ++t) {
        if (!(c.lora_targets & (1 << t))) continue;
        const std::string pre = "blk." + std::to_string(l) + "." + kProjName[t];
        CK(fill(pre + ".lora_a", lora_a_std));
        CK(fill(pre + ".lora_b", lora_b_std));
      }
  }
  (void)V;
  return 0;
}

// ------------------------------------------------------------------ inputs
int LlamaEngine::set_tokens(const long long* ids, int n) {
  if (!realized_ || !ids || n != N()) return -1;
  const int V = cfg_.vocab;
  CK(staged((size_t)n * 4 * 4 + 64));
  int* h = static_cast<int*>(stage_);   // ids | order | seg ids | seg starts (+ count)
  CU(cudaStreamSynchronize(stream_));
  for (int i = 0; i < n; ++i) {
    if (ids[i] < 0 || ids[i] >= V) return -1;
    h[i] = (int)ids[i];
  }
  // rows grouped by id, in row order within an id (the deterministic
  // embedding scatter-add): a stable LSD radix sort of the row indices by id,
  // one pass per byte of the largest id (linear in n)
  int* ord = h + n;
  int* sid = h + 2 * n;
  int* sst = h + 3 * n;
  {
    std::vector<int>& tmp = sort_tmp_;
    tmp.resize(n);
    for (int i = 0; i < n; ++i) ord[i] = i;
    int* src = ord;
    int* dst = tmp.data();
    for (int shift = 0; shift < 32 && (shift == 0 || (V - 1) >> shift); shift += 8) {
      int count[257] = {0};
      for (int i = 0; i < n; ++i) ++count[((h[src[i]] >> shift) & 255) + 1];
      for (int d = 0; d < 256; ++d) count[d + 1] += count[d];
      for (int i = 0; i < n; ++i) dst[count[(h[src[i]] >> shift) & 255]++] = src[i];
      std::swap(src, dst);
    }
    if (src != ord) std::copy(src, src + n, ord);
  }
  int ns = 0;
  for (int i = 0; i < n; ++i) {
    const int id = h[ord[i]];
    if (i == 0 || id != h[ord[i - 1]]) {
      sid[ns] = id;
      sst[ns] = i;
      ++ns;
    }
  }
  sst[ns] = n;
  nseg_ = ns;
  CU(cudaMemcpyAsync(ids_, h, (size_t)n * 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaMemcpyAsync(ord_, ord, (size_t)n * 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaMemcpyAsync(seg_id_, sid, (size_t)ns * 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaMemcpyAsync(seg_start_, sst, (size_t)(ns + 1) * 4, cudaMemcpyHostToDevice, stream_));
  sst[ns + 1] = ns;
  CU(cudaMemcpyAsync(nseg_dev_, sst + ns + 1, 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

int LlamaEngine::set_positions(const long long* pos, int n) {
  if (!realized_ || !pos || n != N()) return -1;
  CK(staged((size_t)n * 4));
  CU(cudaStreamSynchronize(stream_));
  int* h = static_cast<int*>(stage_);
  for (int i = 0; i < n; ++i) {
    if (pos[i] < 0 || pos[i] >= cs_rows_) return -1;
    h[i] = (int)pos[i];
  }
  CU(cudaMemcpyAsync(pos_, h, (size_t)n * 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

int LlamaEngine::set_label_ids(const long long* ids, int n) {
  if (!realized_ || !ids || n != N()) return -1;
  CK(staged((size_t)n * 4));
  CU(cudaStreamSynchronize(stream_));
  int* h = static_cast<int*>(stage_);
  for (int i = 0; i < n; ++i) h[i] = (ids[i] >= 0 && ids[i] < cfg_.vocab) ? (int)ids[i] : -1;
  CU(cudaMemcpyAsync(labels_, h, (size_t)n * 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaStreamSynchronize(stream_));
  dense_labels_ = false;
  return 0;
}

int LlamaEngine::set_labels_dense(const double* lab, long long n) {
  const long long want = (long long)N() * cfg_.vocab;
  if (!realized_ || !lab || n != want) return -1;
  if (!labels_dense_) {
    bufs_.emplace_back();
    CK(alloc(bufs_.back(), (size_t)want * 4));
    labels_dense_ = static_cast<float*>(bufs_.back().p);
  }
  const long long chunk = 4 << 20;
  CK(staged((size_t)chunk * 4));
  float* h = static_cast<float*>(stage_);
  for (long long o = 0; o < want; o += chunk) {
    const long long k = std::min(chunk, want - o);
    CU(cudaStreamSynchronize(stream_));
    for (long long i = 0; i < k; ++i) h[i] = (float)lab[o + i];
    CU(cudaMemcpyAsync(labels_dense_ + o, h, (size_t)k * 4, cudaMemcpyHostToDevice, stream_));
  }
  CU(cudaStreamSynchronize(stream_));
  dense_labels_ = true;
  return 0;
}

int LlamaEngine::set_hp(const double* hp, int n) {
  if (!realized_ || !hp || n != 7) return -1;
  CK(staged(64));
  CU(cudaStreamSynchronize(stream_));
  float* h = static_cast<float*>(stage_);
  for (int i = 0; i < 7; ++i) h[i] = (float)hp[i];
  CU(cudaMemcpyAsync(hp_, h, 7 * 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

// ------------------------------------------------------------------ step program
void LlamaEngine::prof_begin(int kind, double flops) {
  while (evpool_.size() < evnext_ + 2) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    evpool_.push_back(e);
  }
  cur_kind_ = kind;
  cur_flops_ = flops;
  cudaEventRecord(evpool_[evnext_], stream_);
}

void LlamaEngine::prof_end() {
  cudaEventRecord(evpool_[evnext_ + 1], stream_);
  recs_.push_back(Rec{cur_kind_, cur_flops_, evpool_[evnext_], evpool_[evnext_ + 1]});
  evnext_ += 2;
}

int LlamaEngine::gemm(const GemmDesc& d0) {
  if (profiling_) prof_begin(kKGemm, 2.0 * d0.M * d0.N * d0.K * d0.batch);
  GemmDesc d = d0;
  d.alone = d0.alone || (gemm_alone_ && g_plan_alone);
  const int rc = gemm_launch(d, gemm_scratch(), err_, stream_);
  counting_ += gemm_last_launches();
  if (profiling_) prof_end();
  if (rc) fprintf(stderr, "[toy_b200] gemm launch rejected (%d): M=%d N=%d K=%d batch=%d\n", rc, d.M, d.N, d.K, d.batch);
  return rc;
}

int LlamaEngine::gemm_side(const GemmDesc& d0) {
  if (!side_ || !wsc_.ws) return gemm(d0);
  GemmDesc d = d0;
  d.max_ctas = g_side_gemm_ctas > 0 ? g_side_gemm_ctas : (f16w_ ? 100 : 0);
  d.tile_bn = g_side_gemm_bn;
  const int rc = gemm_launch(d, wsc_.ws ? wsc_ : gemm_scratch(), err_, wst_);
  counting_ += gemm_last_launches();
  if (rc) fprintf(stderr, "[toy_b200] gemm launch rejected (%d): M=%d N=%d K=%d batch=%d\n", rc, d.M, d.N, d.K, d.batch);
  return rc;
}

cudaEvent_t LlamaEngine::next_event() {
  if (sev_next_ == sev_.size()) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    sev_.push_back(e);
  }
  return sev_[sev_next_++];
}

int LlamaEngine::fork_side() {
  if (!side_) return 0;
  cudaEvent_t e = next_event();
  if (!e) return -3;
  CU(cudaEventRecord(e, stream_));
  CU(cudaStreamWaitEvent(wst_, e, 0));
  side_forked_ = true;
  return 0;
}

int LlamaEngine::side_read2(Transient& a, Transient& b) {
  if (!side_) return 0;
  cudaEvent_t e = next_event();
  if (!e) return -3;
  CU(cudaEventRecord(e, wst_));
  a.busy[a.cur] = e;
  b.busy[b.cur] = e;
  return 0;
}

int LlamaEngine::side_read(Transient& t) { return side_read2(t, t); }

int LlamaEngine::flip(Transient& t) {
  t.cur ^= 1;
  if (t.busy[t.cur]) {
    CU(cudaStreamWaitEvent(stream_, t.busy[t.cur], 0));
    t.busy[t.cur] = nullptr;
  }
  return 0;
}

int LlamaEngine::join_side() {
  if (!side_ || !side_forked_) return 0;
  side_forked_ = false;
  cudaEvent_t e = next_event();
  if (!e) return -3;
  CU(cudaEventRecord(e, wst_));
  CU(cudaStreamWaitEvent(stream_, e, 0));
  return 0;
}

namespace {
int kind_of(const char* call) {
  static const struct { const char* prefix; int kind; } table[] = {
      {"launch_rmsnorm_fwd", LlamaEngine::kKRmsFwd}, {"launch_rmsnorm_bwd", LlamaEngine::kKRmsBwd},
      {"launch_colsum", LlamaEngine::kKColsum},      {"launch_rope", LlamaEngine::kKRope},
      {"launch_softmax", LlamaEngine::kKSoftmax},    {"launch_swiglu", LlamaEngine::kKSwiglu},
      {"launch_cross_entropy", LlamaEngine::kKCe},   {"launch_loss_reduce", LlamaEngine::kKLoss},
      {"launch_adamw", LlamaEngine::kKAdamw},        {"launch_embed", LlamaEngine::kKEmbed},
      {"launch_split", LlamaEngine::kKSplit},        {"launch_q8_0_ring", LlamaEngine::kKSplit},        {"launch_flash_fwd", LlamaEngine::kKFlashFwd},
      {"launch_flash_bwd_prep", LlamaEngine::kKFlashPrep}, {"launch_flash_bwd", LlamaEngine::kKFlashBwd},
      {"launch_flash_rope", LlamaEngine::kKRope},   {"launch_lora", LlamaEngine::kKLora},
      {"launch_moe", LlamaEngine::kKSwiglu},         {"launch_rms_cols", LlamaEngine::kKRmsFwd}};
  for (const auto& t : table)
    if (strncmp(call, t.prefix, strlen(t.prefix)) == 0) return t.kind;
  return LlamaEngine::kKCount;
}
}  // namespace

// Every non-GEMM launch of the step program goes through KL: it counts the
// launch and, in a profiled step, brackets it with an event pair.
#define KL(x)                                      \
  do {                                             \
    ++counting_;                                   \
    if (profiling_) prof_begin(kind_of(#x), 0.0);  \
    const int rc_k = (x);                          \
    if (profiling_) prof_end();                    \
    if (rc_k) return rc_k;                         \
  } while (0)

// u = X A^T [N][r] (saved for the backward) and B^T [r][d_out] of adapter
// (l, t), ahead of the base GEMM that splices s u B^T into its output.
int LlamaEngine::lora_prep(int l, int t, Planes X, int d_in, int d_out) {
  const LlamaConfig& c = cfg_;
  const int N = this->N(), r = c.lora_rank;
  const std::string pre = "blk." + std::to_string(l) + "." + kProjName[t];
  // u = X A^T, and B^T for the splice in the same launch
  KL(launch_lora_down(X, d_in, N, d_in, P32(P(pre + ".lora_a")), r, 1.0f, lora_u_[l][t], stream_,
                      P32(P(pre + ".lora_b")), d_out, lora_bt_[l][t]));
  return 0;
}

// The splice of adapter (l, t) as a GEMM epilogue addend on output columns [c0, c0 + d_out).
LoraAddend LlamaEngine::lora_addend(int l, int t, int c0, int d_out) const {
  LoraAddend a;
  a.u = lora_u_[l][t];
  a.bt = lora_bt_[l][t];
  a.c0 = c0;
  a.width = d_out;
  a.r = cfg_.lora_rank;
  a.scale = cfg_.lora_alpha / (float)cfg_.lora_rank;
  return a;
}

int LlamaEngine::dequant_layer(int l) {
  if (!q8_planes_) return 0;
  const int slot = l & 1;
  if (ring_layer_[slot] != l) {
    KL(launch_q8_0_ring(ring_desc_[l], stream_));
    ring_layer_[slot] = l;
  }
  if (ring_ev_[slot]) {   // filled ahead on wst_
    CU(cudaStreamWaitEvent(stream_, ring_ev_[slot], 0));
    ring_ev_[slot] = nullptr;
  }
  return 0;
}

int LlamaEngine::fill_ahead(int l) {
  if (!q8_planes_ || !side_ || l < 0 || l >= cfg_.n_layers) return 0;
  const int slot = l & 1;
  if (ring_layer_[slot] == l) return 0;
  CK(fork_side());   // the slot's previous block has been enqueued on the step stream
  KL(launch_q8_0_ring(ring_desc_[l], wst_));
  cudaEvent_t e = next_event();
  if (!e) return -3;
  CU(cudaEventRecord(e, wst_));
  ring_ev_[slot] = e;
  ring_layer_[slot] = l;
  return 0;
}

int LlamaEngine::norm_bwd(const float* x, const float* gamma, const float* dres, const Param& gp, int slot16) {
  const LlamaConfig& c = cfg_;
  const bool trainable = gp.trainable;
  CK(flip(t_dxp_));
  dxp_ = dxp2_[t_dxp_.cur];
  if (trainable) {
    CK(flip(t_gpart_));
    gpart_ = gpart2_[t_gpart_.cur];
  }
  const int nblk = rmsnorm_bwd_blocks();
  KL(launch_rmsnorm_bwd(x, dh_, gamma, dres, dx_, grad16(dxp_, slot16), trainable ? gpart_ : nullptr, nblk, N(),
                        c.d_model, c.rms_eps,
                        stream_, dxp_ld_));
  if (trainable) {   // dgamma: a weight gradient, on the side stream
    CK(fork_side());
    KL(launch_colsum(gpart_, nblk, c.d_model, G32(gp), 0, sst()));
    CK(side_read(t_gpart_));
  }
  return 0;
}

// Fill descriptors of every block's ring operands (pointers into the Q8_0
// arena, the adapters' f32 parameters and the ring slot), built once.
int LlamaEngine::build_ring(long long qvoff) {
  const LlamaConfig& c = cfg_;
  const float s = c.lora_rank > 0 ? c.lora_alpha / (float)c.lora_rank : 0.f;
  static const char* kFirst[4] = {"attn_q.weight", "attn_output.weight", "ffn_gate.weight", "ffn_down.weight"};
  std::vector<RingLayer> host(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    RingLayer& L = host[l];
    bf16* base = static_cast<bf16*>(q8pl_.p) + (long long)(l & 1) * 2 * q8_slot_elems_;
    long long chunk = 0;
    for (int g = 0; g < 4; ++g) {
      const RingGroup& rg = ring_[g];
      const Param& W = P("blk." + std::to_string(l) + "." + kFirst[g]);
      if (W.q8v_offset + (long long)rg.d_out * rg.d_in > qvoff || W.q8s_offset * 32 != W.q8v_offset) return -1;
      RingMat& M = L.m[L.n++];
      M.qv = static_cast<const int8_t*>(q8v_.p) + W.q8v_offset;
      M.qs = static_cast<const uint16_t*>(q8s_.p) + W.q8s_offset;
      M.hi = base + rg.off;
      M.lo = base + q8_slot_elems_ + rg.off;
      M.d_out = rg.d_out; M.d_in = rg.d_in; M.ext = rg.ext; M.r = c.lora_rank; M.s = s;
      M.chunk0 = chunk;
      chunk += (long long)(rg.d_out + rg.ext) * (rg.d_in + rg.ext) / 16;
      if (per_head_ && g == kGroupQKV) {   // the per-head LoRA-Q pairs as one block-diagonal adapter
        const std::string pre = "blk." + std::to_string(l) + ".attn_q";
        RingAdapter& a = M.ad[M.n_ad++];
        a.A = P32(P(pre + ".lora_a"));
        a.B = P32(P(pre + ".lora_b"));
        a.c0 = 0;
        a.width = c.n_heads * c.d_head;
        M.bd_r = c.lora_rank;
        M.bd_w = c.d_head;
        M.s = 1.0f;
      } else if (rg.ext) {
        const LoraGroup G = lora_group(g);
        if (G.n > 3 || c.lora_rank > 16) return -1;
        for (int i = 0; i < G.n; ++i) {
          const std::string pre = "blk." + std::to_string(l) + "." + kProjName[G.t[i]];
          RingAdapter& a = M.ad[M.n_ad++];
          a.A = P32(P(pre + ".lora_a"));
          a.B = P32(P(pre + ".lora_b"));
          a.c0 = G.c0[i];
          a.width = G.w[i];
        }
      }
    }
    L.chunks = chunk;
    if (chunk != ring_chunks_) return -1;
  }
  ring_desc_ = std::move(host);
  return 0;
}

// Y[:, col_off : col_off + d_out] += s * u B^T as a separate kernel (for base
// GEMMs without a fused epilogue); u and B^T come from lora_group_prep.
int LlamaEngine::lora_forward(int l, int t, float* Y, long long ldy, int col_off, int d_out) {
  const LoraAddend a = lora_addend(l, t, col_off, d_out);
  KL(launch_lora_up(a.u, N(), a.r, a.bt, d_out, a.scale, epi_rowmajor(kEpiAccumF32, Y + col_off, ldy), stream_));
  return 0;
}

// Gradients of the adapter on projection (l, t): dB, dA into the gradient
// arena, and dX += s * (dY B) A (row-major [N][d_in] or the given scatter).
int LlamaEngine::lora_backward(int l, int t, Planes X, int d_in, Planes dY, long long ld_dy, int col_off, int d_out,
                               float* dX, const Epilogue* dx_scatter) {
  const LlamaConfig& c = cfg_;
  const int N = this->N(), r = c.lora_rank;
  const float s = c.lora_alpha / (float)r;
  const std::string pre = "blk." + std::to_string(l) + "." + kProjName[t];
  const Param& A = P(pre + ".lora_a");
  const Param& Bp = P(pre + ".lora_b");
  const float* u = lora_u_[l][t];
  const float* bt = lora_bt_[l][t];
  Planes dYo = offset(dY, col_off);
  Epilogue e = dx_scatter ? *dx_scatter : epi_rowmajor(kEpiAccumF32, dX, d_in);
  if (r <= kLoraBwdMaxRank) {   // one fused pass over dY and X, then the fixed-order chunk reduction
    KL(launch_lora_backward(dYo, ld_dy, d_out, X, d_in, d_in, u, bt, P32(A), r, s, N, e, du32_, lora_part_, G32(Bp),
                            G32(A), stream_));
    return 0;
  }
  // dB = s * dY^T u   [d_out][r]
  KL(launch_lora_wgrad(dYo, ld_dy, u, N, d_out, r, s, G32(Bp), r, 1, lora_part_, stream_));
  // du = s * dY B   [N][r]
  KL(launch_lora_down(dYo, ld_dy, N, d_out, bt, r, s, du32_, stream_));
  // dA = du^T X   [r][d_in]
  KL(launch_lora_wgrad(X, d_in, du32_, N, d_in, r, 1.0f, G32(A), 1, d_in, lora_part_, stream_));
  // dX += du A   [N][d_in]
  KL(launch_lora_up(du32_, N, r, P32(A), d_in, 1.0f, e, stream_));
  return 0;
}

LlamaEngine::LoraGroup LlamaEngine::lora_group(int g) const {
  const LlamaConfig& c = cfg_;
  const int d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff;
  LoraGroup G;
  auto add = [&](int t, int c0, int w) {
    if (c.mode == 1 && (c.lora_targets & (1 << t)) && !(per_head_ && t == kLoraQ)) {
      G.t[G.n] = t; G.c0[G.n] = c0; G.w[G.n] = w;
      ++G.n;
    }
  };
  if (g == kGroupQKV) {
    add(kLoraQ, 0, H * dh);
    add(kLoraK, H * dh, KV * dh);
    add(kLoraV, (H + KV) * dh, KV * dh);
  } else if (g == kGroupO) {
    add(kLoraO, 0, d);
  } else if (g == kGroupGU) {
    add(kLoraGate, 0, ff);
    add(kLoraUp, ff, ff);
  } else {
    add(kLoraDown, 0, d);
  }
  return G;
}

// RMSNorm of x into h, and -- for the group of adapters that read h -- their
// down-projections u = h A^T and B^T copies in the same pass when possible.
int LlamaEngine::rmsnorm_lora(int l, const float* x, const float* gamma, Planes h, const LoraGroup& G,
                              long long ldh) {
  const LlamaConfig& c = cfg_;
  const int N = this->N(), d = c.d_model;
  const int ext_base = ldh > d ? d : -1;   // the adapters' u also as h's extra columns
  if (G.n && c.lora_rank <= 16) {
    LoraSegs segs = lora_group_segs(l, G, d, ext_base);
    if (profiling_) prof_begin(kKRmsFwd, 0.0);
    const int rc = launch_rmsnorm_fwd_lora(x, gamma, h, N, d, c.rms_eps, c.lora_rank, segs, stream_, ldh);
    if (profiling_) prof_end();
    if (rc != -2) {   // -2: no variant for this width, run the two passes below
      ++counting_;
      return rc;
    }
  }
  KL(launch_rmsnorm_fwd(x, gamma, h, N, d, c.rms_eps, stream_, ldh));
  if (G.n) CK(lora_group_prep(l, G, h, d, ldh));
  return 0;
}

LoraSegs LlamaEngine::lora_group_segs(int l, const LoraGroup& G, int d_in, int ext_base) {
  LoraSegs segs;
  for (int i = 0; i < G.n; ++i) {
    const std::string pre = "blk." + std::to_string(l) + "." + kProjName[G.t[i]];
    LoraSeg& sg = segs.s[segs.n++];
    sg.col_off = 0; sg.width = d_in;
    sg.w = P32(P(pre + ".lora_a"));
    sg.alpha = 1.0f;
    sg.out = lora_u_[l][G.t[i]];
    sg.b_src = P32(P(pre + ".lora_b")); sg.b_rows = G.w[i]; sg.bt = lora_bt_[l][G.t[i]];
    sg.ext_col = ext_base >= 0 ? ext_base + 16 * i : -1;
  }
  return segs;
}

int LlamaEngine::lora_group_prep(int l, const LoraGroup& G, Planes X, int d_in, long long ldx) {
  const int N = this->N(), r = cfg_.lora_rank;
  if (r > 16) {
    for (int i = 0; i < G.n; ++i) CK(lora_prep(l, G.t[i], X, d_in, G.w[i]));
    return 0;
  }
  if (wg_tc_ && d_in >= kWgTcMinWidth && d_in % 8 == 0 && ldx % 8 == 0) {
    // u = X A^T for the whole group as one tensor-core GEMM against the packed A's
    LoraPackW pw;
    LoraScatterU sc;
    pw.r = sc.r = r;
    sc.X = X;
    sc.ldx = ldx;
    for (int i = 0; i < G.n; ++i) {
      const std::string pre = "blk." + std::to_string(l) + "." + kProjName[G.t[i]];
      pw.p[pw.n] = P32(P(pre + ".lora_a"));
      pw.koff[pw.n] = 0;
      pw.w[pw.n++] = d_in;
      sc.out[sc.n] = lora_u_[l][G.t[i]];
      sc.ext_col[sc.n++] = ldx > d_in ? d_in + 16 * i : -1;
      KL(launch_lora_transpose(P32(P(pre + ".lora_b")), G.w[i], r, lora_bt_[l][G.t[i]], stream_));
    }
    KL(launch_lora_pack_w(pw, kWgTcCols, d_in, wg_wp_, stream_));
    GemmDesc g;
    g.M = N; g.N = kWgTcCols; g.K = d_in;
    g.a = op(X, N, d_in, ldx, 0);
    g.b = op(wg_wp_, kWgTcCols, d_in, d_in, 0);
    g.epi = epi_rowmajor(kEpiStoreF32, wg_u_, kWgTcCols);
    CK(gemm(g));
    KL(launch_lora_scatter_u(wg_u_, N, kWgTcCols, sc, stream_));
    return 0;
  }
  const LoraSegs segs = lora_group_segs(l, G, d_in, ldx > d_in ? d_in : -1);
  KL(launch_lora_down_group(X, ldx, N, r, segs, stream_));
  return 0;
}

int LlamaEngine::lora_group_du(int l, const LoraGroup& G, Planes dY, long long ld_dy, int d_in, Epilogue& dx_epi,
                                int ext_base) {
  const int N = this->N(), r = cfg_.lora_rank;
  const float s = cfg_.lora_alpha / (float)r;
  CK(flip(t_du_));
  du32_ = du2_[t_du_.cur];
  int sw = 0;
  bool contiguous = true;
  for (int i = 0; i < G.n; ++i) {
    sw += G.w[i];
    if (i) contiguous = contiguous && G.c0[i] == G.c0[i - 1] + G.w[i - 1];
  }
  if (wg_tc_ && contiguous && sw >= kWgTcMinWidth && sw % 8 == 0 && G.c0[0] % 8 == 0 && ld_dy % 8 == 0) {
    // du = s dY B for the whole group as one tensor-core GEMM against the
    // block-diagonal packed B's (adapter i's rows only see its own columns)
    LoraPackW pw;
    LoraScatterU sc;
    pw.r = sc.r = r;
    pw.trans = 1;
    sc.alpha = s;
    sc.X = dY;
    sc.ldx = ld_dy;
    for (int i = 0; i < G.n; ++i) {
      const std::string pre = "blk." + std::to_string(l) + "." + kProjName[G.t[i]];
      pw.p[pw.n] = P32(P(pre + ".lora_b"));
      pw.koff[pw.n] = G.c0[i] - G.c0[0];
      pw.w[pw.n++] = G.w[i];
      sc.out[sc.n] = du32_ + (long long)i * N * r;
      sc.ext_col[sc.n++] = ext_base >= 0 ? ext_base + 16 * i : -1;
    }
    KL(launch_lora_pack_w(pw, kWgTcCols, sw, wg_wp_, stream_));
    GemmDesc g;
    g.M = N; g.N = kWgTcCols; g.K = sw;
    g.a = op(Planes{dY.hi + G.c0[0], dY.lo + G.c0[0]}, N, sw, ld_dy, 0);
    g.b = op(wg_wp_, kWgTcCols, sw, sw, 0);
    g.epi = epi_rowmajor(kEpiStoreF32, wg_u_, kWgTcCols);
    CK(gemm(g));
    KL(launch_lora_scatter_u(wg_u_, N, kWgTcCols, sc, stream_));
  } else {
    LoraSegs segs;
    for (int i = 0; i < G.n; ++i) {
      LoraSeg& sg = segs.s[segs.n++];
      sg.col_off = G.c0[i]; sg.width = G.w[i];
      sg.w = lora_bt_[l][G.t[i]];
      sg.alpha = s;
      sg.out = du32_ + (long long)i * N * r;
      sg.ext_col = ext_base >= 0 ? ext_base + 16 * i : -1;
    }
    KL(launch_lora_down_group(dY, ld_dy, N, r, segs, stream_));
  }
  if (ext_base >= 0) return 0;   // the dX GEMM reads du from dY's extra columns
  for (int i = 0; i < G.n; ++i) {
    const std::string pre = "blk." + std::to_string(l) + "." + kProjName[G.t[i]];
    LoraAddend& a = dx_epi.lora[dx_epi.n_lora++];
    a.u = du32_ + (long long)i * N * r;
    a.bt = P32(P(pre + ".lora_a"));   // A [r][d_in]: dX += du A
    a.c0 = 0;
    a.width = d_in;
    a.r = r;
    a.scale = 1.0f;
  }
  return 0;
}

int LlamaEngine::lora_group_wgrad(int l, const LoraGroup& G, Planes X, long long ldx, int d_in, Planes dY,
                                   long long ld_dy) {
  if (wg_tc_ && wsc_.ws && d_in >= kWgTcMinWidth && G.c0[0] % 8 == 0 && ld_dy % 8 == 0 && ldx % 8 == 0) {
    bool contiguous = true;   // the group's output columns one range (q|k|v, gate|up)
    for (int i = 1; i < G.n; ++i) contiguous = contiguous && G.c0[i] == G.c0[i - 1] + G.w[i - 1];
    if (contiguous) return lora_group_wgrad_tc(l, G, X, ldx, d_in, dY, ld_dy);
  }
  const int N = this->N(), r = cfg_.lora_rank;
  const float s = cfg_.lora_alpha / (float)r;
  LoraWgGroup g;
  for (int i = 0; i < G.n; ++i) {
    const std::string pre = "blk." + std::to_string(l) + "." + kProjName[G.t[i]];
    LoraWgSeg& sg = g.s[g.n++];
    sg.col_off = G.c0[i]; sg.width = G.w[i];
    sg.u = lora_u_[l][G.t[i]];
    sg.du = du32_ + (long long)i * N * r;
    sg.dB = G32(P(pre + ".lora_b"));
    sg.dA = G32(P(pre + ".lora_a"));
  }
  KL(launch_lora_wgrad_group(dY, ld_dy, X, ldx, d_in, N, r, s, g, side_ ? lora_part2_ : lora_part_, sst()));
  return 0;
}

// dA_i = du_i^T X and dB_i = s dY_i^T u_i as two tensor-core GEMMs over the
// token dimension (K = N): DA = X^T [du_0 | du_1 | ..] ([d_in][64]) and
// DB = dY[:, group columns]^T [u_0 | u_1 | ..] ([sum of widths][64], of which
// the diagonal r x width blocks are kept), both split-bf16 with three passes
// like every other product, then one scatter into the gradients. On CUDA
// cores these reductions took ~35 % of a Llama-3.2-1B QLoRA step at rank 16.
int LlamaEngine::lora_group_wgrad_tc(int l, const LoraGroup& G, Planes X, long long ldx, int d_in, Planes dY,
                                     long long ld_dy) {
  const int N = this->N(), r = cfg_.lora_rank;
  const float s = cfg_.lora_alpha / (float)r;
  LoraPackSrc us, dus;
  LoraWgGroup g;
  int sw = 0;
  for (int i = 0; i < G.n; ++i) {
    const std::string pre = "blk." + std::to_string(l) + "." + kProjName[G.t[i]];
    us.p[us.n++] = lora_u_[l][G.t[i]];
    dus.p[dus.n++] = du32_ + (long long)i * N * r;
    LoraWgSeg& sg = g.s[g.n++];
    sg.col_off = G.c0[i]; sg.width = G.w[i];
    sg.u = lora_u_[l][G.t[i]];
    sg.du = du32_ + (long long)i * N * r;
    sg.dB = G32(P(pre + ".lora_b"));
    sg.dA = G32(P(pre + ".lora_a"));
    sw += G.w[i];
  }
  KL(launch_lora_pack_planes(us, N, r, kWgTcCols, wg_ubp_, sst()));
  KL(launch_lora_pack_planes(dus, N, r, kWgTcCols, wg_dubp_, sst()));
  GemmDesc ga;
  ga.M = d_in; ga.N = kWgTcCols; ga.K = N;
  ga.a = op(X, N, d_in, ldx, 1);
  ga.b = op(wg_dubp_, N, kWgTcCols, kWgTcCols, 1);
  ga.epi = epi_rowmajor(kEpiStoreF32, wg_da_, kWgTcCols);
  CK(gemm_side(ga));
  GemmDesc gb;
  gb.M = sw; gb.N = kWgTcCols; gb.K = N;
  gb.a = op(Planes{dY.hi + G.c0[0], dY.lo + G.c0[0]}, N, sw, ld_dy, 1);
  gb.b = op(wg_ubp_, N, kWgTcCols, kWgTcCols, 1);
  gb.epi = epi_rowmajor(kEpiStoreF32, wg_db_, kWgTcCols);
  CK(gemm_side(gb));
  KL(launch_lora_wg_extract(wg_da_, wg_db_, d_in, r, kWgTcCols, s, g, sst()));
  return 0;
}

Operand LlamaEngine::experts_op(const Param& p, int rows, int cols, int mn) {
  Operand o = expert_op(p, 0, rows, cols, mn);
  o.nbatch = cfg_.n_experts;   // batch z = expert z of the stacked tensor
  o.bdiv1 = 1;
  o.bmul1 = 1;
  return o;
}

Operand LlamaEngine::expert_op(const Param& p, int e, int rows, int cols, int mn) {
  // expert e of a stacked Q8_0 tensor: rows x cols quants (row-major) and their scales
  Operand o = op(Planes{}, rows, cols, cols, mn);
  const long long first = (long long)e * rows * cols;
  o.q8 = static_cast<const int8_t*>(q8v_.p) + p.q8v_offset + first;
  o.q8_scale = static_cast<const uint16_t*>(q8s_.p) + p.q8s_offset + first / 32;
  return o;
}

// The MoE FFN of block l: router GEMM, routing, slots ordered by expert on the
// host, the experts' gate / up GEMMs over their slot rows (Q8_0 dequantised in
// the GEMM), SwiGLU, down GEMMs, and the weighted sum back onto the tokens
// with the residual: x[l + 1] = x1 + sum_k w_k y_k.
int LlamaEngine::moe_forward(int l) {
  const LlamaConfig& c = cfg_;
  const int N = this->N(), d = c.d_model, ff = c.d_ff, E = c.n_experts, K = c.n_experts_used;
  const long long NK = (long long)N * K;
  const std::string pre = "blk." + std::to_string(l) + ".";
  MoeLayer& M = moe_l_[l];
  GemmDesc gr;
  gr.M = N; gr.N = E; gr.K = d;
  gr.a = op(h2_[l], N, d, d, 0);
  gr.b = op(PP(P(pre + "ffn_gate_inp.weight")), E, d, d, 0);
  gr.epi = epi_rowmajor(kEpiStoreF32, moe_logits_, E);
  CK(gemm(gr));
  KL(launch_moe_route(moe_logits_, N, E, K, c.norm_topk, M.probs, M.idx, M.w, stream_));
  // slots (token * K + choice) in expert order, ascending within an expert
  CU(cudaMemcpyAsync(moe_hidx_.data(), M.idx, NK * 4, cudaMemcpyDeviceToHost, stream_));
  CU(cudaStreamSynchronize(stream_));
  M.count.assign(E, 0);
  for (long long i = 0; i < NK; ++i) {
    const int e = moe_hidx_[i];
    if (e < 0 || e >= E) return -3;
    ++M.count[e];
  }
  M.offset.assign(E + 1, 0);
  for (int e = 0; e < E; ++e) M.offset[e + 1] = M.offset[e] + M.count[e];
  std::vector<int> fill(M.offset.begin(), M.offset.end() - 1);
  for (long long i = 0; i < NK; ++i) {
    const int at = fill[moe_hidx_[i]]++;
    moe_hperm_[at] = (int)i;
    moe_hpos_[i] = at;
  }
  CU(cudaMemcpyAsync(M.perm, moe_hperm_.data(), NK * 4, cudaMemcpyHostToDevice, stream_));
  CU(cudaMemcpyAsync(M.pos, moe_hpos_.data(), NK * 4, cudaMemcpyHostToDevice, stream_));
  // the experts' 128-slot M tiles for the grouped GEMMs (one launch per product for all experts)
  M.htab.clear();
  for (int e = 0; e < E; ++e)
    for (int t0 = 0; t0 < M.count[e]; t0 += 128) {
      M.htab.push_back(e);
      M.htab.push_back(M.offset[e] + t0);
      M.htab.push_back(M.offset[e] + std::min(M.count[e], t0 + 128));
    }
  M.ntiles = (int)(M.htab.size() / 3);
  if (M.ntiles > NK / 128 + E + 1) return -3;
  CU(cudaMemcpyAsync(M.gtab, M.htab.data(), M.htab.size() * 4, cudaMemcpyHostToDevice, stream_));
  KL(launch_moe_gather(h2_[l], d, M.perm, NK, K, d, moe_xs_, stream_));
  const Param& Wg = P(pre + "ffn_gate_exps.weight");
  const Param& Wu = P(pre + "ffn_up_exps.weight");
  const Param& Wd = P(pre + "ffn_down_exps.weight");
  for (int h = 0; h < 2; ++h) {   // gate into columns [0, ff), up into [ff, 2 ff), every expert's slots at once
    GemmDesc g;
    g.M = (int)NK; g.N = ff; g.K = d;
    g.a = op(moe_xs_, (int)NK, d, d, 0);
    g.b = experts_op(h ? Wu : Wg, ff, d, 0);
    g.epi = epi_rowmajor(kEpiStoreF32, M.gu + h * ff, 2 * ff);
    g.group_tiles = M.gtab;
    g.group_mtiles = M.ntiles;
    CK(gemm(g));
  }
  KL(launch_swiglu_fwd(M.gu, M.a, (int)NK, ff, stream_, ff));
  {
    GemmDesc g;
    g.M = (int)NK; g.N = d; g.K = ff;
    g.a = op(M.a, (int)NK, ff, ff, 0);
    g.b = experts_op(Wd, d, ff, 0);
    g.epi = epi_rowmajor(kEpiStoreF32, M.ye, d);
    g.group_tiles = M.gtab;
    g.group_mtiles = M.ntiles;
    CK(gemm(g));
  }
  KL(launch_moe_combine(x1_[l], M.ye, M.pos, M.w, N, K, d, x_[l + 1], stream_));
  return 0;
}

// d(h2) of block l's MoE FFN into dh_ from the output gradient dx_: per slot
// dw = <dy, y> and w dy, back through each expert (down, SwiGLU, gate / up,
// the frozen Q8_0 weights read MN-major), the router's softmax backward, and
// the fixed-order sum of the slots' input gradients onto their tokens.
int LlamaEngine::moe_backward(int l) {
  const LlamaConfig& c = cfg_;
  const int N = this->N(), d = c.d_model, ff = c.d_ff, E = c.n_experts, K = c.n_experts_used;
  const long long NK = (long long)N * K;
  const std::string pre = "blk." + std::to_string(l) + ".";
  MoeLayer& M = moe_l_[l];
  const Param& Wg = P(pre + "ffn_gate_exps.weight");
  const Param& Wu = P(pre + "ffn_up_exps.weight");
  const Param& Wd = P(pre + "ffn_down_exps.weight");
  KL(launch_moe_dy(dx_, M.ye, M.perm, M.w, NK, K, d, moe_dw_, moe_dye_, stream_));
  {
    GemmDesc g;   // through every expert's down projection at once
    g.M = (int)NK; g.N = ff; g.K = d;
    g.a = op(moe_dye_, (int)NK, d, d, 0);
    g.b = experts_op(Wd, d, ff, 1);
    g.epi = epi_rowmajor(kEpiStoreF32, moe_das_, ff);
    g.group_tiles = M.gtab;
    g.group_mtiles = M.ntiles;
    CK(gemm(g));
  }
  KL(launch_swiglu_bwd(M.gu, moe_das_, moe_dgu_, (int)NK, ff, stream_, 2 * ff));
  for (int h = 0; h < 2; ++h) {   // dxs = dgate Wg_e + dup Wu_e
    GemmDesc g;
    g.M = (int)NK; g.N = d; g.K = ff;
    g.a = op(offset(moe_dgu_, (long long)h * ff), (int)NK, ff, 2 * ff, 0);
    g.b = experts_op(h ? Wu : Wg, ff, d, 1);
    g.epi = epi_rowmajor(h ? kEpiAccumF32 : kEpiStoreF32, moe_dxs_, d);
    g.group_tiles = M.gtab;
    g.group_mtiles = M.ntiles;
    CK(gemm(g));
  }
  KL(launch_moe_router_bwd(M.probs, M.idx, M.w, moe_dw_, N, E, K, c.norm_topk, moe_dlog_, stream_));
  GemmDesc gr;
  gr.M = N; gr.N = d; gr.K = E;
  gr.a = op(moe_dlog_, N, E, E, 0);
  gr.b = op(PP(P(pre + "ffn_gate_inp.weight")), E, d, d, 1);
  gr.epi = epi_rowmajor(kEpiStoreF32, dh_, d);
  CK(gemm(gr));
  KL(launch_moe_gather_sum(moe_dxs_, M.pos, N, K, d, dh_, stream_));
  return 0;
}

int LlamaEngine::enqueue_forward() {
  const LlamaConfig& c = cfg_;
  const int N = this->N(), d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff, T = c.T, B = c.B;
  const int W = (H + 2 * KV) * dh, G = H / KV, V = c.vocab;
  const float scale = 1.0f / std::sqrt((float)dh);
  const bool lora = c.mode == 1;
  const Param& E = P("token_embd.weight");
  side_ = wst_ && !profiling_;   // the forward's side work: ring fills one block ahead
  side_forked_ = false;
  sev_next_ = 0;
  ring_layer_[0] = ring_layer_[1] = -1;
  ring_ev_[0] = ring_ev_[1] = nullptr;
  KL(launch_embed_gather(P32(E), ids_, x_[0], N, d, stream_));
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string pre = "blk." + std::to_string(l) + ".";
    CK(dequant_layer(l));
    CK(fill_ahead(l + 1));
    const LoraGroup Gq = lora_group(kGroupQKV);
    const int eq = ext_[kGroupQKV];   // q|k|v adapters folded into the GEMM as extra reduction columns
    CK(rmsnorm_lora(l, x_[l], P32(P(pre + "attn_norm.weight")), h1_[l], Gq, d + eq));   // + the adapters' u
    if (per_head_) {   // u = h A^T of every head's pair, as planes into h's extension columns
      GemmDesc gu;
      gu.M = N; gu.N = H * c.lora_rank; gu.K = d;
      gu.a = op(h1_[l], N, d, d + eq, 0);
      gu.b = op(PP(P(pre + "attn_q.lora_a")), H * c.lora_rank, d, d, 0);
      gu.epi = epi_rowmajor(kEpiStoreSplit, nullptr, d + eq);
      gu.epi.out_hi = h1_[l].hi + d;
      gu.epi.out_lo = h1_[l].lo + d;
      CK(gemm(gu));
    }
    GemmDesc g;
    g.M = N; g.N = W; g.K = d + eq;
    g.a = op(h1_[l], N, d + eq, d + eq, 0);
    g.b = wop(P(pre + "attn_q.weight"), W, d, d, 0);
    const float* bias = c.qkv_bias ? P32(P(pre + "attn_q.bias")) : nullptr;
    const int qkv_t[3] = {kLoraQ, kLoraK, kLoraV};
    const int qkv_c0[3] = {0, H * dh, (H + KV) * dh}, qkv_w[3] = {H * dh, KV * dh, KV * dh};
    if ((dh == 64 || dh == 128) && !c.qk_norm) {
      // one launch: q|k|v projection, adapters, bias, RoPE, head-major Q / K / V planes
      g.epi.mode = kEpiRopeQKV;
      RopeOut& ro = g.epi.rope;
      ro.pos = pos_; ro.cs = cs_; ro.tab_rows = cs_rows_; ro.bias = bias;
      ro.q_hi = Qh_[l].hi; ro.q_lo = Qh_[l].lo; ro.k_hi = Kh_[l].hi; ro.k_lo = Kh_[l].lo;
      ro.v_hi = Vh_[l].hi; ro.v_lo = Vh_[l].lo;
      ro.T = T; ro.H = H; ro.KV = KV; ro.dh = dh;
      for (int i = 0; i < Gq.n && !eq; ++i) g.epi.lora[g.epi.n_lora++] = lora_addend(l, Gq.t[i], Gq.c0[i], Gq.w[i]);
      CK(gemm(g));
    } else {
      g.epi = epi_rowmajor(kEpiStoreF32, qkv_, W);
      CK(gemm(g));
      for (int i = 0; i < Gq.n && !eq; ++i) CK(lora_forward(l, Gq.t[i], qkv_, W, Gq.c0[i], Gq.w[i]));
      if (c.qk_norm) {   // RMSNorm over the whole q and k vectors, before RoPE; pre-norm values kept
        KL(launch_rms_cols_fwd(qkv_, W, 0, H * dh, P32(P(pre + "attn_q_norm.weight")), c.rms_eps, N, qkpre_[l],
                               stream_));
        KL(launch_rms_cols_fwd(qkv_, W, H * dh, KV * dh, P32(P(pre + "attn_k_norm.weight")), c.rms_eps, N,
                               qkpre_[l] + (long long)N * H * dh, stream_));
      }
      KL(launch_rope_qkv_fwd(qkv_, bias, pos_, cs_, cs_rows_, Qh_[l], Kh_[l], Vh_[l], B, T, H, KV, dh, stream_));
    }
    if (flash_) {
      // fused: O (token-major planes) and the row normalisers for the backward
      KL(launch_flash_fwd(Qh_[l], Kh_[l], Vh_[l], O_[l], lse2_[l], B, T, H, KV, dh, scale, err_, stream_, o_ld_));
    } else {
      // scores S = scale * Q K^T per (sequence, head)
      GemmDesc gs;
      gs.M = T; gs.N = T; gs.K = dh; gs.batch = B * H;
      gs.a = bop(Qh_[l], T, dh, dh, B * H, 0);
      gs.b = bop(Kh_[l], T, dh, dh, B * KV, 0, H, KV, G, 1);
      gs.causal = 1;   // tiles above the diagonal are never read by the causal softmax
      gs.epi.mode = kEpiStoreF32; gs.epi.out = S_; gs.epi.alpha = scale; gs.epi.m_s0 = T;
      gs.epi.bstride = (long long)T * T;
      CK(gemm(gs));
      KL(launch_softmax_causal_fwd(S_, Pm_[l], (long long)B * H, T, stream_));
      // O = P V, written token-major [N][H*dh]
      GemmDesc go;
      go.M = T; go.N = dh; go.K = T; go.batch = B * H;
      go.a = bop(Pm_[l], T, T, T, B * H, 0);
      go.b = bop(Vh_[l], T, dh, dh, B * KV, 1, H, KV, G, 1);
      go.causal = 2;   // P is zero for keys past the tile's last query
      go.epi.mode = kEpiStoreSplit; go.epi.out_hi = O_[l].hi; go.epi.out_lo = O_[l].lo;
      go.epi.z_div = H; go.epi.z_s1 = (long long)T * o_ld_; go.epi.bstride = dh; go.epi.m_s0 = o_ld_;
      CK(gemm(go));
    }
    // x1 = x + O Wo^T
    const int eo = ext_[kGroupO];   // o adapter folded in as extra reduction columns
    GemmDesc gw;
    gw.M = N; gw.N = d; gw.K = H * dh + eo;
    gw.a = op(O_[l], N, H * dh + eo, o_ld_, 0);
    gw.b = wop(P(pre + "attn_output.weight"), d, H * dh, H * dh, 0);
    gw.epi = epi_rowmajor(kEpiResidF32, x1_[l], d);
    gw.epi.res = x_[l];
    const LoraGroup Go = lora_group(kGroupO);
    if (Go.n) {
      CK(lora_group_prep(l, Go, O_[l], H * dh, o_ld_));
      if (!eo) gw.epi.lora[gw.epi.n_lora++] = lora_addend(l, kLoraO, 0, d);
    }
    CK(gemm(gw));
    const LoraGroup Gg = lora_group(kGroupGU);
    const int eg = ext_[kGroupGU];
    CK(rmsnorm_lora(l, x1_[l], P32(P(pre + "ffn_norm.weight")), h2_[l], Gg, d + eg));   // + the adapters' u
    if (moe_) {
      CK(moe_forward(l));
      continue;
    }
    GemmDesc gg;
    gg.M = N; gg.N = 2 * ff; gg.K = d + eg;
    gg.a = op(h2_[l], N, d + eg, d + eg, 0);
    const Param& Wgu = P(pre + "ffn_gate.weight");
    gg.b = wop(Wgu, 2 * ff, d, d, 0);
    if (Wgu.q8 && !q8_planes_ && a_ld_ == ff) {   // (the epilogue writes a with a row pitch of d_ff)
      // Q8_0 base: one launch -- gate|up projection (gate and up rows paired per
      // tile), adapters, a = silu(gate) * up as planes; gate|up kept in f32 for
      // the backward. (The dequantising GEMM has operand-feed headroom for the
      // extra epilogue stores; the plane GEMM does not, so full fine-tunes keep
      // SwiGLU as its own kernel.)
      gg.epi = epi_rowmajor(kEpiSwiGLU, gu_[l], 2 * ff);
      gg.epi.out_hi = a_[l].hi; gg.epi.out_lo = a_[l].lo; gg.epi.pair_off = ff;
      for (int i = 0; i < Gg.n; ++i) gg.epi.lora[gg.epi.n_lora++] = lora_addend(l, Gg.t[i], Gg.c0[i], Gg.w[i]);
      CK(gemm(gg));
    } else {
      gg.epi = epi_rowmajor(kEpiStoreF32, gu_[l], 2 * ff);
      CK(gemm(gg));
      for (int i = 0; i < Gg.n && !eg; ++i) CK(lora_forward(l, Gg.t[i], gu_[l], 2 * ff, Gg.c0[i], Gg.w[i]));
      KL(launch_swiglu_fwd(gu_[l], a_[l], N, ff, stream_, a_ld_));
    }
    const int ed = ext_[kGroupDown];   // down adapter folded in as extra reduction columns
    GemmDesc gd;
    gd.M = N; gd.N = d; gd.K = ff + ed;
    gd.a = op(a_[l], N, ff + ed, a_ld_, 0);
    gd.b = wop(P(pre + "ffn_down.weight"), d, ff, ff, 0);
    gd.epi = epi_rowmajor(kEpiResidF32, x_[l + 1], d);
    gd.epi.res = x1_[l];
    const LoraGroup Gd = lora_group(kGroupDown);
    if (Gd.n) {
      CK(lora_group_prep(l, Gd, a_[l], ff, a_ld_));
      if (!ed) gd.epi.lora[gd.epi.n_lora++] = lora_addend(l, kLoraDown, 0, d);
    }
    CK(gemm(gd));
  }
  CK(join_side());
  side_ = false;
  KL(launch_rmsnorm_fwd(x_[c.n_layers], P32(P("output_norm.weight")), xf_, N, d, c.rms_eps, stream_));
  const Param& Wout = c.tied ? E : P("output.weight");
  GemmDesc gl;
  gl.M = N; gl.N = V; gl.K = d;
  gl.a = op(xf_, N, d, d, 0);
  gl.b = op(PP(Wout), V, d, d, 0);
  gl.epi = epi_rowmajor(kEpiStoreF32, logits_, V);
  if (!dense_labels_) {
    // the LM head writes each row's vocab-chunk (max, sum exp) pairs with the
    // logits; the cross-entropy then needs a single pass over them
    gl.epi.mode = kEpiStoreLse;
    gl.epi.lse_part = lse_part_;
    CK(gemm(gl));
    KL(launch_cross_entropy_lse(logits_, lse_part_, lse_ms_, labels_, loss_rows_, dlog_, N, V, stream_));
    ++counting_;   // (two kernels: the logsumexp combine and the gradient pass)
  } else {
    CK(gemm(gl));
    KL(launch_cross_entropy(logits_, labels_, labels_dense_, loss_rows_, dlog_, N, V, stream_));
  }
  KL(launch_loss_reduce(loss_rows_, N, loss_, stream_));
  return 0;
}

int LlamaEngine::enqueue_backward() {
  const LlamaConfig& c = cfg_;
  const int N = this->N(), d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff, T = c.T, B = c.B;
  const int W = (H + 2 * KV) * dh, G = H / KV, V = c.vocab;
  const float scale = 1.0f / std::sqrt((float)dh);
  const bool full = c.mode == 0, lora = c.mode == 1;
  const Param& E = P("token_embd.weight");
  const Param& Wout = c.tied ? E : P("output.weight");
  side_ = wst_ && !profiling_;
  side_forked_ = false;
  t_dxp_ = t_dgu_ = t_dqkv_ = t_du_ = t_gpart_ = Transient{};
  dxp_ = dxp2_[0]; dgu_ = dgu2_[0]; dqkv_ = dqkv2_[0]; du32_ = du2_[0];
  // fp16 weight gradients from the second step a program runs on: the first
  // records the gradients' magnitudes (three-pass products meanwhile)
  const bool w16 = f16w_ && f16w_ready_;
  if (f16w_) KL(launch_f16_scale_update(amax16_, scale16_, inv16_, n16_, stream_));
  const int L = c.n_layers;
  // dxf = dlogits W_out   ([N][V] x [V][d])
  GemmDesc g;
  g.M = N; g.N = d; g.K = V;
  g.a = op(dlog_, N, V, V, 0);
  g.b = op(PP(Wout), V, d, d, 1);
  g.epi = epi_rowmajor(kEpiStoreF32, dh_, d);
  CK(gemm(g));
  if (full) {
    GemmDesc ge;
    ge.M = V; ge.N = d; ge.K = N;
    ge.a = op(dlog_, N, V, V, 1);
    ge.b = op(xf_, N, d, d, 1);
    ge.epi = epi_rowmajor(kEpiStoreF32, G32(Wout), d);
    if (w16) {
      ge.split = false; ge.f16 = true;
      ge.a = op16(dlog_.f16, N, V, V, 1);
      ge.b = op16(xf_.f16, N, d, d, 1);
      ge.epi.alpha_dev = inv16_ + n16_;
    }
    CK(fork_side());
    CK(gemm_side(ge));
  }
  const Param& gf = P("output_norm.weight");
  CK(norm_bwd(x_[c.n_layers], P32(gf), nullptr, gf, 4 * (L - 1)));
  for (int l = c.n_layers - 1; l >= 0; --l) {
    const std::string pre = "blk." + std::to_string(l) + ".";
    CK(dequant_layer(l));   // the forward's last two blocks are still in the ring
    CK(fill_ahead(l - 1));
    const Param& Wo = P(pre + "attn_output.weight");
    const Param& Wq = P(pre + "attn_q.weight");
    // ---- FFN
    if (moe_) {
      CK(moe_backward(l));
    } else {
    const Param& Wd = P(pre + "ffn_down.weight");
    const Param& Wg = P(pre + "ffn_gate.weight");
    const int ed = ext_[kGroupDown];   // dY carries du of the down adapter in its extra columns
    GemmDesc gda;
    gda.M = N; gda.N = ff; gda.K = d + ed;
    gda.a = op(dxp_, N, d + ed, dxp_ld_, 0);
    gda.b = wop(Wd, d, ff, ff, 1);
    gda.epi = epi_rowmajor(kEpiStoreF32, da_, ff);
    const LoraGroup Gd = lora_group(kGroupDown);
    const bool gd_grp = Gd.n && lora_grouped(ff);
    if (gd_grp) CK(lora_group_du(l, Gd, dxp_, dxp_ld_, ff, gda.epi, ed ? d : -1));
    CK(gemm(gda));
    if (gd_grp || full) {   // weight gradients of the down projection, on the side stream
      CK(fork_side());
      if (gd_grp) CK(lora_group_wgrad(l, Gd, a_[l], a_ld_, ff, dxp_, dxp_ld_));
      if (full) {
        GemmDesc gw;
        gw.M = d; gw.N = ff; gw.K = N;
        gw.a = op(dxp_, N, d, dxp_ld_, 1);
        gw.b = op(a_[l], N, ff, a_ld_, 1);
        gw.epi = epi_rowmajor(kEpiStoreF32, G32(Wd), ff);
        if (w16) {
          gw.split = false; gw.f16 = true;
          gw.a = op16(dxp_.f16, N, d, dxp_ld_, 1);
          gw.b = op16(a_[l].f16, N, ff, a_ld_, 1);
          gw.epi.alpha_dev = inv16_ + 4 * l;
        }
        CK(gemm_side(gw));
      }
      CK(side_read2(t_dxp_, t_du_));
    }
    if (Gd.n && !gd_grp) CK(lora_backward(l, kLoraDown, a_[l], ff, dxp_, dxp_ld_, 0, d, da_, nullptr));
    const int eg = ext_[kGroupGU];   // dgu carries du of the gate|up adapters in its extra columns
    CK(flip(t_dgu_));
    dgu_ = dgu2_[t_dgu_.cur];
    KL(launch_swiglu_bwd(gu_[l], da_, grad16(dgu_, 4 * l + 1), N, ff, stream_, 2 * ff + eg));
    GemmDesc gh;
    gh.M = N; gh.N = d; gh.K = 2 * ff + eg;
    gh.a = op(dgu_, N, 2 * ff + eg, 2 * ff + eg, 0);
    gh.b = wop(Wg, 2 * ff, d, d, 1);
    gh.epi = epi_rowmajor(kEpiStoreF32, dh_, d);
    const LoraGroup Gg = lora_group(kGroupGU);
    const bool gg_grp = Gg.n && lora_grouped(d);
    if (gg_grp) CK(lora_group_du(l, Gg, dgu_, 2 * ff + eg, d, gh.epi, eg ? 2 * ff : -1));
    CK(gemm(gh));
    if (gg_grp || full) {
      CK(fork_side());
      if (gg_grp) CK(lora_group_wgrad(l, Gg, h2_[l], d + eg, d, dgu_, 2 * ff + eg));
      if (full) {
        GemmDesc gw;
        gw.M = 2 * ff; gw.N = d; gw.K = N;
        gw.a = op(dgu_, N, 2 * ff, 2 * ff + eg, 1);
        gw.b = op(h2_[l], N, d, d, 1);
        gw.epi = epi_rowmajor(kEpiStoreF32, G32(Wg), d);
        if (w16) {
          gw.split = false; gw.f16 = true;
          gw.a = op16(dgu_.f16, N, 2 * ff, 2 * ff + eg, 1);
          gw.b = op16(h2_[l].f16, N, d, d, 1);
          gw.epi.alpha_dev = inv16_ + 4 * l + 1;
        }
        CK(gemm_side(gw));
      }
      CK(side_read2(t_dgu_, t_du_));
    }
    for (int i = 0; i < Gg.n && !gg_grp; ++i)
      CK(lora_backward(l, Gg.t[i], h2_[l], d, dgu_, 2 * ff, Gg.c0[i], Gg.w[i], dh_, nullptr));
    }
    const Param& g2 = P(pre + "ffn_norm.weight");
    CK(norm_bwd(x1_[l], P32(g2), dx_, g2, 4 * l + 2));
    // ---- attention output projection: dO (head-major f32), dWo
    Epilogue hm;
    hm.mode = kEpiStoreF32; hm.out = dO32_;
    hm.m_div = T; hm.m_s1 = (long long)H * T * dh; hm.m_s0 = dh; hm.n_div = dh; hm.n_s1 = (long long)T * dh;
    const int eo = ext_[kGroupO];   // dY carries du of the o adapter in its extra columns
    GemmDesc gdo;
    gdo.M = N; gdo.N = H * dh; gdo.K = d + eo;
    gdo.a = op(dxp_, N, d + eo, dxp_ld_, 0);
    gdo.b = wop(Wo, d, H * dh, H * dh, 1);
    gdo.epi = hm;
    const LoraGroup Go = lora_group(kGroupO);
    const bool go_grp = Go.n && lora_grouped(H * dh);
    if (go_grp) CK(lora_group_du(l, Go, dxp_, dxp_ld_, H * dh, gdo.epi, eo ? d : -1));
    CK(gemm(gdo));
    if (go_grp || full) {
      CK(fork_side());
      if (go_grp) CK(lora_group_wgrad(l, Go, O_[l], o_ld_, H * dh, dxp_, dxp_ld_));
      if (full) {
        GemmDesc gw;
        gw.M = d; gw.N = H * dh; gw.K = N;
        gw.a = op(dxp_, N, d, dxp_ld_, 1);
        gw.b = op(O_[l], N, H * dh, o_ld_, 1);
        gw.epi = epi_rowmajor(kEpiStoreF32, G32(Wo), H * dh);
        if (w16) {
          gw.split = false; gw.f16 = true;
          gw.a = op16(dxp_.f16, N, d, dxp_ld_, 1);
          gw.b = op16(O_[l].f16, N, H * dh, o_ld_, 1);
          gw.epi.alpha_dev = inv16_ + 4 * l + 2;
        }
        CK(gemm_side(gw));
      }
      CK(side_read2(t_dxp_, t_du_));
    }
    if (Go.n && !go_grp) CK(lora_backward(l, kLoraO, O_[l], H * dh, dxp_, dxp_ld_, 0, d, dO32_, &hm));
    CK(flip(t_dqkv_));   // written by the RoPE backward below
    dqkv_ = dqkv2_[t_dqkv_.cur];
    if (flash_) {
      // ---- attention core, fused: partial dQ / dK / dV summed by the RoPE backward
      KL(launch_flash_bwd_prep(dO32_, O_[l], dO_, dvec_, B, T, H, dh, stream_, o_ld_));
      KL(launch_flash_bwd(Qh_[l], Kh_[l], Vh_[l], dO_, lse2_[l], dvec_, fws_, B, T, H, KV, dh, scale, err_,
                          stream_));
      KL(launch_flash_rope_bwd(fws_, pos_, cs_, cs_rows_, grad16(dqkv_, 4 * l + 3), c.qkv_bias ? qkv_ : nullptr, B,
                               T, H, KV, dh, stream_, W + ext_[kGroupQKV]));
    } else {
      KL(launch_split_f32(dO32_, dO_.hi, dO_.lo, (long long)N * H * dh, stream_));
      // ---- attention core
      GemmDesc gp;
      gp.M = T; gp.N = T; gp.K = dh; gp.batch = B * H;
      gp.a = bop(dO_, T, dh, dh, B * H, 0);
      gp.b = bop(Vh_[l], T, dh, dh, B * KV, 0, H, KV, G, 1);
      gp.causal = 1;
      gp.epi.mode = kEpiStoreF32; gp.epi.out = S_; gp.epi.m_s0 = T; gp.epi.bstride = (long long)T * T;
      CK(gemm(gp));
      KL(launch_softmax_causal_bwd(Pm_[l], S_, dS_, (long long)B * H, T, scale, stream_));
      GemmDesc gq;
      gq.M = T; gq.N = dh; gq.K = T; gq.batch = B * H;
      gq.a = bop(dS_, T, T, T, B * H, 0);
      gq.b = bop(Kh_[l], T, dh, dh, B * KV, 1, H, KV, G, 1);
      gq.causal = 2;   // dS is zero past the diagonal
      gq.epi.mode = kEpiStoreF32; gq.epi.out = dQ_; gq.epi.m_s0 = dh; gq.epi.bstride = (long long)T * dh;
      CK(gemm(gq));
      GemmDesc gk;
      gk.M = T; gk.N = dh; gk.K = G * T; gk.batch = B * KV;
      gk.a = bop(dS_, G * T, T, T, B * KV, 1);
      gk.b = bop(Qh_[l], G * T, dh, dh, B * KV, 1);
      gk.epi.mode = kEpiStoreF32; gk.epi.out = dK_; gk.epi.m_s0 = dh; gk.epi.bstride = (long long)T * dh;
      CK(gemm(gk));
      GemmDesc gv;
      gv.M = T; gv.N = dh; gv.K = G * T; gv.batch = B * KV;
      gv.a = bop(Pm_[l], G * T, T, T, B * KV, 1);
      gv.b = bop(dO_, G * T, dh, dh, B * KV, 1);
      gv.epi.mode = kEpiStoreF32; gv.epi.out = dV_; gv.epi.m_s0 = dh; gv.epi.bstride = (long long)T * dh;
      CK(gemm(gv));
      KL(launch_rope_qkv_bwd(dQ_, dK_, dV_, pos_, cs_, cs_rows_, dqkv_, c.qkv_bias ? qkv_ : nullptr, B, T, H, KV, dh,
                             stream_, W + ext_[kGroupQKV]));
    }
    if (c.qk_norm) {   // back through the whole-vector q / k RMSNorm, on the gradient planes in place
      KL(launch_rms_cols_bwd(dqkv_, W + ext_[kGroupQKV], 0, H * dh, P32(P(pre + "attn_q_norm.weight")), qkpre_[l],
                             c.rms_eps, N, stream_));
      KL(launch_rms_cols_bwd(dqkv_, W + ext_[kGroupQKV], H * dh, KV * dh, P32(P(pre + "attn_k_norm.weight")),
                             qkpre_[l] + (long long)N * H * dh, c.rms_eps, N, stream_));
    }
    if (c.qkv_bias && full) KL(launch_colsum_rows(qkv_, N, W, G32(P(pre + "attn_q.bias")), stream_));
    // ---- QKV projection
    const int eq = ext_[kGroupQKV];   // dqkv carries du of the q|k|v adapters in its extra columns
    GemmDesc gx;
    gx.M = N; gx.N = d; gx.K = W + eq;
    gx.a = op(dqkv_, N, W + eq, W + eq, 0);
    gx.b = wop(Wq, W, d, d, 1);
    gx.epi = epi_rowmajor(kEpiStoreF32, dh_, d);
    const LoraGroup Gq = lora_group(kGroupQKV);
    const bool gq_grp = Gq.n && lora_grouped(d);
    if (gq_grp) CK(lora_group_du(l, Gq, dqkv_, W + eq, d, gx.epi, eq ? W : -1));
    const int Rq = H * c.lora_rank;
    if (per_head_) {   // du = dY_q B (block-diagonal B from the ring operand) into dY's extension columns
      GemmDesc gdu;
      gdu.M = N; gdu.N = Rq; gdu.K = H * dh;
      gdu.a = op(dqkv_, N, H * dh, W + eq, 0);
      gdu.b = op(ring_ext_b(l), H * dh, Rq, d + eq, 1);
      gdu.b.l2_keep = ring_keep_;
      gdu.epi = epi_rowmajor(kEpiStoreSplit, nullptr, W + eq);
      gdu.epi.out_hi = dqkv_.hi + W;
      gdu.epi.out_lo = dqkv_.lo + W;
      CK(gemm(gdu));
    }
    CK(gemm(gx));
    if (per_head_) {   // dA = du^T h and the diagonal blocks of dY_q^T u, on the weight-gradient stream
      CK(fork_side());
      GemmDesc ga;
      ga.M = Rq; ga.N = d; ga.K = N;
      ga.a = op(offset(dqkv_, W), N, Rq, W + eq, 1);
      ga.b = op(h1_[l], N, d, d + eq, 1);
      ga.epi = epi_rowmajor(kEpiStoreF32, G32(P(pre + "attn_q.lora_a")), d);
      CK(gemm_side(ga));
      GemmDesc gb;
      gb.M = H * dh; gb.N = Rq; gb.K = N;
      gb.a = op(dqkv_, N, H * dh, W + eq, 1);
      gb.b = op(offset(h1_[l], d), N, Rq, d + eq, 1);
      gb.epi = epi_rowmajor(kEpiStoreF32, bd_dense_, Rq);
      CK(gemm_side(gb));
      KL(launch_lora_blockdiag_take(bd_dense_, H, dh, c.lora_rank, G32(P(pre + "attn_q.lora_b")), sst()));
      CK(side_read(t_dqkv_));
    }
    if (gq_grp || full) {
      CK(fork_side());
      if (gq_grp) CK(lora_group_wgrad(l, Gq, h1_[l], d + eq, d, dqkv_, W + eq));
      if (full) {
        GemmDesc gw;
        gw.M = W; gw.N = d; gw.K = N;
        gw.a = op(dqkv_, N, W, W + eq, 1);
        gw.b = op(h1_[l], N, d, d, 1);
        gw.epi = epi_rowmajor(kEpiStoreF32, G32(Wq), d);
        if (w16) {
          gw.split = false; gw.f16 = true;
          gw.a = op16(dqkv_.f16, N, W, W + eq, 1);
          gw.b = op16(h1_[l].f16, N, d, d, 1);
          gw.epi.alpha_dev = inv16_ + 4 * l + 3;
        }
        CK(gemm_side(gw));
      }
      CK(side_read2(t_dqkv_, t_du_));
    }
    for (int i = 0; i < Gq.n && !gq_grp; ++i)
      CK(lora_backward(l, Gq.t[i], h1_[l], d, dqkv_, W, Gq.c0[i], Gq.w[i], dh_, nullptr));
    const Param& g1 = P(pre + "attn_norm.weight");
    CK(norm_bwd(x_[l], P32(g1), dx_, g1, l > 0 ? 4 * (l - 1) : -1));
    CK(bucket_ready(layer_grad_lo_[l], false));   // this layer's gradients are final
  }
  CK(join_side());   // the embedding scatter adds to the LM head's (tied) gradient
  if (full) {
    // the scatter adds onto the embedding's gradient: the tied LM head's dW
    // GEMM wrote it above; an untied embedding starts from zero every step
    if (!c.tied) CU(cudaMemsetAsync(G32(E), 0, (size_t)E.numel() * 4, stream_));
    KL(launch_embed_scatter(dx_, ord_, seg_start_, seg_id_, nseg_dev_, N, G32(E), d, stream_));
  }
  CK(bucket_ready(0, true));
  CK(bucket_join());
  side_ = false;
  if (f16w_) f16w_ready_ = true;   // the gradient slots hold this program's magnitudes
  return 0;
}

int LlamaEngine::enqueue_optimizer() {
  Planes pp{static_cast<bf16*>(phi_.p), static_cast<bf16*>(plo_.p)};
  const bool acc = accum_ > 1;
  float* g = static_cast<float*>(acc ? acc_.p : g_.p);
  KL(launch_adamw(static_cast<float*>(p32_.p), g, static_cast<float*>(m_.p), static_cast<float*>(v_.p), pp, n_train_,
                  hp_, grad_scale_ / (float)accum_, stream_));
  if (acc) CU(cudaMemsetAsync(acc_.p, 0, acc_.bytes, stream_));   // the next window starts empty
  return 0;
}

int LlamaEngine::enqueue_step(bool run_optimizer, bool accumulate) {
  counting_ = 0;
  CK(bucket_begin());
  // the backward's GEMMs of an adapter recipe have the GPU to themselves (its
  // second stream carries only CUDA-core adapter work): planned as such. The
  // forward's keep the shared plan, which measured faster there (full FT
  // 222.4k vs 220.1k with the forward planned alone; the isolated timings the
  // alone plan is fitted to lack the forward's L2 reuse between kernels).
  gemm_alone_ = false;
  CK(enqueue_forward());
  gemm_alone_ = cfg_.mode != 0;
  CK(enqueue_backward());
  gemm_alone_ = false;
  if (accumulate)
    KL(launch_add_inplace(static_cast<float*>(acc_.p), static_cast<const float*>(g_.p), n_train_, stream_));
  if (run_optimizer) CK(enqueue_optimizer());
  launches_ = counting_;
  return 0;
}

int LlamaEngine::set_grad_accumulation(int n) {
  if (!realized_ || n < 1) return -1;
  CU(cudaSetDevice(device_));
  if (n > 1 && !acc_.p) CK(alloc(acc_, (size_t)std::max<long long>(n_train_, 64) * 4));
  if (acc_.p) CU(cudaMemsetAsync(acc_.p, 0, acc_.bytes, stream_));
  accum_ = n;
  micro_ = 0;
  graph_valid_ = graph_acc_valid_ = false;
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

int LlamaEngine::step(bool is_first, bool run_optimizer) {
  if (!realized_) return -2;
  CU(cudaSetDevice(device_));
  if (is_first) {
    CU(cudaMemsetAsync(m_.p, 0, m_.bytes, stream_));
    CU(cudaMemsetAsync(v_.p, 0, v_.bytes, stream_));
    if (accum_ > 1) {   // a new accumulation window
      CU(cudaMemsetAsync(acc_.p, 0, acc_.bytes, stream_));
      micro_ = 0;
    }
  }
  // With gradient accumulation every step adds into the arena and the last
  // micro-batch of the window runs the optimiser; the accumulating steps
  // replay a graph of their own.
  const bool acc = accum_ > 1 && run_optimizer;
  const bool opt = run_optimizer && (!acc || micro_ == accum_ - 1);
  if (acc) micro_ = opt ? 0 : micro_ + 1;
  cudaGraphExec_t& gx = (acc && !opt) ? graph_acc_ : graph_;
  bool& gvalid = (acc && !opt) ? graph_acc_valid_ : graph_valid_;
  bool& gdense = (acc && !opt) ? graph_acc_dense_ : graph_dense_;
  const bool can_graph = use_graph_ && run_optimizer;
  if (can_graph && gvalid && gdense == dense_labels_) {
    CU(cudaGraphLaunch(gx, stream_));
    return 0;
  }
  if (!can_graph) return enqueue_step(opt, acc);
  // First use of this configuration: run eagerly once (validates every launch),
  // then capture the same program for replay.
  CK(enqueue_step(opt, acc));
  cudaGraph_t g = nullptr;
  CU(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
  const int rc = enqueue_step(opt, acc);
  cudaError_t ce = cudaStreamEndCapture(stream_, &g);
  if (rc || ce != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return rc ? rc : -3;
  }
  if (gx) cudaGraphExecDestroy(gx);
  gx = nullptr;
  ce = cudaGraphInstantiate(&gx, g, cudaGraphInstantiateFlagUseNodePriority);
  cudaGraphDestroy(g);
  CU(ce);
  gvalid = true;
  gdense = dense_labels_;
  return 0;
}

int LlamaEngine::run_steps(int n, float* ms) {
  if (!realized_ || n <= 0 || !ms) return -1;
  CU(cudaSetDevice(device_));
  if (use_graph_ && !(graph_valid_ && graph_dense_ == dense_labels_)) CK(step(false, true));  // capture
  cudaEvent_t a, b;
  CU(cudaEventCreate(&a));
  CU(cudaEventCreate(&b));
  CU(cudaEventRecord(a, stream_));
  for (int i = 0; i < n; ++i) CK(step(false, true));
  CU(cudaEventRecord(b, stream_));
  if (wait_fn_) {
    const int rc = wait_fn_(wait_ctx_, b);
    if (rc) {
      cudaEventDestroy(a);
      cudaEventDestroy(b);
      return rc;
    }
  }
  CU(cudaEventSynchronize(b));
  CU(cudaEventElapsedTime(ms, a, b));
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return 0;
}

int LlamaEngine::profile_step(bool is_first, int* kinds, float* ms, double* flops, int cap) {
  if (!realized_) return -2;
  CU(cudaSetDevice(device_));
  if (is_first) {
    CU(cudaMemsetAsync(m_.p, 0, m_.bytes, stream_));
    CU(cudaMemsetAsync(v_.p, 0, v_.bytes, stream_));
  }
  profiling_ = true;
  recs_.clear();
  evnext_ = 0;
  const int rc = enqueue_step(true, accum_ > 1);
  profiling_ = false;
  CK(rc);
  CU(cudaStreamSynchronize(stream_));
  const int n = (int)recs_.size();
  for (int i = 0; i < n && i < cap; ++i) {
    float t = 0.f;
    cudaEventElapsedTime(&t, recs_[i].a, recs_[i].b);
    if (kinds) kinds[i] = recs_[i].kind;
    if (ms) ms[i] = t;
    if (flops) flops[i] = recs_[i].flops;
  }
  return n;
}

int LlamaEngine::forward_only() {
  if (!realized_) return -2;
  counting_ = 0;
  return enqueue_forward();
}

float LlamaEngine::last_loss() {
  float h = NAN;
  cudaStreamSynchronize(stream_);
  cudaMemcpy(&h, loss_, 4, cudaMemcpyDeviceToHost);
  return h;
}

int LlamaEngine::sync() {
  CU(cudaStreamSynchronize(stream_));
  return 0;
}

}  // namespace tb2

namespace tb2 {

long long LlamaEngine::debug_activation(int which, int layer, float* dst, long long cap) {
  if (!realized_) return -2;
  const LlamaConfig& c = cfg_;
  const long long N = this->N(), d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff;
  const long long W = (H + 2 * KV) * dh;
  if (layer < 0 || layer > c.n_layers || (layer == c.n_layers && which != 0)) return -1;
  const float* f = nullptr;
  Planes p{};
  long long n = 0, ld = 0, rw = d;   // ld: row pitch of planes with extra columns (rows of rw values)
  switch (which) {
    case 0: f = x_[layer]; n = N * d; break;
    case 1: f = x1_[layer]; n = N * d; break;
    case 2: p = h1_[layer]; n = N * d; ld = d + ext_[kGroupQKV]; break;
    case 3: p = Qh_[layer]; n = N * H * dh; break;
    case 4: p = Kh_[layer]; n = N * KV * dh; break;
    case 5: p = Vh_[layer]; n = N * KV * dh; break;
    case 6:
      if (flash_) return -2;   // the fused attention keeps no probability matrix
      p = Pm_[layer]; n = (long long)c.B * H * c.T * c.T; break;
    case 7: p = O_[layer]; n = N * H * dh; rw = H * dh; ld = o_ld_; break;
    case 8: f = gu_[layer]; n = N * 2 * ff; break;
    case 9: p = a_[layer]; n = N * ff; rw = ff; ld = a_ld_; break;
    case 10: f = logits_; n = N * c.vocab; break;
    case 11: p = h2_[layer]; n = N * d; ld = d + ext_[kGroupGU]; break;
    case 12: f = qkv_; n = N * W; break;
    default: return -1;
  }
  if (!dst || cap < n) return n;
  CU(cudaStreamSynchronize(stream_));
  if (f) {
    CU(cudaMemcpy(dst, f, n * 4, cudaMemcpyDeviceToHost));
    return n;
  }
  std::vector<bf16> hi(n), lo(n);
  if (ld > rw) {
    CU(cudaMemcpy2D(hi.data(), rw * 2, p.hi, ld * 2, rw * 2, N, cudaMemcpyDeviceToHost));
    CU(cudaMemcpy2D(lo.data(), rw * 2, p.lo, ld * 2, rw * 2, N, cudaMemcpyDeviceToHost));
  } else {
    CU(cudaMemcpy(hi.data(), p.hi, n * 2, cudaMemcpyDeviceToHost));
    CU(cudaMemcpy(lo.data(), p.lo, n * 2, cudaMemcpyDeviceToHost));
  }
  for (long long i = 0; i < n; ++i) dst[i] = __bfloat162float(hi[i]) + __bfloat162float(lo[i]);
  return n;
}

}  // namespace tb2
