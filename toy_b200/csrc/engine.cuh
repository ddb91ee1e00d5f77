// The Llama training step on one GPU: the program LlamaSeqEngine#build_training_step
// (lib/toy/llm/engine/llama_seq_engine.rb:1786-1958) builds as a ggml graph,
// expressed here as a fixed sequence of sm_100a kernels on one stream and
// replayed as a CUDA graph.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <string>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"

namespace tb2 {

enum LoraTarget : int { kLoraQ = 0, kLoraK, kLoraV, kLoraO, kLoraGate, kLoraUp, kLoraDown, kLoraCount };

struct LlamaConfig {
  int vocab = 0, d_model = 0, n_heads = 0, n_kv = 0, d_head = 0, d_ff = 0, n_layers = 0;
  float rope_base = 1e4f, rms_eps = 1e-5f, freq_scale = 1.0f;
  int tied = 1, qkv_bias = 0;
  int T = 0, B = 1;
  int mode = 0;           // 0 full fine-tune, 1 QLoRA (frozen Q8_0 base + LoRA adapters)
  int lora_rank = 0;
  float lora_alpha = 0.f;
  int lora_targets = 0;   // bitmask over LoraTarget
  std::vector<float> freq_factors;   // d_head/2 llama3-style factors, or empty
  int attn_impl = 0;      // 0: fused flash attention where supported, 1: materialised scores
  // 1: the reference's LoRA-Q (lora_targets = q only): one (A_h [r][d], B_h
  // [d_head][r]) pair per query head, no alpha / r scale, stored stacked as
  // attn_q.lora_a [H r][d] and attn_q.lora_b [H d_head][r]; needs the Q8_0
  // plane ring (base mode 1)
  int lora_per_head_q = 0;
  // mixture of experts in every block's FFN (QLoRA only): n_experts routed by
  // a frozen f32 router, the top n_experts_used per token (norm_topk: their
  // weights renormalised to sum 1), expert SwiGLU FFNs of width d_ff as frozen
  // Q8_0 -- the OLMoE block (llama_kv_engine.rb build_moe_ffn :2073)
  int n_experts = 0, n_experts_used = 0, norm_topk = 0;
  // 2: RMSNorm over the whole q and k vectors before RoPE (frozen gammas)
  int qk_norm = 0;
};

// One named parameter inside the arenas.
struct Param {
  std::string name;
  long long offset = 0;   // element offset in the arenas
  int rows = 1, cols = 1; // row-major [rows][cols]
  bool trainable = false;
  bool q8 = false;        // frozen projection stored as Q8_0 (no f32 / plane copy: offset unused)
  long long q8_offset = 0;   // bytes into q8_ (the blocks as uploaded)
  long long q8v_offset = 0;  // bytes into q8v_ (int8 quants, row-major)
  long long q8s_offset = 0;  // elements into q8s_ (fp16 scale bits, one per 32 quants)
  int layer = -1;            // block index of a Q8_0 projection
  int ring_group = -1;       // first projection of a ring operand: its adapter group (kGroupQKV ..)
  long long numel() const { return (long long)rows * cols; }
};

// How the step feeds a frozen Q8_0 projection to its GEMMs (read when an engine
// is realised): 1 (default) dequantises each block's projections once per use
// into a two-slot ring of split planes that the plain GEMMs read, with the
// adapters of a group (rank <= 16) appended as extra reduction columns / rows
// (q|k|v and gate|up); 0 hands the quants and scales to the GEMM, which
// dequantises every k-block of B in shared memory for every M tile, and adds
// the adapters in GEMM epilogues. Same values either way. Returns the previous
// mode, or -1 for a mode out of range.
int engine_set_q8_base_mode(int mode);
// 1 (default): engines realised afterwards keep their plane ring resident in
// the L2 (a persisting set-aside of the ring's size, when the device offers
// one); 0: the ring is written and read as ordinary data. Returns the previous
// setting, or -1.
int engine_set_q8_ring_l2(int on);
// Persistent CTAs of each weight-gradient GEMM on the second stream of engines
// realised afterwards: 0 (default) 100 for a full fine-tune's one-pass fp16
// weight gradients and one per SM otherwise, n > 0 at most n (148: one per
// SM; the same work walked by fewer CTAs, leaving SMs to the activation
// chain). Returns the previous setting, or -1 for n outside 0..148.
int engine_set_side_gemm_ctas(int n);
// Output tile width of the weight-gradient GEMMs on the second stream (0: the
// launch plan's choice). Returns the previous width, or -1.
int engine_set_side_gemm_tile_width(int bn);
// 1: an adapter recipe's backward GEMMs (the GPU to themselves) are planned as
// such; 0 (default): every GEMM with the shared-GPU launch plan. Read when a session enqueues its step program.
// Returns the previous setting, or -1.
int engine_set_plan_alone(int on);
// 1 (default): full fine-tunes realised afterwards compute their weight
// gradients in one fp16 tensor-core pass (fp16 copies of the operands; the
// gradients scaled per tensor by a power of two from the previous step's
// largest magnitude); 0: three split-bf16 passes like every other product.
// Returns the previous setting, or -1.
int engine_set_f16_wgrad(int on);

struct DeviceBuf {
  void* p = nullptr;
  size_t bytes = 0;
};

class LlamaEngine {
 public:
  LlamaEngine(const LlamaConfig& cfg, int device);
  ~LlamaEngine();
  int realize();          // allocate everything; returns 0 or negative

  const LlamaConfig& cfg() const { return cfg_; }
  int N() const { return cfg_.T * cfg_.B; }
  cudaStream_t stream() const { return stream_; }
  const std::vector<Param>& params() const { return params_; }
  const Param* find(const std::string& name) const;
  long long n_trainable() const { return n_train_; }
  long long n_total() const { return n_total_; }

  // Parameter I/O (host f32, row-major). Uploading refreshes the planes.
  int set_param(const std::string& name, const float* host, long long n);
  int get_param(const std::string& name, float* host, long long n);
  int get_grad(const std::string& name, float* host, long long n);
  int get_moment(const std::string& name, int which, float* host, long long n);
  int set_moment(const std::string& name, int which, const float* host, long long n);
  int set_param_q8(const std::string& name, const uint8_t* blocks, long long nbytes);
  int get_param_q8(const std::string& name, uint8_t* blocks, long long nbytes);
  // Standard deviations stay f64 end to end: the reference draws in f64 and
  // narrows each value once, so a float std would shift every draw.
  int init_random(long long seed, double init_scale, double std_all, double lora_a_std, double lora_b_std);

  // Per-step inputs.
  int set_tokens(const long long* ids, int n);
  int set_positions(const long long* pos, int n);
  int set_label_ids(const long long* ids, int n);
  int set_labels_dense(const double* lab, long long n);
  int set_hp(const double* hp, int n);

  // One step: forward, CE, backward, (allreduce hook), AdamW. is_first zeroes
  // the Adam moments first (tnn_graph_reset semantics).
  int step(bool is_first, bool run_optimizer = true);
  int forward_only();                    // loss only
  float last_loss();                     // synchronises
  int sync();

  // Gradient-arena access for data-parallel reduction.
  float* grad_arena() { return static_cast<float*>(g_.p); }
  void set_grad_scale(float s) { grad_scale_ = s; }
  void set_allreduce_hook(int (*fn)(void*, float*, long long, cudaStream_t), void* ctx) {
    allreduce_fn_ = fn;
    allreduce_ctx_ = ctx;
    graph_valid_ = graph_acc_valid_ = false;
  }
  // Host wait for the end of a timed run when collectives are in flight: the
  // data-parallel layer polls the event next to its communicator, with a time
  // limit, instead of blocking (0 done, else an error code).
  void set_wait_hook(int (*fn)(void*, cudaEvent_t), void* ctx) {
    wait_fn_ = fn;
    wait_ctx_ = ctx;
  }
  void set_use_graph(bool on) {
    use_graph_ = on;
    graph_valid_ = graph_acc_valid_ = false;
  }
  // Gradient accumulation over n micro-batches (n >= 1; 1 = off): every step
  // adds its gradients into an accumulation arena and only every n-th step
  // runs AdamW, on the accumulated sum times 1/n (times 1/world with data
  // parallelism), then clears the arena. With equal token counts per
  // micro-batch this is the step on the joined batch. A first step
  // (is_first) starts a new window.
  int set_grad_accumulation(int n);
  int grad_accumulation() const { return accum_; }
  int micro_index() const { return micro_; }
  // Gradient buckets. bucket_take is the decision rule of the backward: the
  // gradients at arena offsets >= lo are final; the pending range [pend_lo,
  // pend_hi) becomes a bucket [b_lo, b_hi) once it holds min_floats (or on the
  // final flush). Pure host logic, shared with the data-parallel layer's plan.
  static bool bucket_take(long long& pend_lo, long long& pend_hi, long long lo, bool flush, long long min_floats,
                          long long& b_lo, long long& b_hi) {
    pend_lo = pend_lo < lo ? pend_lo : lo;
    if (pend_hi <= pend_lo || (!flush && pend_hi - pend_lo < min_floats)) return false;
    b_lo = pend_lo;
    b_hi = pend_hi;
    pend_hi = pend_lo;
    return true;
  }
  const std::vector<long long>& layer_grad_lo() const { return layer_grad_lo_; }
  // Read-only views for the decode engine, which shares this engine's weights:
  // a frozen Q8_0 projection as its quants [rows][cols] and fp16 scale bits
  // [rows][cols / 32], any other parameter as its f32 values.
  struct WeightView {
    const float* f32 = nullptr;
    const int8_t* qv = nullptr;
    const uint16_t* qs = nullptr;
    int rows = 0, cols = 0;
  };
  WeightView weight(const std::string& name) const {
    WeightView w;
    const Param* p = find(name);
    if (!p) return w;
    w.rows = p->rows;
    w.cols = p->cols;
    if (p->q8) {
      w.qv = static_cast<const int8_t*>(q8v_.p) + p->q8v_offset;
      w.qs = static_cast<const uint16_t*>(q8s_.p) + p->q8s_offset;
    } else {
      w.f32 = static_cast<const float*>(p32_.p) + p->offset;
    }
    return w;
  }
  const float* rope_table() const { return cs_; }   // [rope_rows][d_head / 2] (cos, sin) pairs
  int rope_rows() const { return cs_rows_; }
  int device() const { return device_; }
  long long bucket_floats() const { return bucket_floats_; }
  void set_bucket_floats(long long n) {
    bucket_floats_ = n;
    graph_valid_ = graph_acc_valid_ = false;
  }
  void drop_graph() {
    if (graph_) cudaGraphExecDestroy(graph_);
    if (graph_acc_) cudaGraphExecDestroy(graph_acc_);
    graph_ = graph_acc_ = nullptr;
    graph_valid_ = graph_acc_valid_ = false;
  }
  int launches_per_step() const { return launches_; }
  // Copy a saved activation of the last step to the host as f32 (planes are
  // reconstructed as hi + lo). Returns the element count, or negative.
  long long debug_activation(int which, int layer, float* dst, long long cap);

  // Timing. run_steps: n steps (graph replay) between two events on the step
  // stream; returns total milliseconds in *ms. profile_step: one eager step with
  // an event pair around every launch; fills per-launch kind, duration and
  // algorithmic FLOPs (GEMMs), returns the launch count.
  enum Kind : int { kKGemm = 0, kKRmsFwd, kKRmsBwd, kKColsum, kKRope, kKSoftmax, kKSwiglu, kKCe, kKLoss, kKAdamw,
                    kKEmbed, kKSplit, kKAllreduce, kKFlashFwd, kKFlashBwd, kKFlashPrep, kKLora, kKCount };
  int run_steps(int n, float* ms);
  int profile_step(bool is_first, int* kinds, float* ms, double* flops, int cap);

 private:
  int alloc(DeviceBuf& b, size_t bytes);
  int add_param(const std::string& name, int rows, int cols, bool trainable, bool q8);
  int enqueue_forward();
  int enqueue_backward();
  int enqueue_optimizer();
  // accumulate: add this step's gradients into the accumulation arena;
  // run_optimizer: AdamW (on the arena when accumulating)
  int enqueue_step(bool run_optimizer, bool accumulate = false);
  int gemm(const GemmDesc& d);
  // Weight gradients (dW GEMMs, adapter dA / dB) feed only the optimiser, so
  // the backward runs them on a second stream, side by side with the chain of
  // activation gradients: wst_ forks from the step stream after their inputs
  // are written and joins it before the optimiser. The transients they read
  // (dY planes, du) alternate between two copies; before the step stream
  // writes a copy again it waits for that copy's last side reader. A profiled
  // step keeps everything on the step stream.
  struct Transient {
    int cur = 0;
    cudaEvent_t busy[2] = {nullptr, nullptr};
  };
  int gemm_side(const GemmDesc& d);
  cudaStream_t sst() const { return side_ ? wst_ : stream_; }
  cudaEvent_t next_event();
  int fork_side();                        // wst_ waits for the step stream so far
  int side_read(Transient& t);            // the copy in use is read by the side work enqueued so far
  int side_read2(Transient& a, Transient& b);
  int flip(Transient& t);                 // switch copies, waiting for the new one's side readers
  int join_side();                        // the step stream waits for wst_
  int lora_forward(int l, int t, float* Y, long long ldy, int col_off, int d_out);
  int lora_prep(int l, int t, Planes X, int d_in, int d_out);
  LoraAddend lora_addend(int l, int t, int c0, int d_out) const;
  int lora_backward(int l, int t, Planes X, int d_in, Planes dY, long long ld_dy, int col_off, int d_out,
                    float* dX, const Epilogue* dx_scatter);
  // Adapter groups: the enabled adapters whose base projections form one GEMM
  // (kGroupQKV: q|k|v, kGroupO, kGroupGU: gate|up, kGroupDown), with their
  // first column and width in the GEMM's output.
  enum { kGroupQKV = 0, kGroupO, kGroupGU, kGroupDown };
  struct LoraGroup {
    int n = 0;
    int t[3] = {0, 0, 0}, c0[3] = {0, 0, 0}, w[3] = {0, 0, 0};
  };
  LoraGroup lora_group(int g) const;
  // forward: u = X A^T and B^T of every adapter of the group, one launch
  int lora_group_prep(int l, const LoraGroup& G, Planes X, int d_in, long long ldx);
  // ext_base >= 0: u of adapter i also goes to X's columns ext_base + 16 i + j
  LoraSegs lora_group_segs(int l, const LoraGroup& G, int d_in, int ext_base);
  int rmsnorm_lora(int l, const float* x, const float* gamma, Planes h, const LoraGroup& G, long long ldh);
  // backward, before the group's dX GEMM: du = s dY B of every adapter (one
  // launch) and the splices dX += du A as addends of that GEMM's epilogue
  // With ext_base >= 0 du goes to dY's columns ext_base + 16 i + j (the dX
  // GEMM's extra reduction columns) instead of the epilogue.
  int lora_group_du(int l, const LoraGroup& G, Planes dY, long long ld_dy, int d_in, Epilogue& dx_epi,
                    int ext_base);
  // backward, after it: dB and dA of every adapter (partials + fixed-order sum)
  int lora_group_wgrad(int l, const LoraGroup& G, Planes X, long long ldx, int d_in, Planes dY, long long ld_dy);
  // the same on tensor cores, for groups whose input is at least kWgTcMinWidth wide
  int lora_group_wgrad_tc(int l, const LoraGroup& G, Planes X, long long ldx, int d_in, Planes dY, long long ld_dy);
  static constexpr int kWgTcMinWidth = 2048;
  static constexpr int kWgTcCols = 64;   // columns of the packed u / du planes and of the DA / DB products
  bool wg_tc_ = false;
  Planes wg_ubp_{}, wg_dubp_{};
  float* wg_da_ = nullptr;
  float* wg_db_ = nullptr;
  float* wg_u_ = nullptr;    // [N][64]: u or du of a wide group before its scatter
  Planes wg_wp_{};           // [64][K]: a wide group's packed A (or block-diagonal B) planes
  bool lora_grouped(int d_in) const { return cfg_.lora_rank <= 16 && d_in % 32 == 0; }
  // Per-head LoRA-Q: the block-diagonal adapter rides the q|k|v GEMMs as extra
  // reduction columns (u = h A^T into h's, du = dY_q B into dY's); dA and dB
  // are tensor-core products on the weight-gradient stream, dB through a dense
  // [H d_head][H r] product whose diagonal blocks are kept.
  bool per_head_ = false;
  float* bd_dense_ = nullptr;
  // Mixture of experts: the step runs eagerly (each block's expert counts come
  // back to the host, which orders the (token, choice) slots by expert and
  // sizes one Q8_0 GEMM per expert and projection). Per block the router's
  // probabilities, the choices and weights, the slot order and its inverse,
  // the experts' gate|up (f32), SwiGLU (planes) and output (f32) per slot.
  bool moe_ = false;
  struct MoeLayer {
    float *probs = nullptr, *w = nullptr, *gu = nullptr, *ye = nullptr;
    int *idx = nullptr, *perm = nullptr, *pos = nullptr;
    int* gtab = nullptr;            // the experts' M tiles (expert, first slot, end slot) for the grouped GEMMs
    int ntiles = 0;
    std::vector<int> htab;
    Planes a;
    std::vector<int> count, offset;
  };
  std::vector<MoeLayer> moe_l_;
  float *moe_logits_ = nullptr, *moe_das_ = nullptr, *moe_dxs_ = nullptr, *moe_dw_ = nullptr;
  Planes moe_xs_, moe_dye_, moe_dgu_, moe_dlog_;
  std::vector<int> moe_hidx_, moe_hperm_, moe_hpos_;
  std::vector<float*> qkpre_;   // QK-norm: per block the pre-norm q | k [N][(H + KV) d_head]
  int moe_forward(int l);
  int moe_backward(int l);
  Operand expert_op(const Param& p, int e, int rows, int cols, int mn);
  Operand experts_op(const Param& p, int rows, int cols, int mn);   // all experts, batch = expert
  Planes ring_ext_b(int l) const;   // B's extension block of block l's q|k|v ring operand
  float* P32(const Param& p) { return static_cast<float*>(p32_.p) + p.offset; }
  float* G32(const Param& p) { return static_cast<float*>(g_.p) + p.offset; }
  Planes PP(const Param& p) {
    return Planes{static_cast<bf16*>(phi_.p) + p.offset, static_cast<bf16*>(plo_.p) + p.offset};
  }
  // GEMM operand over a weight (and, for fused operands, the weights stored
  // after it): split planes, or the quants + scales of a Q8_0 projection.
  Operand wop(const Param& p, int rows, int cols, long long ld, int mn);
  const Param& P(const std::string& n) const;
  int refresh_planes(const Param& p);
  int split_q8(const Param& p);   // blocks -> quants + scales
  // Ring slot l % 2 := block l's ring operands (Q8_0 projections as planes,
  // with the adapters of the groups that fold them in); no launch when the
  // slot already holds them in this step program.
  int dequant_layer(int l);

  LlamaConfig cfg_;
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  bool realized_ = false;
  std::vector<Param> params_;
  std::map<std::string, int> pidx_;
  long long n_train_ = 0, n_total_ = 0, q8_bytes_ = 0;
  // arenas
  DeviceBuf p32_, phi_, plo_, g_, m_, v_, q8_, q8v_, q8s_;
  // Q8_0 base as planes: per block the first quant / scale index and the count
  // of its projections' elements; two slots of slot_elems hi then lo values
  bool q8_planes_ = false;
  bool ring_keep_ = false;
  bool gemm_alone_ = false;   // main-stream GEMMs enqueued now have the GPU to themselves (launch plan)   // the ring holds an L2 persisting set-aside (evict-last writes and reads)
  DeviceBuf q8pl_;
  long long q8_slot_elems_ = 0;
  int ring_layer_[2] = {-1, -1};
  // ring operand of each adapter group: [d_out + ext][d_in + ext] planes at
  // element offset off of a slot's hi (and lo) half; the blocks' fill
  // descriptors (passed with each fill launch) live in ring_desc_
  struct RingGroup {
    int d_out = 0, d_in = 0, ext = 0;
    long long off = 0;
  };
  RingGroup ring_[4];
  std::vector<RingLayer> ring_desc_;
  long long ring_chunks_ = 0;
  // extra reduction width of each group's base GEMMs (0, or 64 with the
  // group's adapters folded into the ring operand)
  int ext_[4] = {0, 0, 0, 0};
  // row pitches of the activations that carry extension columns: the attention
  // output (o group), the SwiGLU output (down group) and the RMSNorm-backward
  // planes (dY of both)
  long long o_ld_ = 0, a_ld_ = 0, dxp_ld_ = 0;
  int build_ring(long long qvoff);
  // the weight-gradient stream and its state (see Transient)
  cudaStream_t wst_ = nullptr;
  GemmScratch wsc_;
  DeviceBuf wsc_ws_;
  bool side_ = false;
  bool side_forked_ = false;   // wst_ has work of this program still to join
  std::vector<cudaEvent_t> sev_;
  size_t sev_next_ = 0;
  Transient t_dxp_, t_dgu_, t_dqkv_, t_du_, t_gpart_;
  Planes dxp2_[2], dgu2_[2], dqkv2_[2];
  float* gpart2_[2] = {nullptr, nullptr};
  cudaEvent_t ring_ev_[2] = {nullptr, nullptr};   // a fill of the slot still running on wst_
  // ring slot (l % 2) := block l on wst_, one block ahead of its use (the
  // slot's previous block is done on the step stream); dequant_layer waits
  int fill_ahead(int l);
  // RMSNorm backward into dx / dxp; for a trainable gamma its column sum on wst_.
  // slot16 >= 0: dxp's fp16 copy too, scaled by that gradient slot
  int norm_bwd(const float* x, const float* gamma, const float* dres, const Param& gp, int slot16 = -1);
  // One-pass fp16 weight gradients (full fine-tune): the fp16 copies hang off
  // the operands' Planes (h1_, h2_, a_, O_, xf_, dlog_, dxp2_, dgu2_, dqkv2_).
  // Gradient slot i (4 per layer: the down projection's dY, dgate|dup, the o
  // projection's dY, dq|dk|dv; then dlogits) is written scaled by scale16_[i]
  // and unscaled by the GEMM epilogue with inv16_[i]; the kernels that write a
  // slot raise amax16_[i], from which the next step's scale is set.
  bool f16w_ = false;
  bool f16w_ready_ = false;   // a finished step has recorded the slots' magnitudes
  int n16_ = 0;
  unsigned* amax16_ = nullptr;
  float *scale16_ = nullptr, *inv16_ = nullptr;
  Planes grad16(Planes p, int slot) const {   // p with its fp16 copy scaled and measured as slot
    if (!f16w_ || slot < 0) {
      p.f16 = nullptr;
      return p;
    }
    p.f16_scale = scale16_ + slot;
    p.f16_amax = amax16_ + slot;
    return p;
  }
  float* du2_[2] = {nullptr, nullptr};
  float* lora_part2_ = nullptr;   // the side stream's weight-gradient partials
  // activations and scratch
  std::vector<DeviceBuf> bufs_;
  std::vector<float*> x_, x1_, gu_;
  std::vector<Planes> h1_, h2_, a_, Qh_, Kh_, Vh_, Pm_, O_;
  bool flash_ = false;             // attention core on the fused flash kernels
  std::vector<float*> lse2_;       // flash: per-layer softmax normalisers [B][H][T]
  float *dvec_ = nullptr, *fws_ = nullptr;   // flash backward: D and partial-gradient workspace
  std::vector<std::vector<float*>> lora_u_;    // [layer][target] u = X A^T, f32 [N][r]
  std::vector<std::vector<float*>> lora_bt_;   // [layer][target] B^T, f32 [r][d_out] (this step's B)
  float* lora_part_ = nullptr;                 // weight-gradient partial sums
  float2* lse_part_ = nullptr;                 // LM head: (max, sum exp) per 64-column vocab chunk [V/64][N]
  float2* lse_ms_ = nullptr;                   // per row (max, sum exp) [N]
  float *qkv_ = nullptr, *S_ = nullptr, *logits_ = nullptr, *loss_rows_ = nullptr, *loss_ = nullptr;
  float *dx_ = nullptr, *dh_ = nullptr, *da_ = nullptr, *dO32_ = nullptr, *dQ_ = nullptr, *dK_ = nullptr,
        *dV_ = nullptr, *gpart_ = nullptr, *du32_ = nullptr;
  Planes xf_, dlog_, dxp_, dgu_, dO_, dS_, dqkv_, up_tmp_;
  // inputs
  int *ids_ = nullptr, *pos_ = nullptr, *labels_ = nullptr, *ord_ = nullptr, *seg_start_ = nullptr,
      *seg_id_ = nullptr, *nseg_dev_ = nullptr;
  float *labels_dense_ = nullptr, *hp_ = nullptr, *cs_ = nullptr;
  int cs_rows_ = 0, nseg_ = 0;
  bool dense_labels_ = false;
  std::vector<int> sort_tmp_;   // set_tokens' radix-sort buffer
  // host staging (pinned)
  void* stage_ = nullptr;
  size_t stage_bytes_ = 0;
  int* err_ = nullptr;
  float grad_scale_ = 1.0f;
  int (*allreduce_fn_)(void*, float*, long long, cudaStream_t) = nullptr;
  void* allreduce_ctx_ = nullptr;
  int (*wait_fn_)(void*, cudaEvent_t) = nullptr;
  void* wait_ctx_ = nullptr;
  // Gradient buckets: the backward finalises the arena from the top down (layer
  // L-1 first); every range of at least bucket_floats_ finished floats is reduced
  // on comm_stream_ while the backward continues, the rest after the backward.
  // bucket_floats_ is the minimum bucket size.
  long long bucket_floats_ = 1LL << 20;
  cudaStream_t comm_stream_ = nullptr;
  std::vector<cudaEvent_t> bucket_ev_;
  size_t bucket_next_ = 0;
  long long pend_lo_ = 0, pend_hi_ = 0;   // finished, not yet reduced: [pend_lo_, pend_hi_)
  std::vector<long long> layer_grad_lo_;  // lowest arena offset of each layer's trainable gradients
  bool comm_used_ = false;
  int bucket_begin();
  int bucket_ready(long long lo, bool flush);
  int bucket_join();
  bool use_graph_ = true;
  cudaGraphExec_t graph_ = nullptr;
  bool graph_valid_ = false;
  bool graph_dense_ = false;
  // gradient accumulation: the arena, the window length and the position in it;
  // the steps that only accumulate replay their own graph
  int accum_ = 1, micro_ = 0;
  DeviceBuf acc_;
  cudaGraphExec_t graph_acc_ = nullptr;
  bool graph_acc_valid_ = false, graph_acc_dense_ = false;
  int launches_ = 0;
  int counting_ = 0;
  int staged(size_t bytes);
  // profiling (eager only)
  struct Rec {
    int kind;
    double flops;
    cudaEvent_t a, b;
  };
  bool profiling_ = false;
  std::vector<Rec> recs_;
  std::vector<cudaEvent_t> evpool_;
  size_t evnext_ = 0;
  int cur_kind_ = 0;
  double cur_flops_ = 0;
  void prof_begin(int kind, double flops);
  void prof_end();
};

}  // namespace tb2
