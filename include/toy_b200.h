/* toy_b200 — B200-native (sm_100a) backend for toy's training step.
 *
 * C ABI. Every entry point takes plain pointers, sizes and opaque handles;
 * nothing in these signatures is a C++ or torch type. Functions that return
 * a handle give NULL on bad arguments; functions that return int give 0 on
 * success and a negative code on failure (-1 bad argument, -2 wrong state,
 * -3 device allocation or launch failure), following the convention of the
 * reference shim tinynn/tinynn_ggml.h.
 *
 * Three groups of entry points:
 *   1. tnn_*  — drop-in replacements for the subset of tinynn/tinynn_ggml.h
 *               that toy's training recipes call (sessions, tensors, uploads,
 *               the primitive op surface, the autograd/step calls).
 *   2. tb2_*  — additions with no counterpart in the reference: the coarse
 *               Llama training-engine realize, an index fast path for labels,
 *               device-pointer primitives used by tests and the step program,
 *               and multi-GPU gradient synchronisation.
 */
#ifndef TOY_B200_H
#define TOY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ===================================================================== */
/* Device-pointer primitives (tb2_*). `stream` is a cudaStream_t or NULL */
/* for the legacy default stream. All enqueue asynchronously.            */
/* ===================================================================== */

/* One GEMM operand stored as two bf16 planes (hi, lo) in device memory.
 * mn_major = 0: stored rows index M (or N) and K is contiguous.
 * mn_major = 1: stored rows index K and M (or N) is contiguous.
 * GEMM batch z reads storage batch (z / bdiv1) * bmul1 + ((z % bdiv1) / bdiv2) * bmul2. */
typedef struct tb2_operand {
  const void *hi;
  const void *lo;
  int mn_major;
  long long ld;
  int rows;
  int cols;
  long long batch_stride;
  int nbatch;
  int bdiv1, bmul1, bdiv2, bmul2;
  /* Q8_0 B operand of a non-batched split GEMM (NULL otherwise; hi / lo are
   * then unused): int8 quants of the stored [rows][cols] matrix, row stride ld
   * bytes, and the fp16 scale bits [rows][cols / 32] -- Q8_0 blocks (ggml
   * block_q8_0) with the scales split off. Tiles are dequantised in shared
   * memory, never in HBM. */
  const void *q8;
  const void *q8_scale;
} tb2_operand;

/* Epilogue: mode 0 store f32, 1 accumulate f32, 2 residual (out = res + acc),
 * 3 store split-bf16 planes, 4 store f32 and split planes. Output element
 * (z, m, n) is at (z/z_div)*z_s1 + (z%z_div)*bstride + (m/m_div)*m_s1 + (m%m_div)*m_s0
 * + (n/n_div)*n_s1 + n%n_div (a divisor <= 0 means "no split"). */
typedef struct tb2_epilogue {
  int mode;
  float alpha;
  float *out;
  const float *res;
  void *out_hi;
  void *out_lo;
  long long bstride;
  int z_div;
  long long z_s1;
  int m_div;
  long long m_s1, m_s0;
  int n_div;
  long long n_s1;
} tb2_epilogue;

/* D_z[m,n] = epilogue(sum_k A_z[m,k] B_z[n,k]) on tcgen05 tensor cores.
 * split = 1: 3 MMAs per k-step over (hi, lo) planes (~fp32 accuracy);
 * split = 0: plain bf16 (hi planes only);
 * split = 2: plain fp16 (the hi arrays hold fp16 values; lo unused).
 * ksplits: K ranges reduced deterministically through a per-device workspace
 * (0 = chosen from the tile count). causal: 0 none, 1 skip output tiles whose
 * columns all exceed their rows (attention scores), 2 limit K to each row
 * tile's last row + 1 (products with causal probabilities).
 * Replaces the arithmetic behind tnn_matmul / tnn_out_prod
 * (tinynn/tinynn_ggml.c:815-835) for the training step. */
int tb2_gemm(int M, int N, int K, int batch, int split, const tb2_operand *a, const tb2_operand *b,
             const tb2_epilogue *epi, int ksplits, int causal, void *stream);

/* tb2_gemm for callers that cannot allocate device memory. No counterpart in
 * the reference. Some hosts own every device buffer (a framework's memory pool,
 * a real-time loop where an allocator call would synchronise the device) and
 * can only hand this library inputs and outputs; tb2_gemm allocates its split-K
 * workspace on first use, this variant uses an 8 MiB workspace compiled into
 * the library (held on every GPU that loads it until exit) and never calls an
 * allocator. An explicit ksplits whose effective count (capped at ceil(K/64),
 * 1 for causal or batched products) times M*N exceeds 2^21 floats returns -5;
 * with ksplits = 0 the split count is chosen to fit. Calls share the workspace:
 * calls that overlap on the GPU race, so serialise them on one stream. The
 * first call on a device looks up the workspace's device address; make it
 * before any stream capture. Same arguments and results as tb2_gemm; a kernel
 * whose bounded wait gave up is reported by tb2_gemm_noalloc_error(), not by
 * tb2_device_error(). */
int tb2_gemm_noalloc(int M, int N, int K, int batch, int split, const tb2_operand *a, const tb2_operand *b,
                     const tb2_epilogue *epi, int ksplits, int causal, void *stream);
/* The error word of tb2_gemm_noalloc on the current device: synchronises the
 * device, returns 0 when the last call's kernels completed their waits, the
 * non-zero code a kernel recorded otherwise (its output is then not valid),
 * or -3 when the word cannot be read; clears it. Allocates nothing. No
 * counterpart in the reference. */
int tb2_gemm_noalloc_error(void);

/* Tile scheduling of every GEMM this library launches: mode 1 runs each GEMM
 * whose shape allows it (split planes, no causal mode) on CTA pairs -- two
 * CTAs on neighbouring SMs sharing one 256-row tensor-core tile
 * (tcgen05 cta_group::2), each holding half of the B tile; 0 never (single
 * CTAs); -1 (the default) only the shapes where pairs measured faster (both
 * operands K-major and N >= 2048: the LM head and the gate|up projections).
 * Results are the same sums in the same order either way. No counterpart in
 * the reference.
 * Returns 0, or -1 for an unknown mode. */
int tb2_gemm_set_pair_mode(int mode);

/* Output tile width (columns of a CTA's tile) of every GEMM launched
 * afterwards: 0 (the default) lets the launch plan's cost model choose; 64,
 * 128, 192 or 256 forces that width wherever the shape and epilogue allow it
 * (the cost model decides otherwise). For measuring the plan; at the same K
 * split count the results are the same sums in the same order at every
 * width. No counterpart in the reference.
 * Returns the previous width, or -1 for another value. */
int tb2_gemm_set_tile_width(int bn);

/* How a QLoRA step feeds its frozen Q8_0 projections to the tensor cores,
 * fixed for each session when its engine is realised: 1 (the default)
 * dequantises each transformer block's projections once per use (once in the
 * forward, once in the backward) into a two-slot ring of bf16 hi / lo planes
 * that the plain GEMMs read; 0 hands the quants and fp16 scales to the GEMM,
 * which dequantises B in shared memory for every 128-row M tile. The values
 * the tensor cores see are bit-identical either way; the resident copy of the
 * base is the Q8_0 data in both. No counterpart in the reference (its
 * ggml_mul_mat dequantises inside the matmul).
 * Returns the previous mode, or -1 for an unknown mode. */
int tb2_set_q8_base_mode(int mode);

/* With the ring of tb2_set_q8_base_mode(1): 1 (the default) keeps each
 * session's ring resident in the L2 -- the session reserves an L2 persisting
 * set-aside of the ring's size (a limit of this process's CUDA context,
 * released with the last session that holds one; nothing when the device
 * offers no set-aside that large) and the ring's planes are written and read
 * with the L2 evict-last policy, so the dequantised weights are read back from
 * the L2 and not written back to HBM; 0 writes and reads them as ordinary
 * data. Applies to engines realised afterwards; results are identical either
 * way. No counterpart in the reference.
 * Returns the previous setting, or -1 for an unknown one. */
int tb2_set_q8_ring_l2(int on);

/* Persistent CTAs of each weight-gradient GEMM the step runs on its second
 * stream: 0 (the default) 100 for the one-pass fp16 weight gradients of a
 * full fine-tune, one per SM otherwise; n > 0 at most n (148: one per SM),
 * the same tiles and K splits walked by fewer CTAs so that more SMs stay with
 * the activation gradient chain. Results are identical. Read when a session
 * enqueues its step program (its first step, which also captures the step's
 * CUDA graph). No counterpart in the reference.
 * Returns the previous setting, or -1 for n outside 0..148. */
int tb2_set_side_gemm_ctas(int n);

/* Output tile width of those weight-gradient GEMMs: 0 lets the launch plan
 * choose, 64 / 128 / 192 / 256 forces it where the shape allows (as
 * tb2_gemm_set_tile_width, for these GEMMs only). Read when a session
 * enqueues its step program. No counterpart in the reference.
 * Returns the previous width, or -1 for another value. */
int tb2_set_side_gemm_tile_width(int bn);

/* 1: the backward's GEMMs of an adapter recipe, which have the GPU to
 * themselves, use the launch plan for a GEMM running alone; 0 (the default,
 * which measured the same within noise): every GEMM uses the plan for a GPU
 * shared with the weight-gradient stream. K-split counts may differ between the two, so
 * the last bits of a step may too; each is deterministic. Read when a session
 * enqueues its step program. No counterpart in the reference.
 * Returns the previous setting, or -1 for another value. */
int tb2_set_plan_alone(int on);
/* 1 (the default): full fine-tunes realised afterwards compute their weight
 * gradients in one fp16 tensor-core pass (the gradient operands scaled per
 * tensor by a power of two set from the previous step's largest magnitude;
 * the first step of a program records those magnitudes on three split-bf16
 * passes); 0: three split-bf16 passes. No counterpart in the reference.
 * Returns the previous setting, or -1 for another value. */
int tb2_set_f16_wgrad(int on);

/* hi = rn_bf16(x), lo = rn_bf16(x - hi) for n f32 values. */
int tb2_split_f32(const float *x, void *hi, void *lo, size_t n, void *stream);

/* f32 [rows][K] -> Q8_0 blocks [rows][K/32*34] (ggml quantize_row_q8_0_ref:
 * d = amax/127 as fp16, q = round-half-away(x * (1/d)); bit-exact).
 * The quantiser behind tnn_cpy into a Q8_0 tensor (tinynn/ab_smoke_q8_kv.rb). */
int tb2_q8_0_quantize(const float *x, void *q, long long rows, int K, void *stream);
/* Q8_0 blocks -> split-bf16 planes (and exact f32 values when f32 != NULL). */
int tb2_q8_0_dequantize(const void *q, void *hi, void *lo, float *f32, long long rows, int K, void *stream);

/* Read and clear the device-side error word of the current device
 * (non-zero when a kernel's bounded wait gave up). Synchronises the device. */
int tb2_device_error(void);

/* Library version string. */
const char *tb2_version(void);

/* ===================================================================== */
/* Sessions (tinynn/tinynn_ggml.h:47-66)                                 */
/* ===================================================================== */

/* backend_kind must be 1 (CUDA); this library has no CPU path and returns
 * NULL (with a message on stderr) for any other kind instead of falling back.
 * Replaces tnn_session_new / tnn_session_new_on (tinynn/tinynn_ggml.h:47,60). */
void *tnn_session_new(int backend_kind);
void *tnn_session_new_on(int backend_kind, int device);
/* tinynn/tinynn_ggml.h:63 */
int tnn_cuda_get_device_count(void);
/* Frees every tensor and device buffer of the session (tinynn/tinynn_ggml.h:64). */
void tnn_session_free(void *sess);
/* tinynn/tinynn_ggml.h:89 */
const char *tnn_backend_name(void *sess);
/* Returns 73 (tinynn/tinynn_ggml.h:90). */
int tnn_link_check(void);

/* ===================================================================== */
/* Training engine: the graph LlamaSeqEngine builds (llama_seq_engine.rb) */
/* ===================================================================== */

#define TB2_MODE_FULL_FINETUNE 0 /* every weight trainable f32 (FromScratch / full fine-tune) */
#define TB2_MODE_QLORA 1         /* frozen Q8_0 base + trainable LoRA adapters (LoRA / QLoRA) */

#define TB2_LORA_Q (1 << 0)
#define TB2_LORA_K (1 << 1)
#define TB2_LORA_V (1 << 2)
#define TB2_LORA_O (1 << 3)
#define TB2_LORA_GATE (1 << 4)
#define TB2_LORA_UP (1 << 5)
#define TB2_LORA_DOWN (1 << 6)

typedef struct tb2_llama_config {
  int vocab, d_model, n_heads, n_kv, d_head, d_ff, n_layers;
  double rope_base, rms_eps, freq_scale;
  int tied, qkv_bias;
  int t_seq, t_batch;
  int mode;
  int lora_rank;
  double lora_alpha;
  int lora_targets;
  const double *rope_freq_factors; /* d_head/2 llama3 factors or NULL */
  int attn_impl;                   /* 0: fused flash attention (d_head 64), 1: materialised scores */
  int lora_per_head_q;             /* 1: toy's LoRA-Q recipe -- one (A_h, B_h) pair per query head, scale 1
                                      (transformer_block.rb:522-579,861-871); lora_targets must be q only;
                                      attn_q.lora_a is the A_h stacked [H r][d], attn_q.lora_b the B_h
                                      stacked [H d_head][r]; needs tb2_set_q8_base_mode(1) */
  /* Mixture of experts in every block's FFN (QLoRA only; llama_kv_engine.rb
   * build_moe_ffn :2073): a frozen f32 router (blk.N.ffn_gate_inp.weight
   * [n_experts x d]) picks the top n_experts_used experts per token by softmax
   * probability (norm_topk: their weights renormalised to sum 1); the experts'
   * SwiGLU FFNs of width d_ff are frozen Q8_0, stacked as
   * blk.N.ffn_{gate,up}_exps.weight [n_experts d_ff x d] and
   * blk.N.ffn_down_exps.weight [n_experts d x d_ff]. Adapters only on q, k, v, o.
   * The backward runs through the experts, the routing weights and the router's
   * softmax. Such a step runs eagerly (one host round trip per block to order
   * the routed tokens by expert). 0 = dense FFN. */
  int n_experts, n_experts_used, norm_topk;
  /* 2: RMSNorm over the whole q and k vectors before RoPE (OLMoE), frozen
   * gammas blk.N.attn_{q,k}_norm.weight; 0 none. QLoRA only. */
  int qk_norm;
} tb2_llama_config;

/* Realize the forward + cross-entropy + backward + AdamW program for a Llama
 * decoder on the session's GPU: allocates weights, Adam moments, activations.
 * Coarse replacement for LlamaSeqEngine#realize_for_random_init / realize_for_mmap
 * + build_training_step (lib/toy/llm/engine/llama_seq_engine.rb:932,713,1786). */
int tb2_llama_realize(void *sess, const tb2_llama_config *cfg);

/* Seeded weights in the reference's draw order (upload_random_init!,
 * llama_seq_engine.rb:1161-1340). std_all > 0 draws every tensor from N(0, std_all)
 * (the frozen base of a QLoRA config, quantised to Q8_0 on upload); LoRA A/B
 * follow from the same stream with the given standard deviations. With
 * lora_per_head_q the adapters follow upload_lora_q_init!(seed, init_scale)
 * (llama_seq_engine.rb:2545-2575) instead: lora_a_std is init_scale, every
 * B_h is 0. */
int tb2_llama_init_random(void *sess, long long seed, double init_scale, double std_all, double lora_a_std,
                          double lora_b_std);

#define TB2_IO_TOKEN_IDS 0
#define TB2_IO_POSITIONS 1
#define TB2_IO_LABELS 2
#define TB2_IO_HP 3
#define TB2_IO_LOSS 4
#define TB2_IO_COUNT 5
/* The step's input/output tensors (the handles build_training_step returns and
 * the engine's t_seq_token_ids / t_seq_positions, llama_seq_engine.rb:1786-1958). */
void *tb2_llama_io(void *sess, int which);
/* Parameter tensor view by GGUF-style name (e.g. "blk.0.attn_q.weight",
 * "blk.3.attn_v.lora_a"); upload/download through the tnn_* I/O calls. */
void *tb2_llama_param(void *sess, const char *name);
int tb2_llama_n_params(void *sess);
const char *tb2_llama_param_name(void *sess, int i);
int tb2_llama_param_trainable(void *sess, const char *name);
long long tb2_llama_n_trainable(void *sess);
int tb2_param_grad_to_f64(void *sess, const char *name, double *dst, size_t n);
/* which = 0: first moment m, 1: second moment v. */
int tb2_param_moment_to_f64(void *sess, const char *name, int which, double *dst, size_t n);
/* Raw Q8_0 blocks (34 bytes per 32 values) of a frozen projection, byte-exact
 * (the bytes tinynn/tinynn_gguf.c copies verbatim from a GGUF file). */
int tb2_param_upload_q8_0(void *sess, const char *name, const void *blocks, size_t nbytes);
int tb2_param_download_q8_0(void *sess, const char *name, void *blocks, size_t nbytes);
/* Index fast path for the labels tensor: one target id per token, -1 = none.
 * Equivalent to uploading the one-hot [T*B, vocab] matrix. */
int tb2_upload_label_ids(void *sess, void *labels_tensor, const long *ids, size_t n);
/* Kernels launched by the last eagerly enqueued step (a graph replay launches the same set). */
int tb2_step_launches(void *sess);
int tb2_set_use_graph(void *sess, int on);
int tb2_forward_only(void *sess);
int tb2_sync(void *sess);
/* Run n training steps on the already-uploaded inputs (CUDA-graph replay) and
 * report their device time in *ms (CUDA events on the step stream). The
 * device-timed counterpart of the reference's TNN_STEP_PROFILE split
 * (tinynn/tinynn_ggml.c:2054-2103). */
int tb2_run_steps(void *sess, int n, float *ms);
/* True gradient accumulation over n_micro micro-batches (1 = off, the
 * default). Each tnn_compute_backward adds its gradients into an accumulation
 * arena; every n_micro-th call also runs AdamW on the accumulated sum times
 * 1/n_micro (times 1/world with data parallelism) and clears the arena. With
 * equal token counts per micro-batch that is exactly the step on the joined
 * batch, where the reference approximates accumulation by running AdamW every
 * micro-batch at lr/N (examples/legacy/06_train_from_scratch.rb:64-78). A
 * tnn_graph_reset (first step) starts a new window. Returns 0, -1 for
 * n_micro < 1, -2 before tb2_llama_realize. No counterpart in the reference. */
int tb2_llama_set_grad_accumulation(void *sess, int n_micro);
/* One eagerly-enqueued step with an event pair around every kernel: fills
 * kinds[i] (0 GEMM, 1 rmsnorm fwd, 2 rmsnorm bwd, 3 column sums, 4 rope,
 * 5 softmax, 6 swiglu, 7 cross-entropy, 8 loss reduce, 9 AdamW, 10 embedding,
 * 11 split, 12 gradient all-reduce), ms[i] and the GEMM algorithmic flops[i].
 * Returns the launch count (at most cap entries are written). */
int tb2_profile_step(void *sess, int is_first, int *kinds, float *ms, double *flops, int cap);
/* Copy a saved activation of the last step to host f32 (for layer-by-layer
 * parity checks): which = 0 x_in, 1 x_after_attn, 2 attn_norm out, 3 Q (head-major,
 * roped), 4 K, 5 V, 6 softmax probs, 7 attention out, 8 gate|up, 9 swiglu out,
 * 10 logits, 11 ffn_norm out. Returns the element count (cap too small: nothing copied). */
long long tb2_debug_activation(void *sess, int which, int layer, float *dst, long long cap);

/* Data parallelism (no counterpart in the reference, which has no multi-GPU
 * training): one process per GPU, each with a full replica and its own batch.
 * Rank 0 gets a NCCL unique id (128 bytes) and shares it with the other ranks
 * through any host channel; every rank then calls tb2_dp_init on its realized
 * session. From then on each step all-reduces the trainable gradients (sum,
 * NCCL over NVLink) before AdamW, which scales them by 1/world, so every
 * replica takes the identical update of the global-batch mean gradient.
 * The reduction runs in buckets on a second stream while the backward goes on:
 * as soon as the finished gradients (the backward completes them from the last
 * layer down) reach the bucket size, they are all-reduced; the rest follows
 * the backward. */
int tb2_nccl_unique_id(void *out, size_t nbytes);
int tb2_dp_init(void *sess, const void *unique_id, int rank, int world);
/* Bucket size in floats (default 2^20); every rank must use the same value.
 * Takes effect at the next step (the step graph is re-captured). */
int tb2_dp_set_bucket_floats(void *sess, long long floats);
/* Releases the step graph (which holds NCCL work) and then the communicator.
 * Releasing a healthy communicator (NCCL finalize + destroy) is collective
 * across the node's ranks: all ranks free together. A rank that leaves on its
 * own calls tb2_dp_abort first, after which this frees local state only. */
int tb2_dp_free(void *sess);

/* Failure handling (host-side; no GPU is made to fault or hang). The
 * communicator is created non-blocking (ncclCommInitRankConfig, blocking = 0);
 * every host wait that depends on a peer polls ncclCommGetAsyncError beside
 * what it waits for, with a time limit: communicator creation (tb2_dp_init),
 * the enqueue of a collective, and the end of each step -- tnn_compute_backward
 * of a data-parallel session returns only once its step (collectives
 * included) is done, and tb2_run_steps waits for its last step the same way.
 * An NCCL error or the limit aborts the communicator (ncclCommAbort ends the
 * collectives still running on this GPU) and returns -3 (NCCL error) or -4
 * (time limit); from then on the session refuses steps (-2) until
 * tb2_dp_free. Process-wide limit in milliseconds (default 120000). */
int tb2_dp_set_timeout_ms(long long ms);
/* Wait, as above, for the session's step stream to be idle: 0, -3 or -4. */
int tb2_dp_wait(void *sess);
/* 0 while the communicator is healthy, else the code that ended it (-3 NCCL
 * error, -4 time limit, -6 tb2_dp_abort). */
int tb2_dp_status(void *sess);
/* Abort the communicator from the host (e.g. when the caller has learnt that
 * a peer rank is gone): collectives in flight on this GPU end, later steps
 * are refused. Returns 0, or -2 without data parallelism. */
int tb2_dp_abort(void *sess);
/* The gradient buckets the backward all-reduces, in issue order, as
 * [lo, hi) float ranges of the trainable-gradient arena: layer_lo[l] is the
 * lowest arena offset of layer l's trainable gradients (non-decreasing in l),
 * n_train the arena size. The backward finalises layers from the last down
 * and reduces the pending range once it holds bucket_floats (the final range,
 * with the embedding and final norm, after the backward). Writes 2 values per
 * bucket while they fit in cap; returns the bucket count, or -1. Pure host
 * logic, the same rule the step program runs; no GPU needed. */
long long tb2_dp_bucket_plan(const long long *layer_lo, int n_layers, long long n_train, long long bucket_floats,
                             long long *out, long long cap);
/* The same plan for a realized session's own layout and bucket size. */
long long tb2_dp_session_bucket_plan(void *sess, long long *out, long long cap);

/* tinynn/tinynn_ggml.h:424 — the next tnn_compute_backward zeroes the Adam moments
 * (of the step program, or of every tnn_opt_step_adamw node of a primitive graph). */
int tnn_graph_reset(void *sess);
/* tinynn/tinynn_ggml.h:419 — gradients are overwritten by every backward; no-op. */
int tnn_graph_reset_grads_only(void *sess);
/* tinynn/tinynn_ggml.h:425 — forward, CE, backward and AdamW in one call: the
 * fused step program after tb2_llama_realize, or the primitive graph built
 * with the calls below. */
int tnn_compute_backward(void *sess);

/* ===================================================================== */
/* Primitive op graph (tinynn/tinynn_ggml.h:97-469): the same calls toy's */
/* graph builders make. Tensors use ggml's shape convention (ne0 fastest; */
/* a "rows x cols" input has ne0 = cols). Ops return NULL on a shape or   */
/* type mismatch; nodes run at tnn_compute / tnn_compute_backward.        */
/* Supported: f32, i32 and Q8_0 (type 8) tensors; RoPE in NEOX mode       */
/* without YaRN (ext_factor 0); soft_max_ext without ALiBi (max_bias 0). */
/* A session uses either this graph or the fused step program.           */
/* ===================================================================== */
/* tinynn_ggml.h:97-141,303-308,394,455 */
void *tnn_input_1d_f32(void *sess, int n);
void *tnn_input_2d_f32(void *sess, int rows, int cols);
void *tnn_input_2d_f32_persistent(void *sess, int rows, int cols);
void *tnn_input_1d_f32_persistent(void *sess, int n);
void *tnn_input_3d_f32_persistent(void *sess, int ne0, int ne1, int ne2);
void *tnn_input_4d_f32_persistent(void *sess, int ne0, int ne1, int ne2, int ne3);
void *tnn_input_2d_persistent_typed(void *sess, int rows, int cols, int ggml_type);
void *tnn_input_1d_i32(void *sess, int n);
void *tnn_input_1d_i32_ctx(void *sess, int n);
void *tnn_rope_freq_factors_alloc(void *sess, int n_dims);
long tnn_row_size(int ggml_type, int ne0);
int tnn_finalize_weights(void *sess);
int tnn_session_set_graph_capacity(void *sess, int capacity);
int tnn_zero_tensor(void *sess, void *tensor);
/* Q8_0 blocks copied verbatim into a type-8 tensor (the bytes tinynn_gguf.c:634-682
 * copies from a GGUF file). No reference counterpart as a single call. */
int tnn_upload_q8_0_blocks(void *sess, void *tensor, const void *blocks, size_t nbytes);
/* tinynn_ggml.c:1715, tinynn_ggml.h:117 */
void *tnn_input_1d_i32_persistent(void *sess, int n);
void *tnn_input_3d_persistent_typed(void *sess, int ne0, int ne1, int ne2, int ggml_type);
/* tinynn_ggml.h:120-131 -- weights whose bytes (F32 or Q8_0 blocks) sit at
 * buf_offset inside a host region the caller attached (e.g. an mmap'd GGUF).
 * The region stays the caller's; the bytes are copied to the device when the
 * tensor is created, so the region may be unmapped afterwards. */
int tnn_session_attach_weight_mmap(void *sess, void *base, size_t size);
void *tnn_input_2d_persistent_mmap(void *sess, int rows, int cols, int ggml_type, size_t buf_offset);
void *tnn_input_3d_persistent_mmap(void *sess, int ne0, int ne1, int ne2, int ggml_type, size_t buf_offset);
void *tnn_input_1d_persistent_mmap(void *sess, int n, int ggml_type, size_t buf_offset);

/* tinynn_ggml.h:157-400 — forward and backward ops */
void *tnn_matmul(void *sess, void *a, void *b);          /* ggml_mul_mat: a [K,M,..] (f32 or Q8_0), b [K,N,..] -> [M,N,..] */
void *tnn_out_prod(void *sess, void *a, void *b);        /* ggml_out_prod: r[n][m] = sum_k a[k][m] b[k][n] */
void *tnn_add(void *sess, void *a, void *b);             /* b broadcast over a */
void *tnn_sub(void *sess, void *a, void *b);
void *tnn_mul(void *sess, void *a, void *b);
void *tnn_scale(void *sess, void *a, double s);
void *tnn_silu(void *sess, void *a);
void *tnn_silu_back(void *sess, void *x, void *dy);
void *tnn_swiglu_split(void *sess, void *gate, void *up);
void *tnn_rms_norm(void *sess, void *x, void *gamma_row, double eps);
void *tnn_rms_norm_back(void *sess, void *x, void *dy, double eps);
void *tnn_rope_ext(void *sess, void *a, void *pos, int n_dims, double freq_base, double freq_scale,
                   double ext_factor, double attn_factor, double beta_fast, double beta_slow, void *freq_factors);
void *tnn_rope_ext_back(void *sess, void *dy, void *pos, int n_dims, double freq_base, double freq_scale,
                        double ext_factor, double attn_factor, double beta_fast, double beta_slow,
                        void *freq_factors);
void *tnn_softmax(void *sess, void *a);
void *tnn_soft_max_ext(void *sess, void *a, void *mask, double scale, double max_bias);
void *tnn_softmax_back(void *sess, void *a, void *dy);
void *tnn_diag_mask_inf(void *sess, void *a, int n_past);
void *tnn_transpose(void *sess, void *a);
void *tnn_permute(void *sess, void *a, int axis0, int axis1, int axis2, int axis3);
void *tnn_cont(void *sess, void *a);
void *tnn_cont_2d(void *sess, void *a, int ne0, int ne1);
void *tnn_reshape_2d(void *sess, void *a, int ne0, int ne1);
void *tnn_reshape_3d(void *sess, void *a, int ne0, int ne1, int ne2);
void *tnn_view_1d(void *sess, void *a, int ne0, long offset);
void *tnn_view_2d(void *sess, void *a, int ne0, int ne1, long nb1, long offset);
void *tnn_view_3d(void *sess, void *a, int ne0, int ne1, int ne2, long nb1, long nb2, long offset);
void *tnn_concat(void *sess, void *a, void *b, int dim);
void *tnn_get_rows(void *sess, void *table, void *idx);
void *tnn_get_rows_back(void *sess, void *d_out, void *idx, void *table_shape);
/* MoE primitives (tinynn_ggml.h:161-175, ggml semantics; forward only, as the
 * reference's graphs use them). tnn_mul_mat_id: as [d_in, d_out, n_experts]
 * (f32 or Q8_0), b [d_in, 1 or n_used, T] f32, ids i32 [n_used, T] ->
 * [d_out, n_used, T], one product with expert ids[u, t] per (u, t); an id
 * outside [0, n_experts) gives zeros. tnn_add_id: a [n0, n1, n2] + b[:, ids]
 * with ids i32 [n1, n2]. tnn_argsort: i32 indices that sort each row of a
 * (descending != 0: largest first), equal values by index; tnn_top_k: the
 * indices of each row's k largest values, largest first. NULL on a shape or
 * type mismatch. */
void *tnn_mul_mat_id(void *sess, void *as, void *b, void *ids);
/* KV-cache graph primitives (tinynn_ggml.h:311-342, 574). tnn_null_ptr: NULL.
 * tnn_detach: a itself for the forward, a cut for the backward.
 * tnn_cpy: a's elements (f32 or i32) written into b's storage; returns b's
 * view, so reads of b that run after it see them. tnn_set_rows: rows idx[i]
 * (i32) of a := rows i of b; returns a's view. tnn_upload_causal_mask: fills
 * f32 [hist, n_tok] with 0 where key j <= pos0 + token i, -inf elsewhere
 * (hist == pos0 + n_tok, else -2; wrong shape or type -3).
 * tnn_upload_cell_mask: the same over a pool of KV cells -- cell c is open
 * to token t when it belongs to t's sequence at a position <= t's, or is a
 * shared-prefix cell (owner -1) below t's shared length; owner -2 is free. */
void *tnn_null_ptr(void);
void *tnn_detach(void *sess, void *a);
void *tnn_cpy(void *sess, void *a, void *b);
void *tnn_set_rows(void *sess, void *a, void *b, void *idx);
int tnn_upload_causal_mask(void *sess, void *tensor, int hist, int n_tok, int pos0);
int tnn_upload_cell_mask(void *sess, void *tensor, int hi, int n_tok, const long *cell_owner, const long *cell_pos,
                         const long *tok_owner, const long *tok_pos, const long *tok_shared);
void *tnn_add_id(void *sess, void *a, void *b, void *ids);
void *tnn_argsort(void *sess, void *a, int descending);
void *tnn_top_k(void *sess, void *a, int k);
void *tnn_cross_entropy_loss(void *sess, void *a, void *b);
void *tnn_sum(void *sess, void *a);
void *tnn_sum_rows(void *sess, void *a);
void *tnn_opt_step_adamw(void *sess, void *a, void *grad, void *m, void *v, void *params);
/* tinynn_ggml.c:2044 -- p = p (1 - alpha wd) - alpha grad, params = [alpha, wd] */
void *tnn_opt_step_sgd(void *sess, void *a, void *grad, void *params);
/* tinynn_ggml.c:1335 (ggml_cast) -- to F32 (dtype 0) only: a copy of an F32
 * tensor, or the dequantised values of a Q8_0 one; NULL for other dtypes. */
void *tnn_cast(void *sess, void *a, int dtype);
/* tinynn_ggml.h:251 (inference, as in the reference): q [dh, Tq, H, B], k, v
 * [dh, Tk, KV, B], mask [Tk, >= Tq] or NULL -> [dh, H, Tq, B]; computed as
 * softmax(scale k^T q + mask) v on the tensor-core GEMM. NULL for
 * logit_softcap != 0 or max_bias != 0 (ALiBi). */
void *tnn_flash_attn_ext(void *sess, void *q, void *k, void *v, void *mask, double scale, double max_bias,
                         double logit_softcap);

/* tinynn_ggml.h:376-469 — programs and autograd */
void tnn_set_param(void *tensor);
void tnn_set_loss(void *tensor);
void tnn_set_output(void *tensor);
int tnn_add_to_graph(void *sess, void *tensor);
int tnn_realize(void *sess, void *result);
int tnn_build_forward_only(void *sess, void *result);
int tnn_build_backward(void *sess);
int tnn_extend_backward_graph(void *sess, void *node);
int tnn_realize_backward(void *sess);
void *tnn_tensor_grad(void *sess, void *tensor);
int tnn_compute(void *sess);
int tnn_reset_for_rebuild(void *sess);
/* tinynn_ggml.h:376 -- every node here keeps its own buffer: a no-op (0) */
int tnn_pin_all_graph_b_nodes(void *sess);

/* tinynn_ggml.h:527-532 — graph introspection */
int tnn_tensor_op(void *t);
const char *tnn_tensor_op_name(void *t);
void *tnn_tensor_src(void *t, int i);
int tnn_tensor_flags(void *t);
int tnn_graph_n_nodes(void *sess);
void *tnn_graph_node(void *sess, int i);

/* ===================================================================== */
/* Tensor I/O (tinynn/tinynn_ggml.h:486-537)                             */
/* ===================================================================== */
int tnn_upload_from_float_array(void *sess, void *tensor, const double *data, size_t n);
int tnn_upload_from_int_array(void *sess, void *tensor, const long *data, size_t n);
int tnn_download_to_f64_array(void *sess, void *tensor, double *dst, size_t n);
/* tinynn_ggml.h:471-484,563-567 -- a 16 MiB f32 host staging area per session:
 * element-wise set / get (f32, or i32 bits), bulk tnn_upload / tnn_download
 * of a whole tensor through it, and statistics over its first n floats. */
void tnn_scratch_set(void *sess, int idx, double v);
double tnn_scratch_get(void *sess, int idx);
void tnn_scratch_set_i32(void *sess, int idx, int value);
int tnn_scratch_get_i32(void *sess, int idx);
int tnn_upload(void *sess, void *tensor);
int tnn_download(void *sess, void *tensor);
double tnn_scratch_min_f32(void *sess, int n);
double tnn_scratch_max_f32(void *sess, int n);
double tnn_scratch_sum_abs_f32(void *sess, int n);
int tnn_scratch_nan_count_f32(void *sess, int n);
/* tinynn_ggml.h:493-497 -- the row-major (br x bc) matrix, transposed: its
 * column j becomes elements j*br .. j*br + br - 1 of the tensor. */
int tnn_upload_transposed_f64(void *sess, void *tensor, const double *src, int br, int bc);
int tnn_tensor_ne0(void *t);
int tnn_tensor_ne1(void *t);
int tnn_tensor_ne2(void *t);
int tnn_tensor_ne3(void *t);
size_t tnn_tensor_nbytes(void *t);
int tnn_tensor_nelements(void *t);
const char *tnn_tensor_name(void *t);
void tnn_tensor_set_name(void *t, const char *name);
int tnn_tensor_dtype(void *t);

/* ===================================================================== */
/* Decode with a KV cache (inference forward)                            */
/* ===================================================================== */
/* The per-token forward toy's KV engine runs for `toy infer` / `serve`
 * (lib/toy/llm/engine/llama_kv_engine.rb: build_block_step :1687,
 * build_attention_qhead_step :2132, SmolLM2KVStepResult.decode_step :2350 /
 * decode_batch :2381, enable_kv_q8! :359; its fused attention is
 * tnn_flash_attn_ext, tinynn/tinynn_ggml.c:1583-1598) on the weights of the
 * session's realised step engine (Q8_0 base or f32, as realised; adapters are
 * not applied). n_seq sequences (1-8 or 16) decode in lockstep, each with its
 * own cache of max_T positions; kv_type 0 keeps K and V in f32, 8 in Q8_0
 * (ggml's quantiser, per head and position in blocks of 32).
 * Returns 0, -1 for a bad argument, -2 without tb2_llama_realize. */
int tb2_kv_realize(void *sess, int max_T, int n_seq, int kv_type);
/* Clear every cache (a new set of sequences). */
int tb2_kv_reset(void *sess);
/* One decode step: token[b] at position positions[b] of sequence b (its
 * cache holds positions 0 .. positions[b] - 1), K / V appended, logits of the
 * next token for every sequence; copied to logits [n_seq][vocab] when
 * non-NULL. The first call captures the step as a CUDA graph. */
int tb2_kv_decode(void *sess, const long long *tokens, const long long *positions, int n_seq, float *logits);
/* The last step's logits [n_seq][vocab] (n = n_seq * vocab). */
int tb2_kv_logits(void *sess, float *out, long long n);
/* steps replays of the last decode step's graph timed by CUDA events (ms);
 * the kernels launched per step. */
int tb2_kv_run(void *sess, int steps, float *ms);
int tb2_kv_launches(void *sess);
int tb2_kv_free(void *sess);

/* ===================================================================== */
/* GGUF files (tinynn/tinynn_gguf.h; writer tinynn/tinynn_ggml.h:538-545) */
/* ===================================================================== */
/* Host-side: a GGUF v2/v3 reader that maps the file read-only in place and a
 * writer. The loaders and the checkpoint writer of toy's training runs
 * (lib/toy/train/toy_gguf_writer.rb) make these calls. */

/* tinynn_gguf.h:89-94 -- the mapping returned by tnn_gguf_mmap_base is
 * followed by at least this many readable zero bytes past tnn_gguf_mmap_size. */
#define TNN_GGUF_MMAP_TAIL 4096
/* tinynn_gguf.h:15 (tinynn_gguf.c:198-280): parse and map; NULL on error. */
void *tnn_gguf_load(const char *path);
void tnn_gguf_free(void *handle);
/* tinynn_gguf.h:45-51: tensor directory (ne0 fastest; ggml type ids: 0 F32,
 * 1 F16, 8 Q8_0, 30 BF16). */
int tnn_gguf_n_tensors(void *handle);
const char *tnn_gguf_tensor_name(void *handle, int i);
int tnn_gguf_tensor_ne(void *handle, int i, int dim);
int tnn_gguf_tensor_type(void *handle, int i);
size_t tnn_gguf_tensor_nbytes(void *handle, int i);
/* tinynn_gguf.h:61-62: values as doubles (F32, F16, BF16, Q8_0 dequantised:
 * scale * quant); 0, or -1 on a bad index, type or element count n. */
int tnn_gguf_read_f32_to_doubles(void *handle, int i, double *out, size_t n);
int tnn_gguf_tensor_is_quantized(void *handle, int i);
/* tinynn_gguf.h:67-86: metadata (-1 / 0.0 / NULL when missing or of another type). */
int tnn_gguf_get_u32(void *handle, const char *key);
double tnn_gguf_get_f32(void *handle, const char *key);
int tnn_gguf_get_bool(void *handle, const char *key);
const char *tnn_gguf_get_str(void *handle, const char *key);
const char *tnn_gguf_arch_prefix(void *handle);
/* tinynn_gguf.c:520-554: 1 when 2-D linears are stored ne=[in, out] (the
 * toy.ggml_native flag, else the stored shape of blk.0.ffn_gate.weight). */
int tnn_gguf_is_native_layout(void *handle);
int tnn_gguf_arr_n(void *handle, const char *key);
const char *tnn_gguf_arr_str(void *handle, const char *key, int i);
int tnn_gguf_arr_i32(void *handle, const char *key, int i);
/* tinynn_gguf.h:95-97: the mapped file, its size, a tensor's absolute offset. */
void *tnn_gguf_mmap_base(void *handle);
size_t tnn_gguf_mmap_size(void *handle);
size_t tnn_gguf_tensor_file_offset(void *handle, int i);
/* tinynn_gguf.h:197: index of a tensor by name, or -1. */
int tnn_gguf_find_index(void *handle, const char *name);
/* tinynn_gguf.h:103: a GGUF with one 2x3 f32 tensor "demo.tensor" = 1..6. */
int tnn_gguf_write_demo_file(const char *path);

/* tinynn_ggml.h:538-545: the checkpoint writer. add_tensor copies a session
 * tensor to the host when called: a step-program parameter (f32 values, or a
 * frozen projection's Q8_0 blocks verbatim) or an f32 primitive-graph node. */
void *tnn_gguf_w_init(void);
void tnn_gguf_w_set_str(void *ctx, const char *key, const char *val);
void tnn_gguf_w_set_u32(void *ctx, const char *key, int val);
void tnn_gguf_w_set_f32(void *ctx, const char *key, double val);
void tnn_gguf_w_set_bool(void *ctx, const char *key, int val);
void tnn_gguf_w_add_tensor(void *ctx, void *t);
int tnn_gguf_w_finalize(void *ctx, const char *path);
void tnn_gguf_w_free(void *ctx);
/* Host-data tensors for the writer (no counterpart in the reference): f32
 * [ne1][ne0], or Q8_0 blocks [ne1][ne0/32*34]. 0 or -1. */
int tb2_gguf_w_add_f32(void *ctx, const char *name, int ne0, int ne1, const float *data);
int tb2_gguf_w_add_q8_0(void *ctx, const char *name, int ne0, int ne1, const void *blocks);

/* The step engine's weights from a GGUF (replaces realize_for_mmap's
 * per-tensor copies, tinynn_gguf.c:612-682, for the fused step): every
 * parameter is found by its GGUF name; a frozen Q8_0 projection takes the
 * file's blocks verbatim (split once into the GEMM's quant / scale layout),
 * f32 / f16 / bf16 / Q8_0 values go to the f32 arenas (Q8_0 dequantised
 * where the step trains the tensor), toy's legacy transposed layout is
 * transposed back, adapters absent from the file keep their init, and the
 * per-head LoRA-Q tensors may come under toy's per-head names
 * (blk.N.attn_q.head_H.lora_{a,b}.weight). flags bit 0: also load Adam
 * moments from "<name>.m" / "<name>.v"; bit 1: a partial file (a checkpoint):
 * tensors it lacks keep their values. Returns the tensor count loaded, -1 for
 * a missing or mis-shaped tensor (named on stderr), -2 before realize. */
int tb2_llama_load_gguf(void *sess, void *gguf, int flags);
/* A checkpoint of the step engine as GGUF v3 with the metadata toy's writer
 * records: what bit 0 is implied (trainable tensors); bit 1 adds the frozen
 * tensors (Q8_0 blocks verbatim); bit 2 adds Adam moments as "<name>.m" /
 * "<name>.v"; bit 3 writes per-head LoRA-Q stacked instead of one pair per
 * head under toy's names. 0 or negative. */
int tb2_llama_save_gguf(void *sess, const char *path, int what);

#ifdef __cplusplus
}
#endif

#endif /* TOY_B200_H */
