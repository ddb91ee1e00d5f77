// Bandwidth-bound kernels of the training step (launch wrappers). All inputs
// and outputs are device pointers; "planes" means a (hi, lo) pair of bf16
// arrays carrying an f32 value as hi + lo (see gemm.cuh).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace tb2 {

using bf16 = __nv_bfloat16;

struct Planes {
  bf16* hi = nullptr;
  bf16* lo = nullptr;
  // Optional fp16 copy of the same values at the same element offsets (the
  // operands of one-pass fp16 weight-gradient GEMMs): f16[i] = rn_f16(x *
  // *f16_scale), saturated to +-65504 (no scale pointer: x itself). Kernels
  // that write gradients also raise *f16_amax to max |x| of what they wrote
  // (unscaled, as f32 bits) when it is set.
  __half* f16 = nullptr;
  const float* f16_scale = nullptr;
  unsigned* f16_amax = nullptr;
};

// hi = rn_bf16(x), lo = rn_bf16(x - hi)
int launch_split_f32(const float* x, bf16* hi, bf16* lo, long long n, cudaStream_t st);

// x0[n, :] = E[ids[n], :]   (ggml get_rows)
int launch_embed_gather(const float* E, const int* ids, float* x0, int N, int d, cudaStream_t st);

// dE[id, :] += sum of dx rows with that id, in a fixed order: `order` lists the
// rows grouped by id, seg_start[k]..seg_start[k+1] is the k-th group (ggml get_rows_back).
// The segment count is read from device memory (*nseg_dev) so a captured graph
// stays valid for any token batch; max_seg bounds the grid.
int launch_embed_scatter(const float* dx, const int* order, const int* seg_start, const int* seg_id,
                         const int* nseg_dev, int max_seg, float* dE, int d, cudaStream_t st);

// h = rmsnorm(x) * gamma written as planes (ggml rms_norm + mul).
int launch_rmsnorm_fwd(const float* x, const float* gamma, Planes h, int N, int d, float eps, cudaStream_t st,
                       long long ldh = 0);   // h rows ldh apart (0: d)

// dx = dres + rms_norm_back(x, dh * gamma) (f32, may alias dres) and its planes;
// per-block partial sums of dh * x * rrms into gpart[nblk][d] (for dgamma;
// none when gpart is null).
struct LoraSegs;
// launch_rmsnorm_fwd plus, in the same pass over each row, u_a = h A_a^T for
// the adapters in g (all reading the whole row: col_off 0, width d; A_a [r][d];
// rank <= 16) and their B^T copies; h rows are ldh apart (0: d), and an
// adapter with ext_col >= 0 also gets u_a as planes in h's columns ext_col + j.
// Returns -2 for a width it has no variant for (the caller then runs the two
// passes).
int launch_rmsnorm_fwd_lora(const float* x, const float* gamma, Planes h, int N, int d, float eps, int r,
                            const LoraSegs& g, cudaStream_t st, long long ldh = 0);
int launch_rmsnorm_bwd(const float* x, const float* dh, const float* gamma, const float* dres, float* dx,
                       Planes dxp, float* gpart, int nblk, int N, int d, float eps, cudaStream_t st,
                       long long ldp = 0);   // dxp rows ldp apart (0: d)
// gout[c] = (accumulate ? gout[c] : 0) + sum_b gpart[b][c]
int launch_colsum(const float* gpart, int nblk, int d, float* gout, int accumulate, cudaStream_t st);
int rmsnorm_bwd_blocks();

// RoPE (NEOX) on the fused q|k|v projection output qkv [N][(H+2KV)*dh] (+ bias),
// written head-major as planes: Q [B][H][T][dh], K [B][KV][T][dh], V [B][KV][T][dh].
int launch_rope_qkv_fwd(const float* qkv, const float* bias, const int* pos, const float* cs_tab, int tab_rows,
                        Planes Q, Planes K, Planes V, int B, int T, int H, int KV, int dh, cudaStream_t st);
// Inverse: head-major f32 dQ, dK, dV -> token-major planes dqkv [N][(H+2KV)*dh]
// (rotation by -theta on dQ, dK).
int launch_rope_qkv_bwd(const float* dQ, const float* dK, const float* dV, const int* pos, const float* cs_tab,
                        int tab_rows, Planes dqkv, float* dqkv_f32, int B, int T, int H, int KV, int dh,
                        cudaStream_t st, long long ld_dqkv = 0);
// Same, with dQ / dK / dV given as sums of partial arrays added in index order:
// dQ of position t sums parts 0 .. t / q_tile (q_tile = 0: one part), q_pstride
// floats apart; dK and dV sum kv_parts parts, kv_pstride floats apart.
int launch_rope_qkv_bwd_sum(const float* dQ, long long q_pstride, int q_tile, const float* dK, const float* dV,
                            long long kv_pstride, int kv_parts, const int* pos, const float* cs_tab, int tab_rows,
                            Planes dqkv, float* dqkv_f32, int B, int T, int H, int KV, int dh, cudaStream_t st,
                            long long ld_dqkv = 0);

// P = softmax(S) over keys k <= q (rows of [Z][T][T]); masked entries 0.
int launch_softmax_causal_fwd(const float* S, Planes P, long long Z, int T, cudaStream_t st);
// dS = P * (dP - sum(P * dP)) * scale (ggml soft_max_back), as planes.
int launch_softmax_causal_bwd(Planes P, const float* dP, Planes dS, long long Z, int T, float scale,
                              cudaStream_t st);

// a = silu(gate) * up from gu [N][2*ff] (gate | up) -> planes [N][ff].
int launch_swiglu_fwd(const float* gu, Planes a, int N, int ff, cudaStream_t st,
                      long long lda = 0);   // a rows lda apart (0: ff)
// dgate = silu_back(gate, da * up), dup = da * silu(gate) -> planes [N][2*ff].
// dgu planes rows are ld_dgu apart (0: 2 ff).
int launch_swiglu_bwd(const float* gu, const float* da, Planes dgu, int N, int ff, cudaStream_t st,
                      long long ld_dgu = 0);

// Cross-entropy over rows of logits [N][V]: loss_rows[n] and dlogits planes
// ((softmax - y) / N). Labels are ids (label_ids, -1 = none) or, when
// label_dense != nullptr, a dense [N][V] distribution.
int launch_cross_entropy(const float* logits, const int* label_ids, const float* label_dense, float* loss_rows,
                         Planes dlogits, int N, int V, cudaStream_t st);
// The same for id labels, from the (max, sum exp) pairs of 64-column vocab
// chunks the LM-head GEMM wrote (kEpiStoreLse, lse_part [ceil(V / 64)][N]):
// one launch combines them per row into ms [N], one pass over the logits
// writes the gradient planes and loss rows.
int launch_cross_entropy_lse(const float* logits, const float2* lse_part, float2* ms, const int* label_ids,
                             float* loss_rows, Planes dlogits, int N, int V, cudaStream_t st);
// Gradient slots of the fp16 weight-gradient operands: scale[i] = 2^k with
// amax[i] * 2^k < 2^12 from the record of the previous step (kept when there
// is none), inv[i] = 2^-k, then amax[i] = 0.
int launch_f16_scale_update(unsigned* amax, float* scale, float* inv, int n, cudaStream_t st);
// loss = sum(loss_rows) / N   (single block, fixed order)
int launch_loss_reduce(const float* loss_rows, int N, float* loss, cudaStream_t st);

// AdamW over a flat arena (opt_step_adamw semantics, hp = device float[7]):
// g_eff = g * grad_scale; writes p, m, v and the planes of p.
int launch_adamw(float* p, const float* g, float* m, float* v, Planes pp, long long n, const float* hp,
                 float grad_scale, cudaStream_t st);

// Q8_0 blocks [rows][K/32*34] -> planes [rows][K] (value = d * q, exact in f32).
// When f32 != nullptr the exact f32 values are written there too.
int launch_q8_0_to_planes(const uint8_t* q, Planes out, float* f32, long long rows, int K, cudaStream_t st);
// f32 [rows][K] -> Q8_0 blocks (ggml quantize_row_q8_0_ref, bit-exact).
int launch_q8_0_quantize(const float* x, uint8_t* q, long long rows, int K, cudaStream_t st);
// The ring copy of one GEMM operand over a transformer block's frozen Q8_0
// projections (the q|k|v rows, o, the gate|up rows or down): planes
// [d_out + ext][d_in + ext], row pitch d_in + ext. Rows < d_out hold the
// dequantised W (columns < d_in; bit-identical to what the Q8_0 GEMM builds in
// shared memory: hi = rn(v), lo = rn(v - hi), v = scale * quant) and, in
// extension column d_in + 16 a + j, s * B_a[row - c0_a][j] for the rows adapter
// a covers; extension row d_out + 16 a + j holds A_a[j][:]; all else is 0. So
// [X | u] times the rows (K-major) is X W^T + s u B^T, and [dY | du] times the
// matrix read MN-major is dY W + du A (du = s dY B).
struct RingAdapter {
  const float* A = nullptr;   // [r][d_in]
  const float* B = nullptr;   // [width][r]
  int c0 = 0, width = 0;
};
//
// Block-diagonal adapter (bd_r > 0, one RingAdapter): the reference's LoRA-Q
// with one (A_h [bd_r][d_in], B_h [bd_w][bd_r]) pair per block of bd_w output
// rows. A is the blocks' A_h stacked ([R][d_in], R = width / bd_w * bd_r), B
// the B_h stacked ([width][bd_r]); extension column d_in + e of row c
// (h = (c - c0) / bd_w) holds s * B[c - c0][e - h bd_r] for e in
// [h bd_r, (h + 1) bd_r), extension row d_out + e holds A[e][:].
struct RingMat {
  const int8_t* qv = nullptr;     // quants [d_out][d_in]
  const uint16_t* qs = nullptr;   // fp16 scale bits [d_out * d_in / 32]
  bf16* hi = nullptr;
  bf16* lo = nullptr;
  int d_out = 0, d_in = 0, ext = 0, n_ad = 0, r = 0;
  int bd_r = 0, bd_w = 0;         // block-diagonal adapter: rank per block, rows per block
  float s = 0.f;
  long long chunk0 = 0;           // first 16-value chunk of this matrix in the launch
  RingAdapter ad[3];
};
constexpr int kRingMats = 4;
struct RingLayer {
  RingMat m[kRingMats];
  int n = 0;
  long long chunks = 0;           // 16-value chunks of all n matrices
  int keep = 0;                   // write the planes with the L2 evict-last policy (the ring stays L2-resident)
};
// Fills the matrices of one transformer block (the descriptors travel with
// the launch).
int launch_q8_0_ring(const RingLayer& desc, cudaStream_t st);
// Q8_0 blocks -> the GEMM's quant layout: the 32 int8 quants of block b at
// qv[32 b ..] and its fp16 scale bits at qs[b] (the same Q8_0 content, scales
// split off so quant tiles are TMA-loadable).
int launch_q8_0_split(const uint8_t* blocks, int8_t* qv, uint16_t* qs, long long nblocks, cudaStream_t st);

// The diagonal blocks of a block-diagonal adapter's dense gradient:
// out[h bw + c][j] = dense[h bw + c][h r + j] (dense [nb bw][nb r], out
// [nb bw][r]), h < nb, c < bw, j < r.
int launch_lora_blockdiag_take(const float* dense, int nb, int bw, int r, float* out, cudaStream_t st);

// out[c] = sum over rows of x[N][W] (fixed order), e.g. bias gradients.
int launch_colsum_rows(const float* x, int N, int W, float* out, cudaStream_t st);

// y[i] += x[i]
int launch_add_inplace(float* y, const float* x, long long n, cudaStream_t st);

}  // namespace tb2

namespace tb2 {
// ---- mixture-of-experts FFN and QK-RMSNorm (moe.cu)
int launch_moe_route(const float* logits, int N, int E, int K, int norm_topk, float* probs, int* idx, float* w,
                     cudaStream_t st);
int launch_moe_gather(Planes h, long long ldh, const int* perm, long long NK, int K, int d, Planes xs, cudaStream_t st);
int launch_moe_combine(const float* x1, const float* ye, const int* pos, const float* w, int N, int K, int d, float* x2,
                       cudaStream_t st);
int launch_moe_dy(const float* dy, const float* ye, const int* perm, const float* w, long long NK, int K, int d,
                  float* dw, Planes dye, cudaStream_t st);
int launch_moe_router_bwd(const float* probs, const int* idx, const float* w, const float* dw, int N, int E, int K,
                          int norm_topk, Planes dlog, cudaStream_t st);
int launch_moe_gather_sum(const float* dxs, const int* pos, int N, int K, int d, float* dh, cudaStream_t st);
int launch_rms_cols_fwd(float* x, long long ld, int c0, int width, const float* g, float eps, int N, float* pre,
                        cudaStream_t st);
int launch_rms_cols_bwd(Planes dy, long long ld, int c0, int width, const float* g, const float* pre, float eps, int N,
                        cudaStream_t st);
}  // namespace tb2
