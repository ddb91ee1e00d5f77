// Low-rank adapter products of the LoRA / QLoRA step on CUDA cores (f32).
//
// With rank r <= 64 every product is skinny (one side is r wide), so these are
// bandwidth-bound kernels rather than tensor-core tiles: reading the activation
// or gradient once dominates, and a tcgen05 GEMM would spend its time filling
// and draining a 128-row pipeline for 8 output columns.
//
// Layouts: activations / gradients are split planes [N][ld] (hi + lo carry the
// f32 value); u, du are f32 [N][r]; adapter matrices are f32 in the layouts the
// kernels name ([r][K] means r rows of K contiguous values).
#pragma once
#include "gemm.cuh"
#include "kernels.cuh"

namespace tb2 {

constexpr int kLoraMaxRank = 64;

// out[n][j] = alpha * sum_k X[n][k] * W[j][k]     (X planes [N][ldx], W [r][K]).
// With bt_out set, the same launch also writes bt_out[j][c] = b_src[c][j]
// (b_src [b_rows][r]): an adapter's B transposed for the splice.
int launch_lora_down(Planes X, long long ldx, int N, int K, const float* W, int r, float alpha, float* out,
                     cudaStream_t st, const float* b_src = nullptr, int b_rows = 0, float* bt_out = nullptr);

// The whole adapter backward of one projection in three launches (r <= 16):
// a row pass du = s dY B (into du [N][r]) and dX(n, k) += sum_j du[n][j] A[j][k]
// (epilogue addressing, as lora_up); one launch of token-chunk partials of
// dB = s dY^T u ([d_out][r]) and dA = du^T X ([r][d_in]); their fixed-order
// sum. dY planes [N][ldy] (d_out columns), X planes [N][ldx], U = u [N][r],
// bt = B^T [r][d_out], A [r][d_in]; `part` holds lora_bwd_partial_floats.
constexpr int kLoraBwdMaxRank = 16;
long long lora_bwd_partial_floats(int N, int d_out, int d_in, int r);
int launch_lora_backward(Planes dY, long long ldy, int d_out, Planes X, long long ldx, int d_in, const float* U,
                         const float* bt, const float* A, int r, float s, int N, const Epilogue& edx, float* du,
                         float* part, float* dB, float* dA, cudaStream_t st);

// ---- adapter groups: the adapters whose base projections form one GEMM
// (q|k|v, gate|up, or a single projection) share one launch per pass.
constexpr int kLoraMaxSegs = 3;

// One adapter of a group for the down pass out[n][j] = alpha * sum_k
// X[n][col_off + k] * w[j][k] (k < width); with bt set the launch also writes
// bt[j][c] = b_src[c][j] for c < b_rows.
//
// With ext_col >= 0 the results are also written as planes into the row's own
// buffer (X for the down pass, h for the fused RMSNorm) at columns ext_col + j:
// the extra reduction columns through which the base GEMM adds the adapter
// (y = [X | u] [W | s B]^T, dX = [dY | du] [W ; A]).
struct LoraSeg {
  int col_off = 0, width = 0;
  const float* w = nullptr;
  float alpha = 1.0f;
  float* out = nullptr;
  const float* b_src = nullptr;
  int b_rows = 0;
  float* bt = nullptr;
  int ext_col = -1;
};
struct LoraSegs {
  LoraSeg s[kLoraMaxSegs];
  int n = 0;
  // launch_lora_down_group internals for adapters whose w exceeds shared
  // memory (the pass then runs over column chunks): w's row stride (0: width),
  // add into out instead of storing, write the extra-column planes (last chunk)
  int ldw = 0, accumulate = 0, write_ext = 1;
};
// Every adapter of the group in one launch (r <= 16; X planes [N][ldx]); an
// adapter set whose w does not fit in shared memory runs as several launches
// over column chunks of the same width, summed in chunk order.
int launch_lora_down_group(Planes X, long long ldx, int N, int r, const LoraSegs& segs, cudaStream_t st);

// Weight gradients of a group: for adapter i, dB_i[c][j] = s sum_n
// dY[n][col_off_i + c] u_i[n][j] (c < width_i) and dA_i[j][k] = sum_n du_i[n][j]
// X[n][k] (k < d_in), as token-chunk partials in one launch and their
// fixed-order sum in a second (r <= 16).
struct LoraWgSeg {
  int col_off = 0, width = 0;
  const float* u = nullptr;
  const float* du = nullptr;
  float* dB = nullptr;   // [width][r]
  float* dA = nullptr;   // [r][d_in]
};
struct LoraWgGroup {
  LoraWgSeg s[kLoraMaxSegs];
  int n = 0;
};
long long lora_group_partial_floats(int N, int r, int d_in, int total_width, int n_adapters);

// The same weight gradients on tensor cores for wide groups (the GEMMs
// DA = X^T [du_0 | ..] and DB = dY^T [u_0 | ..] run by the caller):
// launch_lora_pack_planes lays the group's u or du vectors ([N][r] f32 each)
// side by side as split planes [N][R] (zero past n r columns, R even);
// launch_lora_wg_extract scatters DA [d_in][R] into every dA [r][d_in] and the
// diagonal blocks of DB [sum of widths][R] (the group's output columns in
// order) into every dB [width][r], times s.
struct LoraPackSrc {
  const float* p[kLoraMaxSegs] = {};
  int n = 0;
};
int launch_lora_pack_planes(const LoraPackSrc& src, int N, int r, int R, Planes out, cudaStream_t st);

// Tensor-core down passes of a wide group (the caller runs D = X W^T with the
// packed W): launch_lora_pack_w writes split planes W [R][K] whose rows
// i r + j hold adapter i's row j over columns [koff_i, koff_i + w_i) -- from
// A_i [r][w_i] (trans = 0) or from B_i [w_i][r] read transposed (trans = 1) --
// and zero elsewhere; launch_lora_scatter_u writes out_i[n][j] =
// alpha D[n][i r + j] ([N][r] each) and, with ext_col_i >= 0, the same values
// as planes into X[n][ext_col_i + j].
struct LoraPackW {
  const float* p[kLoraMaxSegs] = {};
  int koff[kLoraMaxSegs] = {}, w[kLoraMaxSegs] = {};
  int n = 0, r = 0, trans = 0;
};
int launch_lora_pack_w(const LoraPackW& src, int R, int K, Planes out, cudaStream_t st);
struct LoraScatterU {
  float* out[kLoraMaxSegs] = {};
  int ext_col[kLoraMaxSegs] = {-1, -1, -1};
  int n = 0, r = 0;
  float alpha = 1.f;
  Planes X{};
  long long ldx = 0;
};
int launch_lora_scatter_u(const float* D, int N, int R, const LoraScatterU& dst, cudaStream_t st);
static_assert(kLoraMaxSegs == 3, "LoraScatterU::ext_col lists one initialiser per segment");
int launch_lora_wg_extract(const float* DA, const float* DB, int d_in, int r, int R, float s, const LoraWgGroup& g,
                           cudaStream_t st);
int launch_lora_wgrad_group(Planes dY, long long ldy, Planes X, long long ldx, int d_in, int N, int r, float s,
                            const LoraWgGroup& g, float* part, cudaStream_t st);

// Y(n, c) += alpha * sum_j U[n][j] * W[j][c]     (U [N][r], W [r][C]); Y(n, c)
// is e.out[epi offset of (z = 0, m = n, n = c)] (gemm.cuh Epilogue addressing;
// e.n_div must be a multiple of 4, rows 16-byte aligned).
int launch_lora_up(const float* U, int N, int r, const float* W, int C, float alpha, const Epilogue& e,
                   cudaStream_t st);

// G(c, j) = alpha * sum_n Big[n][c] * S[n][j]    (Big planes [N][ldb], S [N][r])
// written to out[c * o_sc + j * o_sj]; token chunks are summed in a fixed
// order through `partial` (lora_wgrad_partial_floats floats).
long long lora_wgrad_partial_floats(int N, int C, int r);
int launch_lora_wgrad(Planes Big, long long ldb, const float* S, int N, int C, int r, float alpha, float* out,
                      long long o_sc, long long o_sj, float* partial, cudaStream_t st);

// Wt[j][c] = W[c][j]   (W [C][r] -> Wt [r][C])
int launch_lora_transpose(const float* W, int C, int r, float* Wt, cudaStream_t st);

}  // namespace tb2
