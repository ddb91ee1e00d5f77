// Tensor-core GEMM on split-bf16 operands (sm_100a, tcgen05 + TMA + TMEM).
//
// For every batch z:  D_z[m, n] = epilogue( sum_k A_z[m, k] * B_z[n, k] )
//
// Operands are stored as two bf16 planes, hi = rn_bf16(x) and lo = rn_bf16(x - hi),
// which together carry x to ~2^-17 relative. With `split` set the kernel issues
// three UMMAs per k-step (hi*hi + lo*hi + hi*lo) into one f32 TMEM accumulator,
// giving products accurate to ~2^-16 -- the precision the training step needs to
// hold gradients within 1e-3 relative L2 of an fp64 evaluation. Without `split`
// the lo planes are ignored (one UMMA per k-step, plain bf16).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace tb2 {

// One GEMM operand as it sits in HBM.
//  mn_major = 0: stored rows are the M (or N) index, K is contiguous  -> [MN][ld]
//  mn_major = 1: stored rows are the K index, M (or N) is contiguous  -> [K][ld]
// Storage may hold several batches (nbatch, batch_stride). The batch a GEMM
// batch z reads is (z / bdiv1) * bmul1 + ((z % bdiv1) / bdiv2) * bmul2, which
// covers plain batching (bdiv1 = 1, bmul1 = 1) and grouped-query sharing of one
// K/V head by several query heads.
struct Operand {
  const __nv_bfloat16* hi = nullptr;
  const __nv_bfloat16* lo = nullptr;
  int mn_major = 0;
  long long ld = 0;            // elements between stored rows
  int rows = 0;                // stored rows per batch
  int cols = 0;                // stored columns (contiguous extent)
  long long batch_stride = 0;  // elements between batches
  int nbatch = 1;
  int bdiv1 = 1, bmul1 = 1, bdiv2 = 1, bmul2 = 0;
  // Q8_0 operand (B of a non-batched GEMM only): instead of planes, the int8
  // quants of the stored [rows][cols] matrix (row stride ld bytes) and one fp16
  // scale per 32 consecutive columns of a row ([rows][cols / 32]), so element
  // (r, c) = scale[r][c / 32] * q8[r][c] -- Q8_0 blocks with the scales split
  // off. The GEMM dequantises tiles in shared memory.
  const int8_t* q8 = nullptr;
  const uint16_t* q8_scale = nullptr;
  // B operand only: the planes are kept resident in the L2's persisting
  // set-aside by their producer (written with the evict-last policy); the GEMM
  // loads them with the same policy so reading does not demote them.
  int l2_keep = 0;
};

enum EpiMode : int {
  kEpiStoreF32 = 0,   // out = alpha * acc
  kEpiAccumF32 = 1,   // out += alpha * acc
  kEpiResidF32 = 2,   // out = res + alpha * acc
  kEpiStoreSplit = 3, // (out_hi, out_lo) = split(alpha * acc)
  kEpiStoreBoth = 4,  // out = alpha * acc and (out_hi, out_lo) = split(alpha * acc)
  kEpiRopeQKV = 5,    // fused q|k|v projection: + bias, RoPE (NEOX) on q and k, head-major planes (Epilogue::rope)
  kEpiSwiGLU = 6,     // fused gate|up projection with paired B rows: out = gate|up f32, (out_hi, out_lo) = silu(g) u
  kEpiStoreLse = 7,   // out = acc (logits), and per row and 64-column group the pair (max, sum exp(x - max))
                      // written to lse_part[(n / 64) * M + m] (the vocab-chunked logsumexp of a cross-entropy)
};

// Low-rank adapter added to the accumulator before the epilogue mode (the
// LoRA splice y += s B (A x) of the base projection): for the output columns
// [c0, c0 + width) (multiples of 32), v(m, c) += scale * sum_j u[m][j] * bt[j][c - c0],
// with u = A x saved as f32 [M][r] and bt = B^T as f32 [r][width].
struct LoraAddend {
  const float* u = nullptr;
  const float* bt = nullptr;
  int c0 = 0, width = 0, r = 0;
  float scale = 0.f;
};
constexpr int kMaxLoraAddends = 3;

// kEpiRopeQKV: the output columns are the (H + 2 KV) heads of width dh of one
// token (row m = b * T + t); after bias the q and k heads are rotated by the
// RoPE angle of pos[m] (cos / sin table cs [tab_rows][dh / 2] of float2) and
// every head is written as planes to Q [B][H][T][dh], K and V [B][KV][T][dh].
struct RopeOut {
  const int* pos = nullptr;
  const float* cs = nullptr;
  int tab_rows = 0;
  const float* bias = nullptr;
  __nv_bfloat16 *q_hi = nullptr, *q_lo = nullptr, *k_hi = nullptr, *k_lo = nullptr, *v_hi = nullptr, *v_lo = nullptr;
  int T = 1, H = 0, KV = 0, dh = 64;
};

// Output element (z, m, n) lives at
//   (z / z_div) * z_s1 + (z % z_div) * bstride
//   + (m / m_div) * m_s1 + (m % m_div) * m_s0 + (n / n_div) * n_s1 + (n % n_div)
// (n_div must be a multiple of 32). Row-major [M][ldc] is m_div = n_div = huge,
// m_s0 = ldc; a head-major scatter uses n_div = head width.
struct Epilogue {
  int mode = kEpiStoreF32;
  float alpha = 1.0f;
  // optional device factor: the epilogue's multiplier is alpha * *alpha_dev
  // (the inverse of an operand scale that changes from step to step)
  const float* alpha_dev = nullptr;
  float* out = nullptr;
  const float* res = nullptr;
  __nv_bfloat16* out_hi = nullptr;
  __nv_bfloat16* out_lo = nullptr;
  long long bstride = 0;
  int z_div = 1 << 30;
  long long z_s1 = 0;
  int m_div = 1 << 30;
  long long m_s1 = 0, m_s0 = 0;
  int n_div = 1 << 30;
  long long n_s1 = 0;
  // fused extras (kEpiStoreF32 / AccumF32 / ResidF32 / RopeQKV / SwiGLU, no K splits)
  int n_lora = 0;
  LoraAddend lora[kMaxLoraAddends];
  RopeOut rope;
  // kEpiSwiGLU: B rows are paired -- tile columns [0, BN/2) are gate rows
  // n0/2 .., [BN/2, BN) the matching up rows pair_off + n0/2 .. (pair_off = ff);
  // out (f32 [M][2 ff], m_s0 = 2 ff) keeps gate | up for the backward and
  // (out_hi, out_lo) ([M][ff]) get silu(gate) * up.
  int pair_off = 0;
  // kEpiStoreLse: [ceil(N / 64)][M] (max, sum exp) pairs
  float2* lse_part = nullptr;
};

struct GemmDesc {
  int M = 0, N = 0, K = 0, batch = 1;
  bool split = true;
  // with split = false: the operands' hi arrays hold fp16 (not bf16) values,
  // multiplied in one kind::f16 pass with fp16 inputs (the tensor maps copy
  // 2-byte elements either way; zero fill is 0 in both formats)
  bool f16 = false;
  int splits = 0;   // K ranges reduced through the workspace; 0 = choose from the tile count
  int causal = 0;   // 1: skip tiles with n0 > m0 + 127; 2: clamp K to m0 + 128 (zero beyond)
  int max_ctas = 0; // persistent CTAs at most (0: one per SM); the units are the same, walked by fewer CTAs
  int tile_bn = 0;  // output tile width for this GEMM (0: the launch plan's choice; else as gemm_set_tile_width)
  int alone = 0;    // 1: nothing heavy runs beside it -- plan for a GEMM that has the GPU to itself
  // Grouped product (the experts of a mixture-of-experts block): group_mtiles
  // M tiles listed in device memory as triples (group, first row, end row),
  // rows of at most 128 per tile; a tile's rows read A (unbatched, rows of the
  // whole product) and batch `group` of B, and write only rows below its end.
  // M is the total row count; no K splits, no CTA pairs, batch 1.
  const int* group_tiles = nullptr;
  int group_mtiles = 0;
  Operand a, b;
  Epilogue epi;
};

// Split-K workspace: f32 partial tiles, summed by a separate reduce launch.
// One GEMM at a time may use it.
struct GemmScratch {
  float* ws = nullptr;
  long long ws_floats = 0;
};

// Enqueue the GEMM on `stream`. Returns 0 on success, negative on a rejected
// shape/alignment (nothing launched). `dev_err` is a device int the kernel sets
// to a DeviceError code if one of its bounded waits gives up.
int gemm_launch(const GemmDesc& d, const GemmScratch& scratch, int* dev_err, cudaStream_t stream);
// Kernels the calling thread's last gemm_launch enqueued: 1, or 2 with a
// split-K reduction (0 after a rejected call).
int gemm_last_launches();
// The number of K splits gemm_launch runs for an explicit request of
// `ksplits` (d.splits is ignored): 1 when the shape allows no split (causal,
// batched, fused or logsumexp epilogues), else ksplits capped at the k-block
// count. The workspace then has to hold that many M x N partial tiles.
int gemm_effective_splits(const GemmDesc& d, int ksplits);

// GEMMs on CTA pairs (cta_group::2: 256-row units, each CTA holding half of
// the B tile): -1 (the default) for the shapes where pairs measured faster
// (both operands K-major, N >= 2048), 0 never, 1 wherever the shape allows.
// Process-wide; returns 0 or -1 for a bad mode.
int gemm_set_pair_mode(int mode);
// Output tile width of every later GEMM: 0 (default) by the cost model, else
// 64 / 128 / 192 / 256 wherever the shape allows it. Returns the previous
// width, or -1 for another value.
int gemm_set_tile_width(int bn);

// TMA map over one bf16 plane laid out as `o` describes: dims {cols, rows,
// nbatch}, box {64, box_rows, 1}, 128-byte swizzle. Rows past `rows` inside a
// batch read as zero. Returns 0 or a negative alignment / driver error.
int make_plane_map(CUtensorMap* map, const __nv_bfloat16* base, const Operand& o, int box_rows);

// Row-major helpers used by the step program.
inline Operand op_rowmajor(const __nv_bfloat16* hi, const __nv_bfloat16* lo, int rows, int cols, long long ld,
                           int mn_major) {
  Operand o;
  o.hi = hi; o.lo = lo; o.mn_major = mn_major; o.ld = ld; o.rows = rows; o.cols = cols;
  o.batch_stride = (long long)rows * ld; o.nbatch = 1; o.bdiv1 = 1; o.bmul1 = 0; o.bdiv2 = 1; o.bmul2 = 0;
  return o;
}

inline Epilogue epi_rowmajor(int mode, float* out, long long ldc, float alpha = 1.0f) {
  Epilogue e;
  e.mode = mode; e.out = out; e.alpha = alpha; e.m_s0 = ldc;
  return e;
}

}  // namespace tb2
