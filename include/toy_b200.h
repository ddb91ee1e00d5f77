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
} tb2_operand;

/* Epilogue: mode 0 store f32, 1 accumulate f32, 2 residual (out = res + acc),
 * 3 store split-bf16 planes, 4 store f32 and split planes. Output element
 * (z, m, n) is at z*bstride + (m/m_div)*m_s1 + (m%m_div)*m_s0 + (n/n_div)*n_s1 + n%n_div. */
typedef struct tb2_epilogue {
  int mode;
  float alpha;
  float *out;
  const float *res;
  void *out_hi;
  void *out_lo;
  long long bstride;
  int m_div;
  long long m_s1, m_s0;
  int n_div;
  long long n_s1;
} tb2_epilogue;

/* D_z[m,n] = epilogue(sum_k A_z[m,k] B_z[n,k]) on tcgen05 tensor cores.
 * split = 1: 3 MMAs per k-step over (hi, lo) planes (~fp32 accuracy);
 * split = 0: plain bf16 (hi planes only).
 * Replaces the arithmetic behind tnn_matmul / tnn_out_prod
 * (tinynn/tinynn_ggml.c:815-835) for the training step. */
int tb2_gemm(int M, int N, int K, int batch, int split, const tb2_operand *a, const tb2_operand *b,
             const tb2_epilogue *epi, void *stream);

/* hi = rn_bf16(x), lo = rn_bf16(x - hi) for n f32 values. */
int tb2_split_f32(const float *x, void *hi, void *lo, size_t n, void *stream);

/* Read and clear the device-side error word of the current device
 * (non-zero when a kernel's bounded wait gave up). Synchronises the device. */
int tb2_device_error(void);

/* Library version string. */
const char *tb2_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TOY_B200_H */
