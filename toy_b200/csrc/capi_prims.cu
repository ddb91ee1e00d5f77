// C ABI for the device-pointer primitives (tb2_gemm, tb2_split_f32, ...).
#include "toy_b200.h"
#include "engine.cuh"
#include "gemm.cuh"
#include "kernels.cuh"
#include "runtime.cuh"

namespace {
tb2::Operand to_op(const tb2_operand* o) {
  tb2::Operand r;
  r.hi = static_cast<const __nv_bfloat16*>(o->hi);
  r.lo = static_cast<const __nv_bfloat16*>(o->lo);
  r.mn_major = o->mn_major;
  r.ld = o->ld;
  r.rows = o->rows;
  r.cols = o->cols;
  r.batch_stride = o->batch_stride;
  r.nbatch = o->nbatch;
  r.bdiv1 = o->bdiv1 > 0 ? o->bdiv1 : 1;
  r.bmul1 = o->bmul1;
  r.bdiv2 = o->bdiv2 > 0 ? o->bdiv2 : 1;
  r.bmul2 = o->bmul2;
  r.q8 = static_cast<const int8_t*>(o->q8);
  r.q8_scale = static_cast<const uint16_t*>(o->q8_scale);
  return r;
}
}  // namespace

extern "C" {

int tb2_gemm(int M, int N, int K, int batch, int split, const tb2_operand* a, const tb2_operand* b,
             const tb2_epilogue* epi, int ksplits, int causal, void* stream) {
  if (!a || !b || !epi || ksplits < 0 || split < 0 || split > 2) return -1;
  tb2::GemmDesc d;
  d.M = M; d.N = N; d.K = K; d.batch = batch; d.split = split == 1;
  d.f16 = split == 2;
  d.splits = ksplits;
  d.causal = causal;
  d.a = to_op(a);
  d.b = to_op(b);
  tb2::Epilogue& e = d.epi;
  e.mode = epi->mode;
  e.alpha = epi->alpha;
  e.out = epi->out;
  e.res = epi->res;
  e.out_hi = static_cast<__nv_bfloat16*>(epi->out_hi);
  e.out_lo = static_cast<__nv_bfloat16*>(epi->out_lo);
  e.bstride = epi->bstride;
  e.z_div = epi->z_div > 0 ? epi->z_div : (1 << 30);
  e.z_s1 = epi->z_s1;
  e.m_div = epi->m_div > 0 ? epi->m_div : (1 << 30);
  e.m_s1 = epi->m_s1;
  e.m_s0 = epi->m_s0;
  e.n_div = epi->n_div > 0 ? epi->n_div : (1 << 30);
  e.n_s1 = epi->n_s1;
  int* err = tb2::device_error_word();
  if (!err) return -3;
  const int rc = tb2::gemm_launch(d, tb2::gemm_scratch(), err, static_cast<cudaStream_t>(stream));
  return rc == 0 ? 0 : (rc <= -10 ? -3 : -1);
}

int tb2_gemm_set_pair_mode(int mode) { return tb2::gemm_set_pair_mode(mode); }

int tb2_gemm_set_tile_width(int bn) { return tb2::gemm_set_tile_width(bn); }

int tb2_set_q8_base_mode(int mode) { return tb2::engine_set_q8_base_mode(mode); }

int tb2_set_q8_ring_l2(int on) { return tb2::engine_set_q8_ring_l2(on); }

int tb2_set_side_gemm_ctas(int n) { return tb2::engine_set_side_gemm_ctas(n); }

int tb2_set_side_gemm_tile_width(int bn) { return tb2::engine_set_side_gemm_tile_width(bn); }

int tb2_set_plan_alone(int on) { return tb2::engine_set_plan_alone(on); }
int tb2_set_f16_wgrad(int on) { return tb2::engine_set_f16_wgrad(on); }

int tb2_split_f32(const float* x, void* hi, void* lo, size_t n, void* stream) {
  if (!x || !hi || !lo) return -1;
  return tb2::launch_split_f32(x, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), (long long)n,
                               static_cast<cudaStream_t>(stream));
}

int tb2_q8_0_quantize(const float* x, void* q, long long rows, int K, void* stream) {
  if (!x || !q || rows <= 0 || K <= 0) return -1;
  return tb2::launch_q8_0_quantize(x, static_cast<uint8_t*>(q), rows, K, static_cast<cudaStream_t>(stream));
}

int tb2_q8_0_dequantize(const void* q, void* hi, void* lo, float* f32, long long rows, int K, void* stream) {
  if (!q || !hi || !lo || rows <= 0 || K <= 0) return -1;
  tb2::Planes p{static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo)};
  return tb2::launch_q8_0_to_planes(static_cast<const uint8_t*>(q), p, f32, rows, K,
                                    static_cast<cudaStream_t>(stream));
}

int tb2_device_error(void) { return tb2::read_and_clear_device_error(); }

const char* tb2_version(void) { return "toy_b200 0.1 (sm_100a)"; }

}  // extern "C"
