// tb2_gemm_noalloc: the split-bf16 tensor-core GEMM of tb2_gemm for callers
// that must not allocate device memory.
//
// Who needs this: code that runs where cudaMalloc is unavailable or unsafe —
// inside a memory-pool-restricted process, a real-time loop that forbids
// allocator calls (they can synchronise the device and stall other streams),
// or a host framework that owns all device memory and hands this library only
// its input and output buffers. tb2_gemm allocates a split-K workspace and an
// error word on first use; this entry point instead uses fixed arrays compiled
// into the library image, so it never calls cudaMalloc, cudaFree or any
// allocating library routine.
//
// Limits and sharing:
//   * the split-K workspace holds kNoAllocWsFloats floats (8 MiB); a call whose
//     explicit ksplits, as the GEMM would run them (capped at the k-block count,
//     1 where the shape allows no split), times M * N exceeds it is rejected
//     with -5 and a message; with ksplits = 0 the split count is chosen to fit;
//   * every GPU that loads the library holds these arrays until process exit;
//   * all calls on a device share them and the arrays keep the last call's
//     contents, so calls that overlap on the GPU (different streams, or
//     different host threads) race; serialise them on one stream;
//   * the error word (non-zero when a kernel's bounded wait gave up, so the
//     output is not valid) is cleared, stream-ordered, at the start of every
//     call; tb2_gemm_noalloc_error() reads and clears it.
// The first call on each device resolves the arrays' device addresses
// (cudaGetSymbolAddress with that device current); make that first call before
// any stream capture.
#include <cstdio>
#include <mutex>

#include "gemm.cuh"
#include "toy_b200.h"

namespace {

constexpr long long kNoAllocWsFloats = 2LL << 20;   // 8 MiB of f32 split-K partials
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_ws[kNoAllocWsFloats];
static __device__ __align__(256) int g_noalloc_err[1];

struct DevicePtrs {
  float* ws = nullptr;
  int* err = nullptr;
};

std::mutex g_mu;
DevicePtrs g_ptrs[kMaxDevices];

// Device addresses of the static arrays for the current device (host code must
// not use the arrays' names as device pointers: on the host they are stand-ins).
int resolve(DevicePtrs* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -3;
  std::lock_guard<std::mutex> lk(g_mu);
  DevicePtrs& p = g_ptrs[dev];
  if (!p.ws) {
    void* ws = nullptr;
    void* err = nullptr;
    if (cudaGetSymbolAddress(&ws, g_noalloc_ws) != cudaSuccess) return -3;
    if (cudaGetSymbolAddress(&err, g_noalloc_err) != cudaSuccess) return -3;
    p.ws = static_cast<float*>(ws);
    p.err = static_cast<int*>(err);
  }
  *out = p;
  return 0;
}

}  // namespace

extern "C" int tb2_gemm_noalloc(int M, int N, int K, int batch, int split, const tb2_operand* a, const tb2_operand* b,
                                const tb2_epilogue* epi, int ksplits, int causal, void* stream) {
  if (!a || !b || !epi || ksplits < 0 || split < 0 || split > 2) return -1;
  tb2::GemmDesc d;
  d.M = M; d.N = N; d.K = K; d.batch = batch; d.split = split == 1;
  d.f16 = split == 2;
  d.splits = ksplits;
  d.causal = causal;
  auto cvt = [](const tb2_operand* o) {
    tb2::Operand r;
    r.hi = static_cast<const __nv_bfloat16*>(o->hi);
    r.lo = static_cast<const __nv_bfloat16*>(o->lo);
    r.mn_major = o->mn_major; r.ld = o->ld; r.rows = o->rows; r.cols = o->cols;
    r.batch_stride = o->batch_stride; r.nbatch = o->nbatch;
    r.bdiv1 = o->bdiv1 > 0 ? o->bdiv1 : 1; r.bmul1 = o->bmul1;
    r.bdiv2 = o->bdiv2 > 0 ? o->bdiv2 : 1; r.bmul2 = o->bmul2;
    r.q8 = static_cast<const int8_t*>(o->q8); r.q8_scale = static_cast<const uint16_t*>(o->q8_scale);
    return r;
  };
  d.a = cvt(a);
  d.b = cvt(b);
  tb2::Epilogue& e = d.epi;
  e.mode = epi->mode; e.alpha = epi->alpha; e.out = epi->out; e.res = epi->res;
  e.out_hi = static_cast<__nv_bfloat16*>(epi->out_hi);
  e.out_lo = static_cast<__nv_bfloat16*>(epi->out_lo);
  e.bstride = epi->bstride;
  e.z_div = epi->z_div > 0 ? epi->z_div : (1 << 30);
  e.z_s1 = epi->z_s1;
  e.m_div = epi->m_div > 0 ? epi->m_div : (1 << 30);
  e.m_s1 = epi->m_s1; e.m_s0 = epi->m_s0;
  e.n_div = epi->n_div > 0 ? epi->n_div : (1 << 30);
  e.n_s1 = epi->n_s1;
  const int eff = tb2::gemm_effective_splits(d, ksplits);
  if (eff > 1 && (long long)eff * M * N > kNoAllocWsFloats) {
    fprintf(stderr,
            "[toy_b200] tb2_gemm_noalloc: %d K splits x M x N = %lld floats exceeds the fixed %lld-float "
            "split-K workspace\n",
            eff, (long long)eff * M * N, kNoAllocWsFloats);
    return -5;
  }
  DevicePtrs p;
  if (resolve(&p)) return -3;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(p.err, 0, sizeof(int), st) != cudaSuccess) return -3;
  tb2::GemmScratch sc;
  sc.ws = p.ws;
  sc.ws_floats = kNoAllocWsFloats;
  const int rc = tb2::gemm_launch(d, sc, p.err, st);
  return rc == 0 ? 0 : (rc <= -10 ? -3 : -1);
}

extern "C" int tb2_gemm_noalloc_error(void) {
  DevicePtrs p;
  if (resolve(&p)) return -3;
  if (cudaDeviceSynchronize() != cudaSuccess) return -3;
  int h = 0;
  if (cudaMemcpyFromSymbol(&h, g_noalloc_err, sizeof(int)) != cudaSuccess) return -3;
  if (h) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(int)) != cudaSuccess) return -3;
  }
  return h;
}
