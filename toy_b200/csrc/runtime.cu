// Process-wide device state shared by every entry point: one device error
// word per GPU (written by kernels whose bounded waits give up).
#include "runtime.cuh"

#include <mutex>

namespace tb2 {

namespace {
std::mutex g_mu;
int* g_err[64] = {nullptr};
GemmScratch g_scratch[64];
constexpr long long kWsFloats = 16LL << 20;   // 64 MiB
}  // namespace

const GemmScratch& gemm_scratch() {
  static const GemmScratch none;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return none;
  std::lock_guard<std::mutex> lk(g_mu);
  GemmScratch& s = g_scratch[dev];
  if (!s.ws) {
    float* ws = nullptr;
    if (cudaMalloc(&ws, kWsFloats * sizeof(float)) != cudaSuccess) return none;
    s.ws = ws;
    s.ws_floats = kWsFloats;
  }
  return s;
}

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_err[dev] = p;
  }
  return g_err[dev];
}

int read_and_clear_device_error() {
  int* p = device_error_word();
  if (!p) return -3;
  if (cudaDeviceSynchronize() != cudaSuccess) return -3;
  int h = 0;
  if (cudaMemcpy(&h, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -3;
  if (h) cudaMemset(p, 0, sizeof(int));
  return h;
}

}  // namespace tb2
