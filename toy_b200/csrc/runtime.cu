// Process-wide device state shared by every entry point: one device error
// word per GPU (written by kernels whose bounded waits give up), the split-K
// workspace, and the L2 persisting set-aside the engines' plane rings use.
#include "runtime.cuh"

#include <algorithm>
#include <mutex>

namespace tb2 {

namespace {
std::mutex g_mu;
int* g_err[64] = {nullptr};
GemmScratch g_scratch[64];
constexpr long long kWsFloats = 16LL << 20;   // 64 MiB
struct L2Keep {
  int users = 0;
  size_t held = 0;   // sum of the users' bytes
  size_t prev = 0;   // the context's limit before the first user
};
L2Keep g_l2[64];
}  // namespace

bool l2_keep_acquire(size_t bytes) {
  int dev = 0;
  if (bytes == 0 || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  int maxp = 0;
  if (cudaDeviceGetAttribute(&maxp, cudaDevAttrMaxPersistingL2CacheSize, dev) != cudaSuccess || maxp <= 0 ||
      bytes > (size_t)maxp)
    return false;
  std::lock_guard<std::mutex> lk(g_mu);
  L2Keep& k = g_l2[dev];
  size_t cur = 0;
  if (cudaDeviceGetLimit(&cur, cudaLimitPersistingL2CacheSize) != cudaSuccess) return false;
  const size_t want = std::min(k.held + bytes, (size_t)maxp);
  if (want > cur && cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, want) != cudaSuccess) return false;
  if (k.users == 0) k.prev = cur;
  ++k.users;
  k.held += bytes;
  return true;
}

void l2_keep_release(size_t bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
  std::lock_guard<std::mutex> lk(g_mu);
  L2Keep& k = g_l2[dev];
  if (k.users <= 0) return;
  --k.users;
  k.held = k.held > bytes ? k.held - bytes : 0;
  if (k.users == 0) {
    cudaCtxResetPersistingL2Cache();
    cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, k.prev);
  }
}

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
