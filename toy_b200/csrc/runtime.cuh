#pragma once
#include <cuda_runtime.h>

#include <mutex>

#include "gemm.cuh"

namespace tb2 {
// Set-up that must happen once on every device a launch site runs on (a
// kernel's dynamic shared-memory limit, an occupancy query): ensure(f) calls
// f(device) the first time the current device reaches it and remembers a
// success, so a process that drives several GPUs sets each one up. Host
// threads may call it concurrently.
class DeviceOnce {
 public:
  template <class F>
  int ensure(F&& f) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return -3;
    std::lock_guard<std::mutex> lk(mu_);
    if (done_[dev]) return 0;
    const int rc = f(dev);
    if (rc == 0) done_[dev] = true;
    return rc;
  }

 private:
  static constexpr int kMaxDev = 64;
  std::mutex mu_;
  bool done_[kMaxDev] = {};
};

// Device int the kernels of the current device report wait timeouts into.
int* device_error_word();
// Synchronise, read the word, clear it. Returns the code (0 = none) or -3.
int read_and_clear_device_error();
// Split-K workspace of the current device (allocated on first use: 64 MiB of
// partial tiles). Shared by every GEMM of the device, so GEMMs that use it
// must run on one stream at a time.
const GemmScratch& gemm_scratch();

// L2 persisting set-aside of the current device (a limit of this process's
// context, gone with it): l2_keep_acquire(bytes) grows the set-aside to hold
// the sum of its users' bytes (at most the device's maximum) and returns true
// when `bytes` fit, false (nothing reserved) otherwise; l2_keep_release(bytes)
// gives them back, and the last user restores the context's previous limit and
// returns every persisting line to normal status.
bool l2_keep_acquire(size_t bytes);
void l2_keep_release(size_t bytes);
}  // namespace tb2
