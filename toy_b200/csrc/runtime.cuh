#pragma once
#include <cuda_runtime.h>

#include "gemm.cuh"

namespace tb2 {
// Device int the kernels of the current device report wait timeouts into.
int* device_error_word();
// Synchronise, read the word, clear it. Returns the code (0 = none) or -3.
int read_and_clear_device_error();
// Split-K workspace of the current device (allocated on first use: 64 MiB of
// partial tiles and 64 Ki tile counters). Shared by every GEMM of the device,
// so GEMMs that use it must run on one stream at a time.
const GemmScratch& gemm_scratch();
}  // namespace tb2
