#pragma once
#include <cuda_runtime.h>

namespace tb2 {
// Device int the kernels of the current device report wait timeouts into.
int* device_error_word();
// Synchronise, read the word, clear it. Returns the code (0 = none) or -3.
int read_and_clear_device_error();
}  // namespace tb2
