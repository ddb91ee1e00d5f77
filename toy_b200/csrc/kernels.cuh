// Bandwidth-bound kernels of the training step (launch wrappers).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace tb2 {

// hi = rn_bf16(x), lo = rn_bf16(x - hi)
int launch_split_f32(const float* x, __nv_bfloat16* hi, __nv_bfloat16* lo, long long n, cudaStream_t st);

}  // namespace tb2
