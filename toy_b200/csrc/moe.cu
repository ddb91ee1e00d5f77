// Mixture-of-experts FFN of the training step (OLMoE-style blocks) and the
// whole-vector QK-RMSNorm: the bandwidth kernels around the expert GEMMs.
//
//   route:      per token, softmax of the router logits over the experts, the
//               top-k experts by probability (ties to the lower index) and
//               their weights (renormalised to sum 1 with norm_topk)
//               -- llama_kv_engine.rb build_moe_ffn :2073 (tnn_softmax,
//               tnn_top_k, tnn_get_rows of the probabilities);
//   gather:     the (token, k) slots' input rows in expert order, so each
//               expert's rows are one contiguous GEMM operand (mul_mat_id);
//   combine:    x2 = x1 + sum_k w_k y_(token, k), k ascending (deterministic);
//   backward:   dw_k = <dy, y_k> and dy_k = w_k dy per slot; the router's
//               softmax backward from dw; the fixed-order sum of the slots'
//               input gradients back onto their tokens;
//   QK-norm:    RMSNorm over a column range of the q|k|v rows in place (the
//               pre-norm values kept), and its backward on the gradient planes
//               in place.
//
// A slot is token * k_used + choice; perm lists the slots in expert order,
// pos is its inverse. E <= 256 experts, k_used <= 16; one warp per token or slot.
#include <cuda_bf16.h>

#include <cmath>
#include <cstdint>

#include "kernels.cuh"
#include "pdl.cuh"

namespace tb2 {

namespace {

constexpr int kMoeMaxE = 256;
constexpr int kMoeMaxK = 16;

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void put_planes(const Planes& p, long long i, float v) {
  const bf16 h = __float2bfloat16_rn(v);
  p.hi[i] = h;
  p.lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
}
__device__ __forceinline__ float get_planes(const Planes& p, long long i) {
  return __bfloat162float(p.hi[i]) + __bfloat162float(p.lo[i]);
}

int grid_warps(long long warps) {
  const long long b = (warps + 7) / 8;   // 8 warps per 256-thread block
  return (int)(b < 1 ? 1 : b < 148 * 16 ? b : 148 * 16);
}
int grid_items(long long items) {
  const long long b = (items + 255) / 256;
  return (int)(b < 1 ? 1 : b < 148 * 16 ? b : 148 * 16);
}

#define WARP_LOOP(var, count)                                                                  \
  for (long long var = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; var < (count); \
       var += ((long long)gridDim.x * blockDim.x) >> 5)

__global__ void moe_route_kernel(const float* __restrict__ logits, int N, int E, int K, int norm_topk,
                                 float* __restrict__ probs, int* __restrict__ idx, float* __restrict__ w) {
  griddep_wait();
  const int lane = threadIdx.x & 31;
  WARP_LOOP(n, N) {
    const float* z = logits + n * E;
    float pv[kMoeMaxE / 32];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMoeMaxE / 32; ++j) {
      const int e = lane + 32 * j;
      pv[j] = e < E ? z[e] : -INFINITY;
      m = fmaxf(m, pv[j]);
    }
    m = wmax(m);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kMoeMaxE / 32; ++j) {
      const int e = lane + 32 * j;
      pv[j] = e < E ? expf(pv[j] - m) : 0.f;
      s += pv[j];
    }
    s = wsum(s);
#pragma unroll
    for (int j = 0; j < kMoeMaxE / 32; ++j) {
      const int e = lane + 32 * j;
      pv[j] = pv[j] / s;
      if (e < E) probs[n * E + e] = pv[j];
      else pv[j] = -3.f;   // never selected
    }
    // top-k: k rounds of a warp arg-max (larger probability, then lower index)
    float sel_sum = 0.f, mine = 0.f;
    int mine_i = 0;
    for (int k = 0; k < K; ++k) {
      float bv = -1.f;
      int bi = 1 << 30;
#pragma unroll
      for (int j = 0; j < kMoeMaxE / 32; ++j) {
        const int e = lane + 32 * j;
        if (pv[j] > bv || (pv[j] == bv && e < bi)) {
          bv = pv[j];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
#pragma unroll
      for (int j = 0; j < kMoeMaxE / 32; ++j)
        if (lane + 32 * j == bi) pv[j] = -2.f;   // taken
      sel_sum += bv;
      if (lane == k) {
        mine = bv;
        mine_i = bi;
      }
    }
    if (lane < K) {
      idx[n * K + lane] = mine_i;
      w[n * K + lane] = norm_topk ? mine / sel_sum : mine;
    }
  }
}

// Xs[i] = h[perm[i] / K] (planes, d columns; h has row pitch ldh)
__global__ void moe_gather_kernel(Planes h, long long ldh, const int* __restrict__ perm, long long NK, int K, int d,
                                  Planes xs) {
  griddep_wait();
  const int lane = threadIdx.x & 31;
  WARP_LOOP(i, NK) {
    const long long src = (long long)(perm[i] / K) * ldh, dst = i * d;
    for (int c = lane * 8; c < d; c += 256) {   // 8 bf16 = 16 bytes per plane
      *reinterpret_cast<uint4*>(xs.hi + dst + c) = *reinterpret_cast<const uint4*>(h.hi + src + c);
      *reinterpret_cast<uint4*>(xs.lo + dst + c) = *reinterpret_cast<const uint4*>(h.lo + src + c);
    }
  }
}

// x2[n] = x1[n] + sum_k w[n K + k] ye[pos[n K + k]]
__global__ void moe_combine_kernel(const float* __restrict__ x1, const float* __restrict__ ye,
                                   const int* __restrict__ pos, const float* __restrict__ w, int N, int K, int d,
                                   float* __restrict__ x2) {
  griddep_wait();
  const long long total = (long long)N * (d / 4);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / (d / 4);
    const int c = (int)(i % (d / 4)) * 4;
    float4 acc = *reinterpret_cast<const float4*>(x1 + n * d + c);
    for (int k = 0; k < K; ++k) {
      const float wk = w[n * K + k];
      const float4 y = *reinterpret_cast<const float4*>(ye + (long long)pos[n * K + k] * d + c);
      acc.x += wk * y.x; acc.y += wk * y.y; acc.z += wk * y.z; acc.w += wk * y.w;
    }
    *reinterpret_cast<float4*>(x2 + n * d + c) = acc;
  }
}

// per sorted slot i: dw[slot] = <dy[token], ye[i]>, dye[i] = w[slot] dy[token] (planes)
__global__ void moe_dy_kernel(const float* __restrict__ dy, const float* __restrict__ ye, const int* __restrict__ perm,
                              const float* __restrict__ w, long long NK, int K, int d, float* __restrict__ dw,
                              Planes dye) {
  griddep_wait();
  const int lane = threadIdx.x & 31;
  WARP_LOOP(i, NK) {
    const int slot = perm[i];
    const float* g = dy + (long long)(slot / K) * d;
    const float* y = ye + i * d;
    const float wk = w[slot];
    float s = 0.f;
    for (int c = lane; c < d; c += 32) {
      const float gv = g[c];
      s += gv * y[c];
      put_planes(dye, i * d + c, wk * gv);
    }
    s = wsum(s);
    if (lane == 0) dw[slot] = s;
  }
}

// per token: dprobs from dw at the chosen experts (through the renormalisation
// with norm_topk), dlogits = p (dprobs - <p, dprobs>) as planes [N][E]
__global__ void moe_router_bwd_kernel(const float* __restrict__ probs, const int* __restrict__ idx,
                                      const float* __restrict__ w, const float* __restrict__ dw, int N, int E, int K,
                                      int norm_topk, Planes dlog) {
  griddep_wait();
  const int lane = threadIdx.x & 31;
  WARP_LOOP(n, N) {
    // the chosen experts' gradient: dsel_k = dw_k, or (dw_k - sum_j dw_j w_j) / sum_j p_sel_j
    float dsel = 0.f;
    int ek = -1;
    if (lane < K) {
      dsel = dw[n * K + lane];
      ek = idx[n * K + lane];
    }
    if (norm_topk) {
      const float dww = wsum(lane < K ? dsel * w[n * K + lane] : 0.f);
      const float psum = wsum(lane < K ? probs[n * E + ek] : 0.f);
      dsel = (dsel - dww) / psum;
    }
    float pd = 0.f;   // <p, dprobs>
    for (int k = 0; k < K; ++k) {
      const float dk = __shfl_sync(0xffffffffu, dsel, k);
      const int e = __shfl_sync(0xffffffffu, ek, k);
      pd += probs[n * E + e] * dk;
    }
    for (int e = lane; e < E; e += 32) {
      float dp = 0.f;
      for (int k = 0; k < K; ++k) {
        const float dk = __shfl_sync(0xffffffffu, dsel, k);   // every lane runs the same k loop
        const int ee = __shfl_sync(0xffffffffu, ek, k);
        if (ee == e) dp += dk;
      }
      const float p = probs[n * E + e];
      put_planes(dlog, n * E + e, p * (dp - pd));
    }
  }
}

// dh[n] += sum_k dxs[pos[n K + k]], k ascending
__global__ void moe_gather_sum_kernel(const float* __restrict__ dxs, const int* __restrict__ pos, int N, int K, int d,
                                      float* __restrict__ dh) {
  griddep_wait();
  const long long total = (long long)N * (d / 4);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / (d / 4);
    const int c = (int)(i % (d / 4)) * 4;
    float4 acc = *reinterpret_cast<float4*>(dh + n * d + c);
    for (int k = 0; k < K; ++k) {
      const float4 y = *reinterpret_cast<const float4*>(dxs + (long long)pos[n * K + k] * d + c);
      acc.x += y.x; acc.y += y.y; acc.z += y.z; acc.w += y.w;
    }
    *reinterpret_cast<float4*>(dh + n * d + c) = acc;
  }
}

// RMSNorm of columns [c0, c0 + width) of every row of x [N][ld], in place; the
// pre-norm values go to pre [N][width]
__global__ void rms_cols_fwd_kernel(float* __restrict__ x, long long ld, int c0, int width, const float* __restrict__ g,
                                    float eps, int N, float* __restrict__ pre) {
  griddep_wait();
  const int lane = threadIdx.x & 31;
  WARP_LOOP(n, N) {
    float* r = x + n * ld + c0;
    float ss = 0.f;
    for (int c = lane; c < width; c += 32) {
      const float v = r[c];
      pre[n * width + c] = v;
      ss += v * v;
    }
    ss = wsum(ss);
    const float rr = rsqrtf(ss / (float)width + eps);
    for (int c = lane; c < width; c += 32) r[c] = r[c] * rr * g[c];
  }
}

// the backward of rms_cols_fwd on gradient planes [N][ld], columns [c0, c0 + width),
// in place: dx = (dz - x sum(x dz) / (sum x^2 + n eps)) rrms with dz = dy g
__global__ void rms_cols_bwd_kernel(Planes dyp, long long ld, int c0, int width, const float* __restrict__ g,
                                    const float* __restrict__ pre, float eps, int N) {
  griddep_wait();
  const int lane = threadIdx.x & 31;
  WARP_LOOP(n, N) {
    const float* x = pre + n * width;
    float sxx = 0.f, sxz = 0.f;
    for (int c = lane; c < width; c += 32) {
      const float xv = x[c], dz = get_planes(dyp, n * ld + c0 + c) * g[c];
      sxx += xv * xv;
      sxz += xv * dz;
    }
    sxx = wsum(sxx);
    sxz = wsum(sxz);
    const float rrms = rsqrtf(sxx / (float)width + eps);
    const float f = sxz / (sxx + (float)width * eps);
    for (int c = lane; c < width; c += 32) {
      const long long o = n * ld + c0 + c;
      const float dz = get_planes(dyp, o) * g[c];
      put_planes(dyp, o, (dz - x[c] * f) * rrms);
    }
  }
}

int ok() { return cudaPeekAtLastError() == cudaSuccess ? 0 : -3; }

}  // namespace

int launch_moe_route(const float* logits, int N, int E, int K, int norm_topk, float* probs, int* idx, float* w,
                     cudaStream_t st) {
  if (E < 1 || E > kMoeMaxE || K < 1 || K > kMoeMaxK || K > E || K > 32) return -1;
  launch_pdl(moe_route_kernel, dim3(grid_warps(N)), dim3(256), 0, st, logits, N, E, K, norm_topk, probs, idx, w);
  return ok();
}

int launch_moe_gather(Planes h, long long ldh, const int* perm, long long NK, int K, int d, Planes xs, cudaStream_t st) {
  if (d % 8 || ldh % 8) return -1;
  launch_pdl(moe_gather_kernel, dim3(grid_warps(NK)), dim3(256), 0, st, h, ldh, perm, NK, K, d, xs);
  return ok();
}

int launch_moe_combine(const float* x1, const float* ye, const int* pos, const float* w, int N, int K, int d, float* x2,
                       cudaStream_t st) {
  if (d % 4) return -1;
  launch_pdl(moe_combine_kernel, dim3(grid_items((long long)N * d / 4)), dim3(256), 0, st, x1, ye, pos, w, N, K, d, x2);
  return ok();
}

int launch_moe_dy(const float* dy, const float* ye, const int* perm, const float* w, long long NK, int K, int d,
                  float* dw, Planes dye, cudaStream_t st) {
  launch_pdl(moe_dy_kernel, dim3(grid_warps(NK)), dim3(256), 0, st, dy, ye, perm, w, NK, K, d, dw, dye);
  return ok();
}

int launch_moe_router_bwd(const float* probs, const int* idx, const float* w, const float* dw, int N, int E, int K,
                          int norm_topk, Planes dlog, cudaStream_t st) {
  if (K > 32) return -1;
  launch_pdl(moe_router_bwd_kernel, dim3(grid_warps(N)), dim3(256), 0, st, probs, idx, w, dw, N, E, K, norm_topk, dlog);
  return ok();
}

int launch_moe_gather_sum(const float* dxs, const int* pos, int N, int K, int d, float* dh, cudaStream_t st) {
  if (d % 4) return -1;
  launch_pdl(moe_gather_sum_kernel, dim3(grid_items((long long)N * d / 4)), dim3(256), 0, st, dxs, pos, N, K, d, dh);
  return ok();
}

int launch_rms_cols_fwd(float* x, long long ld, int c0, int width, const float* g, float eps, int N, float* pre,
                        cudaStream_t st) {
  launch_pdl(rms_cols_fwd_kernel, dim3(grid_warps(N)), dim3(256), 0, st, x, ld, c0, width, g, eps, N, pre);
  return ok();
}

int launch_rms_cols_bwd(Planes dy, long long ld, int c0, int width, const float* g, const float* pre, float eps, int N,
                        cudaStream_t st) {
  launch_pdl(rms_cols_bwd_kernel, dim3(grid_warps(N)), dim3(256), 0, st, dy, ld, c0, width, g, pre, eps, N);
  return ok();
}

}  // namespace tb2
