// Bandwidth-bound kernels of the training step: vectorised loads, rows held in
// registers, warp-shuffle reductions, fixed-order (deterministic) reductions,
// grids sized in multiples of the SM count.
#include "kernels.cuh"
#include "lora.cuh"
#include "pdl.cuh"
#include "runtime.cuh"
#include "tc_common.cuh"
#include "warp_reduce.cuh"

#include <cuda_fp16.h>
#include <cstdint>

namespace tb2 {

namespace {

constexpr int kSMs = 148;
constexpr int kRmsBwdBlocks = 2 * kSMs;

__device__ __forceinline__ void split2(float x, bf16& h, bf16& l) {
  h = __float2bfloat16_rn(x);
  l = __float2bfloat16_rn(x - __bfloat162float(h));
}

// rn_f16(x) saturated to the largest finite magnitude (NaN stays NaN)
__device__ __forceinline__ __half f16_sat(float x) {
  return __float2half_rn(x > 65504.f ? 65504.f : (x < -65504.f ? -65504.f : x));
}

__device__ __forceinline__ float f16_scale_of(const Planes& p) { return p.f16_scale ? __ldg(p.f16_scale) : 1.0f; }

// The store helpers take the fp16 copy's scale s as loaded once by the
// kernel (f16_scale_of); the overloads without it load it per call.
__device__ __forceinline__ void store_planes(const Planes& p, long long i, float x, float s) {
  bf16 h, l;
  split2(x, h, l);
  p.hi[i] = h;
  p.lo[i] = l;
  if (p.f16) p.f16[i] = f16_sat(x * s);
}
__device__ __forceinline__ void store_planes(const Planes& p, long long i, float x) {
  store_planes(p, i, x, p.f16 ? f16_scale_of(p) : 1.0f);
}

// Four consecutive values (i % 4 == 0) as two 8-byte stores (three with the fp16 copy).
__device__ __forceinline__ void store_planes4(const Planes& p, long long i, float4 v, float s) {
  __align__(8) bf16 h[4], l[4];
  split2(v.x, h[0], l[0]);
  split2(v.y, h[1], l[1]);
  split2(v.z, h[2], l[2]);
  split2(v.w, h[3], l[3]);
  *reinterpret_cast<uint2*>(p.hi + i) = *reinterpret_cast<const uint2*>(h);
  *reinterpret_cast<uint2*>(p.lo + i) = *reinterpret_cast<const uint2*>(l);
  if (p.f16) {
    __align__(8) __half q[4] = {f16_sat(v.x * s), f16_sat(v.y * s), f16_sat(v.z * s), f16_sat(v.w * s)};
    *reinterpret_cast<uint2*>(p.f16 + i) = *reinterpret_cast<const uint2*>(q);
  }
}
__device__ __forceinline__ void store_planes4(const Planes& p, long long i, float4 v) {
  store_planes4(p, i, v, p.f16 ? f16_scale_of(p) : 1.0f);
}

// Two consecutive values (i % 2 == 0) as two 4-byte stores (three with the fp16 copy).
__device__ __forceinline__ void store_planes2(const Planes& p, long long i, float a, float b) {
  __align__(4) bf16 h[2], l[2];
  split2(a, h[0], l[0]);
  split2(b, h[1], l[1]);
  *reinterpret_cast<uint32_t*>(p.hi + i) = *reinterpret_cast<const uint32_t*>(h);
  *reinterpret_cast<uint32_t*>(p.lo + i) = *reinterpret_cast<const uint32_t*>(l);
  if (p.f16) {
    const float s = f16_scale_of(p);
    __align__(4) __half q[2] = {f16_sat(a * s), f16_sat(b * s)};
    *reinterpret_cast<uint32_t*>(p.f16 + i) = *reinterpret_cast<const uint32_t*>(q);
  }
}

__device__ __forceinline__ float amax4(float m, float4 v) {
  return fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
}

// Raise *amax to the warp's largest m (non-negative floats order like their
// bits). Every lane of the warp calls it. Thousands of warps end on the same
// word: a warp whose maximum the word already holds skips the atomic, so the
// atomics do not queue up on it.
__device__ __forceinline__ void flush_amax(unsigned* amax, float m) {
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m > 0.f && *reinterpret_cast<volatile unsigned*>(amax) < __float_as_uint(m))
    atomicMax(amax, __float_as_uint(m));
}

__device__ __forceinline__ float4 load_planes4(const Planes& p, long long i) {
  const uint2 h = *reinterpret_cast<const uint2*>(p.hi + i);
  const uint2 l = *reinterpret_cast<const uint2*>(p.lo + i);
  const bf16* hh = reinterpret_cast<const bf16*>(&h);
  const bf16* ll = reinterpret_cast<const bf16*>(&l);
  return make_float4(__bfloat162float(hh[0]) + __bfloat162float(ll[0]), __bfloat162float(hh[1]) + __bfloat162float(ll[1]),
                     __bfloat162float(hh[2]) + __bfloat162float(ll[2]), __bfloat162float(hh[3]) + __bfloat162float(ll[3]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }

int grid_for(long long work, int threads, int per_sm = 8) {
  long long b = (work + threads - 1) / threads;
  const long long cap = (long long)kSMs * per_sm;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

int ok() { return cudaPeekAtLastError() == cudaSuccess ? 0 : -3; }

// ------------------------------------------------------------------ split
__global__ void split_f32_kernel(const float* __restrict__ x, bf16* __restrict__ hi, bf16* __restrict__ lo,
                                 long long n) {
  griddep_wait();
  const long long n4 = n / 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  Planes p{hi, lo};
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride)
    store_planes4(p, i * 4, reinterpret_cast<const float4*>(x)[i]);
  for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    store_planes(p, i, x[i]);
}

// ------------------------------------------------------------------ embedding
__global__ void embed_gather_kernel(const float* __restrict__ E, const int* __restrict__ ids, float* __restrict__ x0,
                                    int N, int d4) {
  griddep_wait();
  const long long total = (long long)N * d4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / d4), c = (int)(i % d4);
    reinterpret_cast<float4*>(x0)[i] = reinterpret_cast<const float4*>(E)[(long long)ids[n] * d4 + c];
  }
}

__global__ void embed_scatter_kernel(const float* __restrict__ dx, const int* __restrict__ order,
                                     const int* __restrict__ seg_start, const int* __restrict__ seg_id,
                                     const int* __restrict__ nseg_dev, float* __restrict__ dE, int d) {
  griddep_wait();
  const int nseg = *nseg_dev;
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (int k = blockIdx.x * warps + threadIdx.x / 32; k < nseg; k += gridDim.x * warps) {
    float* dst = dE + (long long)seg_id[k] * d;
    const int r0 = seg_start[k], r1 = seg_start[k + 1];
    for (int c = lane * 4; c < d; c += 128) {
      float4 acc = *reinterpret_cast<float4*>(dst + c);
      for (int r = r0; r < r1; ++r) {
        const float4 v = *reinterpret_cast<const float4*>(dx + (long long)order[r] * d + c);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      *reinterpret_cast<float4*>(dst + c) = acc;
    }
  }
}

// ------------------------------------------------------------------ RMSNorm
// One warp per row; lane l holds float4 chunks c = l + 32*i (i < NC) in registers.
template <int NC>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                          Planes h, long long ldh, int N, int d, float eps) {
  griddep_wait();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  const int d4 = d / 4;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  for (int n = blockIdx.x * warps + threadIdx.x / 32; n < N; n += gridDim.x * warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + (long long)n * d);
    float4 v[NC];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < d4 ? __ldcs(xr + c) : f4_zero();
      ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)d + eps);
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      if (c < d4) {
        const float4 g = g4[c];
        store_planes4(h, (long long)n * ldh + c * 4,
                      make_float4(v[i].x * r * g.x, v[i].y * r * g.y, v[i].z * r * g.z, v[i].w * r * g.w));
      }
    }
  }
}

// dx = dres + (dz - x * sum(x dz) / (sum x^2 + d eps)) * rrms with dz = dh * gamma.
// Block of 8 warps; warp w accumulates dgamma (dh * x * rrms) over its rows in
// shared memory (fixed row order per warp, fixed warp order in the block sum).
template <int NC>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const float* __restrict__ x, const float* __restrict__ dh,
                                                          const float* __restrict__ gamma, const float* dres,
                                                          float* dx, Planes dxp, long long ldp,
                                                          float* __restrict__ gpart, int N, int d, float eps) {
  griddep_wait();
  extern __shared__ float4 gacc4[];  // [warps][d / 4]
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int d4 = d / 4;
  float4* my = gacc4 + warp * d4;
  if (gpart)
    for (int c = lane; c < d4; c += 32) my[c] = f4_zero();
  __syncwarp();
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  float am = 0.f;   // max |dx| written (for the fp16 copy's scale)
  const float s16 = dxp.f16 ? f16_scale_of(dxp) : 1.0f;
  for (int n = blockIdx.x * warps + warp; n < N; n += gridDim.x * warps) {
    const long long base = (long long)n * d;
    const float4* xr = reinterpret_cast<const float4*>(x + base);
    const float4* hr = reinterpret_cast<const float4*>(dh + base);
    const float4* rres = dres ? reinterpret_cast<const float4*>(dres + base) : nullptr;
    // x and dh in registers; the residual gradient is read where it is added
    // (in the first round of loads while the row is short, NC <= 8)
    constexpr bool kRvEarly = NC <= 8;
    float4 xv[NC], hv[NC], rv[kRvEarly ? NC : 1];
    float sxx = 0.f, sxdz = 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      xv[i] = c < d4 ? xr[c] : f4_zero();
      hv[i] = c < d4 ? __ldcs(hr + c) : f4_zero();
      if constexpr (kRvEarly) rv[i] = (rres && c < d4) ? rres[c] : f4_zero();
      const float4 g = c < d4 ? g4[c] : f4_zero();
      sxx += xv[i].x * xv[i].x + xv[i].y * xv[i].y + xv[i].z * xv[i].z + xv[i].w * xv[i].w;
      sxdz += xv[i].x * hv[i].x * g.x + xv[i].y * hv[i].y * g.y + xv[i].z * hv[i].z * g.z + xv[i].w * hv[i].w * g.w;
    }
    sxx = warp_sum(sxx);
    sxdz = warp_sum(sxdz);
    const float rr = 1.0f / sqrtf(sxx / (float)d + eps);
    const float coef = sxdz / (sxx + (float)d * eps);
    float4* out = reinterpret_cast<float4*>(dx + base);
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      if (c >= d4) continue;
      const float4 v = xv[i], gg = hv[i], g = g4[c];
      float4 rs;
      if constexpr (kRvEarly) rs = rv[i];
      else rs = rres ? rres[c] : f4_zero();
      float4 o;
      o.x = rs.x + (gg.x * g.x - v.x * coef) * rr;
      o.y = rs.y + (gg.y * g.y - v.y * coef) * rr;
      o.z = rs.z + (gg.z * g.z - v.z * coef) * rr;
      o.w = rs.w + (gg.w * g.w - v.w * coef) * rr;
      out[c] = o;
      if (dxp.hi) store_planes4(dxp, (long long)n * ldp + c * 4, o, s16);
      am = amax4(am, o);
      if (gpart) {
        float4 a = my[c];
        a.x += gg.x * v.x * rr;
        a.y += gg.y * v.y * rr;
        a.z += gg.z * v.z * rr;
        a.w += gg.w * v.w * rr;
        my[c] = a;
      }
    }
  }
  if (dxp.f16_amax) flush_amax(dxp.f16_amax, am);
  if (!gpart) return;   // frozen gamma: no dgamma partials
  __syncthreads();
  for (int c = threadIdx.x; c < d4; c += blockDim.x) {
    float4 s = f4_zero();
    for (int w = 0; w < warps; ++w) {
      const float4 a = gacc4[w * d4 + c];
      s.x += a.x; s.y += a.y; s.z += a.z; s.w += a.w;
    }
    reinterpret_cast<float4*>(gpart + (long long)blockIdx.x * d)[c] = s;
  }
}

// gout[c] = (accumulate ? gout[c] : 0) + sum_b gpart[b][c]: 32 columns per block,
// 8 row groups summed in fixed order, then the groups in fixed order.
__global__ void colsum_kernel(const float* __restrict__ gpart, int nblk, int d, float* gout, int accumulate) {
  griddep_wait();
  __shared__ float sm[8][33];
  const int cx = threadIdx.x % 32, gy = threadIdx.x / 32;
  const int c = blockIdx.x * 32 + cx;
  float s = 0.f;
  if (c < d)
    for (int b = gy; b < nblk; b += 8) s += gpart[(long long)b * d + c];
  sm[gy][cx] = s;
  __syncthreads();
  if (gy == 0 && c < d) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) t += sm[g][cx];
    gout[c] = accumulate ? gout[c] + t : t;
  }
}

// ------------------------------------------------------------------ RoPE
// One block per token; thread i of the block handles pair (j, j + dh/2) of slot s
// for (s, j) = divmod(i, dh/2) over the H + 2*KV head slots of q | k | v.
__global__ void __launch_bounds__(256) rope_qkv_fwd_kernel(const float* __restrict__ qkv, const float* __restrict__ bias,
                                                           const int* __restrict__ pos, const float2* __restrict__ cs,
                                                           int tab_rows, Planes Q, Planes K, Planes V, int N, int T,
                                                           int H, int KV, int dh) {
  griddep_wait();
  const int half = dh / 2;
  const int slots = H + 2 * KV;
  const int width = slots * dh;
  for (int n = blockIdx.x; n < N; n += gridDim.x) {
    const int b = n / T, t = n - b * T;
    int p = pos[n];
    p = p < 0 ? 0 : (p >= tab_rows ? tab_rows - 1 : p);
    const float* row = qkv + (long long)n * width;
    const float2* crow = cs + (long long)p * half;
    for (int i = threadIdx.x; i < slots * half; i += blockDim.x) {
      const int slot = i / half, j = i - slot * half;
      float x0 = row[slot * dh + j], x1 = row[slot * dh + j + half];
      if (bias) {
        x0 += bias[slot * dh + j];
        x1 += bias[slot * dh + j + half];
      }
      if (slot < H + KV) {
        const float2 c = crow[j];
        const bool isq = slot < H;
        const int hh = isq ? slot : slot - H;
        const long long dst = (((long long)b * (isq ? H : KV) + hh) * T + t) * dh + j;
        const Planes& o = isq ? Q : K;
        store_planes(o, dst, x0 * c.x - x1 * c.y);
        store_planes(o, dst + half, x0 * c.y + x1 * c.x);
      } else {
        const int hh = slot - H - KV;
        const long long dst = (((long long)b * KV + hh) * T + t) * dh + j;
        store_planes(V, dst, x0);
        store_planes(V, dst + half, x1);
      }
    }
  }
}

// dQ / dK / dV may each be a sum of partial arrays: dQ of token t is the sum of
// parts p <= t / q_tile (q_tile = 0: one part), p * q_pstride apart; dK and dV
// are sums of kv_parts parts, kv_pstride apart. Parts are added in index order.
__global__ void __launch_bounds__(256) rope_qkv_bwd_kernel(const float* __restrict__ dQ, long long q_pstride,
                                                           int q_tile, const float* __restrict__ dK,
                                                           const float* __restrict__ dV, long long kv_pstride,
                                                           int kv_parts, const int* __restrict__ pos,
                                                           const float2* __restrict__ cs, int tab_rows, Planes out,
                                                           long long ldo, float* out_f32, int N, int T, int H, int KV,
                                                           int dh) {
  griddep_wait();
  // one item = four consecutive rotation pairs (j .. j + 3, j + half ..) of one
  // head slot of one token; the partial sums are added in part order
  const int half = dh / 2, h4 = half / 4;
  const int slots = H + 2 * KV;
  const int width = slots * dh;
  const long long items = (long long)N * slots * h4;
  float am = 0.f;   // max |dq|, |dk|, |dv| written
  const float s16 = out.f16 ? f16_scale_of(out) : 1.0f;
  for (long long it = blockIdx.x * (long long)blockDim.x + threadIdx.x; it < items;
       it += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(it / (slots * h4));
    const int rem = (int)(it - (long long)n * slots * h4);
    const int slot = rem / h4, j = (rem - slot * h4) * 4;
    const int b = n / T, t = n - b * T;
    float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0;
    const float* srcb;
    long long src, pstride;
    int parts;
    if (slot < H) {
      srcb = dQ; src = (((long long)b * H + slot) * T + t) * dh + j;
      pstride = q_pstride; parts = q_tile > 0 ? t / q_tile + 1 : 1;
    } else if (slot < H + KV) {
      srcb = dK; src = (((long long)b * KV + slot - H) * T + t) * dh + j;
      pstride = kv_pstride; parts = kv_parts;
    } else {
      srcb = dV; src = (((long long)b * KV + slot - H - KV) * T + t) * dh + j;
      pstride = kv_pstride; parts = kv_parts;
    }
    int q = 0;
    for (; q + 4 <= parts; q += 4) {   // four parts' loads in flight
      float4 u0[4], u1[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        u0[k] = *reinterpret_cast<const float4*>(srcb + src + (q + k) * pstride);
        u1[k] = *reinterpret_cast<const float4*>(srcb + src + (q + k) * pstride + half);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        g0.x += u0[k].x; g0.y += u0[k].y; g0.z += u0[k].z; g0.w += u0[k].w;
        g1.x += u1[k].x; g1.y += u1[k].y; g1.z += u1[k].z; g1.w += u1[k].w;
      }
    }
    for (; q < parts; ++q) {
      const float4 u0 = *reinterpret_cast<const float4*>(srcb + src + q * pstride);
      const float4 u1 = *reinterpret_cast<const float4*>(srcb + src + q * pstride + half);
      g0.x += u0.x; g0.y += u0.y; g0.z += u0.z; g0.w += u0.w;
      g1.x += u1.x; g1.y += u1.y; g1.z += u1.z; g1.w += u1.w;
    }
    float4 y0 = g0, y1 = g1;
    if (slot < H + KV) {   // rotation by -theta on dQ, dK
      int p = pos[n];
      p = p < 0 ? 0 : (p >= tab_rows ? tab_rows - 1 : p);
      const float2* c = cs + (long long)p * half + j;
      const float2 c0 = c[0], c1 = c[1], c2 = c[2], c3 = c[3];
      y0 = make_float4(g0.x * c0.x + g1.x * c0.y, g0.y * c1.x + g1.y * c1.y, g0.z * c2.x + g1.z * c2.y,
                       g0.w * c3.x + g1.w * c3.y);
      y1 = make_float4(-g0.x * c0.y + g1.x * c0.x, -g0.y * c1.y + g1.y * c1.x, -g0.z * c2.y + g1.z * c2.x,
                       -g0.w * c3.y + g1.w * c3.x);
    }
    const long long dp = (long long)n * ldo + slot * dh + j;
    store_planes4(out, dp, y0, s16);
    store_planes4(out, dp + half, y1, s16);
    am = amax4(amax4(am, y0), y1);
    if (out_f32) {
      const long long dst = (long long)n * width + slot * dh + j;
      *reinterpret_cast<float4*>(out_f32 + dst) = y0;
      *reinterpret_cast<float4*>(out_f32 + dst + half) = y1;
    }
  }
  if (out.f16_amax) flush_amax(out.f16_amax, am);
}

// ------------------------------------------------------------------ attention softmax
// One warp per score row (z, q); lane l holds float4 chunks l + 32*i (i < NC,
// 128*NC >= T) in registers. Keys k <= q are live, the rest are written as 0.
template <int NC>
__global__ void __launch_bounds__(256) softmax_causal_fwd_kernel(const float* __restrict__ S, Planes P, long long rows,
                                                                 int T) {
  griddep_wait();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  const int T4 = T / 4;
  for (long long row = blockIdx.x * (long long)warps + threadIdx.x / 32; row < rows;
       row += (long long)gridDim.x * warps) {
    const int q = (int)(row % T);
    const float4* s4 = reinterpret_cast<const float4*>(S + row * T);
    const int live4 = q / 4 + 1;   // chunks that hold at least one live key
    float4 v[NC];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < live4 ? __ldcs(s4 + c) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (c < live4) {
        const int k = 4 * c;
        if (k + 1 > q) v[i].y = -INFINITY;
        if (k + 2 > q) v[i].z = -INFINITY;
        if (k + 3 > q) v[i].w = -INFINITY;
      }
      m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
    }
    m = warp_max(m);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      v[i].x = expf(v[i].x - m);
      v[i].y = expf(v[i].y - m);
      v[i].z = expf(v[i].z - m);
      v[i].w = expf(v[i].w - m);
      sum += v[i].x + v[i].y + v[i].z + v[i].w;
    }
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      if (c < T4)
        store_planes4(P, row * T + 4 * c, make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv));
    }
  }
}

// dS = P * (dP - sum(P * dP)) * scale (ggml soft_max_back), zero past the diagonal.
template <int NC>
__global__ void __launch_bounds__(256) softmax_causal_bwd_kernel(Planes P, const float* __restrict__ dP, Planes dS,
                                                                 long long rows, int T, float scale) {
  griddep_wait();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  const int T4 = T / 4;
  for (long long row = blockIdx.x * (long long)warps + threadIdx.x / 32; row < rows;
       row += (long long)gridDim.x * warps) {
    const int q = (int)(row % T);
    const long long base = row * T;
    const int live4 = q / 4 + 1;
    float4 pv[NC], gv[NC];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      if (c < live4) {
        pv[i] = load_planes4(P, base + 4 * c);
        gv[i] = __ldcs(reinterpret_cast<const float4*>(dP + base) + c);
        const int k = 4 * c;
        if (k + 1 > q) pv[i].y = 0.f;
        if (k + 2 > q) pv[i].z = 0.f;
        if (k + 3 > q) pv[i].w = 0.f;
      } else {
        pv[i] = f4_zero();
        gv[i] = f4_zero();
      }
      dot += pv[i].x * gv[i].x + pv[i].y * gv[i].y + pv[i].z * gv[i].z + pv[i].w * gv[i].w;
    }
    dot = warp_sum(dot);
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      if (c < T4)
        store_planes4(dS, base + 4 * c,
                      make_float4(pv[i].x * (gv[i].x - dot) * scale, pv[i].y * (gv[i].y - dot) * scale,
                                  pv[i].z * (gv[i].z - dot) * scale, pv[i].w * (gv[i].w - dot) * scale));
    }
  }
}

// ------------------------------------------------------------------ SwiGLU
// One block per token row, float4 over the ff columns of gate | up.
__global__ void __launch_bounds__(128) swiglu_fwd_kernel(const float* __restrict__ gu, Planes a, long long lda, int N,
                                                         int ff) {
  griddep_wait();
  const int ff4 = ff / 4;
  for (int n = blockIdx.x; n < N; n += gridDim.x) {
    const float4* g4 = reinterpret_cast<const float4*>(gu + (long long)n * 2 * ff);
    const float4* u4 = g4 + ff4;
    for (int c = threadIdx.x; c < ff4; c += blockDim.x) {
      const float4 g = __ldcs(g4 + c), u = __ldcs(u4 + c);
      store_planes4(a, (long long)n * lda + 4 * c,
                    make_float4(g.x / (1.0f + expf(-g.x)) * u.x, g.y / (1.0f + expf(-g.y)) * u.y,
                                g.z / (1.0f + expf(-g.z)) * u.z, g.w / (1.0f + expf(-g.w)) * u.w));
    }
  }
}

__device__ __forceinline__ void swiglu_back1(float g, float u, float dy, float& dg, float& du) {
  const float s = 1.0f / (1.0f + expf(-g));
  dg = dy * u * (s * (1.0f + g * (1.0f - s)));
  du = dy * g * s;
}

__global__ void __launch_bounds__(128) swiglu_bwd_kernel(const float* __restrict__ gu, const float* __restrict__ da,
                                                         Planes dgu, long long ldo, int N, int ff) {
  griddep_wait();
  const int ff4 = ff / 4;
  float am = 0.f;   // max |dgate|, |dup| written
  const float s16 = dgu.f16 ? f16_scale_of(dgu) : 1.0f;
  for (int n = blockIdx.x; n < N; n += gridDim.x) {
    const float4* g4 = reinterpret_cast<const float4*>(gu + (long long)n * 2 * ff);
    const float4* u4 = g4 + ff4;
    const float4* d4 = reinterpret_cast<const float4*>(da + (long long)n * ff);
    for (int c = threadIdx.x; c < ff4; c += blockDim.x) {
      const float4 g = g4[c], u = u4[c], dy = __ldcs(d4 + c);
      float4 dg, du;
      swiglu_back1(g.x, u.x, dy.x, dg.x, du.x);
      swiglu_back1(g.y, u.y, dy.y, dg.y, du.y);
      swiglu_back1(g.z, u.z, dy.z, dg.z, du.z);
      swiglu_back1(g.w, u.w, dy.w, dg.w, du.w);
      store_planes4(dgu, (long long)n * ldo + 4 * c, dg, s16);
      store_planes4(dgu, (long long)n * ldo + ff + 4 * c, du, s16);
      am = amax4(amax4(am, dg), du);
    }
  }
  if (dgu.f16_amax) flush_amax(dgu.f16_amax, am);
}

// ------------------------------------------------------------------ cross-entropy
constexpr int kCeThreads = 512;

__device__ __forceinline__ void ms_combine(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = s * expf(m - mm) + s2 * expf(m2 - mm);
  m = mm;
}

__global__ void __launch_bounds__(kCeThreads) cross_entropy_kernel(const float* __restrict__ logits,
                                                                   const int* __restrict__ label_ids,
                                                                   const float* __restrict__ label_dense,
                                                                   float* __restrict__ loss_rows, Planes dl, int N,
                                                                   int V) {
  griddep_wait();
  __shared__ float sm_m[kCeThreads / 32], sm_s[kCeThreads / 32];
  __shared__ float bc[2];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float invN = 1.0f / (float)N;
  const float s16 = dl.f16 ? f16_scale_of(dl) : 1.0f;
  const bool vec = (V % 4) == 0;
  for (int n = blockIdx.x; n < N; n += gridDim.x) {
    const float* z = logits + (long long)n * V;
    float m = -INFINITY, s = 0.f;
    if (vec) {
      const float4* z4 = reinterpret_cast<const float4*>(z);
      for (int v = threadIdx.x; v < V / 4; v += blockDim.x) {
        const float4 x = z4[v];
        const float mx = fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w));
        if (mx > m) {
          s *= expf(m - mx);
          m = mx;
        }
        s += expf(x.x - m) + expf(x.y - m) + expf(x.z - m) + expf(x.w - m);
      }
    } else {
      for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float x = z[v];
        if (x > m) {
          s = s * expf(m - x) + 1.0f;
          m = x;
        } else {
          s += expf(x - m);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      ms_combine(m, s, m2, s2);
    }
    if (lane == 0) { sm_m[warp] = m; sm_s[warp] = s; }
    __syncthreads();
    if (threadIdx.x == 0) {
      float M = sm_m[0], Sx = sm_s[0];
      for (int w = 1; w < kCeThreads / 32; ++w) ms_combine(M, Sx, sm_m[w], sm_s[w]);
      bc[0] = M;
      bc[1] = Sx;
    }
    __syncthreads();
    const float M = bc[0], Ssum = bc[1];
    const float lse = M + logf(Ssum);
    const float inv = 1.0f / Ssum;
    int lab = label_dense ? -1 : label_ids[n];
    if (lab >= V) lab = -1;
    float dense_acc = 0.f;
    if (vec && !label_dense) {
      const float4* z4 = reinterpret_cast<const float4*>(z);
      for (int v = threadIdx.x; v < V / 4; v += blockDim.x) {
        const float4 x = __ldcs(z4 + v);
        float4 g = make_float4(expf(x.x - M) * inv, expf(x.y - M) * inv, expf(x.z - M) * inv, expf(x.w - M) * inv);
        const int k = lab - 4 * v;
        if (k == 0) g.x -= 1.0f;
        if (k == 1) g.y -= 1.0f;
        if (k == 2) g.z -= 1.0f;
        if (k == 3) g.w -= 1.0f;
        store_planes4(dl, (long long)n * V + 4 * v, make_float4(g.x * invN, g.y * invN, g.z * invN, g.w * invN), s16);
      }
    } else {
      for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float x = z[v];
        float y = 0.f;
        if (label_dense) {
          y = label_dense[(long long)n * V + v];
          dense_acc += y * (x - lse);
        } else if (v == lab) {
          y = 1.0f;
        }
        store_planes(dl, (long long)n * V + v, (expf(x - M) * inv - y) * invN, s16);
      }
    }
    if (label_dense) {
      dense_acc = warp_sum(dense_acc);
      __syncthreads();
      if (lane == 0) sm_m[warp] = dense_acc;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < kCeThreads / 32; ++w) t += sm_m[w];
        loss_rows[n] = -t;
      }
    } else if (threadIdx.x == 0) {
      loss_rows[n] = lab >= 0 ? lse - z[lab] : 0.f;
    }
    __syncthreads();
  }
}

// Row statistics from the LM-head GEMM's vocab-chunk pairs: (max, sum exp(z -
// max)) over the G = ceil(V / 64) chunks of row n, combined in chunk-slice
// order (block: 32 rows x 32 slices; slice y takes chunks y, y + 32, ...;
// then the slices in order).
__global__ void __launch_bounds__(1024) lse_combine_kernel(const float2* __restrict__ part, int G, int N,
                                                           float2* __restrict__ ms) {
  griddep_wait();
  __shared__ float2 sm[32][33];
  const int x = threadIdx.x % 32, y = threadIdx.x / 32;
  const int n = blockIdx.x * 32 + x;
  float m = -INFINITY, s = 0.f;
  if (n < N)
    for (int g = y; g < G; g += 32) {
      const float2 p = part[(long long)g * N + n];
      ms_combine(m, s, p.x, p.y);
    }
  sm[y][x] = make_float2(m, s);
  __syncthreads();
  if (y == 0 && n < N) {
    for (int k = 1; k < 32; ++k) ms_combine(m, s, sm[k][x].x, sm[k][x].y);
    ms[n] = make_float2(m, s);
  }
}

// The cross-entropy gradient in one pass over the logits, given each row's
// (max, sum exp): dz = (softmax(z) - onehot(label)) / N as planes; loss row =
// lse - z[label] (0 for label -1).
__global__ void __launch_bounds__(kCeThreads) cross_entropy_grad_kernel(const float* __restrict__ logits,
                                                                        const float2* __restrict__ ms,
                                                                        const int* __restrict__ label_ids,
                                                                        float* __restrict__ loss_rows, Planes dl,
                                                                        int N, int V) {
  griddep_wait();
  const float invN = 1.0f / (float)N;
  const float s16 = dl.f16 ? f16_scale_of(dl) : 1.0f;
  for (int n = blockIdx.x; n < N; n += gridDim.x) {
    const float2 st = ms[n];
    const float M = st.x, inv = 1.0f / st.y;
    const float* z = logits + (long long)n * V;
    int lab = label_ids[n];
    if (lab >= V) lab = -1;
    if ((V % 4) == 0) {
      const float4* z4 = reinterpret_cast<const float4*>(z);
      for (int v = threadIdx.x; v < V / 4; v += blockDim.x) {
        const float4 x = __ldcs(z4 + v);
        float4 g = make_float4(expf(x.x - M) * inv, expf(x.y - M) * inv, expf(x.z - M) * inv, expf(x.w - M) * inv);
        const int k = lab - 4 * v;
        if (k == 0) g.x -= 1.0f;
        if (k == 1) g.y -= 1.0f;
        if (k == 2) g.z -= 1.0f;
        if (k == 3) g.w -= 1.0f;
        store_planes4(dl, (long long)n * V + 4 * v, make_float4(g.x * invN, g.y * invN, g.z * invN, g.w * invN), s16);
      }
    } else {
      for (int v = threadIdx.x; v < V; v += blockDim.x)
        store_planes(dl, (long long)n * V + v, (expf(z[v] - M) * inv - (v == lab ? 1.0f : 0.0f)) * invN, s16);
    }
    if (threadIdx.x == 0) loss_rows[n] = lab >= 0 ? M + logf(st.y) - z[lab] : 0.f;
  }
}

// Per gradient slot: the power-of-two scale of this step's fp16 copies from
// the largest magnitude the previous step wrote (amax * scale < 2^12, a 16x
// margin below the fp16 range) and its inverse for the GEMM epilogue; then the
// slot's record is cleared for this step. A slot without a finite positive
// record keeps its scale.
__global__ void f16_scale_update_kernel(unsigned* amax, float* scale, float* inv, int n) {
  griddep_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float a = __uint_as_float(amax[i]);
    if (a > 0.f && a <= 3.0e38f) {
      int e;
      frexpf(a, &e);   // a < 2^e
      int k = 12 - e;
      k = k < -126 ? -126 : (k > 126 ? 126 : k);
      scale[i] = ldexpf(1.0f, k);
      inv[i] = ldexpf(1.0f, -k);
    }
    amax[i] = 0u;
  }
}

__global__ void loss_reduce_kernel(const float* __restrict__ rows, int N, float* __restrict__ loss) {
  griddep_wait();
  __shared__ float sm[1024 / 32];
  float s = 0.f;
  for (int i = threadIdx.x; i < N; i += blockDim.x) s += rows[i];
  s = warp_sum(s);
  if (threadIdx.x % 32 == 0) sm[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) t += sm[w];
    *loss = t / (float)N;
  }
}

// ------------------------------------------------------------------ AdamW
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, Planes pp, long long n4, const float* __restrict__ hp,
                             float grad_scale) {
  griddep_wait();
  const float alpha = hp[0], b1 = hp[1], b2 = hp[2], eps = hp[3], wd = hp[4], b1h = hp[5], b2h = hp[6];
  const float keep = 1.0f - alpha * wd;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 P = reinterpret_cast<float4*>(p)[i];
    const float4 G = __ldcs(reinterpret_cast<const float4*>(g) + i);
    float4 M = reinterpret_cast<float4*>(m)[i];
    float4 Vv = reinterpret_cast<float4*>(v)[i];
    float* pe = &P.x;
    const float* ge = &G.x;
    float* me = &M.x;
    float* ve = &Vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gg = ge[k] * grad_scale;
      me[k] = me[k] * b1 + gg * (1.0f - b1);
      ve[k] = ve[k] * b2 + gg * gg * (1.0f - b2);
      pe[k] = pe[k] * keep - alpha * (me[k] * b1h) / (sqrtf(ve[k] * b2h) + eps);
    }
    reinterpret_cast<float4*>(p)[i] = P;
    reinterpret_cast<float4*>(m)[i] = M;
    reinterpret_cast<float4*>(v)[i] = Vv;
    if (pp.hi) store_planes4(pp, i * 4, P);
  }
}

// ------------------------------------------------------------------ Q8_0
__global__ void q8_0_to_planes_kernel(const uint8_t* __restrict__ q, Planes out, float* __restrict__ f32,
                                      long long rows, int K) {
  griddep_wait();
  const long long total = rows * K;
  const int row_bytes = K / 32 * 34;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / K;
    const int k = (int)(i % K);
    const uint8_t* blk = q + r * row_bytes + (k / 32) * 34;
    const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    const float val = d * (float)(int8_t)blk[2 + (k % 32)];
    store_planes(out, i, val);
    if (f32) f32[i] = val;
  }
}

// Ring fill (layout in kernels.cuh): the block's descriptors come by value
// (constant bank); each thread takes kRingPer 16-value chunks spaced a grid
// apart, issuing every chunk's loads before converting and storing any.
constexpr int kRingPer = 1;

__device__ __forceinline__ void ring_chunk_loc(const RingLayer& L, long long i, int& k, int& row, int& col) {
  k = 0;
  while (k + 1 < L.n && i >= L.m[k + 1].chunk0) ++k;
  const RingMat& M = L.m[k];
  const int cpr = (M.d_in + M.ext) / 16;
  const long long c = i - M.chunk0;
  row = (int)(c / cpr);
  col = (int)(c % cpr) * 16;
}

// 16-byte global store with an L2 cache-policy hint
__device__ __forceinline__ void st_keep(uint4* p, uint4 v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w), "l"(pol)
               : "memory");
}

__global__ void __launch_bounds__(256) q8_0_ring_kernel(const __grid_constant__ RingLayer L) {
  griddep_wait();
  const uint64_t pol = L.keep ? l2_policy_evict_last() : 0ull;
  const long long total = L.chunks;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < total; i0 += stride * kRingPer) {
    int4 q[kRingPer];
    float sc[kRingPer];
    float4 av[kRingPer][4];
    int kk[kRingPer], rr[kRingPer], cc[kRingPer];
#pragma unroll
    for (int u = 0; u < kRingPer; ++u) {   // loads of every chunk first
      const long long i = i0 + u * stride;
      kk[u] = -1;
      if (i >= total) continue;
      ring_chunk_loc(L, i, kk[u], rr[u], cc[u]);
      const RingMat& M = L.m[kk[u]];
      if (rr[u] < M.d_out && cc[u] < M.d_in) {
        const long long e = (long long)rr[u] * M.d_in + cc[u];
        q[u] = __ldg(reinterpret_cast<const int4*>(M.qv + e));
        sc[u] = __half2float(__ushort_as_half(__ldg(M.qs + e / 32)));
      } else if (rr[u] >= M.d_out) {
        const int t = rr[u] - M.d_out;
        const bool bd = M.bd_r > 0;
        const int a = bd ? 0 : t / 16, j = bd ? t : t % 16;
        const int jmax = bd ? M.ad[0].width / M.bd_w * M.bd_r : M.r;
        if (cc[u] < M.d_in && a < M.n_ad && j < jmax) {
          const float4* src = reinterpret_cast<const float4*>(M.ad[a].A + (long long)j * M.d_in + cc[u]);
#pragma unroll
          for (int v = 0; v < 4; ++v) av[u][v] = __ldg(src + v);
        } else {
#pragma unroll
          for (int v = 0; v < 4; ++v) av[u][v] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kRingPer; ++u) {
      if (kk[u] < 0) continue;
      const RingMat& M = L.m[kk[u]];
      const int row = rr[u], col = cc[u];
      float v[16];
      if (row < M.d_out && col < M.d_in) {
        const int8_t* b = reinterpret_cast<const int8_t*>(&q[u]);
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] = sc[u] * (float)b[t];
      } else if (row < M.d_out && M.bd_r > 0) {
        // block-diagonal adapter: row's block h owns extension columns [h bd_r, (h + 1) bd_r)
        const RingAdapter& ad = M.ad[0];
        const bool on = row >= ad.c0 && row < ad.c0 + ad.width;
        const int h = on ? (row - ad.c0) / M.bd_w : 0;
        const int e0 = col - M.d_in - h * M.bd_r;
        const float* br = on ? ad.B + (long long)(row - ad.c0) * M.bd_r : nullptr;
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] = (on && e0 + t >= 0 && e0 + t < M.bd_r) ? M.s * br[e0 + t] : 0.f;
      } else if (row < M.d_out) {
        const int a = (col - M.d_in) / 16;
        const bool on = a < M.n_ad && row >= M.ad[a].c0 && row < M.ad[a].c0 + M.ad[a].width;
        const float* br = on ? M.ad[a].B + (long long)(row - M.ad[a].c0) * M.r : nullptr;
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] = (on && t < M.r) ? M.s * br[t] : 0.f;
      } else {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          v[4 * w] = av[u][w].x; v[4 * w + 1] = av[u][w].y; v[4 * w + 2] = av[u][w].z; v[4 * w + 3] = av[u][w].w;
        }
      }
      __align__(16) bf16 h[16], l[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) split2(v[t], h[t], l[t]);
      const long long o = (long long)row * (M.d_in + M.ext) + col;
      uint4* ph = reinterpret_cast<uint4*>(M.hi + o);
      uint4* pl = reinterpret_cast<uint4*>(M.lo + o);
      if (L.keep) {
        st_keep(ph, reinterpret_cast<const uint4*>(h)[0], pol);
        st_keep(ph + 1, reinterpret_cast<const uint4*>(h)[1], pol);
        st_keep(pl, reinterpret_cast<const uint4*>(l)[0], pol);
        st_keep(pl + 1, reinterpret_cast<const uint4*>(l)[1], pol);
      } else {
        ph[0] = reinterpret_cast<const uint4*>(h)[0];
        ph[1] = reinterpret_cast<const uint4*>(h)[1];
        pl[0] = reinterpret_cast<const uint4*>(l)[0];
        pl[1] = reinterpret_cast<const uint4*>(l)[1];
      }
    }
  }
}

// Round half away from zero (C roundf / numpy-gguf np_roundf semantics) spelled
// out so a half-way product always rounds outward: t = trunc(v); v - t is exact
// for |v| < 2^23, so the comparison with 0.5 decides ties exactly.
__device__ __forceinline__ int round_half_away(float v) {
  const float t = truncf(v);
  const float r = fabsf(__fsub_rn(v, t));
  const int ti = (int)t;
  return r >= 0.5f ? (v < 0.f ? ti - 1 : ti + 1) : ti;
}

__global__ void q8_0_quantize_kernel(const float* __restrict__ x, uint8_t* __restrict__ q, long long nblocks) {
  griddep_wait();
  for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblocks;
       b += (long long)gridDim.x * blockDim.x) {
    const float* xb = x + b * 32;
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(xb[j]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    // A block is 17 little-endian 16-bit words: the fp16 scale, then q[2j] | q[2j+1] << 8.
    unsigned short* ow = reinterpret_cast<unsigned short*>(q + b * 34);
    ow[0] = __half_as_ushort(__float2half_rn(d));
    for (int j = 0; j < 16; ++j) {
      const int q0 = round_half_away(__fmul_rn(xb[2 * j], id));
      const int q1 = round_half_away(__fmul_rn(xb[2 * j + 1], id));
      ow[1 + j] = (unsigned short)((q0 & 0xFF) | ((q1 & 0xFF) << 8));
    }
  }
}

// One thread per block: 17 little-endian 16-bit words (scale, then quant pairs).
__global__ void q8_0_split_kernel(const uint8_t* __restrict__ blocks, int8_t* __restrict__ qv,
                                  uint16_t* __restrict__ qs, long long nblocks) {
  griddep_wait();
  for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblocks;
       b += (long long)gridDim.x * blockDim.x) {
    const unsigned short* w = reinterpret_cast<const unsigned short*>(blocks + b * 34);
    qs[b] = w[0];
    uint32_t out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = (uint32_t)w[1 + 2 * j] | ((uint32_t)w[2 + 2 * j] << 16);
    uint4* dst = reinterpret_cast<uint4*>(qv + b * 32);
    dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
  }
}

__global__ void colsum_rows_kernel(const float* __restrict__ x, int N, int W, float* __restrict__ out) {
  griddep_wait();
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < W; c += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int n = 0; n < N; ++n) s += x[(long long)n * W + c];
    out[c] = s;
  }
}

__global__ void add_inplace_kernel(float* __restrict__ y, const float* __restrict__ x, long long n) {
  griddep_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] += x[i];
}

__global__ void blockdiag_take_kernel(const float* __restrict__ dense, int nb, int bw, int r,
                                      float* __restrict__ out) {
  griddep_wait();
  const long long n = (long long)nb * bw * r;
  const long long R = (long long)nb * r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / r;
    const int j = (int)(i % r);
    const int h = (int)(row / bw);
    out[i] = dense[row * R + (long long)h * r + j];
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Register-chunk count (float4 chunks per lane) for a row of `len` floats.
int row_chunks(int len) {
  const int nc = (len / 4 + 31) / 32;
  static const int choices[] = {1, 2, 4, 5, 8, 12, 16, 24, 28, 32};
  for (int c : choices)
    if (nc <= c) return c;
  return -1;
}

template <template <int> class F, typename... A>
int dispatch_nc(int nc, A... a) {
  switch (nc) {
    case 1: return F<1>::run(a...);
    case 2: return F<2>::run(a...);
    case 4: return F<4>::run(a...);
    case 5: return F<5>::run(a...);
    case 8: return F<8>::run(a...);
    case 12: return F<12>::run(a...);
    case 16: return F<16>::run(a...);
    case 24: return F<24>::run(a...);
    case 28: return F<28>::run(a...);
    case 32: return F<32>::run(a...);
    default: return -1;
  }
}

// rmsnorm_fwd fused with the low-rank down-projections of the adapters that
// read its output row: u_a[n][j] = sum_k h[n][k] A_a[j][k] for each adapter a
// (A_a [r][d] brought into shared memory once per block by bulk copies that
// land while the warps load and normalise their first rows), plus the B^T
// copies the splice reads. A warp normalises RW rows at a time, so each A value read from
// shared memory serves RW rows; the r sums of an adapter are reduced across the
// warp with warp_sum_multi. With ext_col >= 0, u_a is also written as planes
// into h's columns ext_col + j.
template <int NC, int RT, int NS, int RW>
__global__ void __launch_bounds__(256) rmsnorm_fwd_lora_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ gamma, Planes h, long long ldh,
                                                               int N, int d, float eps, int r, LoraSegs g, int* err) {
  extern __shared__ __align__(128) float4 asm4[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(asm4);   // bytes 0..15
  float* as = reinterpret_cast<float*>(asm4 + 1);      // NS x [r][d]
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  griddep_wait();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(bar, (uint32_t)(NS * r * d * 4));
#pragma unroll
    for (int a = 0; a < NS; ++a) bulk_load(as + a * r * d, g.s[a].w, (uint32_t)(r * d * 4), bar);
  }
  bool a_ready = false;
#pragma unroll
  for (int a = 0; a < NS; ++a) {
    const LoraSeg& sg = g.s[a];
    if (sg.bt) {
      for (long long i = blockIdx.x * 256LL + threadIdx.x; i < (long long)sg.b_rows * r;
           i += (long long)gridDim.x * 256) {
        const int c = (int)(i / r), j = (int)(i % r);
        sg.bt[(long long)j * sg.b_rows + c] = sg.b_src[i];
      }
    }
  }
  __syncthreads();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  const int d4 = d / 4;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  for (int n0 = (blockIdx.x * warps + threadIdx.x / 32) * RW; n0 < N; n0 += gridDim.x * warps * RW) {
    float4 y[RW][NC];
#pragma unroll
    for (int q = 0; q < RW; ++q) {
      const int n = n0 + q;
      const float4* xr = reinterpret_cast<const float4*>(x + (long long)n * d);
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const int c = lane + 32 * i;
        y[q][i] = (n < N && c < d4) ? __ldcs(xr + c) : f4_zero();
      }
    }
#pragma unroll
    for (int q = 0; q < RW; ++q) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < NC; ++i)
        ss += y[q][i].x * y[q][i].x + y[q][i].y * y[q][i].y + y[q][i].z * y[q][i].z + y[q][i].w * y[q][i].w;
      ss = warp_sum(ss);
      const float rr = 1.0f / sqrtf(ss / (float)d + eps);
      const int n = n0 + q;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const int c = lane + 32 * i;
        if (c < d4) {
          const float4 gg = g4[c];
          y[q][i] = make_float4(y[q][i].x * rr * gg.x, y[q][i].y * rr * gg.y, y[q][i].z * rr * gg.z,
                                y[q][i].w * rr * gg.w);
          if (n < N) store_planes4(h, (long long)n * ldh + c * 4, y[q][i]);
        }
      }
    }
    if (!a_ready) {   // the adapters' A have landed
      if (!mbar_wait(bar, 0, err, kErrWaitBulk)) return;
      a_ready = true;
    }
#pragma unroll
    for (int a = 0; a < NS; ++a) {
      float acc[RW][RT];
#pragma unroll
      for (int q = 0; q < RW; ++q)
#pragma unroll
        for (int j = 0; j < RT; ++j) acc[q][j] = 0.f;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const int c = lane + 32 * i;
        if (c < d4) {
#pragma unroll
          for (int j = 0; j < RT; ++j) {
            if (j < r) {
              const float4 w = *reinterpret_cast<const float4*>(as + (a * r + j) * d + c * 4);
#pragma unroll
              for (int q = 0; q < RW; ++q)
                acc[q][j] += y[q][i].x * w.x + y[q][i].y * w.y + y[q][i].z * w.z + y[q][i].w * w.w;
            }
          }
        }
      }
      const LoraSeg& sg = g.s[a];
      const int j = warp_sum_multi_index<RT>(lane);
#pragma unroll
      for (int q = 0; q < RW; ++q) {
        const float t = sg.alpha * warp_sum_multi<RT>(acc[q], lane);
        const int n = n0 + q;
        if (n < N && j < r && warp_sum_multi_leader<RT>(lane)) {
          sg.out[(long long)n * r + j] = t;
          if (sg.ext_col >= 0) {
            bf16 hh, ll;
            split2(t, hh, ll);
            h.hi[(long long)n * ldh + sg.ext_col + j] = hh;
            h.lo[(long long)n * ldh + sg.ext_col + j] = ll;
          }
        }
      }
    }
  }
}

template <int NC>
struct RmsFwdLora {
  template <int RT, int NS>
  static int go(const float* x, const float* gamma, Planes h, long long ldh, int N, int d, float eps, int r,
                const LoraSegs& g, cudaStream_t st) {
    constexpr int RW = NS * RT <= 32 ? 2 : 1;
    auto* kern = rmsnorm_fwd_lora_kernel<NC, RT, NS, RW>;
    static DeviceOnce setup;
    setup.ensure([&](int) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      return 0;
    });
    const size_t smem = 16 + (size_t)NS * r * d * sizeof(float);
    launch_pdl(kern, dim3(grid_for(((long long)N + RW - 1) / RW * 32, 256)), dim3(256), smem, st, x, gamma, h, ldh, N,
               d, eps, r, g, device_error_word());
    return ok();
  }
  static int run(const float* x, const float* gamma, Planes h, long long ldh, int N, int d, float eps, int r,
                 LoraSegs g, cudaStream_t st) {
    if (r <= 8) {
      if (g.n == 1) return go<8, 1>(x, gamma, h, ldh, N, d, eps, r, g, st);
      if (g.n == 2) return go<8, 2>(x, gamma, h, ldh, N, d, eps, r, g, st);
      return go<8, 3>(x, gamma, h, ldh, N, d, eps, r, g, st);
    }
    if (g.n == 1) return go<16, 1>(x, gamma, h, ldh, N, d, eps, r, g, st);
    if (g.n == 2) return go<16, 2>(x, gamma, h, ldh, N, d, eps, r, g, st);
    return go<16, 3>(x, gamma, h, ldh, N, d, eps, r, g, st);
  }
};

template <int NC>
struct RmsFwd {
  static int run(const float* x, const float* gamma, Planes h, long long ldh, int N, int d, float eps,
                 cudaStream_t st) {
    launch_pdl(rmsnorm_fwd_kernel<NC>, dim3(grid_for((long long)N * 32, 256)), dim3(256), 0, st, x, gamma, h, ldh, N, d,
               eps);
    return ok();
  }
};

template <int NC>
struct RmsBwd {
  static int run(const float* x, const float* dh, const float* gamma, const float* dres, float* dx, Planes dxp,
                 long long ldp, float* gpart, int nblk, int N, int d, float eps, cudaStream_t st) {
    const size_t smem = (size_t)8 * d * sizeof(float);
    static DeviceOnce setup;
    setup.ensure([](int) {
      cudaFuncSetAttribute(rmsnorm_bwd_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      return 0;
    });
    launch_pdl(rmsnorm_bwd_kernel<NC>, dim3(nblk), dim3(256), smem, st, x, dh, gamma, dres, dx, dxp, ldp, gpart, N, d,
               eps);
    return ok();
  }
};

template <int NC>
struct SmFwd {
  static int run(const float* S, Planes P, long long rows, int T, cudaStream_t st) {
    launch_pdl(softmax_causal_fwd_kernel<NC>, dim3(grid_for(rows * 32, 256)), dim3(256), 0, st, S, P, rows, T);
    return ok();
  }
};

template <int NC>
struct SmBwd {
  static int run(Planes P, const float* dP, Planes dS, long long rows, int T, float scale, cudaStream_t st) {
    launch_pdl(softmax_causal_bwd_kernel<NC>, dim3(grid_for(rows * 32, 256)), dim3(256), 0, st, P, dP, dS, rows, T, scale);
    return ok();
  }
};

}  // namespace

int rmsnorm_bwd_blocks() { return kRmsBwdBlocks; }

int launch_split_f32(const float* x, bf16* hi, bf16* lo, long long n, cudaStream_t st) {
  if (n <= 0) return 0;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(hi) & 7u) || (reinterpret_cast<uintptr_t>(lo) & 7u)) return -1;
  launch_pdl(split_f32_kernel, dim3(grid_for(n / 4 + 1, 256)), dim3(256), 0, st, x, hi, lo, n);
  return ok();
}

int launch_embed_gather(const float* E, const int* ids, float* x0, int N, int d, cudaStream_t st) {
  if (d % 4) return -1;
  launch_pdl(embed_gather_kernel, dim3(grid_for((long long)N * d / 4, 256)), dim3(256), 0, st, E, ids, x0, N, d / 4);
  return ok();
}

int launch_embed_scatter(const float* dx, const int* order, const int* seg_start, const int* seg_id,
                         const int* nseg_dev, int max_seg, float* dE, int d, cudaStream_t st) {
  if (d % 4 || max_seg <= 0) return -1;
  launch_pdl(embed_scatter_kernel, dim3(grid_for((long long)max_seg * 32, 256)), dim3(256), 0, st, dx, order, seg_start, seg_id,
                                                                               nseg_dev, dE, d);
  return ok();
}

int launch_rmsnorm_fwd(const float* x, const float* gamma, Planes h, int N, int d, float eps, cudaStream_t st,
                       long long ldh) {
  if (ldh == 0) ldh = d;
  if (d % 4 || ldh % 4 || ldh < d) return -1;
  return dispatch_nc<RmsFwd>(row_chunks(d), x, gamma, h, ldh, N, d, eps, st);
}

int launch_rmsnorm_fwd_lora(const float* x, const float* gamma, Planes h, int N, int d, float eps, int r,
                            const LoraSegs& g, cudaStream_t st, long long ldh) {
  if (ldh == 0) ldh = d;
  if (d % 4 || ldh % 4 || ldh < d || r < 1 || r > 16 || g.n < 1 || g.n > kLoraMaxSegs) return -1;
  for (int a = 0; a < g.n; ++a)
    if (g.s[a].ext_col >= 0 && (g.s[a].ext_col < d || g.s[a].ext_col + r > ldh)) return -1;
  if ((size_t)g.n * r * d * 4 + 16 > 200 * 1024) return -2;   // the adapters' A do not fit in shared memory
  for (int a = 0; a < g.n; ++a)
    if (!g.s[a].w || (reinterpret_cast<uintptr_t>(g.s[a].w) & 15) || !g.s[a].out || g.s[a].col_off != 0 ||
        g.s[a].width != d ||
        (g.s[a].bt && (!g.s[a].b_src || g.s[a].b_rows <= 0)))
      return -1;
  switch (row_chunks(d)) {   // the chunk counts whose register arrays stay small next to the adapter sums
    case 1: return RmsFwdLora<1>::run(x, gamma, h, ldh, N, d, eps, r, g, st);
    case 2: return RmsFwdLora<2>::run(x, gamma, h, ldh, N, d, eps, r, g, st);
    case 4: return RmsFwdLora<4>::run(x, gamma, h, ldh, N, d, eps, r, g, st);
    case 5: return RmsFwdLora<5>::run(x, gamma, h, ldh, N, d, eps, r, g, st);
    case 8: return RmsFwdLora<8>::run(x, gamma, h, ldh, N, d, eps, r, g, st);
    case 16: return RmsFwdLora<16>::run(x, gamma, h, ldh, N, d, eps, r, g, st);
    default: return -2;   // caller falls back to rmsnorm_fwd + the group down-projection
  }
}

int launch_rmsnorm_bwd(const float* x, const float* dh, const float* gamma, const float* dres, float* dx,
                       Planes dxp, float* gpart, int nblk, int N, int d, float eps, cudaStream_t st, long long ldp) {
  if (ldp == 0) ldp = d;
  if (d % 4 || ldp % 4 || ldp < d || nblk != kRmsBwdBlocks) return -1;
  if ((size_t)8 * d * sizeof(float) > 200 * 1024) return -1;
  return dispatch_nc<RmsBwd>(row_chunks(d), x, dh, gamma, dres, dx, dxp, ldp, gpart, nblk, N, d, eps, st);
}

int launch_colsum(const float* gpart, int nblk, int d, float* gout, int accumulate, cudaStream_t st) {
  launch_pdl(colsum_kernel, dim3((d + 31) / 32), dim3(256), 0, st, gpart, nblk, d, gout, accumulate);
  return ok();
}

int launch_rope_qkv_fwd(const float* qkv, const float* bias, const int* pos, const float* cs_tab, int tab_rows,
                        Planes Q, Planes K, Planes V, int B, int T, int H, int KV, int dh, cudaStream_t st) {
  if (dh % 2) return -1;
  const int N = B * T;
  launch_pdl(rope_qkv_fwd_kernel, dim3(N < 8 * kSMs ? N : 8 * kSMs), dim3(256), 0, st,
      qkv, bias, pos, reinterpret_cast<const float2*>(cs_tab), tab_rows, Q, K, V, N, T, H, KV, dh);
  return ok();
}

int launch_rope_qkv_bwd(const float* dQ, const float* dK, const float* dV, const int* pos, const float* cs_tab,
                        int tab_rows, Planes dqkv, float* dqkv_f32, int B, int T, int H, int KV, int dh,
                        cudaStream_t st, long long ld_dqkv) {
  return launch_rope_qkv_bwd_sum(dQ, 0, 0, dK, dV, 0, 1, pos, cs_tab, tab_rows, dqkv, dqkv_f32, B, T, H, KV, dh, st,
                                 ld_dqkv);
}

int launch_rope_qkv_bwd_sum(const float* dQ, long long q_pstride, int q_tile, const float* dK, const float* dV,
                            long long kv_pstride, int kv_parts, const int* pos, const float* cs_tab, int tab_rows,
                            Planes dqkv, float* dqkv_f32, int B, int T, int H, int KV, int dh, cudaStream_t st,
                            long long ld_dqkv) {
  const int N = B * T;
  const long long width = (long long)(H + 2 * KV) * dh;
  if (ld_dqkv == 0) ld_dqkv = width;
  if (q_tile < 0 || kv_parts < 1 || ld_dqkv < width || dh % 8 || ld_dqkv % 4 || q_pstride % 4 || kv_pstride % 4)
    return -1;
  const long long items = (long long)N * (H + 2 * KV) * (dh / 8);
  launch_pdl(rope_qkv_bwd_kernel, dim3(grid_for(items, 256)), dim3(256), 0, st, dQ, q_pstride, q_tile, dK, dV,
             kv_pstride, kv_parts, pos, reinterpret_cast<const float2*>(cs_tab), tab_rows, dqkv, ld_dqkv, dqkv_f32, N,
             T, H, KV, dh);
  return ok();
}

int launch_softmax_causal_fwd(const float* S, Planes P, long long Z, int T, cudaStream_t st) {
  if (T % 4) return -1;
  return dispatch_nc<SmFwd>(row_chunks(T), S, P, Z * T, T, st);
}

int launch_softmax_causal_bwd(Planes P, const float* dP, Planes dS, long long Z, int T, float scale,
                              cudaStream_t st) {
  if (T % 4) return -1;
  return dispatch_nc<SmBwd>(row_chunks(T), P, dP, dS, Z * T, T, scale, st);
}

int launch_swiglu_fwd(const float* gu, Planes a, int N, int ff, cudaStream_t st, long long lda) {
  if (lda == 0) lda = ff;
  if (ff % 4 || lda % 4 || lda < ff) return -1;
  launch_pdl(swiglu_fwd_kernel, dim3(N < 16 * kSMs ? N : 16 * kSMs), dim3(128), 0, st, gu, a, lda, N, ff);
  return ok();
}

int launch_swiglu_bwd(const float* gu, const float* da, Planes dgu, int N, int ff, cudaStream_t st, long long ld_dgu) {
  if (ld_dgu == 0) ld_dgu = 2LL * ff;
  if (ff % 4 || ld_dgu % 4 || ld_dgu < 2LL * ff) return -1;
  launch_pdl(swiglu_bwd_kernel, dim3(N < 16 * kSMs ? N : 16 * kSMs), dim3(128), 0, st, gu, da, dgu, ld_dgu, N, ff);
  return ok();
}

int launch_cross_entropy(const float* logits, const int* label_ids, const float* label_dense, float* loss_rows,
                         Planes dlogits, int N, int V, cudaStream_t st) {
  int g = N < 4 * kSMs ? N : 4 * kSMs;
  launch_pdl(cross_entropy_kernel, dim3(g), dim3(kCeThreads), 0, st, logits, label_ids, label_dense, loss_rows, dlogits, N, V);
  return ok();
}

int launch_cross_entropy_lse(const float* logits, const float2* lse_part, float2* ms, const int* label_ids,
                             float* loss_rows, Planes dlogits, int N, int V, cudaStream_t st) {
  launch_pdl(lse_combine_kernel, dim3((N + 31) / 32), dim3(1024), 0, st, lse_part, (V + 63) / 64, N, ms);
  if (ok()) return -3;
  const int g = N < 4 * kSMs ? N : 4 * kSMs;
  launch_pdl(cross_entropy_grad_kernel, dim3(g), dim3(kCeThreads), 0, st, logits, (const float2*)ms, label_ids,
             loss_rows, dlogits, N, V);
  return ok();
}

int launch_f16_scale_update(unsigned* amax, float* scale, float* inv, int n, cudaStream_t st) {
  if (n <= 0) return 0;
  launch_pdl(f16_scale_update_kernel, dim3((n + 255) / 256), dim3(256), 0, st, amax, scale, inv, n);
  return ok();
}

int launch_loss_reduce(const float* loss_rows, int N, float* loss, cudaStream_t st) {
  launch_pdl(loss_reduce_kernel, dim3(1), dim3(1024), 0, st, loss_rows, N, loss);
  return ok();
}

int launch_adamw(float* p, const float* g, float* m, float* v, Planes pp, long long n, const float* hp,
                 float grad_scale, cudaStream_t st) {
  if (n % 4 || !aligned16(p) || !aligned16(g) || !aligned16(m) || !aligned16(v)) return -1;
  launch_pdl(adamw_kernel, dim3(grid_for(n / 4, 256)), dim3(256), 0, st, p, g, m, v, pp, n / 4, hp, grad_scale);
  return ok();
}

int launch_q8_0_to_planes(const uint8_t* q, Planes out, float* f32, long long rows, int K, cudaStream_t st) {
  if (K % 32) return -1;
  launch_pdl(q8_0_to_planes_kernel, dim3(grid_for(rows * K, 256)), dim3(256), 0, st, q, out, f32, rows, K);
  return ok();
}

int launch_q8_0_ring(const RingLayer& desc, cudaStream_t st) {
  if (desc.chunks <= 0 || desc.n < 1 || desc.n > kRingMats) return -1;
  launch_pdl(q8_0_ring_kernel, dim3(grid_for((desc.chunks + kRingPer - 1) / kRingPer, 256)), dim3(256), 0, st, desc);
  return ok();
}

int launch_q8_0_split(const uint8_t* blocks, int8_t* qv, uint16_t* qs, long long nblocks, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(blocks) & 1u) || (reinterpret_cast<uintptr_t>(qv) & 15u) ||
      (reinterpret_cast<uintptr_t>(qs) & 1u))
    return -1;
  launch_pdl(q8_0_split_kernel, dim3(grid_for(nblocks, 128)), dim3(128), 0, st, blocks, qv, qs, nblocks);
  return ok();
}

int launch_q8_0_quantize(const float* x, uint8_t* q, long long rows, int K, cudaStream_t st) {
  if (K % 32 || (reinterpret_cast<uintptr_t>(q) & 1u) || (reinterpret_cast<uintptr_t>(x) & 3u)) return -1;
  const long long nb = rows * (K / 32);
  launch_pdl(q8_0_quantize_kernel, dim3(grid_for(nb, 128)), dim3(128), 0, st, x, q, nb);
  return ok();
}

int launch_colsum_rows(const float* x, int N, int W, float* out, cudaStream_t st) {
  launch_pdl(colsum_rows_kernel, dim3((W + 127) / 128), dim3(128), 0, st, x, N, W, out);
  return ok();
}

int launch_lora_blockdiag_take(const float* dense, int nb, int bw, int r, float* out, cudaStream_t st) {
  if (!dense || !out || nb < 1 || bw < 1 || r < 1) return -1;
  launch_pdl(blockdiag_take_kernel, dim3(grid_for((long long)nb * bw * r, 256)), dim3(256), 0, st, dense, nb, bw, r,
             out);
  return ok();
}

int launch_add_inplace(float* y, const float* x, long long n, cudaStream_t st) {
  launch_pdl(add_inplace_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, y, x, n);
  return ok();
}

}  // namespace tb2
