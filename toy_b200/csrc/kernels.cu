// Bandwidth-bound kernels of the training step: vectorised loads, warp-shuffle
// reductions, fixed-order (deterministic) reductions, grids sized in multiples
// of the SM count.
#include "kernels.cuh"

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

__device__ __forceinline__ void store_planes(const Planes& p, long long i, float x) {
  bf16 h, l;
  split2(x, h, l);
  p.hi[i] = h;
  p.lo[i] = l;
}

// Four consecutive values (i % 4 == 0) as two 8-byte stores.
__device__ __forceinline__ void store_planes4(const Planes& p, long long i, float4 v) {
  __align__(8) bf16 h[4], l[4];
  split2(v.x, h[0], l[0]);
  split2(v.y, h[1], l[1]);
  split2(v.z, h[2], l[2]);
  split2(v.w, h[3], l[3]);
  *reinterpret_cast<uint2*>(p.hi + i) = *reinterpret_cast<const uint2*>(h);
  *reinterpret_cast<uint2*>(p.lo + i) = *reinterpret_cast<const uint2*>(l);
}

__device__ __forceinline__ float load_planes(const Planes& p, long long i) {
  return __bfloat162float(p.hi[i]) + __bfloat162float(p.lo[i]);
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
__global__ void rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma, Planes h, int N,
                                   int d, float eps) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  const int d4 = d / 4;
  for (int n = blockIdx.x * warps + threadIdx.x / 32; n < N; n += gridDim.x * warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + (long long)n * d);
    float ss = 0.f;
    for (int c = lane; c < d4; c += 32) {
      const float4 v = xr[c];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)d + eps);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    for (int c = lane; c < d4; c += 32) {
      const float4 v = xr[c], g = g4[c];
      store_planes4(h, (long long)n * d + c * 4, make_float4(v.x * r * g.x, v.y * r * g.y, v.z * r * g.z, v.w * r * g.w));
    }
  }
}

// Block of 8 warps; warp w accumulates dgamma over its rows in shared memory
// (fixed row order per warp, fixed warp order in the block sum).
__global__ void rmsnorm_bwd_kernel(const float* __restrict__ x, const float* __restrict__ dh,
                                   const float* __restrict__ gamma, const float* dres, float* dx, Planes dxp,
                                   float* __restrict__ gpart, int N, int d, float eps) {
  extern __shared__ float gacc[];  // [warps][d]
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int d4 = d / 4;
  float* my = gacc + warp * d;
  for (int c = lane; c < d; c += 32) my[c] = 0.f;
  __syncwarp();
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  for (int n = blockIdx.x * warps + warp; n < N; n += gridDim.x * warps) {
    const long long base = (long long)n * d;
    const float4* xr = reinterpret_cast<const float4*>(x + base);
    const float4* hr = reinterpret_cast<const float4*>(dh + base);
    float sxx = 0.f, sxdz = 0.f;
    for (int c = lane; c < d4; c += 32) {
      const float4 v = xr[c], gg = hr[c], g = g4[c];
      sxx += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      sxdz += v.x * gg.x * g.x + v.y * gg.y * g.y + v.z * gg.z * g.z + v.w * gg.w * g.w;
    }
    sxx = warp_sum(sxx);
    sxdz = warp_sum(sxdz);
    const float rr = 1.0f / sqrtf(sxx / (float)d + eps);
    const float coef = sxdz / (sxx + (float)d * eps);
    const float4* rres = dres ? reinterpret_cast<const float4*>(dres + base) : nullptr;
    float4* out = reinterpret_cast<float4*>(dx + base);
    for (int c = lane; c < d4; c += 32) {
      const float4 v = xr[c], gg = hr[c], g = g4[c];
      const float4 rs = rres ? rres[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 o;
      o.x = rs.x + (gg.x * g.x - v.x * coef) * rr;
      o.y = rs.y + (gg.y * g.y - v.y * coef) * rr;
      o.z = rs.z + (gg.z * g.z - v.z * coef) * rr;
      o.w = rs.w + (gg.w * g.w - v.w * coef) * rr;
      out[c] = o;
      if (dxp.hi) store_planes4(dxp, base + c * 4, o);
      my[4 * c + 0] += gg.x * v.x * rr;
      my[4 * c + 1] += gg.y * v.y * rr;
      my[4 * c + 2] += gg.z * v.z * rr;
      my[4 * c + 3] += gg.w * v.w * rr;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < warps; ++w) s += gacc[w * d + c];
    gpart[(long long)blockIdx.x * d + c] = s;
  }
}

__global__ void colsum_kernel(const float* __restrict__ gpart, int nblk, int d, float* gout, int accumulate) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < d; c += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int b = 0; b < nblk; ++b) s += gpart[(long long)b * d + c];
    gout[c] = accumulate ? gout[c] + s : s;
  }
}

// ------------------------------------------------------------------ RoPE
__global__ void rope_qkv_fwd_kernel(const float* __restrict__ qkv, const float* __restrict__ bias,
                                    const int* __restrict__ pos, const float2* __restrict__ cs, int tab_rows, Planes Q,
                                    Planes K, Planes V, int B, int T, int H, int KV, int dh) {
  const int half = dh / 2;
  const int slots = H + 2 * KV;
  const long long total = (long long)B * T * slots * half;
  const int width = slots * dh;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const long long r = i / half;
    const int slot = (int)(r % slots);
    const int n = (int)(r / slots);
    const int b = n / T, t = n % T;
    const long long src = (long long)n * width + slot * dh + j;
    float x0 = qkv[src], x1 = qkv[src + half];
    if (bias) {
      x0 += bias[slot * dh + j];
      x1 += bias[slot * dh + j + half];
    }
    if (slot < H + KV) {
      int p = pos[n];
      p = p < 0 ? 0 : (p >= tab_rows ? tab_rows - 1 : p);
      const float2 c = cs[(long long)p * half + j];
      const float y0 = x0 * c.x - x1 * c.y;
      const float y1 = x0 * c.y + x1 * c.x;
      const bool isq = slot < H;
      const int hh = isq ? slot : slot - H;
      const long long dst = (((long long)b * (isq ? H : KV) + hh) * T + t) * dh + j;
      const Planes& o = isq ? Q : K;
      store_planes(o, dst, y0);
      store_planes(o, dst + half, y1);
    } else {
      const int hh = slot - H - KV;
      const long long dst = (((long long)b * KV + hh) * T + t) * dh + j;
      store_planes(V, dst, x0);
      store_planes(V, dst + half, x1);
    }
  }
}

__global__ void rope_qkv_bwd_kernel(const float* __restrict__ dQ, const float* __restrict__ dK,
                                    const float* __restrict__ dV, const int* __restrict__ pos,
                                    const float2* __restrict__ cs, int tab_rows, Planes out, float* out_f32, int B,
                                    int T, int H, int KV, int dh) {
  const int half = dh / 2;
  const int slots = H + 2 * KV;
  const long long total = (long long)B * T * slots * half;
  const int width = slots * dh;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const long long r = i / half;
    const int slot = (int)(r % slots);
    const int n = (int)(r / slots);
    const int b = n / T, t = n % T;
    float y0, y1;
    if (slot < H + KV) {
      const bool isq = slot < H;
      const int hh = isq ? slot : slot - H;
      const float* srcb = isq ? dQ : dK;
      const long long src = (((long long)b * (isq ? H : KV) + hh) * T + t) * dh + j;
      const float g0 = srcb[src], g1 = srcb[src + half];
      int p = pos[n];
      p = p < 0 ? 0 : (p >= tab_rows ? tab_rows - 1 : p);
      const float2 c = cs[(long long)p * half + j];
      y0 = g0 * c.x + g1 * c.y;
      y1 = -g0 * c.y + g1 * c.x;
    } else {
      const int hh = slot - H - KV;
      const long long src = (((long long)b * KV + hh) * T + t) * dh + j;
      y0 = dV[src];
      y1 = dV[src + half];
    }
    const long long dst = (long long)n * width + slot * dh + j;
    store_planes(out, dst, y0);
    store_planes(out, dst + half, y1);
    if (out_f32) {
      out_f32[dst] = y0;
      out_f32[dst + half] = y1;
    }
  }
}

// ------------------------------------------------------------------ attention softmax
__global__ void softmax_causal_fwd_kernel(const float* __restrict__ S, Planes P, long long rows, int T) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (long long row = blockIdx.x * (long long)warps + threadIdx.x / 32; row < rows;
       row += (long long)gridDim.x * warps) {
    const int q = (int)(row % T);
    const float* s = S + row * T;
    float m = -INFINITY;
    for (int k = lane; k <= q; k += 32) m = fmaxf(m, s[k]);
    m = warp_max(m);
    float sum = 0.f;
    for (int k = lane; k <= q; k += 32) sum += expf(s[k] - m);
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
    for (int k = lane; k < T; k += 32) store_planes(P, row * T + k, k <= q ? expf(s[k] - m) * inv : 0.f);
  }
}

__global__ void softmax_causal_bwd_kernel(Planes P, const float* __restrict__ dP, Planes dS, long long rows, int T,
                                          float scale) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (long long row = blockIdx.x * (long long)warps + threadIdx.x / 32; row < rows;
       row += (long long)gridDim.x * warps) {
    const int q = (int)(row % T);
    const long long base = row * T;
    float dot = 0.f;
    for (int k = lane; k <= q; k += 32) dot += load_planes(P, base + k) * dP[base + k];
    dot = warp_sum(dot);
    for (int k = lane; k < T; k += 32) {
      const float v = k <= q ? load_planes(P, base + k) * (dP[base + k] - dot) * scale : 0.f;
      store_planes(dS, base + k, v);
    }
  }
}

// ------------------------------------------------------------------ SwiGLU
__global__ void swiglu_fwd_kernel(const float* __restrict__ gu, Planes a, int N, int ff) {
  const long long total = (long long)N * ff;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / ff;
    const int j = (int)(i % ff);
    const float g = gu[n * 2 * ff + j], u = gu[n * 2 * ff + ff + j];
    store_planes(a, i, g / (1.0f + expf(-g)) * u);
  }
}

__global__ void swiglu_bwd_kernel(const float* __restrict__ gu, const float* __restrict__ da, Planes dgu, int N,
                                  int ff) {
  const long long total = (long long)N * ff;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / ff;
    const int j = (int)(i % ff);
    const float g = gu[n * 2 * ff + j], u = gu[n * 2 * ff + ff + j];
    const float s = 1.0f / (1.0f + expf(-g));
    const float dy = da[i];
    store_planes(dgu, n * 2 * ff + j, dy * u * (s * (1.0f + g * (1.0f - s))));
    store_planes(dgu, n * 2 * ff + ff + j, dy * g * s);
  }
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
  __shared__ float sm_m[kCeThreads / 32], sm_s[kCeThreads / 32];
  __shared__ float bc[2];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float invN = 1.0f / (float)N;
  for (int n = blockIdx.x; n < N; n += gridDim.x) {
    const float* z = logits + (long long)n * V;
    float m = -INFINITY, s = 0.f;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const float x = z[v];
      if (x > m) {
        s = s * expf(m - x) + 1.0f;
        m = x;
      } else {
        s += expf(x - m);
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
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const float x = z[v];
      float y = 0.f;
      if (label_dense) {
        y = label_dense[(long long)n * V + v];
        dense_acc += y * (x - lse);
      } else if (v == lab) {
        y = 1.0f;
      }
      store_planes(dl, (long long)n * V + v, (expf(x - M) * inv - y) * invN);
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

__global__ void loss_reduce_kernel(const float* __restrict__ rows, int N, float* __restrict__ loss) {
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
  const float alpha = hp[0], b1 = hp[1], b2 = hp[2], eps = hp[3], wd = hp[4], b1h = hp[5], b2h = hp[6];
  const float keep = 1.0f - alpha * wd;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 P = reinterpret_cast<float4*>(p)[i];
    const float4 G = reinterpret_cast<const float4*>(g)[i];
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

__global__ void colsum_rows_kernel(const float* __restrict__ x, int N, int W, float* __restrict__ out) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < W; c += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int n = 0; n < N; ++n) s += x[(long long)n * W + c];
    out[c] = s;
  }
}

__global__ void add_inplace_kernel(float* __restrict__ y, const float* __restrict__ x, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] += x[i];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int rmsnorm_bwd_blocks() { return kRmsBwdBlocks; }

int launch_split_f32(const float* x, bf16* hi, bf16* lo, long long n, cudaStream_t st) {
  if (n <= 0) return 0;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(hi) & 7u) || (reinterpret_cast<uintptr_t>(lo) & 7u)) return -1;
  split_f32_kernel<<<grid_for(n / 4 + 1, 256), 256, 0, st>>>(x, hi, lo, n);
  return ok();
}

int launch_embed_gather(const float* E, const int* ids, float* x0, int N, int d, cudaStream_t st) {
  if (d % 4) return -1;
  embed_gather_kernel<<<grid_for((long long)N * d / 4, 256), 256, 0, st>>>(E, ids, x0, N, d / 4);
  return ok();
}

int launch_embed_scatter(const float* dx, const int* order, const int* seg_start, const int* seg_id,
                         const int* nseg_dev, int max_seg, float* dE, int d, cudaStream_t st) {
  if (d % 4 || max_seg <= 0) return -1;
  embed_scatter_kernel<<<grid_for((long long)max_seg * 32, 256), 256, 0, st>>>(dx, order, seg_start, seg_id,
                                                                               nseg_dev, dE, d);
  return ok();
}

int launch_rmsnorm_fwd(const float* x, const float* gamma, Planes h, int N, int d, float eps, cudaStream_t st) {
  if (d % 4) return -1;
  rmsnorm_fwd_kernel<<<grid_for((long long)N * 32, 256), 256, 0, st>>>(x, gamma, h, N, d, eps);
  return ok();
}

int launch_rmsnorm_bwd(const float* x, const float* dh, const float* gamma, const float* dres, float* dx,
                       Planes dxp, float* gpart, int nblk, int N, int d, float eps, cudaStream_t st) {
  if (d % 4 || nblk != kRmsBwdBlocks) return -1;
  const int threads = 256;
  const size_t smem = (size_t)(threads / 32) * d * sizeof(float);
  if (smem > 200 * 1024) return -1;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  rmsnorm_bwd_kernel<<<nblk, threads, smem, st>>>(x, dh, gamma, dres, dx, dxp, gpart, N, d, eps);
  return ok();
}

int launch_colsum(const float* gpart, int nblk, int d, float* gout, int accumulate, cudaStream_t st) {
  colsum_kernel<<<(d + 255) / 256, 256, 0, st>>>(gpart, nblk, d, gout, accumulate);
  return ok();
}

int launch_rope_qkv_fwd(const float* qkv, const float* bias, const int* pos, const float* cs_tab, int tab_rows,
                        Planes Q, Planes K, Planes V, int B, int T, int H, int KV, int dh, cudaStream_t st) {
  if (dh % 2) return -1;
  const long long total = (long long)B * T * (H + 2 * KV) * (dh / 2);
  rope_qkv_fwd_kernel<<<grid_for(total, 256), 256, 0, st>>>(qkv, bias, pos, reinterpret_cast<const float2*>(cs_tab),
                                                            tab_rows, Q, K, V, B, T, H, KV, dh);
  return ok();
}

int launch_rope_qkv_bwd(const float* dQ, const float* dK, const float* dV, const int* pos, const float* cs_tab,
                        int tab_rows, Planes dqkv, float* dqkv_f32, int B, int T, int H, int KV, int dh,
                        cudaStream_t st) {
  const long long total = (long long)B * T * (H + 2 * KV) * (dh / 2);
  rope_qkv_bwd_kernel<<<grid_for(total, 256), 256, 0, st>>>(dQ, dK, dV, pos, reinterpret_cast<const float2*>(cs_tab),
                                                            tab_rows, dqkv, dqkv_f32, B, T, H, KV, dh);
  return ok();
}

int launch_softmax_causal_fwd(const float* S, Planes P, long long Z, int T, cudaStream_t st) {
  softmax_causal_fwd_kernel<<<grid_for(Z * T * 32, 256), 256, 0, st>>>(S, P, Z * T, T);
  return ok();
}

int launch_softmax_causal_bwd(Planes P, const float* dP, Planes dS, long long Z, int T, float scale,
                              cudaStream_t st) {
  softmax_causal_bwd_kernel<<<grid_for(Z * T * 32, 256), 256, 0, st>>>(P, dP, dS, Z * T, T, scale);
  return ok();
}

int launch_swiglu_fwd(const float* gu, Planes a, int N, int ff, cudaStream_t st) {
  swiglu_fwd_kernel<<<grid_for((long long)N * ff, 256), 256, 0, st>>>(gu, a, N, ff);
  return ok();
}

int launch_swiglu_bwd(const float* gu, const float* da, Planes dgu, int N, int ff, cudaStream_t st) {
  swiglu_bwd_kernel<<<grid_for((long long)N * ff, 256), 256, 0, st>>>(gu, da, dgu, N, ff);
  return ok();
}

int launch_cross_entropy(const float* logits, const int* label_ids, const float* label_dense, float* loss_rows,
                         Planes dlogits, int N, int V, cudaStream_t st) {
  int g = N < 4 * kSMs ? N : 4 * kSMs;
  cross_entropy_kernel<<<g, kCeThreads, 0, st>>>(logits, label_ids, label_dense, loss_rows, dlogits, N, V);
  return ok();
}

int launch_loss_reduce(const float* loss_rows, int N, float* loss, cudaStream_t st) {
  loss_reduce_kernel<<<1, 1024, 0, st>>>(loss_rows, N, loss);
  return ok();
}

int launch_adamw(float* p, const float* g, float* m, float* v, Planes pp, long long n, const float* hp,
                 float grad_scale, cudaStream_t st) {
  if (n % 4 || !aligned16(p) || !aligned16(g) || !aligned16(m) || !aligned16(v)) return -1;
  adamw_kernel<<<grid_for(n / 4, 256), 256, 0, st>>>(p, g, m, v, pp, n / 4, hp, grad_scale);
  return ok();
}

int launch_q8_0_to_planes(const uint8_t* q, Planes out, float* f32, long long rows, int K, cudaStream_t st) {
  if (K % 32) return -1;
  q8_0_to_planes_kernel<<<grid_for(rows * K, 256), 256, 0, st>>>(q, out, f32, rows, K);
  return ok();
}

int launch_q8_0_quantize(const float* x, uint8_t* q, long long rows, int K, cudaStream_t st) {
  if (K % 32 || (reinterpret_cast<uintptr_t>(q) & 1u) || (reinterpret_cast<uintptr_t>(x) & 3u)) return -1;
  const long long nb = rows * (K / 32);
  q8_0_quantize_kernel<<<grid_for(nb, 128), 128, 0, st>>>(x, q, nb);
  return ok();
}

int launch_colsum_rows(const float* x, int N, int W, float* out, cudaStream_t st) {
  colsum_rows_kernel<<<(W + 127) / 128, 128, 0, st>>>(x, N, W, out);
  return ok();
}

int launch_add_inplace(float* y, const float* x, long long n, cudaStream_t st) {
  add_inplace_kernel<<<grid_for(n, 256), 256, 0, st>>>(y, x, n);
  return ok();
}

}  // namespace tb2
