// Low-rank adapter kernels (see lora.cuh). Every reduction runs in a fixed
// order, so results do not depend on scheduling.
#include "lora.cuh"

#include <algorithm>

#include "pdl.cuh"
#include "runtime.cuh"
#include "tc_common.cuh"
#include "warp_reduce.cuh"

namespace tb2 {

namespace {

constexpr int kWgradChunks = 32;   // token chunks of the weight-gradient reduction (at least)
constexpr int kWgradSmem = 16 * 1024;   // a chunk's S rows staged in shared memory

// Chunking of the N tokens: at least kWgradChunks chunks, each small enough
// for its S rows to fit kWgradSmem.
void wgrad_chunks(int N, int r, int& nch, int& chunk) {
  chunk = (N + kWgradChunks - 1) / kWgradChunks;
  const int cap = kWgradSmem / (4 * r);
  if (chunk > cap) chunk = cap;
  if (chunk < 1) chunk = 1;
  nch = (N + chunk - 1) / chunk;
}

__device__ __forceinline__ float4 load_planes4(Planes p, long long i) {
  const uint2 h = *reinterpret_cast<const uint2*>(p.hi + i);
  const uint2 l = *reinterpret_cast<const uint2*>(p.lo + i);
  return make_float4(__uint_as_float(h.x << 16) + __uint_as_float(l.x << 16),
                     __uint_as_float(h.x & 0xffff0000u) + __uint_as_float(l.x & 0xffff0000u),
                     __uint_as_float(h.y << 16) + __uint_as_float(l.y << 16),
                     __uint_as_float(h.y & 0xffff0000u) + __uint_as_float(l.y & 0xffff0000u));
}

__device__ __forceinline__ float2 load_planes2(Planes p, long long i) {
  const uint32_t h = *reinterpret_cast<const uint32_t*>(p.hi + i);
  const uint32_t l = *reinterpret_cast<const uint32_t*>(p.lo + i);
  return make_float2(__uint_as_float(h << 16) + __uint_as_float(l << 16),
                     __uint_as_float(h & 0xffff0000u) + __uint_as_float(l & 0xffff0000u));
}

// Output element (0, m, n) of the GEMM epilogue addressing (gemm.cuh).
__device__ __forceinline__ long long out_offset(const Epilogue& e, int m, int n) {
  return (long long)(m / e.m_div) * e.m_s1 + (long long)(m % e.m_div) * e.m_s0 + (long long)(n / e.n_div) * e.n_s1 +
         (n % e.n_div);
}

// One warp per row: lane l covers columns 4l, 4l + 128, ...; the r partial
// sums are reduced across the warp by butterfly shuffles. W is staged in
// shared memory ([r][K], read as float4 along K: conflict-free) when it fits;
// each warp keeps two rows in flight.
template <int RT, bool SMEM_W>
__global__ void __launch_bounds__(256) lora_down_kernel(Planes X, long long ldx, int N, int K,
                                                        const float* __restrict__ W, int r, float alpha,
                                                        float* __restrict__ out, const float* __restrict__ bsrc,
                                                        int bc, float* __restrict__ bt) {
  griddep_wait();
  // side job: bt[j][c] = bsrc[c][j] (the adapter's B transposed for the splice)
  if (bt) {
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < (long long)bc * r; i += (long long)gridDim.x * 256) {
      const int c = (int)(i / r), j = (int)(i % r);
      bt[(long long)j * bc + c] = bsrc[i];
    }
  }
  extern __shared__ float4 wsm4[];
  const float* w = W;
  if (SMEM_W) {
    float* wsm = reinterpret_cast<float*>(wsm4);
    for (int i = threadIdx.x * 4; i < r * K; i += 256 * 4)
      *reinterpret_cast<float4*>(wsm + i) = __ldg(reinterpret_cast<const float4*>(W + i));
    __syncthreads();
    w = wsm;
  }
  const int lane = threadIdx.x % 32;
  const int warps = gridDim.x * 8;
  for (int n = (blockIdx.x * 8 + threadIdx.x / 32) * 2; n < N; n += warps * 2) {
    const bool two = n + 1 < N;
    float acc0[RT], acc1[RT];
#pragma unroll
    for (int j = 0; j < RT; ++j) acc0[j] = acc1[j] = 0.f;
    for (int k = lane * 4; k < K; k += 128) {
      const float4 x0 = load_planes4(X, (long long)n * ldx + k);
      const float4 x1 = two ? load_planes4(X, (long long)(n + 1) * ldx + k) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < RT; ++j) {
        if (j < r) {
          const float4 wv = *reinterpret_cast<const float4*>(w + (long long)j * K + k);
          acc0[j] += x0.x * wv.x + x0.y * wv.y + x0.z * wv.z + x0.w * wv.w;
          acc1[j] += x1.x * wv.x + x1.y * wv.y + x1.z * wv.z + x1.w * wv.w;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < RT; ++j) {
      float v0 = acc0[j], v1 = acc1[j];
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        v0 += __shfl_xor_sync(0xffffffffu, v0, o);
        v1 += __shfl_xor_sync(0xffffffffu, v1, o);
      }
      if (j < r && lane == (j & 31)) {
        out[(long long)n * r + j] = alpha * v0;
        if (two) out[(long long)(n + 1) * r + j] = alpha * v1;
      }
    }
  }
}

// Tile of 32 rows x 128 columns: thread (ty, tx) owns rows 4 ty .. 4 ty + 3 and
// columns 4 tx .. 4 tx + 3.
template <int RT>
__global__ void __launch_bounds__(256) lora_up_kernel(const float* __restrict__ U, int N, int r,
                                                      const float* __restrict__ W, int C, float alpha, Epilogue e) {
  griddep_wait();
  __shared__ float us[32][RT];
  __shared__ __align__(16) float ws[RT][128];
  const int tid = threadIdx.x, tx = tid % 32, ty = tid / 32;
  const int c0 = blockIdx.x * 128, n0 = blockIdx.y * 32;
  for (int i = tid; i < 32 * r; i += 256) {
    const int rr = i / r, j = i % r;
    us[rr][j] = n0 + rr < N ? U[(long long)(n0 + rr) * r + j] : 0.f;
  }
  for (int i = tid; i < r * 128; i += 256) {
    const int j = i / 128, cc = i % 128;
    ws[j][cc] = c0 + cc < C ? W[(long long)j * C + c0 + cc] : 0.f;
  }
  __syncthreads();
  float4 acc[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < RT; ++j) {
    if (j < r) {
      const float4 w = *reinterpret_cast<const float4*>(&ws[j][tx * 4]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float u = us[ty * 4 + q][j];
        acc[q].x += u * w.x; acc[q].y += u * w.y; acc[q].z += u * w.z; acc[q].w += u * w.w;
      }
    }
  }
  const int c = c0 + tx * 4;
  if (c >= C) return;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int n = n0 + ty * 4 + q;
    if (n >= N) break;
    float4* y = reinterpret_cast<float4*>(e.out + out_offset(e, n, c));
    float4 v = *y;
    v.x += alpha * acc[q].x; v.y += alpha * acc[q].y; v.z += alpha * acc[q].z; v.w += alpha * acc[q].w;
    *y = v;
  }
}

// Block of WARPS warps over 64 columns (lane: columns 2 l, 2 l + 1) and the
// token chunk by; warp w takes tokens n0 + w, n0 + w + WARPS, ... and the
// warps' sums are added in warp order: partial[by][c][j] = sum over the chunk
// of Big[n][c] * S[n][j].
template <int RT>
struct WgradCfg {
  static constexpr int kWarps = RT <= 16 ? 8 : (RT <= 32 ? 4 : 2);
};

template <int RT>
__global__ void __launch_bounds__(WgradCfg<RT>::kWarps * 32)
    lora_wgrad_partial_kernel(Planes Big, long long ldb, const float* __restrict__ S, int N, int C, int r, int chunk,
                              float* __restrict__ partial) {
  griddep_wait();
  constexpr int WARPS = WgradCfg<RT>::kWarps;
  extern __shared__ float ss[];          // [chunk][r] S rows, then [WARPS][64][RT] warp sums
  float* red = ss + chunk * r;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int c = blockIdx.x * 64 + lane * 2;
  const int n0 = blockIdx.y * chunk;
  const int n1 = min(N, n0 + chunk);
  for (int i = threadIdx.x; i < (n1 - n0) * r; i += WARPS * 32) ss[i] = S[(long long)n0 * r + i];
  __syncthreads();
  float a0[RT], a1[RT];
#pragma unroll
  for (int j = 0; j < RT; ++j) a0[j] = a1[j] = 0.f;
  if (c < C) {
#pragma unroll 4
    for (int n = n0 + warp; n < n1; n += WARPS) {
      const float2 b = load_planes2(Big, (long long)n * ldb + c);
      const float* sr = ss + (n - n0) * r;
#pragma unroll
      for (int j = 0; j < RT; ++j) {
        if (j < r) {
          const float sv = sr[j];
          a0[j] += b.x * sv;
          a1[j] += b.y * sv;
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < RT; ++j) {
    red[(warp * 64 + lane * 2) * RT + j] = a0[j];
    red[(warp * 64 + lane * 2 + 1) * RT + j] = a1[j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * r; i += WARPS * 32) {
    const int cc = i / r, j = i % r;
    if (blockIdx.x * 64 + cc >= C) continue;
    float sum = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < WARPS; ++w2) sum += red[(w2 * 64 + cc) * RT + j];
    partial[((long long)blockIdx.y * C + blockIdx.x * 64 + cc) * r + j] = sum;
  }
}

__global__ void lora_wgrad_reduce_kernel(const float* __restrict__ partial, int nch, int C, int r, float alpha,
                                         float* __restrict__ out, long long o_sc, long long o_sj) {
  griddep_wait();
  const long long total = (long long)C * r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int ch = 0; ch < nch; ++ch) s += partial[(long long)ch * total + i];
    const int c = (int)(i / r), j = (int)(i % r);
    out[(long long)c * o_sc + (long long)j * o_sj] = alpha * s;
  }
}

__global__ void lora_transpose_kernel(const float* __restrict__ W, int C, int r, float* __restrict__ Wt) {
  griddep_wait();
  const long long total = (long long)C * r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i / C), c = (int)(i % C);
    Wt[i] = W[(long long)c * r + j];
  }
}

// Tensor-core weight gradients of a wide adapter group (lora.cuh): the group's
// u (or du) vectors side by side as split planes, out[n][i r + j] = src_i[n][j],
// zero in the columns past n_src r.
__global__ void lora_pack_planes_kernel(LoraPackSrc src, int N, int r, int R, Planes out) {
  griddep_wait();
  const long long total = (long long)N * (R / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / (R / 2);
    const int c = (int)(i % (R / 2)) * 2;
    float v[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int seg = (c + e) / r, j = (c + e) % r;
      v[e] = seg < src.n ? src.p[seg][n * r + j] : 0.f;
    }
    uint32_t h, l;
    split_pair(v[0], v[1], h, l);
    *reinterpret_cast<uint32_t*>(out.hi + n * R + c) = h;
    *reinterpret_cast<uint32_t*>(out.lo + n * R + c) = l;
  }
}

// Packed adapter weights W [R][K] as split planes (lora.cuh launch_lora_pack_w).
__global__ void lora_pack_w_kernel(LoraPackW src, int R, int K, Planes out) {
  griddep_wait();
  const long long total = (long long)R * (K / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / (K / 2)), k0 = (int)(i % (K / 2)) * 2;
    const int a = row / src.r, j = row % src.r;
    float v[2] = {0.f, 0.f};
    if (a < src.n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = k0 + e - src.koff[a];
        if (c >= 0 && c < src.w[a])
          v[e] = src.trans ? src.p[a][(long long)c * src.r + j] : src.p[a][(long long)j * src.w[a] + c];
      }
    }
    uint32_t h, l;
    split_pair(v[0], v[1], h, l);
    *reinterpret_cast<uint32_t*>(out.hi + (long long)row * K + k0) = h;
    *reinterpret_cast<uint32_t*>(out.lo + (long long)row * K + k0) = l;
  }
}

// u of each adapter from D [N][R] (lora.cuh launch_lora_scatter_u).
__global__ void lora_scatter_u_kernel(const float* __restrict__ D, int N, int R, LoraScatterU dst) {
  griddep_wait();
  const long long total = (long long)N * dst.n * dst.r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / (dst.n * dst.r);
    const int c = (int)(i % (dst.n * dst.r)), a = c / dst.r, j = c % dst.r;
    const float v = dst.alpha * D[n * R + c];
    dst.out[a][n * dst.r + j] = v;
    if (dst.ext_col[a] >= 0) {
      const __nv_bfloat16 h = __float2bfloat16_rn(v);
      const long long e = n * dst.ldx + dst.ext_col[a] + j;
      dst.X.hi[e] = h;
      dst.X.lo[e] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
  }
}

// dA_i[j][k] = DA[k][i r + j] (DA = X^T [du_0 | du_1 | ..], [d_in][R]) and
// dB_i[c][j] = s DB[o_i + c][i r + j] (DB = dY^T [u_0 | u_1 | ..] over the
// group's contiguous output columns, [sum w][R]; only the diagonal blocks).
__global__ void lora_wg_extract_kernel(const float* __restrict__ DA, const float* __restrict__ DB, int d_in, int r,
                                       int R, float s, LoraWgGroup g) {
  griddep_wait();
  long long na = (long long)g.n * r * d_in, nb = 0;
  for (int a = 0; a < g.n; ++a) nb += (long long)g.s[a].width * r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < na + nb;
       i += (long long)gridDim.x * blockDim.x) {
    if (i < na) {
      const int a = (int)(i / ((long long)r * d_in));
      const long long t = i % ((long long)r * d_in);
      const int j = (int)(t / d_in), k = (int)(t % d_in);
      g.s[a].dA[t] = DA[(long long)k * R + a * r + j];
    } else {
      long long t = i - na;
      int a = 0, off = 0;
      while (t >= (long long)g.s[a].width * r) {
        t -= (long long)g.s[a].width * r;
        off += g.s[a].width;
        ++a;
      }
      const int c = (int)(t / r), j = (int)(t % r);
      g.s[a].dB[t] = s * DB[(long long)(off + c) * R + a * r + j];
    }
  }
}

// Adapter backward, row pass: one warp per token row (two rows in flight)
//   du[n][j] = s sum_c dY[n][c] bt[j][c]     (saved for the weight gradients)
//   dX(n, k) += sum_j du[n][j] A[j][k]        (epilogue addressing, as lora_up)
// bt = B^T [r][d_out] is staged in shared memory when it fits.
template <int RT, bool SMEM_B>
__global__ void __launch_bounds__(256) lora_bwd_rows_kernel(Planes dY, long long ldy, int d_out, int d_in,
                                                            const float* __restrict__ bt,
                                                            const float* __restrict__ A, int r, float s, int N,
                                                            float* __restrict__ du, Epilogue edx) {
  griddep_wait();
  extern __shared__ float4 bsm4[];
  const float* b = bt;
  if (SMEM_B) {
    float* bsm = reinterpret_cast<float*>(bsm4);
    for (int i = threadIdx.x * 4; i < r * d_out; i += 256 * 4)
      *reinterpret_cast<float4*>(bsm + i) = __ldg(reinterpret_cast<const float4*>(bt + i));
    __syncthreads();
    b = bsm;
  }
  const int lane = threadIdx.x % 32;
  const int warps = gridDim.x * 8;
  for (int n = (blockIdx.x * 8 + threadIdx.x / 32) * 2; n < N; n += warps * 2) {
    const bool two = n + 1 < N;
    float acc0[RT], acc1[RT];
#pragma unroll
    for (int j = 0; j < RT; ++j) acc0[j] = acc1[j] = 0.f;
    for (int c = lane * 4; c < d_out; c += 128) {
      const float4 y0 = load_planes4(dY, (long long)n * ldy + c);
      const float4 y1 = two ? load_planes4(dY, (long long)(n + 1) * ldy + c) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < RT; ++j) {
        if (j < r) {
          const float4 w = *reinterpret_cast<const float4*>(b + (long long)j * d_out + c);
          acc0[j] += y0.x * w.x + y0.y * w.y + y0.z * w.z + y0.w * w.w;
          acc1[j] += y1.x * w.x + y1.y * w.y + y1.z * w.z + y1.w * w.w;
        }
      }
    }
    // full sums in every lane (butterfly), scaled
#pragma unroll
    for (int j = 0; j < RT; ++j) {
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        acc0[j] += __shfl_xor_sync(0xffffffffu, acc0[j], o);
        acc1[j] += __shfl_xor_sync(0xffffffffu, acc1[j], o);
      }
      acc0[j] *= s;
      acc1[j] *= s;
      if (j < r && lane == (j & 31)) {
        du[(long long)n * r + j] = acc0[j];
        if (two) du[(long long)(n + 1) * r + j] = acc1[j];
      }
    }
    for (int k = lane * 4; k < d_in; k += 128) {
      float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
#pragma unroll
      for (int j = 0; j < RT; ++j) {
        if (j < r) {
          const float4 a4 = __ldg(reinterpret_cast<const float4*>(A + (long long)j * d_in + k));
          x0.x += acc0[j] * a4.x; x0.y += acc0[j] * a4.y; x0.z += acc0[j] * a4.z; x0.w += acc0[j] * a4.w;
          x1.x += acc1[j] * a4.x; x1.y += acc1[j] * a4.y; x1.z += acc1[j] * a4.z; x1.w += acc1[j] * a4.w;
        }
      }
      float4* y = reinterpret_cast<float4*>(edx.out + out_offset(edx, n, k));
      float4 v = *y;
      v.x += x0.x; v.y += x0.y; v.z += x0.z; v.w += x0.w;
      *y = v;
      if (two) {
        y = reinterpret_cast<float4*>(edx.out + out_offset(edx, n + 1, k));
        v = *y;
        v.x += x1.x; v.y += x1.y; v.z += x1.z; v.w += x1.w;
        *y = v;
      }
    }
  }
}

// Adapter backward, weight-gradient partials of both factors in one launch:
// blocks x < gy take 64 columns of dY with S = u (dB, scaled by s), the rest 64
// columns of X with S = du (dA); block y is a token chunk. Within a block the
// warps' sums are added in warp order: part[y][col][j], col over d_out then d_in.
template <int RT>
__global__ void __launch_bounds__(WgradCfg<RT>::kWarps * 32)
    lora_bwd_wgrad_kernel(Planes dY, long long ldy, int d_out, const float* __restrict__ U, Planes X, long long ldx,
                          int d_in, const float* __restrict__ du, int gy, int N, int r, float s, int chunk,
                          float* __restrict__ part) {
  griddep_wait();
  constexpr int WARPS = WgradCfg<RT>::kWarps;
  extern __shared__ float ss[];          // [chunk][r] S rows, then [WARPS][64][RT] warp sums
  float* red = ss + chunk * r;
  const bool on_y = (int)blockIdx.x < gy;
  const Planes big = on_y ? dY : X;
  const long long ldb = on_y ? ldy : ldx;
  const int C = on_y ? d_out : d_in;
  const float* S = on_y ? U : du;
  const float alpha = on_y ? s : 1.0f;
  const int cb = on_y ? (int)blockIdx.x * 64 : ((int)blockIdx.x - gy) * 64;
  const long long col0 = on_y ? 0 : d_out;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int c = cb + lane * 2;
  const int n0 = blockIdx.y * chunk;
  const int n1 = min(N, n0 + chunk);
  for (int i = threadIdx.x; i < (n1 - n0) * r; i += WARPS * 32) ss[i] = S[(long long)n0 * r + i];
  __syncthreads();
  float a0[RT], a1[RT];
#pragma unroll
  for (int j = 0; j < RT; ++j) a0[j] = a1[j] = 0.f;
  if (c < C) {
#pragma unroll 4
    for (int n = n0 + warp; n < n1; n += WARPS) {
      const float2 bv = load_planes2(big, (long long)n * ldb + c);
      const float* sr = ss + (n - n0) * r;
#pragma unroll
      for (int j = 0; j < RT; ++j) {
        if (j < r) {
          const float sv = sr[j];
          a0[j] += bv.x * sv;
          a1[j] += bv.y * sv;
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < RT; ++j) {
    red[(warp * 64 + lane * 2) * RT + j] = a0[j];
    red[(warp * 64 + lane * 2 + 1) * RT + j] = a1[j];
  }
  __syncthreads();
  const long long ct = (long long)d_out + d_in;
  for (int i = threadIdx.x; i < 64 * r; i += WARPS * 32) {
    const int cc = i / r, j = i % r;
    if (cb + cc >= C) continue;
    float sum = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < WARPS; ++w2) sum += red[(w2 * 64 + cc) * RT + j];
    part[((long long)blockIdx.y * ct + col0 + cb + cc) * r + j] = alpha * sum;
  }
}

// dB[c][j] = sum_chunk part[chunk][c][j] (c < d_out); dA[j][k] = sum_chunk part[chunk][d_out + k][j]
__global__ void lora_bwd_reduce_kernel(const float* __restrict__ part, int nch, int d_out, int d_in, int r,
                                       float* __restrict__ dB, float* __restrict__ dA) {
  griddep_wait();
  const long long total = ((long long)d_out + d_in) * r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int b = 0; b < nch; ++b) s += part[(long long)b * total + i];
    const int c = (int)(i / r), j = (int)(i % r);
    if (c < d_out) dB[(long long)c * r + j] = s;
    else dA[(long long)j * d_in + (c - d_out)] = s;
  }
}

template <int RT>
struct Bwd {
  static int run(Planes dY, long long ldy, int d_out, Planes X, long long ldx, int d_in, const float* U,
                 const float* bt, const float* A, int r, float s, int N, const Epilogue& e, float* du, float* part,
                 cudaStream_t st) {
    long long blocks = (N + 15) / 16;
    if (blocks > 148 * 2) blocks = 148 * 2;
    const size_t bbytes = (size_t)r * d_out * sizeof(float);
    int rc = bbytes <= 48 * 1024
                 ? launch_pdl(lora_bwd_rows_kernel<RT, true>, dim3((unsigned)blocks), dim3(256), bbytes, st, dY, ldy,
                              d_out, d_in, bt, A, r, s, N, du, e)
                 : launch_pdl(lora_bwd_rows_kernel<RT, false>, dim3((unsigned)blocks), dim3(256), 0, st, dY, ldy,
                              d_out, d_in, bt, A, r, s, N, du, e);
    if (rc) return rc;
    int nch, chunk;
    wgrad_chunks(N, r, nch, chunk);
    constexpr int WARPS = WgradCfg<RT>::kWarps;
    const size_t smem = ((size_t)chunk * r + (size_t)WARPS * 64 * RT) * sizeof(float);
    if (smem > 48 * 1024) return -1;
    const int gy = (d_out + 63) / 64, gx = (d_in + 63) / 64;
    return launch_pdl(lora_bwd_wgrad_kernel<RT>, dim3((unsigned)(gy + gx), (unsigned)nch), dim3(WARPS * 32), smem, st,
                      dY, ldy, d_out, U, X, ldx, d_in, (const float*)du, gy, N, r, s, chunk, part);
  }
};

// Group down pass: one warp per two token rows. Every adapter's w is staged
// in shared memory ([r][width] each, read as float4 along k: conflict-free).
// When all adapters read the same columns of X (the forward: one normalised
// input, several adapters) each X chunk is loaded once for all of them. Four
// 128-column chunks of both rows are loaded before they are used; the r sums
// of an adapter are reduced with warp_sum_multi. Also writes the B^T copies,
// and, for adapters with ext_col >= 0, the results as planes into X's columns
// ext_col + j.
template <int RT, int NS, bool SHARED>
__global__ void __launch_bounds__(256) lora_down_group_kernel(Planes X, long long ldx, int N, int r, LoraSegs g) {
  griddep_wait();
  extern __shared__ float4 wsm4[];
  float* wsm = reinterpret_cast<float*>(wsm4);
  int wofs[kLoraMaxSegs];
  {
    int o = 0;
#pragma unroll
    for (int a = 0; a < NS; ++a) {
      wofs[a] = o;
      o += r * g.s[a].width;
    }
  }
#pragma unroll
  for (int a = 0; a < NS; ++a) {
    const LoraSeg& sg = g.s[a];
    const int n4 = r * sg.width / 4, w4 = sg.width / 4, ld4 = (g.ldw ? g.ldw : sg.width) / 4;
    const float4* src = reinterpret_cast<const float4*>(sg.w);
    float4* dst = wsm4 + wofs[a] / 4;
    for (int i0 = threadIdx.x; i0 < n4; i0 += 4 * 256) {   // four loads in flight per thread
      float4 t[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * 256;
        if (i < n4) t[u] = __ldg(src + (long long)(i / w4) * ld4 + i % w4);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * 256 < n4) dst[i0 + u * 256] = t[u];
    }
    if (sg.bt) {
      for (long long i = blockIdx.x * 256LL + threadIdx.x; i < (long long)sg.b_rows * r;
           i += (long long)gridDim.x * 256) {
        const int c = (int)(i / r), j = (int)(i % r);
        sg.bt[(long long)j * sg.b_rows + c] = sg.b_src[i];
      }
    }
  }
  __syncthreads();
  const int lane = threadIdx.x % 32;
  const int warps = gridDim.x * 8;
  for (int n = (blockIdx.x * 8 + threadIdx.x / 32) * 2; n < N; n += warps * 2) {
    const bool two = n + 1 < N;
    float acc0[NS][RT], acc1[NS][RT];
#pragma unroll
    for (int a = 0; a < NS; ++a)
#pragma unroll
      for (int j = 0; j < RT; ++j) acc0[a][j] = acc1[a][j] = 0.f;
    auto dot = [&](int a, int k, const float4& x0, const float4& x1) {
      const int w = g.s[a].width;
#pragma unroll
      for (int j = 0; j < RT; ++j) {
        if (j < r) {
          const float4 wv = *reinterpret_cast<const float4*>(wsm + wofs[a] + j * w + k);
          acc0[a][j] += x0.x * wv.x + x0.y * wv.y + x0.z * wv.z + x0.w * wv.w;
          acc1[a][j] += x1.x * wv.x + x1.y * wv.y + x1.z * wv.z + x1.w * wv.w;
        }
      }
    };
    // columns [col_off, col_off + width) of rows n, n + 1, four chunks at a time
    auto pass = [&](int col_off, int width, auto&& use) {
      const long long r0 = (long long)n * ldx + col_off;
      for (int k0 = lane * 4; k0 < width; k0 += 4 * 128) {
        float4 x0[4], x1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int k = k0 + u * 128;
          x0[u] = k < width ? load_planes4(X, r0 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
          x1[u] = (k < width && two) ? load_planes4(X, r0 + ldx + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (k0 + u * 128 < width) use(k0 + u * 128, x0[u], x1[u]);
      }
    };
    if constexpr (SHARED) {
      pass(g.s[0].col_off, g.s[0].width, [&](int k, const float4& x0, const float4& x1) {
#pragma unroll
        for (int a = 0; a < NS; ++a) dot(a, k, x0, x1);
      });
    } else {
#pragma unroll
      for (int a = 0; a < NS; ++a)
        pass(g.s[a].col_off, g.s[a].width, [&](int k, const float4& x0, const float4& x1) { dot(a, k, x0, x1); });
    }
    const int j = warp_sum_multi_index<RT>(lane);
    const bool lead = warp_sum_multi_leader<RT>(lane) && j < r;
#pragma unroll
    for (int a = 0; a < NS; ++a) {
      const LoraSeg& sg = g.s[a];
      float v0 = sg.alpha * warp_sum_multi<RT>(acc0[a], lane);
      float v1 = sg.alpha * warp_sum_multi<RT>(acc1[a], lane);
      if (lead) {
        if (g.accumulate) {   // a later column chunk: add to the earlier chunks' sum
          v0 += sg.out[(long long)n * r + j];
          if (two) v1 += sg.out[(long long)(n + 1) * r + j];
        }
        sg.out[(long long)n * r + j] = v0;
        if (two) sg.out[(long long)(n + 1) * r + j] = v1;
        if (sg.ext_col >= 0 && g.write_ext) {
          const long long e0 = (long long)n * ldx + sg.ext_col + j;
          __nv_bfloat16 h, l;
          h = __float2bfloat16_rn(v0);
          l = __float2bfloat16_rn(v0 - __bfloat162float(h));
          X.hi[e0] = h;
          X.lo[e0] = l;
          if (two) {
            h = __float2bfloat16_rn(v1);
            l = __float2bfloat16_rn(v1 - __bfloat162float(h));
            X.hi[e0 + ldx] = h;
            X.lo[e0 + ldx] = l;
          }
        }
      }
    }
  }
}

// Bulk-staged group down pass: a block of 8 warps takes kDownRows consecutive
// rows. Warp 0 issues bulk copies of every adapter's w and of the columns each
// adapter reads from those rows (both planes) into shared memory, all
// completing on one mbarrier, so every block's loads are in flight at once;
// warp w then reduces rows w and w + 8 from shared memory. Shared memory:
// the barrier, w of each adapter ([r][width] f32), then per row and staged
// segment the hi and the lo columns. Results, B^T copies and extra-column
// planes as lora_down_group_kernel.
constexpr int kDownRows = 16;

template <int RT, int NS, bool SHARED>
__global__ void __launch_bounds__(256) lora_down_bulk_kernel(Planes X, long long ldx, int N, int r, LoraSegs g,
                                                            int* err) {
  extern __shared__ __align__(128) uint8_t dsm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(dsm);
  float* wsm = reinterpret_cast<float*>(dsm + 16);
  constexpr int NSEG = SHARED ? 1 : NS;   // column segments staged per row
  int wofs[NS], sofs[NSEG], wtot = 0, rowb = 0;
#pragma unroll
  for (int a = 0; a < NS; ++a) {
    wofs[a] = wtot;
    wtot += r * g.s[a].width;
  }
#pragma unroll
  for (int q = 0; q < NSEG; ++q) {
    sofs[q] = rowb;
    rowb += g.s[q].width;
  }
  bf16* rsm = reinterpret_cast<bf16*>(wsm + wtot);   // [kDownRows][2 rowb]
  const int n0 = blockIdx.x * kDownRows;
  const int rows = min(kDownRows, N - n0);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  griddep_wait();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(wtot * 4 + rows * rowb * 4));
    __syncwarp();
    const int ncopy = NS + rows * NSEG * 2;
    for (int c = lane; c < ncopy; c += 32) {
      if (c < NS) {
        bulk_load(wsm + wofs[c], g.s[c].w, (uint32_t)(r * g.s[c].width * 4), bar);
      } else {
        const int k = c - NS, t = k / (NSEG * 2), q = (k / 2) % NSEG, pl = k % 2;
        const int w = g.s[q].width;
        bf16* dst = rsm + (long long)t * 2 * rowb + 2 * sofs[q] + pl * w;
        const bf16* src = (pl ? X.lo : X.hi) + (long long)(n0 + t) * ldx + g.s[q].col_off;
        bulk_load(dst, src, (uint32_t)(w * 2), bar);
      }
    }
  }
#pragma unroll
  for (int a = 0; a < NS; ++a) {   // B^T copies for the splice, while the copies land
    const LoraSeg& sg = g.s[a];
    if (sg.bt) {
      for (long long i = blockIdx.x * 256LL + threadIdx.x; i < (long long)sg.b_rows * r;
           i += (long long)gridDim.x * 256) {
        const int c = (int)(i / r), j = (int)(i % r);
        sg.bt[(long long)j * sg.b_rows + c] = sg.b_src[i];
      }
    }
  }
  if (!mbar_wait(bar, 0, err, kErrWaitBulk)) return;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int t0 = warp, t1 = warp + 8;
  const bool two = t1 < rows;
  if (t0 >= rows) return;
  const int j = warp_sum_multi_index<RT>(lane);
  const bool lead = warp_sum_multi_leader<RT>(lane) && j < r;
#pragma unroll
  for (int a = 0; a < NS; ++a) {
    const LoraSeg& sg = g.s[a];
    const int q = SHARED ? 0 : a;
    const int w = sg.width;
    const bf16* h0 = rsm + (long long)t0 * 2 * rowb + 2 * sofs[q];
    const bf16* h1 = rsm + (long long)t1 * 2 * rowb + 2 * sofs[q];
    float acc0[RT], acc1[RT];
#pragma unroll
    for (int jj = 0; jj < RT; ++jj) acc0[jj] = acc1[jj] = 0.f;
    for (int k = lane * 4; k < w; k += 128) {
      const float4 x0 = load_planes4(Planes{const_cast<bf16*>(h0), const_cast<bf16*>(h0 + w)}, k);
      const float4 x1 = two ? load_planes4(Planes{const_cast<bf16*>(h1), const_cast<bf16*>(h1 + w)}, k)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int jj = 0; jj < RT; ++jj) {
        if (jj < r) {
          const float4 wv = *reinterpret_cast<const float4*>(wsm + wofs[a] + jj * w + k);
          acc0[jj] += x0.x * wv.x + x0.y * wv.y + x0.z * wv.z + x0.w * wv.w;
          acc1[jj] += x1.x * wv.x + x1.y * wv.y + x1.z * wv.z + x1.w * wv.w;
        }
      }
    }
    const float v0 = sg.alpha * warp_sum_multi<RT>(acc0, lane);
    const float v1 = sg.alpha * warp_sum_multi<RT>(acc1, lane);
    if (lead) {
      const long long n = n0 + t0;
      sg.out[n * r + j] = v0;
      if (two) sg.out[(n + 8) * r + j] = v1;
      if (sg.ext_col >= 0) {
        const long long e0 = n * ldx + sg.ext_col + j;
        bf16 h = __float2bfloat16_rn(v0);
        X.hi[e0] = h;
        X.lo[e0] = __float2bfloat16_rn(v0 - __bfloat162float(h));
        if (two) {
          h = __float2bfloat16_rn(v1);
          X.hi[e0 + 8 * ldx] = h;
          X.lo[e0 + 8 * ldx] = __float2bfloat16_rn(v1 - __bfloat162float(h));
        }
      }
    }
  }
}

template <int RT, int NS>
int down_bulk(Planes X, long long ldx, int N, int r, const LoraSegs& segs, bool shared, size_t smem, cudaStream_t st) {
  static DeviceOnce setup[2];
  auto* k0 = lora_down_bulk_kernel<RT, NS, false>;
  auto* k1 = lora_down_bulk_kernel<RT, NS, true>;
  if (setup[shared].ensure([&](int) {
        return cudaFuncSetAttribute(shared ? k1 : k0, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) ==
                       cudaSuccess
                   ? 0
                   : -3;
      }))
    return -3;
  int* err = device_error_word();
  const unsigned blocks = (unsigned)((N + kDownRows - 1) / kDownRows);
  return shared ? launch_pdl(k1, dim3(blocks), dim3(256), smem, st, X, ldx, N, r, segs, err)
                : launch_pdl(k0, dim3(blocks), dim3(256), smem, st, X, ldx, N, r, segs, err);
}

template <int RT>
int down_bulk_ns(Planes X, long long ldx, int N, int r, const LoraSegs& segs, bool shared, size_t smem,
                 cudaStream_t st) {
  if (segs.n == 1) return down_bulk<RT, 1>(X, ldx, N, r, segs, shared, smem, st);
  if (segs.n == 2) return down_bulk<RT, 2>(X, ldx, N, r, segs, shared, smem, st);
  return down_bulk<RT, 3>(X, ldx, N, r, segs, shared, smem, st);
}

template <int RT, int NS>
int down_group(Planes X, long long ldx, int N, int r, const LoraSegs& segs, bool shared, size_t smem,
               cudaStream_t st) {
  static DeviceOnce setup[2];
  auto* k0 = lora_down_group_kernel<RT, NS, false>;
  auto* k1 = lora_down_group_kernel<RT, NS, true>;
  if (setup[shared].ensure([&](int) {
        return cudaFuncSetAttribute(shared ? k1 : k0, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) ==
                       cudaSuccess
                   ? 0
                   : -3;
      }))
    return -3;
  // one row pair per warp: the pass is latency-bound, so every row's loads are
  // in flight at once (each block restages w, a few KB of L2 reads)
  const unsigned blocks = (unsigned)std::min<long long>(148 * 4, (N + 15) / 16);
  return shared ? launch_pdl(k1, dim3(blocks), dim3(256), smem, st, X, ldx, N, r, segs)
                : launch_pdl(k0, dim3(blocks), dim3(256), smem, st, X, ldx, N, r, segs);
}

template <int RT>
int down_group_ns(Planes X, long long ldx, int N, int r, const LoraSegs& segs, bool shared, size_t smem,
                  cudaStream_t st) {
  if (segs.n == 1) return down_group<RT, 1>(X, ldx, N, r, segs, shared, smem, st);
  if (segs.n == 2) return down_group<RT, 2>(X, ldx, N, r, segs, shared, smem, st);
  return down_group<RT, 3>(X, ldx, N, r, segs, shared, smem, st);
}

// Group weight gradients as factors: dB_i = s dY_i^T u_i (columns of dY,
// S = u_i) for each adapter, and dA = du^T X over X's columns with the S row
// [du_0 | du_1 | ..] of all adapters at once (or one dA factor per adapter
// when their ranks add up past kWgMaxS). A block takes 64 columns of one
// factor and one token chunk: lane l owns columns 2l, 2l + 1; warp w the
// tokens n0 + w + 8 k, loaded eight at a time; the S rows of the chunk are
// staged in shared memory. Warp sums are added in warp order, so
// partial[chunk][col][q] (q < the factor's S width) is a fixed-order sum.
constexpr int kWgChunks = 32;   // token chunks of a group's weight gradients
constexpr int kWgMaxS = 16;
constexpr int kWgMaxFactors = 2 * kLoraMaxSegs;

struct WgFactor {
  int big = 0;                 // 0: dY columns (dB), 1: X columns (dA)
  int col_off = 0, C = 0;      // columns [col_off, col_off + C) of the big matrix
  int n_src = 0;               // S = [src_0 | src_1 | ..], each [N][r]
  const float* src[kLoraMaxSegs] = {nullptr, nullptr, nullptr};
  float* dst[kLoraMaxSegs] = {nullptr, nullptr, nullptr};   // dB [C][r] or dA_a [r][C]
  float alpha = 1.f;
  int gbase = 0, cbase = 0;    // first 64-column group (blockIdx.x) / output column
};
struct WgPlan {
  WgFactor f[kWgMaxFactors];
  int nf = 0, groups = 0, ct = 0, r = 0;
};

template <int RS>
__global__ void __launch_bounds__(256) lora_wgrad2_kernel(Planes dY, long long ldy, Planes X, long long ldx, int N,
                                                         int chunk, WgPlan p, float* __restrict__ part) {
  griddep_wait();
  extern __shared__ float4 wss4[];
  float* ss = reinterpret_cast<float*>(wss4);   // [chunk][RS] S rows
  float* red = ss + chunk * RS;                 // [8 warps][RS][64] warp sums
  int fi = 0;
  while (fi + 1 < p.nf && (int)blockIdx.x >= p.f[fi + 1].gbase) ++fi;
  const WgFactor& F = p.f[fi];
  const int r = p.r, rs = F.n_src * r;
  const Planes big = F.big ? X : dY;
  const long long ldb = F.big ? ldx : ldy;
  const int cb = ((int)blockIdx.x - F.gbase) * 64;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int n0 = blockIdx.y * chunk;
  const int n1 = min(N, n0 + chunk);
  const int stot = (n1 - n0) * RS;
  for (int i0 = threadIdx.x; i0 < stot; i0 += 8 * 256) {   // eight loads in flight per thread
    float t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * 256, n = i / RS, q = i % RS;
      t[u] = (i < stot && q < rs) ? F.src[q / r][(long long)(n0 + n) * r + q % r] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + u * 256 < stot) ss[i0 + u * 256] = t[u];
  }
  __syncthreads();
  const int c = cb + lane * 2;
  float a0[RS], a1[RS];
#pragma unroll
  for (int q = 0; q < RS; ++q) a0[q] = a1[q] = 0.f;
  if (c < F.C) {
    const long long col = F.col_off + c;
    for (int nb = n0 + warp; nb < n1; nb += 64) {
      float2 bv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int n = nb + 8 * u;
        bv[u] = n < n1 ? load_planes2(big, (long long)n * ldb + col) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int n = nb + 8 * u;
        if (n < n1) {
          const float4* sr = reinterpret_cast<const float4*>(ss + (n - n0) * RS);
#pragma unroll
          for (int q4 = 0; q4 < RS / 4; ++q4) {
            const float4 sv = sr[q4];
            a0[4 * q4] += bv[u].x * sv.x; a1[4 * q4] += bv[u].y * sv.x;
            a0[4 * q4 + 1] += bv[u].x * sv.y; a1[4 * q4 + 1] += bv[u].y * sv.y;
            a0[4 * q4 + 2] += bv[u].x * sv.z; a1[4 * q4 + 2] += bv[u].y * sv.z;
            a0[4 * q4 + 3] += bv[u].x * sv.w; a1[4 * q4 + 3] += bv[u].y * sv.w;
          }
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < RS; ++q)
    *reinterpret_cast<float2*>(red + (warp * RS + q) * 64 + lane * 2) = make_float2(a0[q], a1[q]);
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * RS; i += 256) {
    const int cc = i % 64, q = i / 64;
    if (cb + cc >= F.C || q >= rs) continue;
    float sum = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < 8; ++w2) sum += red[(w2 * RS + q) * 64 + cc];
    part[((long long)blockIdx.y * p.ct + F.cbase + cb + cc) * RS + q] = F.alpha * sum;
  }
}

// Fixed-order sum of the chunk partials, scattered into dB / dA: four
// consecutive lanes share an output, lane k summing chunks k, k + 4, .. in
// order, and the four sums are added as (s0 + s1) + (s2 + s3).
template <int RS>
__global__ void lora_wgrad2_reduce_kernel(const float* __restrict__ part, int nch, WgPlan p) {
  griddep_wait();
  const long long total = (long long)p.ct * RS;
  const int sub = threadIdx.x & 3;
  const long long span = (total + 7) / 8 * 8;   // whole warps stay in the shuffles
  for (long long i0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) / 4; i0 < span;
       i0 += (long long)gridDim.x * blockDim.x / 4) {
    const long long i = i0 < total ? i0 : total - 1;
    float s = 0.f;
    int b = sub;
    for (; b + 12 < nch; b += 16) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = part[(long long)(b + 4 * u) * total + i];
#pragma unroll
      for (int u = 0; u < 4; ++u) s += v[u];
    }
    for (; b < nch; b += 4) s += part[(long long)b * total + i];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (sub || i0 >= total) continue;
    const int col = (int)(i / RS), q = (int)(i % RS);
    int fi = 0;
    while (fi + 1 < p.nf && col >= p.f[fi + 1].cbase) ++fi;
    const WgFactor& F = p.f[fi];
    const int r = p.r;
    if (q >= F.n_src * r) continue;
    const int cc = col - F.cbase;
    if (!F.big) F.dst[0][(long long)cc * r + q] = s;
    else F.dst[q / r][(long long)(q % r) * F.C + cc] = s;
  }
}

template <template <int> class F, typename... A>
int by_rank(int r, A... a) {
  if (r <= 8) return F<8>::run(a...);
  if (r <= 16) return F<16>::run(a...);
  if (r <= 32) return F<32>::run(a...);
  return F<64>::run(a...);
}

template <int RT>
struct Down {
  static int run(Planes X, long long ldx, int N, int K, const float* W, int r, float alpha, float* out,
                 const float* bsrc, int bc, float* bt, cudaStream_t st) {
    long long blocks = (N + 15) / 16;
    if (blocks > 148 * 2) blocks = 148 * 2;
    const size_t wbytes = (size_t)r * K * sizeof(float);
    if (wbytes <= 48 * 1024)
      return launch_pdl(lora_down_kernel<RT, true>, dim3((unsigned)blocks), dim3(256), wbytes, st, X, ldx, N, K, W, r,
                        alpha, out, bsrc, bc, bt);
    return launch_pdl(lora_down_kernel<RT, false>, dim3((unsigned)blocks), dim3(256), 0, st, X, ldx, N, K, W, r,
                      alpha, out, bsrc, bc, bt);
  }
};

template <int RT>
struct Up {
  static int run(const float* U, int N, int r, const float* W, int C, float alpha, Epilogue e, cudaStream_t st) {
    return launch_pdl(lora_up_kernel<RT>, dim3((unsigned)((C + 127) / 128), (unsigned)((N + 31) / 32)), dim3(256), 0,
                      st, U, N, r, W, C, alpha, e);
  }
};

template <int RT>
struct Wgrad {
  static int run(Planes Big, long long ldb, const float* S, int N, int C, int r, int nch, int chunk, float* partial,
                 cudaStream_t st) {
    constexpr int WARPS = WgradCfg<RT>::kWarps;
    const size_t smem = ((size_t)chunk * r + (size_t)WARPS * 64 * RT) * sizeof(float);
    if (smem > 48 * 1024) return -1;
    return launch_pdl(lora_wgrad_partial_kernel<RT>, dim3((unsigned)((C + 63) / 64), (unsigned)nch),
                      dim3(WARPS * 32), smem, st, Big, ldb, S, N, C, r, chunk, partial);
  }
};

bool rank_ok(int r) { return r >= 1 && r <= kLoraMaxRank; }

}  // namespace

int launch_lora_down(Planes X, long long ldx, int N, int K, const float* W, int r, float alpha, float* out,
                     cudaStream_t st, const float* b_src, int b_rows, float* bt_out) {
  if (!rank_ok(r) || N <= 0 || K <= 0 || K % 4 || ldx % 4 || (bt_out && (!b_src || b_rows <= 0))) return -1;
  return by_rank<Down>(r, X, ldx, N, K, W, r, alpha, out, b_src, b_rows, bt_out, st) ? -3 : 0;
}

int launch_lora_up(const float* U, int N, int r, const float* W, int C, float alpha, const Epilogue& e,
                   cudaStream_t st) {
  if (!rank_ok(r) || N <= 0 || C <= 0 || C % 4 || e.n_div % 4 || e.m_s0 % 4 || e.m_s1 % 4 || e.n_s1 % 4) return -1;
  return by_rank<Up>(r, U, N, r, W, C, alpha, e, st) ? -3 : 0;
}

long long lora_wgrad_partial_floats(int N, int C, int r) {
  if (!rank_ok(r) || N <= 0) return 0;
  int nch, chunk;
  wgrad_chunks(N, r, nch, chunk);
  return (long long)nch * C * r;
}

int launch_lora_wgrad(Planes Big, long long ldb, const float* S, int N, int C, int r, float alpha, float* out,
                      long long o_sc, long long o_sj, float* partial, cudaStream_t st) {
  if (!rank_ok(r) || N <= 0 || C <= 0 || C % 2 || ldb % 2) return -1;
  int nch, chunk;
  wgrad_chunks(N, r, nch, chunk);
  int rc = by_rank<Wgrad>(r, Big, ldb, S, N, C, r, nch, chunk, partial, st);
  if (rc) return rc < 0 ? rc : -3;
  const long long total = (long long)C * r;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_wgrad_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, st, partial, nch, C, r, alpha,
                    out, o_sc, o_sj)
             ? -3 : 0;
}

long long lora_bwd_partial_floats(int N, int d_out, int d_in, int r) {
  if (!rank_ok(r) || N <= 0) return 0;
  int nch, chunk;
  wgrad_chunks(N, r, nch, chunk);
  return (long long)nch * ((long long)d_out + d_in) * r;
}

int launch_lora_backward(Planes dY, long long ldy, int d_out, Planes X, long long ldx, int d_in, const float* U,
                         const float* bt, const float* A, int r, float s, int N, const Epilogue& edx, float* du,
                         float* part, float* dB, float* dA, cudaStream_t st) {
  if (r < 1 || r > kLoraBwdMaxRank || N <= 0 || d_out % 4 || d_in % 4 || ldy % 4 || ldx % 4 || edx.n_div % 4 ||
      edx.m_s0 % 4 || edx.m_s1 % 4 || edx.n_s1 % 4)
    return -1;
  const int rc = r <= 8 ? Bwd<8>::run(dY, ldy, d_out, X, ldx, d_in, U, bt, A, r, s, N, edx, du, part, st)
                        : Bwd<16>::run(dY, ldy, d_out, X, ldx, d_in, U, bt, A, r, s, N, edx, du, part, st);
  if (rc) return rc < 0 ? rc : -3;
  int nch, chunk;
  wgrad_chunks(N, r, nch, chunk);
  const long long total = ((long long)d_out + d_in) * r;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_bwd_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, st, (const float*)part, nch, d_out,
                    d_in, r, dB, dA)
             ? -3 : 0;
}

int launch_lora_down_group(Planes X, long long ldx, int N, int r, const LoraSegs& segs, cudaStream_t st) {
  if (r < 1 || r > 16 || N <= 0 || segs.n < 1 || segs.n > kLoraMaxSegs || ldx % 4) return -1;
  size_t wfloats = 0;
  bool shared = true;
  for (int a = 0; a < segs.n; ++a) {
    const LoraSeg& sg = segs.s[a];
    if (!sg.w || !sg.out || sg.width <= 0 || sg.width % 4 || sg.col_off % 4 || (sg.bt && (!sg.b_src || sg.b_rows <= 0)))
      return -1;
    if (sg.ext_col >= 0 && sg.ext_col + r > ldx) return -1;
    wfloats += (size_t)r * sg.width;
    shared = shared && sg.col_off == segs.s[0].col_off && sg.width == segs.s[0].width;
  }
  const size_t smem = wfloats * sizeof(float);
  // w of more than 100 KB (the wide layers of 1B+ models): column chunks of
  // at most 48 KB of w, so that four blocks share an SM and hide the row
  // loads' latency
  constexpr size_t kChunkSmem = 48 * 1024;
  if (smem > 100 * 1024) {
    // w of the whole set in column chunks of one width (a multiple of 4), each
    // staged in shared memory, added in chunk order into out
    int w_all = segs.s[0].width;
    bool same = true;
    for (int a = 1; a < segs.n; ++a) same = same && segs.s[a].width == w_all;
    if (!same) {   // adapters of different widths: one set each
      for (int a = 0; a < segs.n; ++a) {
        LoraSegs one;
        one.s[0] = segs.s[a];
        one.n = 1;
        if (const int rc = launch_lora_down_group(X, ldx, N, r, one, st)) return rc;
      }
      return 0;
    }
    const size_t per_col = (size_t)r * segs.n * sizeof(float);
    int wc = (int)(kChunkSmem / per_col) / 4 * 4;
    if (wc < 4) return -1;
    for (int c0 = 0; c0 < w_all; c0 += wc) {
      LoraSegs part = segs;
      part.ldw = w_all;
      part.accumulate = c0 > 0;
      part.write_ext = c0 + wc >= w_all;
      const int width = std::min(wc, w_all - c0);
      for (int a = 0; a < segs.n; ++a) {
        part.s[a].col_off = segs.s[a].col_off + c0;
        part.s[a].width = width;
        part.s[a].w = segs.s[a].w + c0;
        if (c0 > 0) part.s[a].bt = nullptr;   // the B^T copy once
      }
      const size_t psmem = (size_t)r * segs.n * width * sizeof(float);
      const int rc = r <= 8 ? down_group_ns<8>(X, ldx, N, r, part, shared, psmem, st)
                            : down_group_ns<16>(X, ldx, N, r, part, shared, psmem, st);
      if (rc) return -3;
    }
    return 0;
  }
  // bulk-staged variant: 16-byte aligned rows, segments and w; its shared
  // memory holds w plus kDownRows rows of the staged segments
  bool bulk = ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(X.hi) & 15) == 0 &&
              (reinterpret_cast<uintptr_t>(X.lo) & 15) == 0;
  size_t seg_elems = 0;
  for (int a = 0; a < segs.n; ++a) {
    const LoraSeg& sg = segs.s[a];
    bulk = bulk && sg.col_off % 8 == 0 && sg.width % 8 == 0 && (reinterpret_cast<uintptr_t>(sg.w) & 15) == 0;
    if (a == 0 || !shared) seg_elems += sg.width;
  }
  const size_t bsmem = 16 + smem + (size_t)kDownRows * seg_elems * 4;
  int rc;
  if (bulk && bsmem <= 200 * 1024)
    rc = r <= 8 ? down_bulk_ns<8>(X, ldx, N, r, segs, shared, bsmem, st)
                : down_bulk_ns<16>(X, ldx, N, r, segs, shared, bsmem, st);
  else
    rc = r <= 8 ? down_group_ns<8>(X, ldx, N, r, segs, shared, smem, st)
                : down_group_ns<16>(X, ldx, N, r, segs, shared, smem, st);
  return rc ? -3 : 0;
}

namespace {
// Token chunks of the group weight gradients: kWgChunks of them, each small
// enough for its S rows (kWgMaxS wide) to stay within 64 KB.
void wg_chunks(int N, int& nch, int& chunk) {
  chunk = (N + kWgChunks - 1) / kWgChunks;
  chunk = std::min(chunk, 64 * 1024 / (4 * kWgMaxS));
  chunk = std::max(chunk, 1);
  nch = (N + chunk - 1) / chunk;
}

WgPlan wg_plan(const LoraWgGroup& g, int d_in, int r, float s) {
  WgPlan p;
  p.r = r;
  auto add = [&](const WgFactor& f0) {
    WgFactor f = f0;
    f.gbase = p.groups;
    f.cbase = p.ct;
    p.groups += (f.C + 63) / 64;
    p.ct += f.C;
    p.f[p.nf++] = f;
  };
  for (int a = 0; a < g.n; ++a) {
    WgFactor f;
    f.big = 0; f.col_off = g.s[a].col_off; f.C = g.s[a].width;
    f.n_src = 1; f.src[0] = g.s[a].u; f.dst[0] = g.s[a].dB; f.alpha = s;
    add(f);
  }
  if (g.n * r <= kWgMaxS) {   // one pass over X for every adapter's dA
    WgFactor f;
    f.big = 1; f.col_off = 0; f.C = d_in; f.n_src = g.n; f.alpha = 1.f;
    for (int a = 0; a < g.n; ++a) {
      f.src[a] = g.s[a].du;
      f.dst[a] = g.s[a].dA;
    }
    add(f);
  } else {
    for (int a = 0; a < g.n; ++a) {
      WgFactor f;
      f.big = 1; f.col_off = 0; f.C = d_in; f.n_src = 1; f.alpha = 1.f;
      f.src[0] = g.s[a].du; f.dst[0] = g.s[a].dA;
      add(f);
    }
  }
  return p;
}

template <int RS>
int wgrad2(Planes dY, long long ldy, Planes X, long long ldx, int N, const WgPlan& p, float* part, cudaStream_t st) {
  int nch, chunk;
  wg_chunks(N, nch, chunk);
  auto* kern = lora_wgrad2_kernel<RS>;
  const size_t smem = ((size_t)chunk * RS + (size_t)8 * RS * 64) * sizeof(float);
  static DeviceOnce setup;
  if (setup.ensure([&](int) {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024) == cudaSuccess
                   ? 0
                   : -3;
      }))
    return -3;
  if (launch_pdl(kern, dim3((unsigned)p.groups, (unsigned)nch), dim3(256), smem, st, dY, ldy, X, ldx, N, chunk, p,
                 part))
    return -3;
  const long long total = (long long)p.ct * RS;
  long long blocks = (4 * ((total + 7) / 8 * 8) + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_wgrad2_reduce_kernel<RS>, dim3((unsigned)blocks), dim3(256), 0, st, (const float*)part, nch, p)
             ? -3 : 0;
}
}  // namespace

long long lora_group_partial_floats(int N, int r, int d_in, int total_width, int n_adapters) {
  if (r < 1 || r > 16 || N <= 0) return 0;
  int nch, chunk;
  wg_chunks(N, nch, chunk);
  const long long dcols = (long long)n_adapters * r <= kWgMaxS ? d_in : (long long)n_adapters * d_in;
  return (long long)nch * ((long long)total_width + dcols) * kWgMaxS;
}

int launch_lora_wgrad_group(Planes dY, long long ldy, Planes X, long long ldx, int d_in, int N, int r, float s,
                            const LoraWgGroup& g, float* part, cudaStream_t st) {
  if (r < 1 || r > 16 || N <= 0 || g.n < 1 || g.n > kLoraMaxSegs || d_in % 2 || ldy % 2 || ldx % 2) return -1;
  for (int a = 0; a < g.n; ++a) {
    const LoraWgSeg& sg = g.s[a];
    if (!sg.u || !sg.du || !sg.dB || !sg.dA || sg.width <= 0 || sg.width % 2 || sg.col_off % 2) return -1;
  }
  const WgPlan p = wg_plan(g, d_in, r, s);
  int rs_max = r;
  for (int f = 0; f < p.nf; ++f) rs_max = std::max(rs_max, p.f[f].n_src * r);
  return rs_max <= 8 ? wgrad2<8>(dY, ldy, X, ldx, N, p, part, st) : wgrad2<16>(dY, ldy, X, ldx, N, p, part, st);
}

int launch_lora_pack_planes(const LoraPackSrc& src, int N, int r, int R, Planes out, cudaStream_t st) {
  if (src.n < 1 || src.n > kLoraMaxSegs || r < 1 || R % 2 || src.n * r > R || N <= 0 || !out.hi || !out.lo) return -1;
  for (int a = 0; a < src.n; ++a)
    if (!src.p[a]) return -1;
  long long blocks = ((long long)N * (R / 2) + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_pack_planes_kernel, dim3((unsigned)blocks), dim3(256), 0, st, src, N, r, R, out) ? -3 : 0;
}

int launch_lora_pack_w(const LoraPackW& src, int R, int K, Planes out, cudaStream_t st) {
  if (src.n < 1 || src.n > kLoraMaxSegs || src.r < 1 || src.n * src.r > R || K <= 0 || K % 2 || !out.hi || !out.lo)
    return -1;
  for (int a = 0; a < src.n; ++a)
    if (!src.p[a] || src.w[a] <= 0 || src.koff[a] < 0 || src.koff[a] + src.w[a] > K) return -1;
  long long blocks = ((long long)R * (K / 2) + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_pack_w_kernel, dim3((unsigned)blocks), dim3(256), 0, st, src, R, K, out) ? -3 : 0;
}

int launch_lora_scatter_u(const float* D, int N, int R, const LoraScatterU& dst, cudaStream_t st) {
  if (!D || N <= 0 || dst.n < 1 || dst.n > kLoraMaxSegs || dst.r < 1 || dst.n * dst.r > R) return -1;
  for (int a = 0; a < dst.n; ++a)
    if (!dst.out[a] || (dst.ext_col[a] >= 0 && (!dst.X.hi || !dst.X.lo || dst.ext_col[a] + dst.r > dst.ldx))) return -1;
  long long blocks = ((long long)N * dst.n * dst.r + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_scatter_u_kernel, dim3((unsigned)blocks), dim3(256), 0, st, D, N, R, dst) ? -3 : 0;
}

int launch_lora_wg_extract(const float* DA, const float* DB, int d_in, int r, int R, float s, const LoraWgGroup& g,
                           cudaStream_t st) {
  if (!DA || !DB || g.n < 1 || g.n > kLoraMaxSegs || g.n * r > R || d_in <= 0) return -1;
  long long total = (long long)g.n * r * d_in;
  for (int a = 0; a < g.n; ++a) {
    if (!g.s[a].dA || !g.s[a].dB || g.s[a].width <= 0) return -1;
    total += (long long)g.s[a].width * r;
  }
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_wg_extract_kernel, dim3((unsigned)blocks), dim3(256), 0, st, DA, DB, d_in, r, R, s, g) ? -3
                                                                                                                 : 0;
}

int launch_lora_transpose(const float* W, int C, int r, float* Wt, cudaStream_t st) {
  if (!rank_ok(r) || C <= 0) return -1;
  long long blocks = ((long long)C * r + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_transpose_kernel, dim3((unsigned)blocks), dim3(256), 0, st, W, C, r, Wt) ? -3 : 0;
}

}  // namespace tb2
