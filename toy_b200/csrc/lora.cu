// Low-rank adapter kernels (see lora.cuh). Every reduction runs in a fixed
// order, so results do not depend on scheduling.
#include "lora.cuh"

#include <algorithm>

#include "pdl.cuh"
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
    const int n4 = r * sg.width / 4;
    const float4* src = reinterpret_cast<const float4*>(sg.w);
    float4* dst = wsm4 + wofs[a] / 4;
    for (int i0 = threadIdx.x; i0 < n4; i0 += 4 * 256) {   // four loads in flight per thread
      float4 t[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * 256 < n4) t[u] = __ldg(src + i0 + u * 256);
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
      const float v0 = sg.alpha * warp_sum_multi<RT>(acc0[a], lane);
      const float v1 = sg.alpha * warp_sum_multi<RT>(acc1[a], lane);
      if (lead) {
        sg.out[(long long)n * r + j] = v0;
        if (two) sg.out[(long long)(n + 1) * r + j] = v1;
        if (sg.ext_col >= 0) {
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

template <int RT, int NS>
int down_group(Planes X, long long ldx, int N, int r, const LoraSegs& segs, bool shared, size_t smem,
               cudaStream_t st) {
  static bool attr[2] = {false, false};
  auto* k0 = lora_down_group_kernel<RT, NS, false>;
  auto* k1 = lora_down_group_kernel<RT, NS, true>;
  if (!attr[shared]) {
    if (cudaFuncSetAttribute(shared ? k1 : k0, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
        cudaSuccess)
      return -3;
    attr[shared] = true;
  }
  const unsigned blocks = (unsigned)std::min<long long>(148, (N + 15) / 16);
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

// Group weight-gradient partials. Factor f = 2 i (dB of adapter i: dY columns
// col_off_i .., S = u_i, scaled by s) or 2 i + 1 (dA: X columns, S = du_i);
// blockIdx.x walks the 64-column groups of all factors (gbase[f] = first
// group of factor f), blockIdx.y the token chunks. Partials are [chunk][col][r]
// over the concatenated columns (cbase[f] = first column of factor f).
struct WgLayout {
  int nf;
  int gbase[2 * kLoraMaxSegs + 1];
  int cbase[2 * kLoraMaxSegs + 1];
};

template <int RT>
__global__ void __launch_bounds__(WgradCfg<RT>::kWarps * 32)
    lora_wgrad_group_kernel(Planes dY, long long ldy, Planes X, long long ldx, int d_in, int N, int r, float s,
                            int chunk, LoraWgGroup g, WgLayout lay, float* __restrict__ part) {
  griddep_wait();
  constexpr int WARPS = WgradCfg<RT>::kWarps;
  extern __shared__ float ss[];   // [chunk][r] S rows, then [WARPS][64][RT] warp sums
  float* red = ss + chunk * r;
  int f = 0;
  while (f + 1 < lay.nf && (int)blockIdx.x >= lay.gbase[f + 1]) ++f;
  const LoraWgSeg& sg = g.s[f / 2];
  const bool dB = (f & 1) == 0;
  const Planes big = dB ? dY : X;
  const long long ldb = dB ? ldy : ldx;
  const int off = dB ? sg.col_off : 0;
  const int C = dB ? sg.width : d_in;
  const float* S = dB ? sg.u : sg.du;
  const float alpha = dB ? s : 1.0f;
  const int cb = ((int)blockIdx.x - lay.gbase[f]) * 64;
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
      const float2 bv = load_planes2(big, (long long)n * ldb + off + c);
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
  const long long ct = lay.cbase[lay.nf];
  for (int i = threadIdx.x; i < 64 * r; i += WARPS * 32) {
    const int cc = i / r, j = i % r;
    if (cb + cc >= C) continue;
    float sum = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < WARPS; ++w2) sum += red[(w2 * 64 + cc) * RT + j];
    part[((long long)blockIdx.y * ct + lay.cbase[f] + cb + cc) * r + j] = alpha * sum;
  }
}

__global__ void lora_group_reduce_kernel(const float* __restrict__ part, int nch, int r, int d_in, LoraWgGroup g,
                                         WgLayout lay) {
  griddep_wait();
  const long long ct = lay.cbase[lay.nf];
  const long long total = ct * r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int b = 0; b < nch; ++b) s += part[(long long)b * total + i];
    const int col = (int)(i / r), j = (int)(i % r);
    int f = 0;
    while (f + 1 < lay.nf && col >= lay.cbase[f + 1]) ++f;
    const LoraWgSeg& sg = g.s[f / 2];
    const int c = col - lay.cbase[f];
    if ((f & 1) == 0) sg.dB[(long long)c * r + j] = s;
    else sg.dA[(long long)j * d_in + c] = s;
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
  if (smem > 200 * 1024) return -1;
  const int rc = r <= 8 ? down_group_ns<8>(X, ldx, N, r, segs, shared, smem, st)
                        : down_group_ns<16>(X, ldx, N, r, segs, shared, smem, st);
  return rc ? -3 : 0;
}

namespace {
WgLayout wg_layout(const LoraWgGroup& g, int d_in) {
  WgLayout l;
  l.nf = 2 * g.n;
  l.gbase[0] = l.cbase[0] = 0;
  for (int f = 0; f < l.nf; ++f) {
    const int C = (f & 1) ? d_in : g.s[f / 2].width;
    l.gbase[f + 1] = l.gbase[f] + (C + 63) / 64;
    l.cbase[f + 1] = l.cbase[f] + C;
  }
  return l;
}
}  // namespace

long long lora_group_partial_floats(int N, int r, int d_in, int total_width, int n_adapters) {
  if (r < 1 || r > 16 || N <= 0) return 0;
  int nch, chunk;
  wgrad_chunks(N, r, nch, chunk);
  return (long long)nch * ((long long)total_width + (long long)n_adapters * d_in) * r;
}

int launch_lora_wgrad_group(Planes dY, long long ldy, Planes X, long long ldx, int d_in, int N, int r, float s,
                            const LoraWgGroup& g, float* part, cudaStream_t st) {
  if (r < 1 || r > 16 || N <= 0 || g.n < 1 || g.n > kLoraMaxSegs || d_in % 2 || ldy % 2 || ldx % 2) return -1;
  for (int a = 0; a < g.n; ++a) {
    const LoraWgSeg& sg = g.s[a];
    if (!sg.u || !sg.du || !sg.dB || !sg.dA || sg.width <= 0 || sg.width % 2 || sg.col_off % 2) return -1;
  }
  const WgLayout lay = wg_layout(g, d_in);
  int nch, chunk;
  wgrad_chunks(N, r, nch, chunk);
  int rc;
  if (r <= 8) {
    const size_t smem = ((size_t)chunk * r + (size_t)WgradCfg<8>::kWarps * 64 * 8) * sizeof(float);
    rc = launch_pdl(lora_wgrad_group_kernel<8>, dim3((unsigned)lay.gbase[lay.nf], (unsigned)nch),
                    dim3(WgradCfg<8>::kWarps * 32), smem, st, dY, ldy, X, ldx, d_in, N, r, s, chunk, g, lay, part);
  } else {
    const size_t smem = ((size_t)chunk * r + (size_t)WgradCfg<16>::kWarps * 64 * 16) * sizeof(float);
    rc = launch_pdl(lora_wgrad_group_kernel<16>, dim3((unsigned)lay.gbase[lay.nf], (unsigned)nch),
                    dim3(WgradCfg<16>::kWarps * 32), smem, st, dY, ldy, X, ldx, d_in, N, r, s, chunk, g, lay, part);
  }
  if (rc) return -3;
  const long long total = (long long)lay.cbase[lay.nf] * r;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_group_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, st, (const float*)part, nch, r, d_in,
                    g, lay)
             ? -3 : 0;
}

int launch_lora_transpose(const float* W, int C, int r, float* Wt, cudaStream_t st) {
  if (!rank_ok(r) || C <= 0) return -1;
  long long blocks = ((long long)C * r + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(lora_transpose_kernel, dim3((unsigned)blocks), dim3(256), 0, st, W, C, r, Wt) ? -3 : 0;
}

}  // namespace tb2
