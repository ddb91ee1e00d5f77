// The tnn_* primitive op surface: a lazily built tensor graph with ggml shape
// semantics (ne[0] fastest), executed on the device, with reverse-mode
// autograd emitting the backward node types ggml's autograd emits for the
// training graph (OUT_PROD, RMS_NORM_BACK, ROPE_BACK, SOFT_MAX_BACK,
// SILU_BACK, CROSS_ENTROPY_LOSS_BACK, GET_ROWS_BACK) and in-place
// OPT_STEP_ADAMW nodes.
//
// Session flow (tinynn/tinynn_ggml.h): create inputs and op nodes; either
// tnn_realize(result) + tnn_compute (inference), or tnn_set_param / tnn_set_loss,
// tnn_build_forward_only(loss), tnn_build_backward, tnn_tensor_grad,
// tnn_opt_step_adamw + tnn_extend_backward_graph, tnn_realize_backward, then per
// step tnn_graph_reset(_grads_only), uploads, tnn_compute_backward, downloads.
//
// Matrix products run on the split-bf16 tcgen05 GEMM (gemm.cuh); F32 operands
// are split into planes per launch, Q8_0 weights are dequantised inside the
// GEMM. Every other op is an f32 CUDA-core kernel. Buffers are allocated per
// node at realize time (no reuse): this surface trades memory for simplicity;
// the fused step program (engine.cu) is the fast path for the recipes.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <unordered_set>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"
#include "pdl.cuh"
#include "prims.cuh"
#include "runtime.cuh"

namespace tb2 {

Session::~Session() {
  if (device >= 0) cudaSetDevice(device);
  kv_free(this);   // the decode engine reads the step engine's weights: it goes first
  dp_free(this);
  for (auto& t : tensors) {
    if (t->data && !t->view_of) cudaFree(t->data);
    if (t->q8v && !t->view_of) cudaFree(t->q8v);
    if (t->q8s && !t->view_of) cudaFree(t->q8s);
    if (t->planes) cudaFree(t->planes);
    if (t->outpad) cudaFree(t->outpad);
  }
  if (pstream) cudaStreamDestroy(pstream);
}

const char* prim_op_name(int op) {
  static const char* names[kOpCount] = {
      "NONE", "ADD", "SUB", "MUL", "SCALE", "SILU", "SILU_BACK", "SWIGLU", "MUL_MAT", "OUT_PROD", "MUL_MAT_AT",
      "RMS_NORM", "RMS_NORM_BACK", "ROPE", "ROPE_BACK", "SOFT_MAX", "SOFT_MAX_BACK", "DIAG_MASK_INF",
      "DIAG_MASK_ZERO", "TRANSPOSE", "CONT", "RESHAPE", "VIEW", "CONCAT", "SLICE", "GET_ROWS", "GET_ROWS_BACK",
      "CROSS_ENTROPY_LOSS", "CROSS_ENTROPY_LOSS_BACK", "SUM", "SUM_ROWS", "REPEAT", "REPEAT_BACK", "OPT_STEP_ADAMW",
      "ACC_VIEW", "CPY", "OPT_STEP_SGD"};
  return op >= 0 && op < kOpCount ? names[op] : "?";
}

namespace {

constexpr int kSMs = 148;

int grid_for(long long work, int threads) {
  long long b = (work + threads - 1) / threads;
  if (b > kSMs * 16) b = kSMs * 16;
  return (int)(b < 1 ? 1 : b);
}

struct Sh {
  int n0, n1, n2, n3;
};

Sh shape(const Tensor* t) { return Sh{t->ne[0], t->ne[1], t->ne[2], t->ne[3]}; }

// ------------------------------------------------------------------ kernels
#define GRID_LOOP(i, n) for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (n); i += (long long)gridDim.x * blockDim.x)

// o = a (op) b with b broadcast over any dimension where it has extent 1 /
// a divisor of a's (ggml_can_repeat)
__global__ void k_binary(int op, const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o,
                         Sh sa, Sh sb, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    long long t = i;
    const int i0 = (int)(t % sa.n0); t /= sa.n0;
    const int i1 = (int)(t % sa.n1); t /= sa.n1;
    const int i2 = (int)(t % sa.n2);
    const int i3 = (int)(t / sa.n2);
    const long long bi =
        (((long long)(i3 % sb.n3) * sb.n2 + i2 % sb.n2) * sb.n1 + i1 % sb.n1) * sb.n0 + i0 % sb.n0;
    const float x = a[i], y = b[bi];
    o[i] = op == 0 ? x + y : (op == 1 ? x - y : x * y);
  }
}

// out (shape so) = sum of g (shape sg, each extent a multiple of so's) over the
// repeats, in a fixed order
__global__ void k_repeat_back(const float* __restrict__ g, float* __restrict__ out, Sh sg, Sh so, long long n) {
  griddep_wait();
  const int r0 = sg.n0 / so.n0, r1 = sg.n1 / so.n1, r2 = sg.n2 / so.n2, r3 = sg.n3 / so.n3;
  GRID_LOOP(j, n) {
    long long t = j;
    const int j0 = (int)(t % so.n0); t /= so.n0;
    const int j1 = (int)(t % so.n1); t /= so.n1;
    const int j2 = (int)(t % so.n2);
    const int j3 = (int)(t / so.n2);
    float s = 0.f;
    for (int k3 = 0; k3 < r3; ++k3)
      for (int k2 = 0; k2 < r2; ++k2)
        for (int k1 = 0; k1 < r1; ++k1)
          for (int k0 = 0; k0 < r0; ++k0) {
            const long long gi = (((long long)(j3 + k3 * so.n3) * sg.n2 + (j2 + k2 * so.n2)) * sg.n1 +
                                  (j1 + k1 * so.n1)) * sg.n0 + (j0 + k0 * so.n0);
            s += g[gi];
          }
    out[j] = s;
  }
}

// out = broadcast of a (shape sa) to shape so
__global__ void k_repeat(const float* __restrict__ a, float* __restrict__ out, Sh sa, Sh so, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    long long t = i;
    const int i0 = (int)(t % so.n0); t /= so.n0;
    const int i1 = (int)(t % so.n1); t /= so.n1;
    const int i2 = (int)(t % so.n2);
    const int i3 = (int)(t / so.n2);
    out[i] = a[(((long long)(i3 % sa.n3) * sa.n2 + i2 % sa.n2) * sa.n1 + i1 % sa.n1) * sa.n0 + i0 % sa.n0];
  }
}

// 0 scale, 1 silu, 2 silu_back (a = x, b = dy), 3 swiglu (a = gate, b = up)
__global__ void k_unary(int op, const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o,
                        float s, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    const float x = a[i];
    float y;
    if (op == 0) {
      y = x * s;
    } else if (op == 1) {
      y = x / (1.0f + expf(-x));
    } else if (op == 2) {
      const float sg = 1.0f / (1.0f + expf(-x));
      y = b[i] * (sg * (1.0f + x * (1.0f - sg)));
    } else {
      y = x / (1.0f + expf(-x)) * b[i];
    }
    o[i] = y;
  }
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

// ggml rms_norm over each row of ne0
__global__ void k_rms_norm(const float* __restrict__ x, float* __restrict__ y, long long rows, int n, float eps) {
  griddep_wait();
  const int lane = threadIdx.x % 32, warps = blockDim.x / 32;
  for (long long r = blockIdx.x * (long long)warps + threadIdx.x / 32; r < rows; r += (long long)gridDim.x * warps) {
    const float* xr = x + r * n;
    float ss = 0.f;
    for (int i = lane; i < n; i += 32) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    const float sc = 1.0f / sqrtf(ss / n + eps);
    for (int i = lane; i < n; i += 32) y[r * n + i] = xr[i] * sc;
  }
}

// ggml rms_norm_back: dx = (dz - x * sum(x dz) / (sum x^2 + n eps)) * rrms
__global__ void k_rms_norm_back(const float* __restrict__ x, const float* __restrict__ dz, float* __restrict__ dx,
                                long long rows, int n, float eps) {
  griddep_wait();
  const int lane = threadIdx.x % 32, warps = blockDim.x / 32;
  for (long long r = blockIdx.x * (long long)warps + threadIdx.x / 32; r < rows; r += (long long)gridDim.x * warps) {
    const float* xr = x + r * n;
    const float* gr = dz + r * n;
    float ss = 0.f, sxg = 0.f;
    for (int i = lane; i < n; i += 32) {
      ss += xr[i] * xr[i];
      sxg += xr[i] * gr[i];
    }
    ss = warp_sum(ss);
    sxg = warp_sum(sxg);
    const float rr = 1.0f / sqrtf(ss / n + eps);
    const float k = sxg / (ss + n * eps);
    for (int i = lane; i < n; i += 32) dx[r * n + i] = (gr[i] - xr[i] * k) * rr;
  }
}

// per-row softmax of scale * a + mask (mask row = row % mask_rows); max_bias 0
__global__ void k_softmax(const float* __restrict__ a, const float* __restrict__ mask, float* __restrict__ y,
                          long long rows, int n, float scale, long long mask_rows) {
  griddep_wait();
  const int lane = threadIdx.x % 32, warps = blockDim.x / 32;
  for (long long r = blockIdx.x * (long long)warps + threadIdx.x / 32; r < rows; r += (long long)gridDim.x * warps) {
    const float* ar = a + r * n;
    const float* mr = mask ? mask + (r % mask_rows) * n : nullptr;
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, ar[i] * scale + (mr ? mr[i] : 0.f));
    m = warp_max(m);
    float s = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float v = ar[i] * scale + (mr ? mr[i] : 0.f);
      s += v == -INFINITY ? 0.f : expf(v - m);
    }
    s = warp_sum(s);
    const float inv = s > 0.f ? 1.0f / s : 0.f;
    for (int i = lane; i < n; i += 32) {
      const float v = ar[i] * scale + (mr ? mr[i] : 0.f);
      y[r * n + i] = v == -INFINITY ? 0.f : expf(v - m) * inv;
    }
  }
}

// ggml soft_max_ext_back: dx = scale * y * (dy - sum(y dy))
__global__ void k_softmax_back(const float* __restrict__ y, const float* __restrict__ dy, float* __restrict__ dx,
                               long long rows, int n, float scale) {
  griddep_wait();
  const int lane = threadIdx.x % 32, warps = blockDim.x / 32;
  for (long long r = blockIdx.x * (long long)warps + threadIdx.x / 32; r < rows; r += (long long)gridDim.x * warps) {
    float d = 0.f;
    for (int i = lane; i < n; i += 32) d += y[r * n + i] * dy[r * n + i];
    d = warp_sum(d);
    for (int i = lane; i < n; i += 32) dx[r * n + i] = scale * y[r * n + i] * (dy[r * n + i] - d);
  }
}

// element (k, q) of each [n0 x n1] slice is masked when k > n_past + q
__global__ void k_diag_mask(const float* __restrict__ a, float* __restrict__ o, int n0, int n1, int n_past, float val,
                            long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    const int k = (int)(i % n0), q = (int)((i / n0) % n1);
    o[i] = k > n_past + q ? val : a[i];
  }
}

// NEOX RoPE on [ne0 = head dim, ne1 = heads, ne2 = tokens, ne3]: pairs (i, i + n_dims/2)
// rotated by theta_i = freq_scale * pos * theta_scale^i / ff_i with ggml's f32
// recurrence; columns >= n_dims pass through. dir = -1 rotates back.
__global__ void k_rope(const float* __restrict__ a, const int* __restrict__ pos, const float* __restrict__ ff,
                       float* __restrict__ o, int ne0, int ne1, int ne2, long long rows, int n_dims, float theta_scale,
                       float freq_scale, float attn_factor, float dir) {
  griddep_wait();
  const int half = n_dims / 2;
  GRID_LOOP(r, rows) {   // one (token, head) row per thread
    const int tok = (int)((r / ne1) % ne2);
    const float* ar = a + r * ne0;
    float* orow = o + r * ne0;
    float theta = (float)pos[tok];
    for (int i = 0; i < half; ++i) {
      const float f = ff ? ff[i] : 1.0f;
      const float th = freq_scale * (theta / f);
      const float c = cosf(th) * attn_factor, s = sinf(th) * attn_factor * dir;
      const float x0 = ar[i], x1 = ar[i + half];
      orow[i] = x0 * c - x1 * s;
      orow[i + half] = x0 * s + x1 * c;
      theta *= theta_scale;
    }
    for (int i = n_dims; i < ne0; ++i) orow[i] = ar[i];
  }
}

// 4-D permutation copy: out index (j0..j3) = in index with axes permuted:
// in dim d goes to out dim perm[d]
__global__ void k_permute(const float* __restrict__ a, float* __restrict__ o, Sh si, Sh so, int p0, int p1, int p2,
                          int p3, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    long long t = i;
    int idx[4];
    idx[0] = (int)(t % si.n0); t /= si.n0;
    idx[1] = (int)(t % si.n1); t /= si.n1;
    idx[2] = (int)(t % si.n2);
    idx[3] = (int)(t / si.n2);
    int od[4];
    od[p0] = idx[0];
    od[p1] = idx[1];
    od[p2] = idx[2];
    od[p3] = idx[3];
    o[(((long long)od[3] * so.n2 + od[2]) * so.n1 + od[1]) * so.n0 + od[0]] = a[i];
  }
}

// out = a with its dimension `dim` cut to [start, start + out extent)
__global__ void k_slice(const float* __restrict__ a, float* __restrict__ o, Sh sa, Sh so, int dim, int start,
                        long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    long long t = i;
    int idx[4];
    idx[0] = (int)(t % so.n0); t /= so.n0;
    idx[1] = (int)(t % so.n1); t /= so.n1;
    idx[2] = (int)(t % so.n2);
    idx[3] = (int)(t / so.n2);
    idx[dim] += start;
    o[i] = a[(((long long)idx[3] * sa.n2 + idx[2]) * sa.n1 + idx[1]) * sa.n0 + idx[0]];
  }
}

// concatenation of a and b along `dim`
__global__ void k_concat(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o, Sh sa,
                         Sh sb, Sh so, int dim, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    long long t = i;
    int idx[4];
    idx[0] = (int)(t % so.n0); t /= so.n0;
    idx[1] = (int)(t % so.n1); t /= so.n1;
    idx[2] = (int)(t % so.n2);
    idx[3] = (int)(t / so.n2);
    const int ad[4] = {sa.n0, sa.n1, sa.n2, sa.n3};
    if (idx[dim] < ad[dim]) {
      o[i] = a[(((long long)idx[3] * sa.n2 + idx[2]) * sa.n1 + idx[1]) * sa.n0 + idx[0]];
    } else {
      idx[dim] -= ad[dim];
      o[i] = b[(((long long)idx[3] * sb.n2 + idx[2]) * sb.n1 + idx[1]) * sb.n0 + idx[0]];
    }
  }
}

// strided view copy: rows of ne0 elements, row r at src + r1 * s1 + r2 * s2 + r3 * s3 (elements)
__global__ void k_view_copy(const float* __restrict__ src, float* __restrict__ o, Sh so, long long s1, long long s2,
                            long long s3, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    long long t = i;
    const int i0 = (int)(t % so.n0); t /= so.n0;
    const int i1 = (int)(t % so.n1); t /= so.n1;
    const int i2 = (int)(t % so.n2);
    const int i3 = (int)(t / so.n2);
    o[i] = src[i0 + i1 * s1 + i2 * s2 + i3 * s3];
  }
}

// dst (zero-initialised) += g placed at a strided view position
__global__ void k_view_acc(float* __restrict__ dst, const float* __restrict__ g, Sh so, long long s1, long long s2,
                           long long s3, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    long long t = i;
    const int i0 = (int)(t % so.n0); t /= so.n0;
    const int i1 = (int)(t % so.n1); t /= so.n1;
    const int i2 = (int)(t % so.n2);
    const int i3 = (int)(t / so.n2);
    dst[i0 + i1 * s1 + i2 * s2 + i3 * s3] += g[i];
  }
}

__global__ void k_get_rows(const float* __restrict__ table, const int* __restrict__ idx, float* __restrict__ o,
                           int ne0, int nrows_table, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    const long long r = i / ne0;
    int id = idx[r];
    id = id < 0 ? 0 : (id >= nrows_table ? nrows_table - 1 : id);
    o[i] = table[(long long)id * ne0 + i % ne0];
  }
}

// ggml_mul_mat_id: o[t][u][r] = sum_k W[e][r][k] x[t][u or 0][k], e = ids[t][u]
// (W [E][d_out][d_in] f32, or Q8_0 quants and fp16 scales); one warp per
// output element, lanes along k, an expert index outside [0, E) gives 0.
__global__ void k_mul_mat_id(const float* __restrict__ w32, const int8_t* __restrict__ wq,
                             const uint16_t* __restrict__ ws, const float* __restrict__ x, const int* __restrict__ ids,
                             float* __restrict__ o, int d_in, int d_out, int E, int n_used, int nx1, long long nout) {
  griddep_wait();
  const int lane = threadIdx.x & 31;
  for (long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) / 32; w < nout;
       w += (long long)gridDim.x * blockDim.x / 32) {
    const long long slot = w / d_out;   // t * n_used + u
    const int r = (int)(w % d_out), u = (int)(slot % n_used);
    const long long t = slot / n_used;
    const int e = ids[slot];
    float acc = 0.f;
    if (e >= 0 && e < E) {
      const float* xr = x + (t * nx1 + (nx1 == 1 ? 0 : u)) * d_in;
      const long long row = (long long)e * d_out + r;
      for (int k = lane; k < d_in; k += 32) {
        const float wv = w32 ? w32[row * d_in + k]
                             : __half2float(__ushort_as_half(ws[row * (d_in / 32) + k / 32])) * (float)wq[row * d_in + k];
        acc = fmaf(wv, xr[k], acc);
      }
    }
#pragma unroll
    for (int m = 16; m; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (lane == 0) o[w] = acc;
  }
}

// ggml_set_rows: o[idx[r]][c] = b[r][c] for the rows of b (indices outside o skipped)
__global__ void k_set_rows(const float* __restrict__ b, const int* __restrict__ idx, float* __restrict__ o, int ne0,
                           int o_rows, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    const int r = idx[i / ne0];
    if (r >= 0 && r < o_rows) o[(long long)r * ne0 + i % ne0] = b[i];
  }
}

// ggml_add_id: o[i2][i1][i0] = a[i2][i1][i0] + b[ids[i2][i1]][i0]
__global__ void k_add_id(const float* __restrict__ a, const float* __restrict__ b, const int* __restrict__ ids,
                         float* __restrict__ o, int ne0, int nb_rows, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    int id = ids[i / ne0];
    id = id < 0 ? 0 : (id >= nb_rows ? nb_rows - 1 : id);
    o[i] = a[i] + b[(long long)id * ne0 + i % ne0];
  }
}

// ggml_argsort / ggml_top_k over each row of ne0 values: o[row][rank] = i for
// the rank of element i (ascending, or descending), ties by the lower index
// first; top_k keeps the k leading ranks of a descending sort. One block per row.
__global__ void k_argsort(const float* __restrict__ a, int* __restrict__ o, int ne0, long long rows, int desc,
                          int keep) {
  griddep_wait();
  for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* v = a + row * ne0;
    for (int i = threadIdx.x; i < ne0; i += blockDim.x) {
      const float vi = v[i];
      int rank = 0;
      for (int j = 0; j < ne0; ++j) {
        const float vj = v[j];
        rank += (desc ? vj > vi : vj < vi) || (vj == vi && j < i);
      }
      if (rank < keep) o[row * keep + rank] = i;
    }
  }
}

__global__ void k_get_rows_back(const float* __restrict__ g, const int* __restrict__ idx, float* __restrict__ o,
                                int ne0, int nrows_table, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) {
    const long long r = i / ne0;
    const int id = idx[r];
    if (id >= 0 && id < nrows_table) atomicAdd(&o[(long long)id * ne0 + i % ne0], g[i]);
  }
}

// ggml cross_entropy_loss: loss = -(1/rows) sum_rows sum_v y log softmax(z); one block
// per row writes its term, a second kernel sums them in order
__global__ void k_ce_rows(const float* __restrict__ z, const float* __restrict__ y, float* __restrict__ term,
                          long long rows, int n) {
  griddep_wait();
  __shared__ float red[32];
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* zr = z + r * n;
    const float* yr = y + r * n;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, zr[i]);
    m = warp_max(m);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
      v = warp_max(v);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    float s = 0.f, sy = 0.f, syz = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      s += expf(zr[i] - m);
      sy += yr[i];
      syz += yr[i] * zr[i];
    }
    s = warp_sum(s);
    sy = warp_sum(sy);
    syz = warp_sum(syz);
    __shared__ float r3[3][32];
    if (threadIdx.x % 32 == 0) {
      r3[0][threadIdx.x / 32] = s;
      r3[1][threadIdx.x / 32] = sy;
      r3[2][threadIdx.x / 32] = syz;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float a = 0.f, b = 0.f, c = 0.f;
      for (int w = 0; w < (int)blockDim.x / 32; ++w) {
        a += r3[0][w];
        b += r3[1][w];
        c += r3[2][w];
      }
      // -sum y (z - m - log s)
      term[r] = -(c - b * (m + logf(a)));
    }
    __syncthreads();
  }
}

__global__ void k_sum_ordered(const float* __restrict__ x, long long n, float scale, float* __restrict__ out) {
  griddep_wait();
  __shared__ float red[32];
  float s = 0.f;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  s = warp_sum(s);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) t += red[w];
    out[0] = t * scale;
  }
}

// (softmax(z) - y) * dloss / rows
__global__ void k_ce_back(const float* __restrict__ dl, const float* __restrict__ z, const float* __restrict__ y,
                          float* __restrict__ o, long long rows, int n) {
  griddep_wait();
  const int lane = threadIdx.x % 32, warps = blockDim.x / 32;
  const float g = dl[0] / (float)rows;
  for (long long r = blockIdx.x * (long long)warps + threadIdx.x / 32; r < rows; r += (long long)gridDim.x * warps) {
    const float* zr = z + r * n;
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, zr[i]);
    m = warp_max(m);
    float s = 0.f;
    for (int i = lane; i < n; i += 32) s += expf(zr[i] - m);
    s = warp_sum(s);
    const float inv = 1.0f / s;
    for (int i = lane; i < n; i += 32) o[r * n + i] = (expf(zr[i] - m) * inv - y[r * n + i]) * g;
  }
}

// per-row sum of ne0
__global__ void k_sum_rows(const float* __restrict__ a, float* __restrict__ o, long long rows, int n) {
  griddep_wait();
  const int lane = threadIdx.x % 32, warps = blockDim.x / 32;
  for (long long r = blockIdx.x * (long long)warps + threadIdx.x / 32; r < rows; r += (long long)gridDim.x * warps) {
    float s = 0.f;
    for (int i = lane; i < n; i += 32) s += a[r * n + i];
    s = warp_sum(s);
    if (lane == 0) o[r] = s;
  }
}

// opt_step_adamw (tinynn_ggml.h:457-465); hp = [alpha, b1, b2, eps, wd, beta1h, beta2h]
__global__ void k_adamw(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                        float* __restrict__ v, const float* __restrict__ hp, long long n) {
  griddep_wait();
  const float alpha = hp[0], b1 = hp[1], b2 = hp[2], eps = hp[3], wd = hp[4], b1h = hp[5], b2h = hp[6];
  const float keep = 1.0f - alpha * wd;
  GRID_LOOP(i, n) {
    const float gi = g[i];
    const float mi = m[i] * b1 + gi * (1.0f - b1);
    const float vi = v[i] * b2 + gi * gi * (1.0f - b2);
    m[i] = mi;
    v[i] = vi;
    const float mh = mi * b1h;
    const float vh = sqrtf(vi * b2h) + eps;
    p[i] = p[i] * keep - alpha * mh / vh;
  }
}

// hi = rn_bf16(x), lo = rn_bf16(x - hi) of `rows` rows of `cols` floats, written
// with a row pitch of `ldp` elements (a multiple of 8, TMA's 16-byte stride
// rule); the pad columns are zero
__global__ void k_split_pad(const float* __restrict__ x, bf16* __restrict__ hi, bf16* __restrict__ lo, int cols,
                            int ldp, long long rows) {
  griddep_wait();
  GRID_LOOP(i, rows * ldp) {
    const long long r = i / ldp;
    const int c = (int)(i % ldp);
    const float v = c < cols ? x[r * cols + c] : 0.f;
    const bf16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

// rows of `cols` floats taken from a buffer with row pitch `ldp`
__global__ void k_unpad(const float* __restrict__ src, float* __restrict__ o, int cols, int ldp, long long n) {
  griddep_wait();
  GRID_LOOP(i, n) o[i] = src[(i / cols) * ldp + i % cols];
}

// Q8_0 -> f32: value = fp16 scale * int8 quant (from the split quant / scale arrays)
__global__ void k_dequant(const int8_t* __restrict__ q, const uint16_t* __restrict__ sc, float* __restrict__ o,
                          long long n) {
  griddep_wait();
  GRID_LOOP(i, n) o[i] = __half2float(__ushort_as_half(sc[i / 32])) * (float)q[i];
}

// ggml opt_step_sgd: p = p (1 - alpha wd) - alpha g; hp = [alpha, wd]
__global__ void k_sgd(float* __restrict__ p, const float* __restrict__ g, const float* __restrict__ hp, long long n) {
  griddep_wait();
  const float alpha = hp[0], keep = 1.0f - hp[0] * hp[1];
  GRID_LOOP(i, n) p[i] = p[i] * keep - alpha * g[i];
}

#undef GRID_LOOP

// ------------------------------------------------------------------ graph helpers
float* F(Tensor* t) { return static_cast<float*>(t->data); }
const int* I(Tensor* t) { return static_cast<const int*>(t->data); }

bool same_shape(const Tensor* a, const Tensor* b) {
  return a->ne[0] == b->ne[0] && a->ne[1] == b->ne[1] && a->ne[2] == b->ne[2] && a->ne[3] == b->ne[3];
}

bool can_repeat(const Tensor* small, const Tensor* big) {
  for (int d = 0; d < 4; ++d)
    if (small->ne[d] <= 0 || big->ne[d] % small->ne[d]) return false;
  return true;
}

bool is_f32(const Tensor* t) { return t && t->type == 0; }

// ggml's broadcast of a matrix product over the batch dims (b batch (i2, i3)
// reads a batch (i2 / r2, i3 / r3)); the GEMM maps flat batch z to z / r, which
// is that map when a has one batch or a's ne3 equals b's
bool batch_ok(const Tensor* a, const Tensor* b) {
  if (b->ne[2] % a->ne[2] || b->ne[3] % a->ne[3]) return false;
  return (a->ne[2] == 1 && a->ne[3] == 1) || a->ne[3] == b->ne[3];
}

}  // namespace

Tensor* prim_new(Session* s, int type, int ne0, int ne1, int ne2, int ne3, int op, bool persistent) {
  if (ne0 <= 0 || ne1 <= 0 || ne2 <= 0 || ne3 <= 0) return nullptr;
  auto t = std::make_unique<Tensor>();
  t->sess = s;
  t->role = Tensor::kPrim;
  t->type = type;
  t->ne[0] = ne0; t->ne[1] = ne1; t->ne[2] = ne2; t->ne[3] = ne3;
  t->op = op;
  t->persistent = persistent;
  Tensor* r = t.get();
  s->tensors.push_back(std::move(t));
  if (persistent && prim_alloc(s, r)) return nullptr;
  return r;
}

// Device storage of a tensor (aliasing views share their parent's).
int prim_alloc(Session* s, Tensor* t) {
  if (t->data || t->q8v) return 0;
  if (cudaSetDevice(s->device) != cudaSuccess) return -3;
  if (t->view_of) {
    Tensor* p = t->view_of;
    if (prim_alloc(s, p)) return -3;
    if (p->type == 8) {
      const long long row0 = (long long)(t->view_off / ((size_t)p->ne[0] / 32 * 34));
      t->q8v = static_cast<int8_t*>(p->q8v) + row0 * p->ne[0];
      t->q8s = static_cast<uint16_t*>(p->q8s) + row0 * (p->ne[0] / 32);
      t->data = static_cast<uint8_t*>(p->data) + t->view_off;
    } else {
      t->data = static_cast<uint8_t*>(p->data) + t->view_off;
    }
    t->bytes = (size_t)t->nel() * 4;
    return 0;
  }
  if (t->type == 8) {
    const long long n = t->nel();
    t->bytes = (size_t)(n / 32 * 34);
    if (cudaMalloc(&t->data, t->bytes) != cudaSuccess || cudaMalloc(&t->q8v, (size_t)n) != cudaSuccess ||
        cudaMalloc(&t->q8s, (size_t)(n / 32) * 2) != cudaSuccess)
      return -3;
    cudaMemset(t->data, 0, t->bytes);
    cudaMemset(t->q8v, 0, (size_t)n);
    cudaMemset(t->q8s, 0, (size_t)(n / 32) * 2);
    return 0;
  }
  t->bytes = (size_t)t->nel() * 4;
  if (cudaMalloc(&t->data, t->bytes ? t->bytes : 4) != cudaSuccess) {
    t->data = nullptr;
    return -3;
  }
  return cudaMemset(t->data, 0, t->bytes ? t->bytes : 4) == cudaSuccess ? 0 : -3;
}

// ------------------------------------------------------------------ uploads / downloads
int prim_upload_f64(Session* s, Tensor* t, const double* data, size_t n) {
  if ((long long)n > t->nel() || (t->type != 0 && t->type != 8)) return -2;
  if (prim_alloc(s, t)) return -3;
  std::vector<float> h(n);
  for (size_t i = 0; i < n; ++i) h[i] = (float)data[i];
  if (t->type == 0) return cudaMemcpy(t->data, h.data(), n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -3;
  // Q8_0 tensor: quantise on the device (ggml quantize_row_q8_0), then split for the GEMM
  if ((long long)n != t->nel() || t->ne[0] % 32) return -2;
  float* tmp = nullptr;
  if (cudaMalloc(&tmp, n * 4) != cudaSuccess) return -3;
  int rc = cudaMemcpy(tmp, h.data(), n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -3;
  if (!rc) rc = launch_q8_0_quantize(tmp, static_cast<uint8_t*>(t->data), t->rows(), t->ne[0], nullptr);
  if (!rc)
    rc = launch_q8_0_split(static_cast<const uint8_t*>(t->data), static_cast<int8_t*>(t->q8v),
                           static_cast<uint16_t*>(t->q8s), (long long)n / 32, nullptr);
  if (cudaDeviceSynchronize() != cudaSuccess && !rc) rc = -3;
  cudaFree(tmp);
  return rc;
}

int prim_upload_q8_0(Session* s, Tensor* t, const void* blocks, size_t nbytes) {
  if (t->type != 8 || nbytes != (size_t)(t->nel() / 32 * 34) || t->view_of) return -2;
  if (prim_alloc(s, t)) return -3;
  if (cudaMemcpy(t->data, blocks, nbytes, cudaMemcpyHostToDevice) != cudaSuccess) return -3;
  int rc = launch_q8_0_split(static_cast<const uint8_t*>(t->data), static_cast<int8_t*>(t->q8v),
                             static_cast<uint16_t*>(t->q8s), t->nel() / 32, nullptr);
  if (cudaDeviceSynchronize() != cudaSuccess && !rc) rc = -3;
  return rc;
}

int prim_upload_i64(Session* s, Tensor* t, const long* data, size_t n) {
  if (t->type != 26 || (long long)n > t->nel()) return -2;
  if (prim_alloc(s, t)) return -3;
  std::vector<int> h(n);
  for (size_t i = 0; i < n; ++i) h[i] = (int)data[i];
  return cudaMemcpy(t->data, h.data(), n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -3;
}

int prim_download_f64(Session* s, Tensor* t, double* dst, size_t n) {
  (void)s;
  if ((long long)n > t->nel() || !t->data) return -2;
  if (cudaDeviceSynchronize() != cudaSuccess) return -3;
  if (t->type == 26) {
    std::vector<int> h(n);
    if (cudaMemcpy(h.data(), t->data, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -3;
    for (size_t i = 0; i < n; ++i) dst[i] = h[i];
    return 0;
  }
  if (t->type == 8) {   // dequantise: value = fp16 scale * int8 quant
    std::vector<uint8_t> b((size_t)(t->nel() / 32 * 34));
    if (cudaMemcpy(b.data(), t->data, b.size(), cudaMemcpyDeviceToHost) != cudaSuccess) return -3;
    for (size_t i = 0; i < n; ++i) {
      const uint8_t* blk = b.data() + (i / 32) * 34;
      __half_raw hr;
      hr.x = (unsigned short)(blk[0] | (blk[1] << 8));
      dst[i] = (double)(__half2float(__half(hr)) * (float)(int8_t)blk[2 + i % 32]);
    }
    return 0;
  }
  std::vector<float> h(n);
  if (cudaMemcpy(h.data(), t->data, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -3;
  for (size_t i = 0; i < n; ++i) dst[i] = h[i];
  return 0;
}

int prim_zero(Session* s, Tensor* t) {
  if (prim_alloc(s, t)) return -3;
  return cudaMemset(t->data, 0, t->bytes) == cudaSuccess ? 0 : -3;
}

// ------------------------------------------------------------------ node constructors
namespace {

Tensor* node(Session* s, int op, const Tensor* like, Tensor* a, Tensor* b = nullptr, Tensor* c = nullptr) {
  Tensor* t = prim_new(s, 0, like->ne[0], like->ne[1], like->ne[2], like->ne[3], op, false);
  if (!t) return nullptr;
  t->src[0] = a; t->src[1] = b; t->src[2] = c;
  return t;
}

}  // namespace

Tensor* prim_binary(Session* s, int op, Tensor* a, Tensor* b) {
  if (!is_f32(a) || !is_f32(b) || !can_repeat(b, a)) return nullptr;
  return node(s, op, a, a, b);
}

Tensor* prim_scale(Session* s, Tensor* a, double v) {
  if (!is_f32(a)) return nullptr;
  Tensor* t = node(s, kOpScale, a, a);
  if (t) t->fp[0] = v;
  return t;
}

Tensor* prim_unary(Session* s, int op, Tensor* a, Tensor* b) {
  if (!is_f32(a) || (b && (!is_f32(b) || !same_shape(a, b)))) return nullptr;
  return node(s, op, a, a, b);
}

// ggml_mul_mat(a, b): a [K, M, A2, A3], b [K, N, B2, B3] (A2 | B2, A3 | B3) -> [M, N, B2, B3]
Tensor* prim_mul_mat(Session* s, Tensor* a, Tensor* b) {
  if (!a || !is_f32(b) || (a->type != 0 && a->type != 8) || a->ne[0] != b->ne[0]) return nullptr;
  if (!batch_ok(a, b) || (a->type == 8 && (a->ne[2] != 1 || a->ne[3] != 1))) return nullptr;
  Tensor* t = prim_new(s, 0, a->ne[1], b->ne[1], b->ne[2], b->ne[3], kOpMulMat, false);
  if (t) { t->src[0] = a; t->src[1] = b; }
  return t;
}

// ggml_out_prod(a, b): a [M, K, A2, A3], b [N, K, B2, B3] -> [M, N, B2, B3], r[n][m] = sum_k a[k][m] b[k][n]
Tensor* prim_out_prod(Session* s, Tensor* a, Tensor* b) {
  if (!is_f32(a) || !is_f32(b) || a->ne[1] != b->ne[1] || !batch_ok(a, b)) return nullptr;
  Tensor* t = prim_new(s, 0, a->ne[0], b->ne[0], b->ne[2], b->ne[3], kOpOutProd, false);
  if (t) { t->src[0] = a; t->src[1] = b; }
  return t;
}

// internal: r[n][k] = sum_m g[n][m] a[m][k]  (the gradient of mul_mat's b), a [K, M, ..], g [M, N, ..]
Tensor* prim_mul_mat_at(Session* s, Tensor* a, Tensor* g, const Tensor* b_like) {
  Tensor* t = node(s, kOpMulMatAT, b_like, a, g);
  return t;
}

Tensor* prim_rms_norm(Session* s, Tensor* x, double eps) {
  if (!is_f32(x)) return nullptr;
  Tensor* t = node(s, kOpRmsNorm, x, x);
  if (t) t->fp[0] = eps;
  return t;
}

Tensor* prim_rms_norm_back(Session* s, Tensor* x, Tensor* dy, double eps) {
  if (!is_f32(x) || !is_f32(dy) || !same_shape(x, dy)) return nullptr;
  Tensor* t = node(s, kOpRmsNormBack, x, x, dy);
  if (t) t->fp[0] = eps;
  return t;
}

Tensor* prim_rope(Session* s, int op, Tensor* a, Tensor* pos, int n_dims, double base, double fscale, double ext,
                  double attn, Tensor* ff) {
  if (!is_f32(a) || !pos || pos->type != 26 || pos->nel() < a->ne[2] || n_dims <= 0 || n_dims > a->ne[0] ||
      n_dims % 2 || ext != 0.0)
    return nullptr;
  if (ff && (!is_f32(ff) || ff->nel() < n_dims / 2)) return nullptr;
  Tensor* t = node(s, op, a, a, pos, ff);
  if (t) {
    t->ip[0] = n_dims;
    t->fp[0] = base; t->fp[1] = fscale; t->fp[2] = attn;
  }
  return t;
}

Tensor* prim_softmax(Session* s, Tensor* a, Tensor* mask, double scale, double max_bias) {
  if (!is_f32(a) || max_bias != 0.0) return nullptr;
  // mask [ne0, >= ne1, 1, 1]: row i1 of the mask applies to row i1 of every a slice
  if (mask && (!is_f32(mask) || mask->ne[0] != a->ne[0] || mask->ne[1] < a->ne[1] || mask->ne[2] != 1 ||
               mask->ne[3] != 1))
    return nullptr;
  Tensor* t = node(s, kOpSoftMax, a, a, mask);
  if (t) t->fp[0] = scale;
  return t;
}

Tensor* prim_softmax_back(Session* s, Tensor* y, Tensor* dy, double scale) {
  if (!is_f32(y) || !is_f32(dy) || !same_shape(y, dy)) return nullptr;
  Tensor* t = node(s, kOpSoftMaxBack, y, y, dy);
  if (t) t->fp[0] = scale;
  return t;
}

Tensor* prim_diag_mask(Session* s, int op, Tensor* a, int n_past) {
  if (!is_f32(a)) return nullptr;
  Tensor* t = node(s, op, a, a);
  if (t) t->ip[0] = n_past;
  return t;
}

Tensor* prim_permute(Session* s, Tensor* a, int p0, int p1, int p2, int p3) {
  if (!is_f32(a)) return nullptr;
  const int p[4] = {p0, p1, p2, p3};
  int seen = 0;
  for (int d = 0; d < 4; ++d) {
    if (p[d] < 0 || p[d] > 3) return nullptr;
    seen |= 1 << p[d];
  }
  if (seen != 15) return nullptr;
  int ne[4];
  for (int d = 0; d < 4; ++d) ne[p[d]] = a->ne[d];
  Tensor* t = prim_new(s, 0, ne[0], ne[1], ne[2], ne[3], kOpTranspose, false);
  if (t) {
    t->src[0] = a;
    for (int d = 0; d < 4; ++d) t->ip[d] = p[d];
  }
  return t;
}

Tensor* prim_reshape(Session* s, Tensor* a, int ne0, int ne1, int ne2, int ne3) {
  if (!a || (long long)ne0 * ne1 * ne2 * ne3 != a->nel() || a->type == 8) return nullptr;
  Tensor* t = prim_new(s, a->type, ne0, ne1, ne2, ne3, kOpReshape, false);
  if (t) {
    t->src[0] = a;
    t->view_of = a->view_of ? a->view_of : a;
    t->view_off = a->view_of ? a->view_off : 0;
  }
  return t;
}

Tensor* prim_cont(Session* s, Tensor* a, int ne0, int ne1, int ne2, int ne3) {
  if (!is_f32(a) || (long long)ne0 * ne1 * ne2 * ne3 != a->nel()) return nullptr;
  Tensor* t = prim_new(s, 0, ne0, ne1, ne2, ne3, kOpCont, false);
  if (t) t->src[0] = a;
  return t;
}

// view with element strides: contiguous views alias their parent, others are
// gathered (kOpView); Q8_0 views must be whole contiguous rows
Tensor* prim_view(Session* s, Tensor* a, int ne0, int ne1, int ne2, size_t nb1, size_t nb2, size_t offset) {
  if (!a || ne0 <= 0 || ne1 <= 0 || ne2 <= 0) return nullptr;
  Tensor* root = a->view_of ? a->view_of : a;
  const size_t base = (a->view_of ? a->view_off : 0) + offset;
  if (a->type == 8) {
    const size_t row = (size_t)root->ne[0] / 32 * 34;
    if (ne0 != root->ne[0] || (ne1 > 1 && nb1 != row) || base % row || ne2 != 1 ||
        base + (size_t)ne1 * row > (size_t)root->nel() / 32 * 34)
      return nullptr;
    Tensor* t = prim_new(s, 8, ne0, ne1, 1, 1, kOpReshape, false);
    if (t) { t->src[0] = a; t->view_of = root; t->view_off = base; }
    return t;
  }
  if (!is_f32(a) || offset % 4 || nb1 % 4 || nb2 % 4) return nullptr;
  // the last element of the view must lie inside a
  if (offset + (size_t)(ne2 - 1) * nb2 + (size_t)(ne1 - 1) * nb1 + (size_t)ne0 * 4 > (size_t)a->nel() * 4) return nullptr;
  const bool contiguous = (ne1 == 1 || nb1 == (size_t)ne0 * 4) && (ne2 == 1 || nb2 == (size_t)ne0 * ne1 * 4);
  if (contiguous && base + (size_t)ne0 * ne1 * ne2 * 4 <= (size_t)root->nel() * 4) {
    Tensor* t = prim_new(s, 0, ne0, ne1, ne2, 1, kOpReshape, false);
    if (t) { t->src[0] = a; t->view_of = root; t->view_off = base; }
    return t;
  }
  Tensor* t = prim_new(s, 0, ne0, ne1, ne2, 1, kOpView, false);
  if (t) {
    t->src[0] = a;
    t->fp[0] = (double)(offset / 4);
    t->fp[1] = (double)(nb1 / 4);
    t->fp[2] = (double)(nb2 / 4);
  }
  return t;
}

Tensor* prim_concat(Session* s, Tensor* a, Tensor* b, int dim) {
  if (!is_f32(a) || !is_f32(b) || dim < 0 || dim > 3) return nullptr;
  for (int d = 0; d < 4; ++d)
    if (d != dim && a->ne[d] != b->ne[d]) return nullptr;
  int ne[4] = {a->ne[0], a->ne[1], a->ne[2], a->ne[3]};
  ne[dim] += b->ne[dim];
  Tensor* t = prim_new(s, 0, ne[0], ne[1], ne[2], ne[3], kOpConcat, false);
  if (t) { t->src[0] = a; t->src[1] = b; t->ip[0] = dim; }
  return t;
}

Tensor* prim_slice(Session* s, Tensor* a, int dim, int start, int len) {
  int ne[4] = {a->ne[0], a->ne[1], a->ne[2], a->ne[3]};
  ne[dim] = len;
  Tensor* t = prim_new(s, 0, ne[0], ne[1], ne[2], ne[3], kOpSlice, false);
  if (t) { t->src[0] = a; t->ip[0] = dim; t->ip[1] = start; }
  return t;
}

// ggml_mul_mat_id: as [d_in][d_out][E] (ne order; f32 or Q8_0), b [d_in][1 or
// n_used][T] f32, ids [n_used][T] i32 -> [d_out][n_used][T]. No backward (as in
// the reference, whose MoE graphs do not differentiate through it).
Tensor* prim_mul_mat_id(Session* s, Tensor* as, Tensor* b, Tensor* ids) {
  if (!as || !b || !ids || ids->type != 26 || !is_f32(b) || (as->type != 0 && as->type != 8)) return nullptr;
  const int d_in = as->ne[0], d_out = as->ne[1], n_used = ids->ne[0], T = ids->ne[1];
  if (as->ne[3] != 1 || ids->ne[2] != 1 || ids->ne[3] != 1 || b->ne[0] != d_in || b->ne[2] != T || b->ne[3] != 1 ||
      (b->ne[1] != 1 && b->ne[1] != n_used) || (as->type == 8 && d_in % 32))
    return nullptr;
  Tensor* t = prim_new(s, 0, d_out, n_used, T, 1, kOpMulMatId, false);
  if (t) { t->src[0] = as; t->src[1] = b; t->src[2] = ids; }
  return t;
}

// ggml_add_id: a [n0][n1][n2] f32, b [n0][rows] f32, ids [n1][n2] i32 -> a + b[ids]
Tensor* prim_add_id(Session* s, Tensor* a, Tensor* b, Tensor* ids) {
  if (!is_f32(a) || !is_f32(b) || !ids || ids->type != 26 || b->ne[0] != a->ne[0] || ids->ne[0] != a->ne[1] ||
      ids->ne[1] != a->ne[2] || a->ne[3] != 1 || b->ne[2] != 1 || b->ne[3] != 1)
    return nullptr;
  Tensor* t = prim_new(s, 0, a->ne[0], a->ne[1], a->ne[2], 1, kOpAddId, false);
  if (t) { t->src[0] = a; t->src[1] = b; t->src[2] = ids; }
  return t;
}

// ggml_argsort (k = 0: every index, ascending or descending) and ggml_top_k
// (k > 0: the indices of the k largest, largest first): i32 [k or ne0][rows]
Tensor* prim_argsort(Session* s, Tensor* a, int descending, int k) {
  if (!is_f32(a) || k < 0 || k > a->ne[0]) return nullptr;
  Tensor* t = prim_new(s, 26, k ? k : a->ne[0], a->ne[1], a->ne[2], a->ne[3], k ? kOpTopK : kOpArgsort, false);
  if (t) { t->src[0] = a; t->ip[0] = k ? 1 : (descending ? 1 : 0); }
  return t;
}

// ggml_detach-style cut: an alias of a that the backward does not pass through
Tensor* prim_detach(Session* s, Tensor* a) {
  if (!a || a->type == 8) return nullptr;
  Tensor* t = prim_new(s, a->type, a->ne[0], a->ne[1], a->ne[2], a->ne[3], kOpDetach, false);
  if (t) {
    t->src[0] = a;
    t->view_of = a->view_of ? a->view_of : a;
    t->view_off = a->view_of ? a->view_off : 0;
  }
  return t;
}

// ggml_cpy: the elements of a written into b's storage (same count, same type,
// f32 or i32); the result is b's view, so later reads of b see them
Tensor* prim_cpy(Session* s, Tensor* a, Tensor* b) {
  if (!a || !b || a->type != b->type || (a->type != 0 && a->type != 26) || a->nel() != b->nel()) return nullptr;
  Tensor* t = prim_new(s, b->type, b->ne[0], b->ne[1], b->ne[2], b->ne[3], kOpCpy, false);
  if (t) {
    t->src[0] = a;
    t->src[1] = b;
    t->view_of = b->view_of ? b->view_of : b;
    t->view_off = b->view_of ? b->view_off : 0;
  }
  return t;
}

// ggml_set_rows: rows idx[i] of a (f32 [ne0][rows]) := rows i of b (f32 [ne0][n]),
// idx i32 [n]; the result is a's view (indices outside a's rows are skipped)
Tensor* prim_set_rows(Session* s, Tensor* a, Tensor* b, Tensor* idx) {
  if (!is_f32(a) || !is_f32(b) || !idx || idx->type != 26 || a->ne[0] != b->ne[0] || b->rows() != idx->nel())
    return nullptr;
  Tensor* t = prim_new(s, 0, a->ne[0], a->ne[1], a->ne[2], a->ne[3], kOpSetRows, false);
  if (t) {
    t->src[0] = a;
    t->src[1] = b;
    t->src[2] = idx;
    t->view_of = a->view_of ? a->view_of : a;
    t->view_off = a->view_of ? a->view_off : 0;
  }
  return t;
}

Tensor* prim_get_rows(Session* s, Tensor* table, Tensor* idx) {
  if (!is_f32(table) || !idx || idx->type != 26) return nullptr;
  Tensor* t = prim_new(s, 0, table->ne[0], (int)idx->nel(), 1, 1, kOpGetRows, false);
  if (t) { t->src[0] = table; t->src[1] = idx; }
  return t;
}

Tensor* prim_get_rows_back(Session* s, Tensor* g, Tensor* idx, Tensor* like) {
  if (!is_f32(g) || !idx || idx->type != 26 || !like || g->ne[0] != like->ne[0]) return nullptr;
  Tensor* t = prim_new(s, 0, like->ne[0], like->ne[1], 1, 1, kOpGetRowsBack, false);
  if (t) { t->src[0] = g; t->src[1] = idx; }
  return t;
}

Tensor* prim_cross_entropy(Session* s, Tensor* a, Tensor* b) {
  if (!is_f32(a) || !is_f32(b) || !same_shape(a, b)) return nullptr;
  Tensor* t = prim_new(s, 0, 1, 1, 1, 1, kOpCrossEntropy, false);
  if (t) { t->src[0] = a; t->src[1] = b; }
  return t;
}

Tensor* prim_sum(Session* s, int op, Tensor* a) {
  if (!is_f32(a)) return nullptr;
  Tensor* t = op == kOpSum ? prim_new(s, 0, 1, 1, 1, 1, op, false)
                           : prim_new(s, 0, 1, a->ne[1], a->ne[2], a->ne[3], op, false);
  if (t) t->src[0] = a;
  return t;
}

Tensor* prim_opt_adamw(Session* s, Tensor* a, Tensor* g, Tensor* m, Tensor* v, Tensor* hp) {
  if (!is_f32(a) || !is_f32(g) || !is_f32(m) || !is_f32(v) || !is_f32(hp) || a->nel() != g->nel() ||
      a->nel() != m->nel() || a->nel() != v->nel() || hp->nel() < 7)
    return nullptr;
  Tensor* t = prim_new(s, 0, a->ne[0], a->ne[1], a->ne[2], a->ne[3], kOpOptAdamw, false);
  if (t) {
    t->src[0] = a; t->src[1] = g; t->src[2] = m; t->src[3] = v; t->src[4] = hp;
    t->view_of = a;   // the result is the updated parameter itself
  }
  return t;
}

Tensor* prim_opt_sgd(Session* s, Tensor* a, Tensor* g, Tensor* hp) {
  if (!is_f32(a) || !is_f32(g) || !is_f32(hp) || a->nel() != g->nel() || hp->nel() < 2) return nullptr;
  Tensor* t = prim_new(s, 0, a->ne[0], a->ne[1], a->ne[2], a->ne[3], kOpOptSgd, false);
  if (t) {
    t->src[0] = a; t->src[1] = g; t->src[2] = hp;
    t->view_of = a;   // updated in place
  }
  return t;
}

Tensor* prim_cast(Session* s, Tensor* a, int type) {
  if (!a || type != 0) return nullptr;
  if (a->type == 0) return prim_cont(s, a, a->ne[0], a->ne[1], a->ne[2], a->ne[3]);
  if (a->type != 8) return nullptr;
  Tensor* t = prim_new(s, 0, a->ne[0], a->ne[1], a->ne[2], a->ne[3], kOpDequant, false);
  if (t) t->src[0] = a;
  return t;
}

Tensor* prim_flash_attn_ext(Session* s, Tensor* q, Tensor* k, Tensor* v, Tensor* mask, double scale,
                            double max_bias) {
  if (!is_f32(q) || !is_f32(k) || !is_f32(v) || q->ne[0] != k->ne[0] || !same_shape(k, v) || q->ne[3] != k->ne[3])
    return nullptr;
  Tensor* kq = prim_mul_mat(s, k, q);                                    // [Tk, Tq, H, B]
  Tensor* p = kq ? prim_softmax(s, kq, mask, scale, max_bias) : nullptr;
  Tensor* vt = p ? prim_permute(s, v, 1, 0, 2, 3) : nullptr;            // [Tk, dh, KV, B]
  Tensor* o = vt ? prim_mul_mat(s, vt, p) : nullptr;                     // [dh, Tq, H, B]
  return o ? prim_permute(s, o, 0, 2, 1, 3) : nullptr;                   // [dh, H, Tq, B]
}

int prim_upload_f32_raw(Session* s, Tensor* t, const float* src, size_t n) {
  if (t->type != 0 || (long long)n > t->nel()) return -2;
  if (prim_alloc(s, t)) return -3;
  return cudaMemcpy(t->data, src, n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -3;
}

int prim_download_f32_raw(Session* s, Tensor* t, float* dst, size_t n) {
  (void)s;
  if (!t->data || (long long)n > t->nel()) return -2;
  if (t->type == 8) {
    std::vector<double> d(n);
    const int rc = prim_download_f64(s, t, d.data(), n);
    for (size_t i = 0; i < n && !rc; ++i) dst[i] = (float)d[i];
    return rc;
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return -3;
  if (t->type == 26) {
    std::vector<int> h(n);
    if (cudaMemcpy(h.data(), t->data, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -3;
    for (size_t i = 0; i < n; ++i) dst[i] = (float)h[i];
    return 0;
  }
  return cudaMemcpy(dst, t->data, n * 4, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -3;
}

// ------------------------------------------------------------------ execution
namespace {

int gemm_ws(GemmScratch& sc) {
  sc = gemm_scratch();
  return 0;
}

int run_gemm(const GemmDesc& d, cudaStream_t st) {
  GemmScratch sc;
  gemm_ws(sc);
  const int rc = gemm_launch(d, sc, device_error_word(), st);
  return rc;
}

int pitch8(int cols) { return (cols + 7) / 8 * 8; }

// split an f32 tensor into planes held in t->planes (allocated once), rows of
// ne0 elements at a pitch of pitch8(ne0)
int planes_of(Tensor* t, Planes& p, cudaStream_t st) {
  const int ldp = pitch8(t->ne[0]);
  const long long np = (t->rows() * ldp + 127) / 128 * 128;
  if (!t->planes) {
    if (cudaMalloc(&t->planes, (size_t)np * 4) != cudaSuccess) return -3;
  }
  p.hi = static_cast<bf16*>(t->planes);
  p.lo = p.hi + np;
  return launch_pdl(k_split_pad, dim3(grid_for(t->rows() * ldp, 256)), dim3(256), 0, st, (const float*)F(t), p.hi,
                    p.lo, t->ne[0], ldp, t->rows());
}

// operand over planes from planes_of: `nbatch` batches of rows x cols
Operand plane_op(Planes p, int rows, int cols, int nbatch, int mn, int bdiv = 1, int bmul = 1) {
  Operand o;
  o.hi = p.hi; o.lo = p.lo; o.mn_major = mn; o.ld = pitch8(cols); o.rows = rows; o.cols = cols;
  o.batch_stride = (long long)rows * o.ld; o.nbatch = nbatch;
  o.bdiv1 = bdiv; o.bmul1 = bmul; o.bdiv2 = 1; o.bmul2 = 0;
  return o;
}

// f32 store epilogue into t (rows of `cols` = t->ne[0] floats); rows whose
// length is not a multiple of 4 go through a padded buffer, copied out after
int gemm_store(Tensor* t, GemmDesc& d, cudaStream_t st) {
  const int cols = t->ne[0];
  const long long rows_per_batch = d.M;
  d.epi.mode = kEpiStoreF32;
  if (cols % 4 == 0) {
    d.epi.out = F(t); d.epi.m_s0 = cols; d.epi.bstride = rows_per_batch * cols;
    return run_gemm(d, st);
  }
  const int ldp = (cols + 3) / 4 * 4;
  if (!t->outpad && cudaMalloc(&t->outpad, (size_t)t->rows() * ldp * 4) != cudaSuccess) return -3;
  float* buf = static_cast<float*>(t->outpad);
  d.epi.out = buf; d.epi.m_s0 = ldp; d.epi.bstride = rows_per_batch * ldp;
  const int rc = run_gemm(d, st);
  if (rc) return rc;
  return launch_pdl(k_unpad, dim3(grid_for(t->nel(), 256)), dim3(256), 0, st, (const float*)buf, F(t), cols, ldp,
                    t->nel());
}

int exec(Session* s, Tensor* t) {
  cudaStream_t st = s->pstream;
  Tensor *a = t->src[0], *b = t->src[1];
  const long long n = t->nel();
  const int threads = 256;
  switch (t->op) {
    case kOpNone:
    case kOpReshape:
      return 0;
    case kOpAdd: case kOpSub: case kOpMul:
      return launch_pdl(k_binary, dim3(grid_for(n, threads)), dim3(threads), 0, st,
                        t->op == kOpAdd ? 0 : (t->op == kOpSub ? 1 : 2), F(a), F(b), F(t), shape(a), shape(b), n);
    case kOpScale:
      return launch_pdl(k_unary, dim3(grid_for(n, threads)), dim3(threads), 0, st, 0, F(a), (const float*)nullptr,
                        F(t), (float)t->fp[0], n);
    case kOpSilu:
      return launch_pdl(k_unary, dim3(grid_for(n, threads)), dim3(threads), 0, st, 1, F(a), (const float*)nullptr,
                        F(t), 0.f, n);
    case kOpSiluBack:
      return launch_pdl(k_unary, dim3(grid_for(n, threads)), dim3(threads), 0, st, 2, F(a), (const float*)F(b), F(t),
                        0.f, n);
    case kOpSwiglu:
      return launch_pdl(k_unary, dim3(grid_for(n, threads)), dim3(threads), 0, st, 3, F(a), (const float*)F(b), F(t),
                        0.f, n);
    case kOpRepeat:
      return launch_pdl(k_repeat, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), F(t), shape(a), shape(t), n);
    case kOpRepeatBack:
      return launch_pdl(k_repeat_back, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), F(t), shape(a),
                        shape(t), n);
    case kOpRmsNorm:
      return launch_pdl(k_rms_norm, dim3(grid_for(t->rows() * 32, threads)), dim3(threads), 0, st, F(a), F(t),
                        t->rows(), t->ne[0], (float)t->fp[0]);
    case kOpRmsNormBack:
      return launch_pdl(k_rms_norm_back, dim3(grid_for(t->rows() * 32, threads)), dim3(threads), 0, st, F(a), F(b),
                        F(t), t->rows(), t->ne[0], (float)t->fp[0]);
    case kOpRope: case kOpRopeBack: {
      const int nd = t->ip[0];
      const float ts = powf((float)t->fp[0], -2.0f / (float)nd);
      return launch_pdl(k_rope, dim3(grid_for(t->rows(), 128)), dim3(128), 0, st, F(a), I(b),
                        t->src[2] ? (const float*)F(t->src[2]) : (const float*)nullptr, F(t), t->ne[0], t->ne[1],
                        t->ne[2], t->rows(), nd, ts, (float)t->fp[1], (float)t->fp[2],
                        t->op == kOpRope ? 1.0f : -1.0f);
    }
    case kOpSoftMax:
      return launch_pdl(k_softmax, dim3(grid_for(t->rows() * 32, threads)), dim3(threads), 0, st, F(a),
                        b ? (const float*)F(b) : (const float*)nullptr, F(t), t->rows(), t->ne[0], (float)t->fp[0],
                        (long long)t->ne[1]);
    case kOpSoftMaxBack:
      return launch_pdl(k_softmax_back, dim3(grid_for(t->rows() * 32, threads)), dim3(threads), 0, st, F(a), F(b),
                        F(t), t->rows(), t->ne[0], (float)t->fp[0]);
    case kOpDiagMaskInf: case kOpDiagMaskZero:
      return launch_pdl(k_diag_mask, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), F(t), t->ne[0],
                        t->ne[1], t->ip[0], t->op == kOpDiagMaskInf ? -INFINITY : 0.0f, n);
    case kOpTranspose:
      return launch_pdl(k_permute, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), F(t), shape(a), shape(t),
                        t->ip[0], t->ip[1], t->ip[2], t->ip[3], n);
    case kOpCont:
      return cudaMemcpyAsync(F(t), F(a), (size_t)n * 4, cudaMemcpyDeviceToDevice, st) == cudaSuccess ? 0 : -3;
    case kOpView: {
      const long long off = (long long)t->fp[0], s1 = (long long)t->fp[1], s2 = (long long)t->fp[2];
      return launch_pdl(k_view_copy, dim3(grid_for(n, threads)), dim3(threads), 0, st, (const float*)(F(a) + off),
                        F(t), shape(t), s1, s2, 0LL, n);
    }
    case kOpAccView: {   // t (shape of the viewed parent) = zeros + a placed at the view position
      Tensor* v = t->src[1];   // the view node (holds offset / strides)
      if (cudaMemsetAsync(F(t), 0, (size_t)n * 4, st) != cudaSuccess) return -3;
      long long off = 0, s1 = v->ne[0], s2 = (long long)v->ne[0] * v->ne[1];
      if (v->op == kOpView) {
        off = (long long)v->fp[0]; s1 = (long long)v->fp[1]; s2 = (long long)v->fp[2];
      } else {   // aliasing view: its offset is into the root buffer, a may itself start inside it
        off = (long long)((v->view_off - (a->view_of ? a->view_off : 0)) / 4);
      }
      return launch_pdl(k_view_acc, dim3(grid_for(a->nel(), threads)), dim3(threads), 0, st, F(t) + off,
                        (const float*)F(a), shape(v), s1, s2, 0LL, a->nel());
    }
    case kOpConcat:
      return launch_pdl(k_concat, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), F(b), F(t), shape(a),
                        shape(b), shape(t), t->ip[0], n);
    case kOpSlice:
      return launch_pdl(k_slice, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), F(t), shape(a), shape(t),
                        t->ip[0], t->ip[1], n);
    case kOpDetach:
      return 0;
    case kOpCpy:
      return cudaMemcpyAsync(t->data, a->data, (size_t)n * 4, cudaMemcpyDeviceToDevice, st) == cudaSuccess ? 0 : -3;
    case kOpSetRows:
      return launch_pdl(k_set_rows, dim3(grid_for(b->nel(), threads)), dim3(threads), 0, st, (const float*)F(b),
                        (const int*)I(t->src[2]), F(t), t->ne[0], (int)t->rows(), b->nel());
    case kOpMulMatId: {
      Tensor* ids = t->src[2];
      const long long nout = t->nel();
      long long blocks = (nout * 32 + 255) / 256;
      if (blocks > 148 * 16) blocks = 148 * 16;
      const bool q8 = a->type == 8;
      return launch_pdl(k_mul_mat_id, dim3((unsigned)blocks), dim3(256), 0, st, q8 ? (const float*)nullptr : F(a),
                        q8 ? static_cast<const int8_t*>(a->q8v) : (const int8_t*)nullptr,
                        q8 ? static_cast<const uint16_t*>(a->q8s) : (const uint16_t*)nullptr, (const float*)F(b),
                        (const int*)I(ids), F(t), a->ne[0], a->ne[1], a->ne[2], ids->ne[0], b->ne[1], nout);
    }
    case kOpAddId:
      return launch_pdl(k_add_id, dim3(grid_for(n, threads)), dim3(threads), 0, st, (const float*)F(a),
                        (const float*)F(b), (const int*)I(t->src[2]), F(t), t->ne[0], (int)b->rows(), n);
    case kOpArgsort: case kOpTopK: {
      const long long rows = a->rows();
      const unsigned blocks = (unsigned)std::min<long long>(rows, 148 * 8);
      return launch_pdl(k_argsort, dim3(blocks), dim3(128), 0, st, (const float*)F(a), static_cast<int*>(t->data), a->ne[0], rows,
                        t->ip[0], t->ne[0]);
    }
    case kOpGetRows:
      return launch_pdl(k_get_rows, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), I(b), F(t), t->ne[0],
                        (int)a->rows(), n);
    case kOpGetRowsBack:
      if (cudaMemsetAsync(F(t), 0, (size_t)n * 4, st) != cudaSuccess) return -3;
      return launch_pdl(k_get_rows_back, dim3(grid_for(a->nel(), threads)), dim3(threads), 0, st, F(a), I(b), F(t),
                        t->ne[0], (int)t->rows(), a->nel());
    case kOpCrossEntropy: {
      const long long rows = a->rows();
      if (!t->planes && cudaMalloc(&t->planes, (size_t)rows * 4) != cudaSuccess) return -3;
      float* term = static_cast<float*>(t->planes);
      int rc = launch_pdl(k_ce_rows, dim3(grid_for(rows * 256, 256)), dim3(256), 0, st, F(a), F(b), term, rows,
                          a->ne[0]);
      if (rc) return rc;
      return launch_pdl(k_sum_ordered, dim3(1), dim3(1024), 0, st, (const float*)term, rows, 1.0f / (float)rows,
                        F(t));
    }
    case kOpCrossEntropyBack: {   // src: dloss (scalar), logits, labels
      Tensor* z = t->src[1];
      Tensor* y = t->src[2];
      return launch_pdl(k_ce_back, dim3(grid_for(z->rows() * 32, threads)), dim3(threads), 0, st, (const float*)F(a),
                        (const float*)F(z), (const float*)F(y), F(t), z->rows(), z->ne[0]);
    }
    case kOpSum:
      return launch_pdl(k_sum_ordered, dim3(1), dim3(1024), 0, st, (const float*)F(a), a->nel(), 1.0f, F(t));
    case kOpSumRows:
      return launch_pdl(k_sum_rows, dim3(grid_for(t->nel() * 32, threads)), dim3(threads), 0, st, F(a), F(t),
                        a->rows(), a->ne[0]);
    case kOpDequant:
      return launch_pdl(k_dequant, dim3(grid_for(n, threads)), dim3(threads), 0, st, (const int8_t*)a->q8v,
                        (const uint16_t*)a->q8s, F(t), n);
    case kOpOptSgd:
      return launch_pdl(k_sgd, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), (const float*)F(b),
                        (const float*)F(t->src[2]), n);
    case kOpOptAdamw:
      return launch_pdl(k_adamw, dim3(grid_for(n, threads)), dim3(threads), 0, st, F(a), (const float*)F(b),
                        F(t->src[2]), F(t->src[3]), (const float*)F(t->src[4]), n);
    case kOpMulMat: case kOpMulMatAT: {
      // kOpMulMat:   r[z][n][m] = sum_k a[za][m][k] b[z][n][k]   (ggml_mul_mat)
      // kOpMulMatAT: r[z][n][k] = sum_m b[z][n][m] a[za][m][k]   (d loss / d b of a mul_mat)
      // with za = z / (batch / abatch); one shared a folds b's batches into rows
      const bool at = t->op == kOpMulMatAT;
      const int K = a->ne[0], M = a->ne[1], Nn = b->ne[1];
      const int batch = b->ne[2] * b->ne[3], abatch = a->ne[2] * a->ne[3];
      const bool fold = abatch == 1;
      const int red = at ? M : K;        // reduction length (ne0 of b)
      Planes pb;
      if (planes_of(b, pb, st)) return -3;
      GemmDesc d;
      d.M = fold ? Nn * batch : Nn; d.N = at ? K : M; d.K = red; d.batch = fold ? 1 : batch;
      d.a = plane_op(pb, d.M, red, d.batch, 0);
      if (a->type == 8) {
        d.b = plane_op(Planes{}, M, K, 1, at ? 1 : 0);
        d.b.ld = K;
        d.b.q8 = static_cast<const int8_t*>(a->q8v);
        d.b.q8_scale = static_cast<const uint16_t*>(a->q8s);
      } else {
        Planes pa;
        if (planes_of(a, pa, st)) return -3;
        d.b = plane_op(pa, M, K, abatch, at ? 1 : 0, fold ? 1 : batch / abatch, 1);
      }
      return gemm_store(t, d, st);
    }
    case kOpOutProd: {   // r[z][n][m] = sum_k a[za][k][m] b[z][k][n]
      Planes pa, pb;
      if (planes_of(a, pa, st) || planes_of(b, pb, st)) return -3;
      const int M = a->ne[0], Kk = a->ne[1], Nn = b->ne[0];
      const int batch = b->ne[2] * b->ne[3], abatch = a->ne[2] * a->ne[3];
      GemmDesc d;
      d.M = Nn; d.N = M; d.K = Kk; d.batch = batch;
      d.a = plane_op(pb, Kk, Nn, batch, 1);
      d.b = plane_op(pa, Kk, M, abatch, 1, batch / abatch, 1);
      return gemm_store(t, d, st);
    }
    default:
      return -1;
  }
}

// Tensors reachable from the roots, sources first.
void topo(Tensor* t, std::unordered_set<Tensor*>& seen, std::vector<Tensor*>& out) {
  if (!t || seen.count(t)) return;
  seen.insert(t);
  for (Tensor* sc : t->src) topo(sc, seen, out);
  out.push_back(t);
}

int alloc_all(Session* s, const std::vector<Tensor*>& ns) {
  for (Tensor* t : ns)
    if (prim_alloc(s, t)) return -3;
  return 0;
}

int ensure_stream(Session* s) {
  if (cudaSetDevice(s->device) != cudaSuccess) return -3;
  if (!s->pstream && cudaStreamCreateWithFlags(&s->pstream, cudaStreamNonBlocking) != cudaSuccess) return -3;
  return 0;
}

// d(src) += contribution
void accumulate(Session* s, Tensor* src, Tensor* contrib) {
  if (!contrib) return;
  if (!src->grad) {
    src->grad = contrib;
  } else {
    Tensor* sum = node(s, kOpAdd, src->grad, src->grad, contrib);
    s->bwd.push_back(sum);
    src->grad = sum;
  }
}

// the gradient reduced to the shape of a broadcast operand
Tensor* reduce_to(Session* s, Tensor* g, Tensor* like) {
  if (same_shape(g, like)) return g;
  Tensor* r = node(s, kOpRepeatBack, like, g);
  s->bwd.push_back(r);
  return r;
}

}  // namespace

// ------------------------------------------------------------------ program control
int prim_build_forward(Session* s, Tensor* result) {
  if (ensure_stream(s)) return -3;
  std::unordered_set<Tensor*> seen;
  std::vector<Tensor*> order;
  for (Tensor* r : s->roots) topo(r, seen, order);
  topo(result, seen, order);
  s->nodes = order;
  return 0;
}

int prim_realize(Session* s, Tensor* result) {
  if (prim_build_forward(s, result)) return -3;
  if (alloc_all(s, s->nodes)) return -3;
  s->prim_realized = true;
  return 0;
}

int prim_compute(Session* s) {
  if (ensure_stream(s)) return -3;
  for (Tensor* t : s->nodes) {
    if (prim_alloc(s, t)) return -3;
    const int rc = exec(s, t);
    if (rc) return rc;
  }
  return cudaStreamSynchronize(s->pstream) == cudaSuccess ? 0 : -3;
}

// Reverse-mode autograd over the forward program: gradients of every node on a
// path from a parameter to the loss, as new backward nodes.
int prim_build_backward(Session* s) {
  if (!s->loss) return -2;
  if (s->nodes.empty() && prim_build_forward(s, s->loss)) return -3;
  // which nodes depend on a parameter
  std::unordered_set<Tensor*> needs;
  for (Tensor* t : s->nodes) {
    if (t->op == kOpNone) {
      if (t->is_param) needs.insert(t);
      continue;
    }
    for (Tensor* sc : t->src)
      if (sc && needs.count(sc)) {
        needs.insert(t);
        break;
      }
  }
  for (Tensor* t : s->nodes) t->grad = nullptr;
  s->bwd.clear();
  s->ones = prim_new(s, 0, 1, 1, 1, 1, kOpNone, true);
  if (!s->ones) return -3;
  s->loss->grad = s->ones;
  auto want = [&](Tensor* x) { return x && needs.count(x); };
  auto add = [&](Tensor* x) { if (x) s->bwd.push_back(x); return x; };
  for (auto it = s->nodes.rbegin(); it != s->nodes.rend(); ++it) {
    Tensor* t = *it;
    Tensor* g = t->grad;
    if (!g || t->op == kOpNone) continue;
    Tensor *a = t->src[0], *b = t->src[1];
    switch (t->op) {
      case kOpAdd:
        if (want(a)) accumulate(s, a, g);
        if (want(b)) accumulate(s, b, reduce_to(s, g, b));
        break;
      case kOpSub:
        if (want(a)) accumulate(s, a, g);
        if (want(b)) accumulate(s, b, reduce_to(s, add(prim_scale(s, g, -1.0)), b));
        break;
      case kOpMul:
        if (want(a)) accumulate(s, a, add(prim_binary(s, kOpMul, g, b)));
        if (want(b)) accumulate(s, b, reduce_to(s, add(prim_binary(s, kOpMul, g, a)), b));
        break;
      case kOpScale:
        if (want(a)) accumulate(s, a, add(prim_scale(s, g, t->fp[0])));
        break;
      case kOpSilu:
        if (want(a)) accumulate(s, a, add(prim_unary(s, kOpSiluBack, a, g)));
        break;
      case kOpSwiglu:   // silu(a) * b
        if (want(a)) accumulate(s, a, add(prim_unary(s, kOpSiluBack, a, add(prim_binary(s, kOpMul, g, b)))));
        if (want(b)) accumulate(s, b, add(prim_binary(s, kOpMul, g, add(prim_unary(s, kOpSilu, a, nullptr)))));
        break;
      case kOpMulMat:
        if (want(a) && a->type == 0) {
          const long long batch = (long long)b->ne[2] * b->ne[3], abatch = (long long)a->ne[2] * a->ne[3];
          Tensor* ga;
          if (abatch == 1 && batch > 1) {
            // one shared a: a single product over all of b's rows
            const int rows = (int)(b->ne[1] * batch);
            Tensor* b2 = add(prim_reshape(s, b, b->ne[0], rows, 1, 1));
            Tensor* g2 = add(prim_reshape(s, g, g->ne[0], rows, 1, 1));
            ga = b2 && g2 ? add(prim_out_prod(s, b2, g2)) : nullptr;   // [K, M]
          } else {
            ga = add(prim_out_prod(s, b, g));   // [K, M, B2, B3]
            if (ga && abatch != batch) {
              // b batch z reads a batch z / r: sum the r consecutive batches of each group
              const int r = (int)(batch / abatch);
              Tensor* g4 = add(prim_reshape(s, ga, a->ne[0], a->ne[1], r, (int)abatch));
              Tensor* like = prim_new(s, 0, a->ne[0], a->ne[1], 1, (int)abatch, kOpNone, false);
              Tensor* red = g4 && like ? add(node(s, kOpRepeatBack, like, g4)) : nullptr;
              ga = red ? add(prim_reshape(s, red, a->ne[0], a->ne[1], a->ne[2], a->ne[3])) : nullptr;
            }
          }
          accumulate(s, a, ga);
        }
        if (want(b)) accumulate(s, b, add(prim_mul_mat_at(s, a, g, b)));
        break;
      case kOpRmsNorm:
        if (want(a)) accumulate(s, a, add(prim_rms_norm_back(s, a, g, t->fp[0])));
        break;
      case kOpRope:
        if (want(a))
          accumulate(s, a, add(prim_rope(s, kOpRopeBack, g, b, t->ip[0], t->fp[0], t->fp[1], 0.0, t->fp[2],
                                         t->src[2])));
        break;
      case kOpSoftMax:
        if (want(a)) accumulate(s, a, add(prim_softmax_back(s, t, g, t->fp[0])));
        break;
      case kOpDiagMaskInf:
        if (want(a)) accumulate(s, a, add(prim_diag_mask(s, kOpDiagMaskZero, g, t->ip[0])));
        break;
      case kOpTranspose: {
        if (want(a)) {
          int inv[4];
          for (int d = 0; d < 4; ++d) inv[t->ip[d]] = d;
          accumulate(s, a, add(prim_permute(s, g, inv[0], inv[1], inv[2], inv[3])));
        }
        break;
      }
      case kOpCont:
        if (want(a)) accumulate(s, a, add(prim_reshape(s, g, a->ne[0], a->ne[1], a->ne[2], a->ne[3])));
        break;
      case kOpReshape:
        if (want(a)) {
          if (t->view_of && (t->view_off != (a->view_of ? a->view_off : 0) || t->nel() != a->nel())) {
            Tensor* acc = node(s, kOpAccView, a, g, t);
            accumulate(s, a, add(acc));
          } else {
            accumulate(s, a, add(prim_reshape(s, g, a->ne[0], a->ne[1], a->ne[2], a->ne[3])));
          }
        }
        break;
      case kOpView:
        if (want(a)) accumulate(s, a, add(node(s, kOpAccView, a, g, t)));
        break;
      case kOpConcat: {
        const int dim = t->ip[0];
        if (want(a)) accumulate(s, a, add(prim_slice(s, g, dim, 0, a->ne[dim])));
        if (want(b)) accumulate(s, b, add(prim_slice(s, g, dim, a->ne[dim], b->ne[dim])));
        break;
      }
      case kOpSlice:
        break;
      case kOpGetRows:
        if (want(a)) accumulate(s, a, add(prim_get_rows_back(s, g, b, a)));
        break;
      case kOpCrossEntropy:
        if (want(a)) {
          Tensor* gb = node(s, kOpCrossEntropyBack, a, g, a, b);
          accumulate(s, a, add(gb));
        }
        break;
      case kOpSum:
        if (want(a)) {
          Tensor* r = node(s, kOpRepeat, a, g);
          accumulate(s, a, add(r));
        }
        break;
      case kOpSumRows:
        if (want(a)) {
          Tensor* r = node(s, kOpRepeat, a, g);
          accumulate(s, a, add(r));
        }
        break;
      default:
        break;
    }
  }
  s->bwd_built = true;
  return 0;
}

int prim_realize_backward(Session* s) {
  if (ensure_stream(s)) return -3;
  if (alloc_all(s, s->nodes) || alloc_all(s, s->bwd)) return -3;
  std::unordered_set<Tensor*> seen(s->nodes.begin(), s->nodes.end());
  for (Tensor* t : s->bwd) seen.insert(t);
  for (Tensor* e : s->ext) {
    std::vector<Tensor*> extra;
    topo(e, seen, extra);
    for (Tensor* x : extra)
      if (prim_alloc(s, x)) return -3;
    s->bwd.insert(s->bwd.end(), extra.begin(), extra.end());
  }
  s->ext.clear();
  if (s->ones) {
    const float one = 1.0f;
    if (cudaMemcpy(s->ones->data, &one, 4, cudaMemcpyHostToDevice) != cudaSuccess) return -3;
  }
  s->prim_realized = true;
  return 0;
}

int prim_compute_backward(Session* s) {
  if (ensure_stream(s)) return -3;
  if (!s->prim_realized && prim_realize_backward(s)) return -3;
  if (s->reset_pending) {   // tnn_graph_reset: zero the optimizer moments
    for (Tensor* t : s->bwd)
      if (t->op == kOpOptAdamw) {
        cudaMemsetAsync(t->src[2]->data, 0, t->src[2]->bytes, s->pstream);
        cudaMemsetAsync(t->src[3]->data, 0, t->src[3]->bytes, s->pstream);
      }
    s->reset_pending = false;
  }
  for (Tensor* t : s->nodes) {
    const int rc = exec(s, t);
    if (rc) return rc;
  }
  for (Tensor* t : s->bwd) {
    const int rc = exec(s, t);
    if (rc) return rc;
  }
  return cudaStreamSynchronize(s->pstream) == cudaSuccess ? 0 : -3;
}

}  // namespace tb2
