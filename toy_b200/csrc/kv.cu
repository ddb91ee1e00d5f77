// The decode (inference forward) path with a KV cache: what toy's KV engine
// runs for `toy infer` / `serve` (lib/toy/llm/engine/llama_kv_engine.rb:
// build_block_step :1687, build_attention_qhead_step :2132, decode_step :2350,
// decode_batch :2381; enable_kv_q8! :359 stores K and V as Q8_0; the fused
// attention is tnn_flash_attn_ext, tinynn/tinynn_ggml.c:1583-1598).
//
// B200 design. A decode step moves every weight once per step for n_seq
// tokens, so it is HBM-bound: the projections are GEMVs over the frozen Q8_0
// base read as int8 quants + fp16 scales (1.06 bytes per weight, dequantised
// in registers, never widened in memory), the tied LM head reads the f32
// embedding, and the n_seq sequences that decode in lockstep share each
// weight read. Per block: the q|k|v GEMV with the RMSNorm folded in
// (y = r * sum_k W x gamma, r = rsqrt(mean x^2 + eps) computed by each CTA),
// an append kernel (bias, NEOX RoPE from the training engine's table, K / V
// written into the cache -- quantised to Q8_0 with ggml's quantiser when the
// cache is Q8_0), a split-history flash-decode attention (per query head and
// 128-key chunk, one key per thread; GQA by reading KV head h / G), the o GEMV
// that assembles the chunks' partial softmax sums while it stages its input and
// adds the residual, the gate|up
// GEMV (RMSNorm folded, SwiGLU on the paired rows) and the down GEMV with the
// residual add; then the final norm folded into the LM-head GEMV. The whole
// step is one CUDA graph; tokens and positions are copied in before it.
//
// The weights are the realised training engine's (same session): decoding
// after training, or after tb2_llama_load_gguf, uses them in place. Adapters
// are not applied on this path.
#include <cuda_fp16.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <memory>
#include <vector>

#include "pdl.cuh"
#include "runtime.cuh"
#include "session.cuh"
#include "toy_b200.h"

namespace tb2 {

namespace {

constexpr int kGemvWarps = 8;
constexpr int kChunk = 128;   // keys per attention CTA (one per thread)
constexpr int kMaxSeq = 16;

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

// ---------------------------------------------------------------- GEMV
// out(b, n) for the n_seq rows of x: y = r_b * sum_k W[n][k] x[b][k] g[k]
// (r_b = 1 and g = 1 without a norm). mode 0 store (+ bias), 1 residual
// (out = res + y), 2 SwiGLU over paired rows (n and n + pair: out = silu(y_n) y_{n+pair}).

// A LoRA adapter on the output rows [c0, c0 + width) of a GEMV (in pair mode:
// of the gate rows, on = 0, or of the up rows, on = 1): y(b, n) +=
// s * sum_j B[n - c0][j] u[b][o(n) + j], with u = A x computed by an earlier
// GEMV and o(n) = ((n - c0) / bd_w) r for toy's per-head LoRA-Q (one adapter
// pair per block of bd_w rows), 0 for a plain adapter.
struct GemvLora {
  const float* B = nullptr;        // [width][r]
  const float* u = nullptr;        // [n_seq][ldu]
  long long ldu = 0;
  int c0 = 0, width = 0, r = 0, bd_w = 0, on = 0;
  float s = 1.f;
};
constexpr int kGemvLoras = 3;

struct GemvArgs {
  const float* w32 = nullptr;      // f32 weights [rows][K], or
  const int8_t* wq = nullptr;      // Q8_0 quants [rows][K] and
  const uint16_t* ws = nullptr;    //   fp16 scale bits [rows][K / 32]
  int rows = 0, K = 0;
  const float* x = nullptr;        // [n_seq][ldx]
  long long ldx = 0;
  const float* gamma = nullptr;    // RMSNorm folded in when set
  float eps = 0.f;
  const float* bias = nullptr;
  float* out = nullptr;            // [n_seq][ldo]
  long long ldo = 0;
  const float* res = nullptr;      // [n_seq][ldo]
  int mode = 0, pair = 0;
  // x is the attention output to assemble from the chunks' partials
  // [n_seq][H][nsplit][dh + 2] (o, m, l): x[b][h dh + d] = sum_s o_s e^(m_s - m) / sum_s l_s e^(m_s - m)
  const float* part = nullptr;
  int nsplit = 0, dh = 0;
  // low-rank adapters added to the product before the mode's epilogue
  GemvLora lora[kGemvLoras];
  int n_lora = 0;
};

// One output row (or gate / up pair) of weights held in registers: lane l
// holds 16-value chunks l, l + 32, ... (Q8_0: int8 quants and the block
// scale) or 4-value chunks (f32). Rows up to kRegK columns are read this way,
// the next row's loads issued before the current row's arithmetic; the first
// row's before the grid wait, beside the previous kernel.
constexpr int kQ8Chunks = 3;   // Q8_0 rows of K <= 1536
constexpr int kF32Chunks = 5;  // f32 rows of K <= 640

template <bool Q8>
struct RowRegs {
  static constexpr int kC = Q8 ? kQ8Chunks : kF32Chunks;
  static constexpr int kRows = Q8 ? 2 : 1;   // f32 rows: single rows only (not the gate / up pairs)
  int4 v[kRows][kC];
  float d[kRows][kC];
};

template <bool Q8>
__device__ __forceinline__ bool row_fits(int K, int mode) {
  return Q8 ? K <= kQ8Chunks * 32 * 16 : (K <= kF32Chunks * 32 * 4 && mode != 2);
}

template <bool Q8>
__device__ __forceinline__ void row_load(const GemvArgs& a, int n, int nrow, int lane, RowRegs<Q8>& r) {
  constexpr int kC = RowRegs<Q8>::kC;
  const int nch = Q8 ? a.K / 16 : a.K / 4;
#pragma unroll
  for (int h = 0; h < RowRegs<Q8>::kRows; ++h) {
#pragma unroll
    for (int i = 0; i < kC; ++i) {
      const int c = lane + 32 * i;
      r.v[h][i] = make_int4(0, 0, 0, 0);
      r.d[h][i] = 0.f;
      if (h >= nrow || c >= nch) continue;
      const long long row = n + (long long)h * a.pair;
      if (Q8) {
        r.v[h][i] = __ldg(reinterpret_cast<const int4*>(a.wq + row * a.K) + c);
        r.d[h][i] = __half2float(__ushort_as_half(__ldg(a.ws + row * (a.K / 32) + c / 2)));
      } else {
        r.v[h][i] = __ldg(reinterpret_cast<const int4*>(a.w32 + row * a.K) + c);
      }
    }
  }
}

template <int NB, bool Q8>
__device__ __forceinline__ void row_dot(const GemvArgs& a, const float* xs, int lane, const RowRegs<Q8>& r,
                                        float (&acc)[2][NB]) {
  constexpr int kC = RowRegs<Q8>::kC;
  const int nch = Q8 ? a.K / 16 : a.K / 4;
#pragma unroll
  for (int h = 0; h < RowRegs<Q8>::kRows; ++h) {
#pragma unroll
    for (int i = 0; i < kC; ++i) {
      const int c = lane + 32 * i;
      if (c >= nch) continue;
      if (Q8) {
        const int8_t* qb = reinterpret_cast<const int8_t*>(&r.v[h][i]);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float wv = r.d[h][i] * (float)qb[j];
#pragma unroll
          for (int b = 0; b < NB; ++b) acc[h][b] = fmaf(wv, xs[b * a.K + c * 16 + j], acc[h][b]);
        }
      } else {
        const int4 wi = r.v[h][i];
        const float4 wv = make_float4(__int_as_float(wi.x), __int_as_float(wi.y), __int_as_float(wi.z),
                                      __int_as_float(wi.w));
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float* xb = xs + b * a.K + c * 4;
          acc[h][b] = fmaf(wv.x, xb[0], fmaf(wv.y, xb[1], fmaf(wv.z, xb[2], fmaf(wv.w, xb[3], acc[h][b]))));
        }
      }
    }
  }
}

template <int NB, bool Q8>
__global__ void __launch_bounds__(256) kv_gemv_kernel(const GemvArgs a) {
  // xs [NB][K]: the input rows (times gamma when a norm is folded in); with
  // the attention partials, fs [NB][H][nsplit] holds each chunk's factor
  // e^(m_s - m) / L; then gs [K]: gamma
  extern __shared__ float xs[];
  __shared__ float rs[NB];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_out = a.mode == 2 ? a.pair : a.rows;
  const int nrow = a.mode == 2 ? 2 : 1;
  const int H = a.part ? a.K / a.dh : 0;
  float* fs = xs + NB * a.K;
  float* gs = fs + NB * H * a.nsplit;
  // prologue on weights only (nothing the previous kernels write): gamma into
  // shared memory, this warp's first row into registers
  if (a.gamma)
    for (int k = threadIdx.x; k < a.K; k += blockDim.x) gs[k] = __ldg(a.gamma + k);
  // (wider batches keep the streaming loop: their per-row arithmetic hides the
  // loads, and the row registers would cost occupancy)
  const bool regs = NB <= 4 && row_fits<Q8>(a.K, a.mode);
  const int n_first = blockIdx.x * kGemvWarps + warp, n_step = gridDim.x * kGemvWarps;
  RowRegs<Q8> cur;
  if (NB <= 4 && regs && n_first < n_out) row_load<Q8>(a, n_first, nrow, lane, cur);
  griddep_wait_release();
  if (a.part) {
    const int ns = a.nsplit, stride = a.dh + 2;
    for (int j = threadIdx.x; j < NB * H; j += blockDim.x) {
      const float* p = a.part + (long long)j * ns * stride;
      float m = -INFINITY;
      for (int sp = 0; sp < ns; ++sp) m = fmaxf(m, p[sp * stride + a.dh]);
      float l = 0.f;
      for (int sp = 0; sp < ns; ++sp) {
        const float ms = p[sp * stride + a.dh];
        const float f = ms == -INFINITY ? 0.f : expf(ms - m);
        fs[j * ns + sp] = f;
        l += p[sp * stride + a.dh + 1] * f;
      }
      for (int sp = 0; sp < ns; ++sp) fs[j * ns + sp] /= l;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NB * a.K; i += blockDim.x) {
      const int b = i / a.K, k = i % a.K, hh = k / a.dh, dd = k % a.dh;
      const float* p = a.part + ((long long)b * H + hh) * ns * stride + dd;
      const float* f = fs + (b * H + hh) * ns;
      float o = 0.f;
#pragma unroll 4
      for (int sp = 0; sp < ns; ++sp) o += p[sp * stride] * f[sp];
      xs[i] = o;
    }
  } else {
#pragma unroll 4
    for (int i = threadIdx.x; i < NB * a.K; i += blockDim.x) {
      const int b = i / a.K, k = i % a.K;
      xs[i] = a.x[(long long)b * a.ldx + k];
    }
  }
  if (!a.gamma && threadIdx.x < NB) rs[threadIdx.x] = 1.0f;
  __syncthreads();
  if (a.gamma) {   // per-sequence rsqrt(mean x^2 + eps) from shared memory, then x * gamma in place
    for (int b = warp; b < NB; b += kGemvWarps) {
      float s = 0.f;
      for (int k = lane; k < a.K; k += 32) {
        const float v = xs[b * a.K + k];
        s += v * v;
      }
      s = warp_sum(s);
      if (lane == 0) rs[b] = rsqrtf(s / (float)a.K + a.eps);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NB * a.K; i += blockDim.x) xs[i] *= gs[i % a.K];
    __syncthreads();
  }
  for (int n = n_first; n < n_out; n += n_step) {
    float acc[2][NB];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[h][b] = 0.f;
    if (NB <= 4 && regs) {
      RowRegs<Q8> nxt;
      const bool more = n + n_step < n_out;
      if (more) row_load<Q8>(a, n + n_step, nrow, lane, nxt);   // in flight during this row's arithmetic
      row_dot<NB, Q8>(a, xs, lane, cur, acc);
      if (more) cur = nxt;
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {   // (unrolled: acc is indexed by constants)
        if (h >= nrow) break;
        const long long row = n + (long long)h * a.pair;
        if (Q8) {
          const int8_t* q = a.wq + row * a.K;
          const uint16_t* sc = a.ws + row * (a.K / 32);
#pragma unroll 3
          for (int c = lane; c < a.K / 16; c += 32) {
            const int4 raw = __ldg(reinterpret_cast<const int4*>(q + c * 16));
            const float d = __half2float(__ushort_as_half(__ldg(sc + c / 2)));
            const int8_t* qb = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float wv = d * (float)qb[j];
#pragma unroll
              for (int b = 0; b < NB; ++b) acc[h][b] = fmaf(wv, xs[b * a.K + c * 16 + j], acc[h][b]);
            }
          }
        } else {
          const float* wr = a.w32 + row * a.K;
#pragma unroll 5
          for (int c = lane; c < a.K / 4; c += 32) {
            const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + c * 4));
#pragma unroll
            for (int b = 0; b < NB; ++b) {
              const float* xb = xs + b * a.K + c * 4;
              acc[h][b] = fmaf(wv.x, xb[0], fmaf(wv.y, xb[1], fmaf(wv.z, xb[2], fmaf(wv.w, xb[3], acc[h][b]))));
            }
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float y0 = warp_sum(acc[0][b]) * rs[b];
      float y1 = a.mode == 2 ? warp_sum(acc[1][b]) * rs[b] : 0.f;
#pragma unroll
      for (int i = 0; i < kGemvLoras; ++i) {   // adapters, before the bias / residual / SwiGLU
        if (i >= a.n_lora) break;
        const GemvLora& L = a.lora[i];
        if (n < L.c0 || n >= L.c0 + L.width) continue;
        const int rr = n - L.c0;
        const float* ur = L.u + b * L.ldu + (L.bd_w ? (rr / L.bd_w) * L.r : 0);
        const float* br = L.B + (long long)rr * L.r;
        float t = 0.f;
        for (int j = lane; j < L.r; j += 32) t = fmaf(br[j], ur[j], t);
        t = warp_sum(t) * L.s;
        if (L.on) y1 += t;
        else y0 += t;
      }
      if (lane == 0) {
        float* o = a.out + (long long)b * a.ldo + n;
        if (a.mode == 0) *o = y0 + (a.bias ? a.bias[n] : 0.f);
        else if (a.mode == 1) *o = a.res[(long long)b * a.ldo + n] + y0;
        else *o = y0 / (1.0f + expf(-y0)) * y1;
      }
    }
  }
}

// ---------------------------------------------------------------- embedding
__global__ void kv_embed_kernel(const float* __restrict__ E, const int* __restrict__ tok, int d, float* __restrict__ x) {
  griddep_wait_release();
  const int b = blockIdx.x;
  const float* src = E + (long long)tok[b] * d;
  for (int k = threadIdx.x; k < d; k += blockDim.x) x[(long long)b * d + k] = src[k];
}

// ---------------------------------------------------------------- append: bias, RoPE, K / V into the cache
struct KvCache {
  float* k32 = nullptr;            // f32 cache [n_seq][KV][max_T][dh], or
  float* v32 = nullptr;
  int8_t* kq = nullptr;            // Q8_0: quants [n_seq][KV][max_T][dh]
  int8_t* vq = nullptr;
  uint16_t* ks = nullptr;          //       fp16 scale bits [n_seq][KV][max_T][dh / 32]
  uint16_t* vs = nullptr;
};

struct AppendArgs {
  float* qkv = nullptr;            // [n_seq][W], W = (H + 2 KV) dh
  const float* bias = nullptr;
  const int* pos = nullptr;
  const float2* cs = nullptr;      // [rows][dh / 2] (cos, sin)
  int tab_rows = 0;
  int H = 0, KV = 0, dh = 0, max_T = 0;
  KvCache c;
};

// ggml's Q8_0 rounding: round half away from zero
__device__ __forceinline__ int round_away(float v) {
  const float t = truncf(v);
  const int ti = (int)t;
  return fabsf(__fsub_rn(v, t)) >= 0.5f ? (v < 0.f ? ti - 1 : ti + 1) : ti;
}

// grid (n_seq, H + KV), block dh threads: q heads are rotated in place; KV
// head j rotates k and writes k and v at the sequence's position.
__global__ void kv_append_kernel(const AppendArgs a) {
  extern __shared__ float sh[];   // [2][dh]
  griddep_wait_release();
  const int b = blockIdx.x, hh = blockIdx.y, t = threadIdx.x, dh = a.dh, half = dh / 2;
  const int W = (a.H + 2 * a.KV) * dh;
  float* row = a.qkv + (long long)b * W;
  const int p = a.pos[b];
  const int c0 = hh < a.H ? hh * dh : (a.H + (hh - a.H)) * dh;   // q head or k head
  float x = row[c0 + t] + (a.bias ? a.bias[c0 + t] : 0.f);
  sh[t] = x;
  float v = 0.f;
  if (hh >= a.H) {
    const int cv = (a.H + a.KV + (hh - a.H)) * dh;
    v = row[cv + t] + (a.bias ? a.bias[cv + t] : 0.f);
  }
  __syncthreads();
  const int i = t < half ? t : t - half;
  const float2 cs = a.cs[(long long)p * half + i];
  const float r = t < half ? sh[t] * cs.x - sh[t + half] * cs.y : sh[t - half] * cs.y + sh[t] * cs.x;
  if (hh < a.H) {
    row[c0 + t] = r;
    return;
  }
  const int j = hh - a.H;
  const long long slot = ((long long)b * a.KV + j) * a.max_T + p;
  if (a.c.k32) {
    a.c.k32[slot * dh + t] = r;
    a.c.v32[slot * dh + t] = v;
    return;
  }
  // Q8_0 (ggml quantize_row_q8_0_ref): one warp per 32-value block of the head
  const int lane = t & 31, blk = t >> 5;
  for (int which = 0; which < 2; ++which) {
    const float val = which ? v : r;
    const float amax = warp_max(fabsf(val));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const int q = round_away(__fmul_rn(val, id));
    int8_t* qd = which ? a.c.vq : a.c.kq;
    uint16_t* sd = which ? a.c.vs : a.c.ks;
    qd[slot * dh + t] = (int8_t)q;
    if (lane == 0) sd[slot * (dh / 32) + blk] = __half_as_ushort(__float2half_rn(d));
  }
}

// ---------------------------------------------------------------- flash-decode attention
struct AttnArgs {
  const float* qkv = nullptr;
  const int* pos = nullptr;
  KvCache c;
  int H = 0, KV = 0, dh = 0, max_T = 0, nsplit = 0;
  float scale = 1.f;
  float* part = nullptr;           // [n_seq][H][nsplit][dh + 2]: o (unnormalised), m, l
};

__device__ __forceinline__ float cache_val(const KvCache& c, bool v, long long slot, int dh, int d) {
  if (c.k32) return (v ? c.v32 : c.k32)[slot * dh + d];
  const int8_t* q = v ? c.vq : c.kq;
  const uint16_t* s = v ? c.vs : c.ks;
  return __half2float(__ushort_as_half(s[slot * (dh / 32) + d / 32])) * (float)q[slot * dh + d];
}

// grid (n_seq * H, nsplit), block 128: keys [split * kChunk, ...) of the
// history. Scores: one key per thread (its K row read as 16-byte vectors, q
// from shared memory); the chunk's max and sum by block reductions; P V: each
// thread owns one head dimension for a slice of the keys, reading V rows
// coalesced across threads, P from shared memory. Writes the chunk's
// unnormalised o, its max m and its sum l.
__global__ void __launch_bounds__(kChunk) kv_attn_kernel(const AttnArgs a) {
  // the chunk's V rows as stored: f32 [kChunk][dh], or Q8_0 quants
  // [kChunk][dh] followed by their fp16 scales [kChunk][dh / 32]
  extern __shared__ __align__(16) uint8_t vsm[];
  __shared__ float qs[128];
  __shared__ float ps[kChunk];
  __shared__ float red[kChunk / 32];
  __shared__ float osum[kChunk];
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, j = h / (a.H / a.KV), split = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, dh = a.dh;
  // positions are copied in before the step's first kernel, so the chunk's
  // extent is known before the grid wait: its K and V rows are pulled toward
  // the L2 while the previous kernel (the append of the new row) runs
  const int hist = a.pos[b] + 1;
  const int t0 = split * kChunk, t1 = min(t0 + kChunk, hist);
  const long long base = ((long long)b * a.KV + j) * a.max_T;
  const bool f32c = a.c.k32 != nullptr;
  const int row_bytes = f32c ? dh * 4 : dh;
  if (t0 + tid < t1) {
    const long long slot = base + t0 + tid;
    const uint8_t* kr = f32c ? reinterpret_cast<const uint8_t*>(a.c.k32 + slot * dh)
                             : reinterpret_cast<const uint8_t*>(a.c.kq + slot * dh);
    const uint8_t* vr = f32c ? reinterpret_cast<const uint8_t*>(a.c.v32 + slot * dh)
                             : reinterpret_cast<const uint8_t*>(a.c.vq + slot * dh);
    for (int o = 0; o < row_bytes; o += 128) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kr + o));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(vr + o));
    }
  }
  griddep_wait_release();
  float* out = a.part + ((long long)bh * a.nsplit + split) * (dh + 2);
  if (t0 >= t1) {   // this chunk is past the history
    for (int d = tid; d < dh; d += blockDim.x) out[d] = 0.f;
    if (tid == 0) {
      out[dh] = -INFINITY;
      out[dh + 1] = 0.f;
    }
    return;
  }
  // V rows of the chunk into shared memory by 16-byte async copies (rows are
  // contiguous in the cache), in flight while the scores are computed
  {
    const uint8_t* src = f32c ? reinterpret_cast<const uint8_t*>(a.c.v32 + (base + t0) * dh)
                              : reinterpret_cast<const uint8_t*>(a.c.vq + (base + t0) * dh);
    const int n16 = (t1 - t0) * row_bytes / 16;
    for (int i = tid; i < n16; i += blockDim.x)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(vsm + 16 * i)),
                   "l"(src + 16 * i)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (!f32c) {   // the rows' scales after the quants
      uint16_t* vsc = reinterpret_cast<uint16_t*>(vsm + kChunk * dh);
      const int ns = (t1 - t0) * (dh / 32);
      for (int i = tid; i < ns; i += blockDim.x) vsc[i] = a.c.vs[(base + t0) * (dh / 32) + i];
    }
  }
  const float* q = a.qkv + (long long)b * (a.H + 2 * a.KV) * dh + h * dh;
  for (int d = tid; d < dh; d += blockDim.x) qs[d] = q[d];
  __syncthreads();
  const int t = t0 + tid;
  float s = -INFINITY;
  if (t < t1) {
    float acc = 0.f;
    const long long slot = base + t;
    if (a.c.k32) {
      const float4* kr = reinterpret_cast<const float4*>(a.c.k32 + slot * dh);
#pragma unroll 8
      for (int c = 0; c < dh / 4; ++c) {
        const float4 kv = __ldg(kr + c);
        acc += kv.x * qs[4 * c] + kv.y * qs[4 * c + 1] + kv.z * qs[4 * c + 2] + kv.w * qs[4 * c + 3];
      }
    } else {
      const int4* kr = reinterpret_cast<const int4*>(a.c.kq + slot * dh);
      const uint16_t* ks = a.c.ks + slot * (dh / 32);
#pragma unroll 4
      for (int c = 0; c < dh / 16; ++c) {
        const int4 raw = __ldg(kr + c);
        const int8_t* qb = reinterpret_cast<const int8_t*>(&raw);
        const float sc = __half2float(__ushort_as_half(__ldg(ks + c / 2)));
        float part = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) part += (float)qb[e] * qs[16 * c + e];
        acc += sc * part;
      }
    }
    s = acc * a.scale;
  }
  float m = warp_max(s);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  const float p = t < t1 ? expf(s - m) : 0.f;
  ps[tid] = p;
  __syncthreads();   // red is read above before it is reused below
  float l = warp_sum(p);
  if (lane == 0) red[warp] = l;
  __syncthreads();
  l = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) l += red[w];
  // P V: thread (g, d) sums keys g, g + G, ... of the chunk for dimension d (G = blockDim / dh groups)
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const int groups = blockDim.x / dh, g = tid / dh, d = tid % dh;
  float o = 0.f;
  if (g < groups) {
    const int n = t1 - t0;
    if (f32c) {
      const float* vs32 = reinterpret_cast<const float*>(vsm);
#pragma unroll 8
      for (int k = g; k < n; k += groups) o += ps[k] * vs32[k * dh + d];
    } else {
      const int8_t* vq = reinterpret_cast<const int8_t*>(vsm);
      const uint16_t* vsc = reinterpret_cast<const uint16_t*>(vsm + kChunk * dh);
#pragma unroll 8
      for (int k = g; k < n; k += groups)
        o += ps[k] * (__half2float(__ushort_as_half(vsc[k * (dh / 32) + d / 32])) * (float)vq[k * dh + d]);
    }
  }
  osum[tid] = o;
  __syncthreads();
  if (tid < dh) {
    float acc = 0.f;
    for (int gg = 0; gg < groups; ++gg) acc += osum[gg * dh + tid];
    out[tid] = acc;
  }
  if (tid == 0) {
    out[dh] = m;
    out[dh + 1] = l;
  }
}

}  // namespace

// ---------------------------------------------------------------- the decode engine
// adapter parameter names by target, in the training engine's order (q, k, v, o, gate, up, down)
const char* const kAdName[7] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};

class KvEngine {
 public:
  KvEngine(LlamaEngine& e, int max_T, int n_seq, int kv_type) : e_(e), max_T_(max_T), nb_(n_seq), q8_(kv_type == 8) {}
  ~KvEngine() {
    cudaSetDevice(e_.device());
    if (graph_) cudaGraphExecDestroy(graph_);
    for (void* p : bufs_) cudaFree(p);
    if (host_in_) cudaFreeHost(host_in_);
    if (st_) cudaStreamDestroy(st_);
  }

  int realize() {
    const LlamaConfig& c = e_.cfg();
    if (max_T_ < 1 || max_T_ > e_.rope_rows() || nb_ < 1 || (nb_ > 8 && nb_ != kMaxSeq)) return -1;
    if (c.d_head % 32 || c.d_head > 128 || c.d_model % 16 || c.d_ff % 16) return -1;
    if (c.qk_norm || c.n_experts) return -1;   // QK-RMSNorm and expert blocks: training-step only
    const long long nsplit = (max_T_ + kChunk - 1) / kChunk;
    const long long max_k = std::max(c.d_ff, std::max(c.d_model, c.n_heads * c.d_head));
    if (((long long)nb_ * max_k + (long long)nb_ * c.n_heads * nsplit + max_k) * 4 > 200 * 1024)
      return -1;
    if (cudaSetDevice(e_.device()) != cudaSuccess) return -3;
    if (cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking) != cudaSuccess) return -3;
    const int d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff, V = c.vocab, L = c.n_layers;
    const int W = (H + 2 * KV) * dh;
    nsplit_ = (max_T_ + kChunk - 1) / kChunk;
    attn_smem_ = q8_ ? (size_t)kChunk * dh + (size_t)kChunk * (dh / 32) * 2 : (size_t)kChunk * dh * 4;
    static DeviceOnce attn_setup;   // the largest chunk any engine stages: f32 rows of d_head 128
    if (attn_setup.ensure([](int) {
          return cudaFuncSetAttribute(kv_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kChunk * 128 * 4) ==
                         cudaSuccess
                     ? 0
                     : -3;
        }))
      return -3;
    auto f32 = [&](long long n) -> float* {
      void* p = nullptr;
      if (cudaMalloc(&p, (size_t)std::max<long long>(n, 1) * 4) != cudaSuccess) return nullptr;
      cudaMemset(p, 0, (size_t)std::max<long long>(n, 1) * 4);
      bufs_.push_back(p);
      return static_cast<float*>(p);
    };
    x_ = f32((long long)nb_ * d);
    x1_ = f32((long long)nb_ * d);
    qkv_ = f32((long long)nb_ * W);
    a_ = f32((long long)nb_ * ff);
    part_ = f32((long long)nb_ * H * nsplit_ * (dh + 2));
    logits_ = f32((long long)nb_ * V);
    int* io = reinterpret_cast<int*>(f32(2 * kMaxSeq));
    tok_ = io;
    pos_ = io + kMaxSeq;
    const long long cache = (long long)L * nb_ * KV * max_T_ * dh;
    if (q8_) {
      void* p = nullptr;
      for (int w = 0; w < 2; ++w) {
        if (cudaMalloc(&p, (size_t)cache) != cudaSuccess) return -3;
        bufs_.push_back(p);
        (w ? vq_ : kq_) = static_cast<int8_t*>(p);
        if (cudaMalloc(&p, (size_t)cache / 32 * 2) != cudaSuccess) return -3;
        bufs_.push_back(p);
        (w ? vs_ : ks_) = static_cast<uint16_t*>(p);
      }
    } else {
      k32_ = f32(cache);
      v32_ = f32(cache);
    }
    // the recipe's adapters, applied as the training step applies them
    if (c.mode == 1 && c.lora_rank > 0) {
      const float s = c.lora_per_head_q ? 1.0f : c.lora_alpha / (float)c.lora_rank;
      for (int t = 0; t < kAdapters; ++t) {
        if (!(c.lora_targets & (1 << t))) continue;
        const LlamaEngine::WeightView A = e_.weight(std::string("blk.0.") + kAdName[t] + ".lora_a");
        if (!A.f32) return -1;
        Adapter& ad = ad_[t];
        ad.on = true;
        ad.rows = A.rows;
        ad.u = f32((long long)nb_ * A.rows);
        ad.s = s;
        ad.bd_w = c.lora_per_head_q && t == 0 ? dh : 0;
      }
    }
    for (void* p : bufs_)
      if (!p) return -3;
    if (cudaMallocHost(&host_in_, 2 * kMaxSeq * sizeof(int)) != cudaSuccess) return -3;
    // every weight view must exist (the training engine was realised with this model)
    for (int l = 0; l < L; ++l) {
      const std::string pre = "blk." + std::to_string(l) + ".";
      for (const char* n : {"attn_norm.weight", "attn_q.weight", "attn_output.weight", "ffn_norm.weight",
                            "ffn_gate.weight", "ffn_down.weight"})
        if (!e_.find(pre + n)) return -1;
    }
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -3;
  }

  int reset() {
    cudaSetDevice(e_.device());
    const LlamaConfig& c = e_.cfg();
    const long long cache = (long long)c.n_layers * nb_ * c.n_kv * max_T_ * c.d_head;
    if (q8_) {
      if (cudaMemsetAsync(kq_, 0, cache, st_) || cudaMemsetAsync(vq_, 0, cache, st_)) return -3;
      if (cudaMemsetAsync(ks_, 0, cache / 32 * 2, st_) || cudaMemsetAsync(vs_, 0, cache / 32 * 2, st_)) return -3;
    } else if (cudaMemsetAsync(k32_, 0, cache * 4, st_) || cudaMemsetAsync(v32_, 0, cache * 4, st_)) {
      return -3;
    }
    return cudaStreamSynchronize(st_) == cudaSuccess ? 0 : -3;
  }

  int decode(const long long* tokens, const long long* positions, int n, float* logits_host) {
    const LlamaConfig& c = e_.cfg();
    if (!tokens || !positions || n != nb_) return -1;
    if (cudaSetDevice(e_.device()) != cudaSuccess) return -3;
    if (cudaStreamSynchronize(st_) != cudaSuccess) return -3;
    if (e_.sync()) return -3;   // weights written by training steps are final
    for (int b = 0; b < nb_; ++b) {
      if (tokens[b] < 0 || tokens[b] >= c.vocab || positions[b] < 0 || positions[b] >= max_T_) return -1;
      host_in_[b] = (int)tokens[b];
      host_in_[kMaxSeq + b] = (int)positions[b];
    }
    if (cudaMemcpyAsync(tok_, host_in_, 2 * kMaxSeq * sizeof(int), cudaMemcpyHostToDevice, st_) != cudaSuccess)
      return -3;
    if (!graph_) {   // first step: eager (validates every launch), then captured for replay
      if (int rc = enqueue()) return rc;
      cudaGraph_t g = nullptr;
      if (cudaStreamBeginCapture(st_, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -3;
      const int rc = enqueue();
      if (cudaStreamEndCapture(st_, &g) != cudaSuccess || rc) {
        if (g) cudaGraphDestroy(g);
        return rc ? rc : -3;
      }
      const cudaError_t ce = cudaGraphInstantiate(&graph_, g, 0);
      cudaGraphDestroy(g);
      if (ce != cudaSuccess) return -3;
    } else if (cudaGraphLaunch(graph_, st_) != cudaSuccess) {
      return -3;
    }
    if (logits_host) {
      if (cudaMemcpyAsync(logits_host, logits_, (size_t)nb_ * c.vocab * 4, cudaMemcpyDeviceToHost, st_) != cudaSuccess)
        return -3;
    }
    return cudaStreamSynchronize(st_) == cudaSuccess ? 0 : -3;
  }

  int run(int steps, float* ms) {   // n graph replays at the positions last copied in, timed by events
    if (!graph_ || steps < 1 || !ms) return -2;
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) || cudaEventCreate(&b)) return -3;
    cudaEventRecord(a, st_);
    for (int i = 0; i < steps; ++i)
      if (cudaGraphLaunch(graph_, st_) != cudaSuccess) return -3;
    cudaEventRecord(b, st_);
    cudaEventSynchronize(b);
    cudaEventElapsedTime(ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return 0;
  }

  int logits(float* out, long long n) {
    const LlamaConfig& c = e_.cfg();
    if (!out || n != (long long)nb_ * c.vocab) return -1;
    if (cudaStreamSynchronize(st_) != cudaSuccess) return -3;
    return cudaMemcpy(out, logits_, n * 4, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -3;
  }

  int launches() const { return launches_; }

 private:
  template <int NB>
  int gemv_nb(const GemvArgs& g) {
    const bool q8 = g.wq != nullptr;
    const size_t smem =
        ((size_t)NB * g.K + (g.part ? (size_t)NB * (g.K / g.dh) * g.nsplit : 0) + (g.gamma ? g.K : 0)) * 4;
    auto* k = q8 ? kv_gemv_kernel<NB, true> : kv_gemv_kernel<NB, false>;
    static DeviceOnce setup[2];
    if (setup[q8].ensure([&](int) {
          return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) == cudaSuccess ? 0
                                                                                                               : -3;
        }))
      return -3;
    const int n_out = g.mode == 2 ? g.pair : g.rows;
    const int blocks = std::min(4 * 148, (n_out + kGemvWarps - 1) / kGemvWarps);
    return launch_pdl(k, dim3(blocks), dim3(32 * kGemvWarps), smem, st_, g);
  }

  int gemv(GemvArgs g) {
    if ((g.wq && g.K % 32) || (!g.wq && g.K % 4)) return -1;
    ++launches_;
    switch (nb_) {
      case 1: return gemv_nb<1>(g);
      case 2: return gemv_nb<2>(g);
      case 3: return gemv_nb<3>(g);
      case 4: return gemv_nb<4>(g);
      case 5: return gemv_nb<5>(g);
      case 6: return gemv_nb<6>(g);
      case 7: return gemv_nb<7>(g);
      case 8: return gemv_nb<8>(g);
      case 16: return gemv_nb<16>(g);
      default: return -1;
    }
  }

  // u = A x of adapter t of block l into its buffer; `in` carries the input of
  // the GEMV the adapter belongs to (rows and folded norm, or the partials)
  int adapter_u(int l, int t, const GemvArgs& in) {
    if (!ad_[t].on) return 0;
    const LlamaEngine::WeightView A = e_.weight("blk." + std::to_string(l) + "." + kAdName[t] + ".lora_a");
    if (!A.f32) return -1;
    GemvArgs g = in;
    g.w32 = A.f32; g.wq = nullptr; g.ws = nullptr; g.rows = A.rows; g.K = A.cols;
    g.out = ad_[t].u; g.ldo = A.rows; g.mode = 0; g.pair = 0; g.res = nullptr; g.bias = nullptr; g.n_lora = 0;
    return gemv(g);
  }

  void add_lora(GemvArgs& g, int l, int t, int c0, int width, int on) {
    if (!ad_[t].on) return;
    GemvLora& L = g.lora[g.n_lora++];
    L.B = e_.weight("blk." + std::to_string(l) + "." + kAdName[t] + ".lora_b").f32;
    L.u = ad_[t].u; L.ldu = ad_[t].rows;
    L.c0 = c0; L.width = width; L.r = e_.cfg().lora_rank; L.bd_w = ad_[t].bd_w; L.on = on; L.s = ad_[t].s;
  }

  GemvArgs wargs(const std::string& name, int rows, int K) {
    const LlamaEngine::WeightView w = e_.weight(name);
    GemvArgs g;
    g.w32 = w.f32;
    g.wq = w.qv;
    g.ws = w.qs;
    g.rows = rows;
    g.K = K;
    return g;
  }

  int enqueue() {
    const LlamaConfig& c = e_.cfg();
    const int d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff, V = c.vocab;
    const int W = (H + 2 * KV) * dh;
    launches_ = 0;
    const LlamaEngine::WeightView E = e_.weight("token_embd.weight");
    ++launches_;
    if (launch_pdl(kv_embed_kernel, dim3(nb_), dim3(256), 0, st_, E.f32, (const int*)tok_, d, x_)) return -3;
    KvCache cache;
    for (int l = 0; l < c.n_layers; ++l) {
      const std::string pre = "blk." + std::to_string(l) + ".";
      const long long loff = (long long)l * nb_ * KV * max_T_ * dh;
      if (q8_) {
        cache.kq = kq_ + loff; cache.vq = vq_ + loff; cache.ks = ks_ + loff / 32; cache.vs = vs_ + loff / 32;
      } else {
        cache.k32 = k32_ + loff; cache.v32 = v32_ + loff;
      }
      // q | k | v with the attention RMSNorm folded in (and their adapters)
      GemvArgs g = wargs(pre + "attn_q.weight", W, d);
      g.x = x_; g.ldx = d; g.gamma = e_.weight(pre + "attn_norm.weight").f32; g.eps = c.rms_eps;
      g.out = qkv_; g.ldo = W;
      for (int t = 0; t < 3; ++t)
        if (int rc = adapter_u(l, t, g)) return rc;
      add_lora(g, l, 0, 0, H * dh, 0);
      add_lora(g, l, 1, H * dh, KV * dh, 0);
      add_lora(g, l, 2, (H + KV) * dh, KV * dh, 0);
      if (int rc = gemv(g)) return rc;
      AppendArgs ap;
      ap.qkv = qkv_;
      ap.bias = c.qkv_bias ? e_.weight(pre + "attn_q.bias").f32 : nullptr;
      ap.pos = pos_; ap.cs = reinterpret_cast<const float2*>(e_.rope_table()); ap.tab_rows = e_.rope_rows();
      ap.H = H; ap.KV = KV; ap.dh = dh; ap.max_T = max_T_; ap.c = cache;
      ++launches_;
      if (launch_pdl(kv_append_kernel, dim3(nb_, H + KV), dim3(dh), (size_t)2 * dh * 4, st_, ap)) return -3;
      AttnArgs at;
      at.qkv = qkv_; at.pos = pos_; at.c = cache; at.H = H; at.KV = KV; at.dh = dh; at.max_T = max_T_;
      at.nsplit = nsplit_; at.scale = 1.0f / std::sqrt((float)dh); at.part = part_;
      ++launches_;
      if (launch_pdl(kv_attn_kernel, dim3(nb_ * H, nsplit_), dim3(kChunk), attn_smem_, st_, at)) return -3;
      // x1 = x + att Wo^T, the attention output assembled from the chunks while staging
      g = wargs(pre + "attn_output.weight", d, H * dh);
      g.part = part_; g.nsplit = nsplit_; g.dh = dh;
      g.ldx = H * dh; g.out = x1_; g.ldo = d; g.res = x_; g.mode = 1;
      if (int rc = adapter_u(l, 3, g)) return rc;
      add_lora(g, l, 3, 0, d, 0);
      if (int rc = gemv(g)) return rc;
      // a = silu(h2 Wg^T) * (h2 Wu^T), the FFN RMSNorm folded in (gate | up rows paired)
      g = wargs(pre + "ffn_gate.weight", 2 * ff, d);
      g.x = x1_; g.ldx = d; g.gamma = e_.weight(pre + "ffn_norm.weight").f32; g.eps = c.rms_eps;
      g.out = a_; g.ldo = ff; g.mode = 2; g.pair = ff;
      for (int t = 4; t < 6; ++t)
        if (int rc = adapter_u(l, t, g)) return rc;
      add_lora(g, l, 4, 0, ff, 0);
      add_lora(g, l, 5, 0, ff, 1);
      if (int rc = gemv(g)) return rc;
      // x = x1 + a Wd^T
      g = wargs(pre + "ffn_down.weight", d, ff);
      g.x = a_; g.ldx = ff; g.out = x_; g.ldo = d; g.res = x1_; g.mode = 1;
      if (int rc = adapter_u(l, 6, g)) return rc;
      add_lora(g, l, 6, 0, d, 0);
      if (int rc = gemv(g)) return rc;
    }
    // logits = norm(x) W_out^T (tied: the embedding)
    GemvArgs g = wargs(c.tied ? "token_embd.weight" : "output.weight", V, d);
    g.x = x_; g.ldx = d; g.gamma = e_.weight("output_norm.weight").f32; g.eps = c.rms_eps;
    g.out = logits_; g.ldo = V;
    return gemv(g);
  }

  LlamaEngine& e_;
  int max_T_, nb_;
  bool q8_;
  int nsplit_ = 1, launches_ = 0;
  size_t attn_smem_ = 0;   // dynamic shared memory of the attention kernel (the chunk's V rows)
  // adapters by target (q, k, v, o, gate, up, down): u = A x buffer [n_seq][rows]
  struct Adapter {
    bool on = false;
    int rows = 0, bd_w = 0;
    float s = 1.f;
    float* u = nullptr;
  };
  static constexpr int kAdapters = 7;
  Adapter ad_[kAdapters];
  cudaStream_t st_ = nullptr;
  cudaGraphExec_t graph_ = nullptr;
  std::vector<void*> bufs_;
  float *x_ = nullptr, *x1_ = nullptr, *qkv_ = nullptr, *a_ = nullptr, *part_ = nullptr,
        *logits_ = nullptr;
  float *k32_ = nullptr, *v32_ = nullptr;
  int8_t *kq_ = nullptr, *vq_ = nullptr;
  uint16_t *ks_ = nullptr, *vs_ = nullptr;
  int *tok_ = nullptr, *pos_ = nullptr;
  int* host_in_ = nullptr;
};

void kv_free(Session* s) {
  delete s->kv;
  s->kv = nullptr;
}

}  // namespace tb2

extern "C" {

int tb2_kv_realize(void* sess, int max_T, int n_seq, int kv_type) {
  if (!sess || (kv_type != 0 && kv_type != 8)) return -1;
  tb2::Session* s = static_cast<tb2::Session*>(sess);
  if (!s->eng || s->kv) return -2;
  auto k = std::make_unique<tb2::KvEngine>(*s->eng, max_T, n_seq, kv_type);
  const int rc = k->realize();
  if (rc) return rc;
  s->kv = k.release();
  return 0;
}

int tb2_kv_reset(void* sess) {
  if (!sess || !static_cast<tb2::Session*>(sess)->kv) return -2;
  return static_cast<tb2::Session*>(sess)->kv->reset();
}

int tb2_kv_decode(void* sess, const long long* tokens, const long long* positions, int n_seq, float* logits) {
  if (!sess) return -1;
  tb2::Session* s = static_cast<tb2::Session*>(sess);
  if (!s->kv) return -2;
  return s->kv->decode(tokens, positions, n_seq, logits);
}

int tb2_kv_logits(void* sess, float* out, long long n) {
  if (!sess || !static_cast<tb2::Session*>(sess)->kv) return -2;
  return static_cast<tb2::Session*>(sess)->kv->logits(out, n);
}

int tb2_kv_run(void* sess, int steps, float* ms) {
  if (!sess || !static_cast<tb2::Session*>(sess)->kv) return -2;
  return static_cast<tb2::Session*>(sess)->kv->run(steps, ms);
}

int tb2_kv_launches(void* sess) {
  if (!sess || !static_cast<tb2::Session*>(sess)->kv) return -2;
  return static_cast<tb2::Session*>(sess)->kv->launches();
}

int tb2_kv_free(void* sess) {
  if (!sess) return -1;
  tb2::kv_free(static_cast<tb2::Session*>(sess));
  return 0;
}

}  // extern "C"
