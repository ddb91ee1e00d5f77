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
};

template <int NB, bool Q8>
__global__ void __launch_bounds__(256) kv_gemv_kernel(const GemvArgs a) {
  // xs [NB][K]: the input rows (times gamma when a norm is folded in); with the
  // attention partials, fs [NB][H][nsplit] holds each chunk's factor e^(m_s - m) / L
  extern __shared__ float xs[];
  __shared__ float rs[NB];
  griddep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (a.part) {
    const int H = a.K / a.dh, ns = a.nsplit, stride = a.dh + 2;
    float* fs = xs + NB * a.K;
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
    for (int i = threadIdx.x; i < NB * a.K; i += blockDim.x) xs[i] *= a.gamma[i % a.K];
    __syncthreads();
  }
  const int n_out = a.mode == 2 ? a.pair : a.rows;
  for (int n = blockIdx.x * kGemvWarps + warp; n < n_out; n += gridDim.x * kGemvWarps) {
    float acc[2][NB];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[h][b] = 0.f;
    const int nrow = a.mode == 2 ? 2 : 1;
    for (int h = 0; h < nrow; ++h) {
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
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float y0 = warp_sum(acc[0][b]) * rs[b];
      const float y1 = a.mode == 2 ? warp_sum(acc[1][b]) * rs[b] : 0.f;
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
  griddep_wait();
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
  griddep_wait();
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
  __shared__ float qs[128];
  __shared__ float ps[kChunk];
  __shared__ float red[kChunk / 32];
  __shared__ float osum[kChunk];
  griddep_wait();
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, j = h / (a.H / a.KV), split = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, dh = a.dh;
  const int hist = a.pos[b] + 1;
  const int t0 = split * kChunk, t1 = min(t0 + kChunk, hist);
  float* out = a.part + ((long long)bh * a.nsplit + split) * (dh + 2);
  if (t0 >= t1) {   // this chunk is past the history
    for (int d = tid; d < dh; d += blockDim.x) out[d] = 0.f;
    if (tid == 0) {
      out[dh] = -INFINITY;
      out[dh + 1] = 0.f;
    }
    return;
  }
  const float* q = a.qkv + (long long)b * (a.H + 2 * a.KV) * dh + h * dh;
  for (int d = tid; d < dh; d += blockDim.x) qs[d] = q[d];
  __syncthreads();
  const long long base = ((long long)b * a.KV + j) * a.max_T;
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
  const int groups = blockDim.x / dh, g = tid / dh, d = tid % dh;
  float o = 0.f;
  if (g < groups) {
    const int n = t1 - t0;
#pragma unroll 8
    for (int k = g; k < n; k += groups) {
      const long long slot = base + t0 + k;
      const float v = a.c.v32 ? __ldg(a.c.v32 + slot * dh + d)
                              : __half2float(__ushort_as_half(__ldg(a.c.vs + slot * (dh / 32) + d / 32))) *
                                    (float)__ldg(a.c.vq + slot * dh + d);
      o += ps[k] * v;
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
    const long long nsplit = (max_T_ + kChunk - 1) / kChunk;
    if (((long long)nb_ * std::max(c.d_ff, std::max(c.d_model, c.n_heads * c.d_head)) +
         (long long)nb_ * c.n_heads * nsplit) * 4 > 200 * 1024)
      return -1;
    if (cudaSetDevice(e_.device()) != cudaSuccess) return -3;
    if (cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking) != cudaSuccess) return -3;
    const int d = c.d_model, H = c.n_heads, KV = c.n_kv, dh = c.d_head, ff = c.d_ff, V = c.vocab, L = c.n_layers;
    const int W = (H + 2 * KV) * dh;
    nsplit_ = (max_T_ + kChunk - 1) / kChunk;
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
    const size_t smem = ((size_t)NB * g.K + (g.part ? (size_t)NB * (g.K / g.dh) * g.nsplit : 0)) * 4;
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
      // q | k | v with the attention RMSNorm folded in
      GemvArgs g = wargs(pre + "attn_q.weight", W, d);
      g.x = x_; g.ldx = d; g.gamma = e_.weight(pre + "attn_norm.weight").f32; g.eps = c.rms_eps;
      g.out = qkv_; g.ldo = W;
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
      if (launch_pdl(kv_attn_kernel, dim3(nb_ * H, nsplit_), dim3(kChunk), 0, st_, at)) return -3;
      // x1 = x + att Wo^T, the attention output assembled from the chunks while staging
      g = wargs(pre + "attn_output.weight", d, H * dh);
      g.part = part_; g.nsplit = nsplit_; g.dh = dh;
      g.ldx = H * dh; g.out = x1_; g.ldo = d; g.res = x_; g.mode = 1;
      if (int rc = gemv(g)) return rc;
      // a = silu(h2 Wg^T) * (h2 Wu^T), the FFN RMSNorm folded in (gate | up rows paired)
      g = wargs(pre + "ffn_gate.weight", 2 * ff, d);
      g.x = x1_; g.ldx = d; g.gamma = e_.weight(pre + "ffn_norm.weight").f32; g.eps = c.rms_eps;
      g.out = a_; g.ldo = ff; g.mode = 2; g.pair = ff;
      if (int rc = gemv(g)) return rc;
      // x = x1 + a Wd^T
      g = wargs(pre + "ffn_down.weight", d, ff);
      g.x = a_; g.ldx = ff; g.out = x_; g.ldo = d; g.res = x1_; g.mode = 1;
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
