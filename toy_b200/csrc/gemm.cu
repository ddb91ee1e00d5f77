// Split-bf16 tensor-core GEMM for sm_100a: persistent CTAs, TMA-fed
// shared-memory pipeline, single-thread tcgen05.mma issue into one of two TMEM
// accumulators, 4-warp epilogue.
//
// CTA = warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, then 4 or 8
// epilogue warps (warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31; with 8,
// the two warps of a lane quarter take one column half of the tile each),
// plus 8 converter warps for a Q8_0 B operand.
// Each CTA walks the work units u = blockIdx.x, blockIdx.x + gridDim.x, ...;
// a unit is one 128 x BN output tile (of one batch entry) over a range of K.
// The producer's stage ring runs across units; the MMA issuer alternates
// between two TMEM accumulators so the epilogue of unit i overlaps the
// mainloop of unit i+1.
//
// Split-K: when the tile grid is too small for the 148 SMs, K is cut into S
// ranges. Every unit writes its f32 partial tile to slab s of a workspace and
// a second, bandwidth-bound kernel sums the S slabs in split order (so the
// result does not depend on scheduling) and applies the epilogue.
//
// Causal modes for attention: 1 skips tiles whose keys all exceed their
// queries (n0 > m0 + 127); 2 clamps K (keys) to m0 + 128 because P / dS are
// zero beyond the diagonal.
#include "gemm.cuh"
#include "pdl.cuh"
#include "runtime.cuh"
#include "tc_common.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <mutex>

namespace tb2 {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;          // one 128-byte swizzle atom of bf16 along K
constexpr int kThreads = 192;   // producer, MMA issuer, 4 epilogue warps (the role warps of a 4-warp epilogue)
constexpr int kConvWarps = 8;   // Q8_0 B operand: warps 6.. dequantise into the B tiles
constexpr int kSmemBudget = 200 * 1024;
constexpr int kNumSMs = 148;

// Epilogue warps: 8 (two per TMEM lane quarter, one per column half) for the
// plain instantiations whose tile splits into halves of whole 64-column
// groups; 4 for the fused epilogues, the Q8_0 B operand and 64-wide tiles.
template <int BN, bool Q8, bool FUSED>
__host__ __device__ constexpr int epi_warps() {
  return (Q8 || FUSED || BN == 64) ? 4 : 8;
}
template <int BN, bool Q8, bool FUSED>
__host__ __device__ constexpr int threads_of() {
  return 64 + 32 * epi_warps<BN, Q8, FUSED>() + (Q8 ? 32 * kConvWarps : 0);
}

// kernels the calling thread's last gemm_launch enqueued (the product, and
// the split-K reduction when there is one)
thread_local int t_last_launches = 0;

struct KArgs {
  int M, N, K, batch;
  int a_mn, b_mn;
  int a_bdiv1, a_bmul1, a_bdiv2, a_bmul2;
  int b_bdiv1, b_bmul1, b_bdiv2, b_bmul2;
  int tiles_m, tiles_n, splits, units, kb_total, causal;
  int f16;   // operands are fp16 (one pass), not bf16
  Epilogue epi;
  float* ws;
  const int* gtab;   // grouped product: per M tile (group, first row, end row); null otherwise
  int b_keep;   // B is an operand kept resident in the L2: evict-last loads
  int* err;
  const uint16_t* q8_scale;   // Q8_0 B operand: scales and stored extent
  int q8_rows, q8_cols;
};

__device__ __forceinline__ int batch_index(int z, int d1, int m1, int d2, int m2) {
  return (z / d1) * m1 + ((z % d1) / d2) * m2;
}

template <int BN, bool PAIR = false>
struct Cfg {
  static constexpr int kRowsB = PAIR ? BN / 2 : BN;   // B rows in this CTA's shared memory
  static constexpr int kTileA = BM * BK * 2;  // bytes per plane
  static constexpr int kTileB = kRowsB * BK * 2;
  static constexpr uint32_t kAccCols = BN <= 64 ? 64 : BN <= 128 ? 128 : 256;  // one accumulator
  static constexpr uint32_t kTmemCols = 2 * kAccCols;                           // double buffered
};

// A stage holds the A and B plane tiles and, for a Q8_0 B operand, the int8
// quant tile the converters read (B rows x 64 bytes, or B rows / 64 blocks of
// 64 x 64 bytes when B is MN-major). kTxBytes is what the `full` barrier
// counts: the planes TMA writes (of both CTAs of a pair). Quants count on a
// per-CTA `qfull` barrier, so the converters start as soon as they land.
template <int BN, bool SPLIT, bool Q8 = false, bool PAIR = false>
struct Stages {
  using C = Cfg<BN, PAIR>;
  static constexpr int kQBytes = Q8 ? C::kRowsB * 64 : 0;
  static constexpr int kStageBytes = (SPLIT ? 2 : 1) * (C::kTileA + C::kTileB) + kQBytes;
  static constexpr int kTxBytes = (PAIR ? 2 : 1) * (Q8 ? 2 * C::kTileA : kStageBytes);
  static constexpr int kBudget = Q8 ? 216 * 1024 : kSmemBudget;
  static constexpr int kStages = (kBudget / kStageBytes) > 6 ? 6 : (kBudget / kStageBytes);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align slack*/ + 256 /*barriers*/;
};

struct Unit {
  int z, m0, m1, n0, kb0, kb1, tile;   // m1: end of the rows this unit may write
  bool skip;
};

// unit u -> (batch, first output row, first output column, K range); a unit
// covers BMT rows (BM, or 2 BM for a CTA pair)
template <int BN, int BMT = BM>
__device__ __forceinline__ Unit decode(const KArgs& a, int u) {
  Unit r;
  const int s = u % a.splits;
  int t = u / a.splits;
  r.tile = t;
  r.n0 = (t % a.tiles_n) * BN;
  t /= a.tiles_n;
  if (a.gtab) {   // grouped product: the M tile's group (its B batch) and row range
    const int* g = a.gtab + 3 * (t % a.tiles_m);
    r.z = g[0];
    r.m0 = g[1];
    r.m1 = g[2];
  } else {
    r.m0 = (t % a.tiles_m) * BMT;
    r.z = t / a.tiles_m;
    r.m1 = a.M;
  }
  r.skip = a.causal == 1 && r.n0 > r.m0 + BM - 1;
  int kbt = a.kb_total;
  if (a.causal == 2) {
    const int kmax = min(a.K, r.m0 + BM);
    kbt = (kmax + BK - 1) / BK;
  }
  r.kb0 = (int)((long long)s * kbt / a.splits);
  r.kb1 = (int)((long long)(s + 1) * kbt / a.splits);
  return r;
}

__device__ __forceinline__ long long epi_offset(const Epilogue& e, int z, int m, int nc) {
  return (long long)(z / e.z_div) * e.z_s1 + (long long)(z % e.z_div) * e.bstride +
         (long long)(m / e.m_div) * e.m_s1 + (long long)(m % e.m_div) * e.m_s0 + (long long)(nc / e.n_div) * e.n_s1 +
         (nc % e.n_div);
}

// The 32 addend values of a residual / accumulate epilogue for chunk (m, nc),
// loaded ahead of the chunk's accumulator (they do not depend on the MMA).
__device__ __forceinline__ void epi_prefetch(const Epilogue& e, int N, long long off, int nc, float4 (&r)[8]) {
  if (nc + 32 > N || (e.mode != kEpiAccumF32 && e.mode != kEpiResidF32)) return;
  const float4* src = reinterpret_cast<const float4*>((e.mode == kEpiAccumF32 ? e.out : e.res) + off);
#pragma unroll
  for (int i = 0; i < 8; ++i) r[i] = src[i];
}

// Apply the epilogue to the 32 consecutive outputs (m, nc .. nc+31) held in v.
// `pre` holds the addend loaded by epi_prefetch (used when the chunk is full).
__device__ __forceinline__ void epi_store(const Epilogue& e, int N, long long off, int nc, float (&v)[32],
                                          const float4 (&pre)[8]) {
  const float alpha = e.alpha_dev ? e.alpha * __ldg(e.alpha_dev) : e.alpha;
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] *= alpha;
  const bool full_chunk = nc + 32 <= N;
  if (e.mode == kEpiStoreF32 || e.mode == kEpiAccumF32 || e.mode == kEpiResidF32 || e.mode == kEpiStoreBoth ||
      e.mode == kEpiStoreLse) {
    float* dst = e.out + off;
    if (full_chunk) {
      float4* d4 = reinterpret_cast<float4*>(dst);
      if (e.mode == kEpiAccumF32 || e.mode == kEpiResidF32) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 r = pre[i];
          d4[i] = make_float4(r.x + v[4 * i], r.y + v[4 * i + 1], r.z + v[4 * i + 2], r.w + v[4 * i + 3]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (nc + i < N) {
          if (e.mode == kEpiAccumF32) dst[i] += v[i];
          else if (e.mode == kEpiResidF32) dst[i] = e.res[off + i] + v[i];
          else dst[i] = v[i];
        }
      }
    }
  }
  if (e.mode == kEpiStoreSplit || e.mode == kEpiStoreBoth) {
    __nv_bfloat16* dh = e.out_hi + off;
    __nv_bfloat16* dl = e.out_lo + off;
    if (full_chunk) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float x0 = v[8 * i + 2 * j], x1 = v[8 * i + 2 * j + 1];
          const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
          const __nv_bfloat16 l0 = __float2bfloat16_rn(x0 - __bfloat162float(h0));
          const __nv_bfloat16 l1 = __float2bfloat16_rn(x1 - __bfloat162float(h1));
          h[j] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
          l[j] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
        }
        reinterpret_cast<uint4*>(dh)[i] = make_uint4(h[0], h[1], h[2], h[3]);
        reinterpret_cast<uint4*>(dl)[i] = make_uint4(l[0], l[1], l[2], l[3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (nc + i < N) {
          const __nv_bfloat16 h0 = __float2bfloat16_rn(v[i]);
          dh[i] = h0;
          dl[i] = __float2bfloat16_rn(v[i] - __bfloat162float(h0));
        }
      }
    }
  }
}

// v(m, nc + i) += scale * sum_j u[m][j] * bt[j][nc + i - c0] for every LoRA
// addend whose column range holds the chunk (ranges are multiples of 32). All
// lanes of a warp read the same bt chunk (broadcast); u is the lane's own row.
template <int W>
__device__ __forceinline__ void lora_add(const Epilogue& e, int m, int nc, float (&v)[W]) {
#pragma unroll 1
  for (int a = 0; a < e.n_lora; ++a) {
    const LoraAddend& L = e.lora[a];
    if (nc < L.c0 || nc >= L.c0 + L.width) continue;
    const float* ur = L.u + (long long)m * L.r;
    const float* bt = L.bt + (nc - L.c0);
#pragma unroll 1
    for (int j = 0; j < L.r; ++j) {
      const float su = L.scale * ur[j];
      const float4* b4 = reinterpret_cast<const float4*>(bt + (long long)j * L.width);
#pragma unroll
      for (int q = 0; q < W / 4; ++q) {
        const float4 w4 = __ldg(b4 + q);
        v[4 * q] = fmaf(su, w4.x, v[4 * q]);
        v[4 * q + 1] = fmaf(su, w4.y, v[4 * q + 1]);
        v[4 * q + 2] = fmaf(su, w4.z, v[4 * q + 2]);
        v[4 * q + 3] = fmaf(su, w4.w, v[4 * q + 3]);
      }
    }
  }
}

// 32 values as hi / lo bf16 planes at 16-byte aligned addresses.
__device__ __forceinline__ void store_split32(__nv_bfloat16* hi, __nv_bfloat16* lo, const float (&v)[32]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) split_pair(v[8 * u + 2 * j], v[8 * u + 2 * j + 1], h[j], l[j]);
    reinterpret_cast<uint4*>(hi)[u] = make_uint4(h[0], h[1], h[2], h[3]);
    reinterpret_cast<uint4*>(lo)[u] = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// 16 values as hi / lo bf16 planes at 16-byte aligned addresses.
__device__ __forceinline__ void store_split16(__nv_bfloat16* hi, __nv_bfloat16* lo, const float (&v)[16]) {
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) split_pair(v[8 * u + 2 * j], v[8 * u + 2 * j + 1], h[j], l[j]);
    reinterpret_cast<uint4*>(hi)[u] = make_uint4(h[0], h[1], h[2], h[3]);
    reinterpret_cast<uint4*>(lo)[u] = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// The warp has read its accumulator lanes: hand the accumulator back to the
// MMA issuer (rank 0's barrier for a CTA pair).
template <bool PAIR>
__device__ __forceinline__ void release_acc(uint64_t* tempty, int lane) {
  tc_fence_before();
  __syncwarp();
  if (lane == 0) {
    if constexpr (PAIR) mbar_arrive_cluster(cluster_addr(tempty, 0));
    else mbar_arrive(tempty);
  }
}

// kEpiRopeQKV for one tile row: one head (NCH chunks of 32 columns) at a time,
// sixteen rotation pairs per step -- LoRA addends, bias, RoPE rotation of q / k
// heads by pos[m], head-major planes.
template <int BN, int NCH, bool PAIR>
__device__ __forceinline__ void epi_rope(const Epilogue& e, int m, int n0, bool row_ok, int N, uint32_t acc,
                                         uint64_t* tempty, int lane) {
  constexpr int DH = NCH * 32, HALF = DH / 2;
  const RopeOut& R = e.rope;
  int bq = 0, t = 0, p = 0;
  if (row_ok) {
    bq = m / R.T;
    t = m - bq * R.T;
    p = R.pos[m];
    p = p < 0 ? 0 : (p >= R.tab_rows ? R.tab_rows - 1 : p);
  }
  const float2* crow = reinterpret_cast<const float2*>(R.cs) + (long long)p * HALF;
#pragma unroll 1
  for (int hb = 0; hb < BN; hb += DH) {
    const int c0 = n0 + hb;
    const bool live = row_ok && c0 < N;
    const int slot = c0 / DH;
    __nv_bfloat16 *oh, *ol;
    long long dst;
    bool rot = true;
    if (slot < R.H) {
      dst = (((long long)bq * R.H + slot) * R.T + t) * DH;
      oh = R.q_hi; ol = R.q_lo;
    } else if (slot < R.H + R.KV) {
      dst = (((long long)bq * R.KV + (slot - R.H)) * R.T + t) * DH;
      oh = R.k_hi; ol = R.k_lo;
    } else {
      dst = (((long long)bq * R.KV + (slot - R.H - R.KV)) * R.T + t) * DH;
      oh = R.v_hi; ol = R.v_lo;
      rot = false;
    }
    // rotation pairs (j, j + dh/2) sixteen at a time: x0 = columns j.., x1 = j + dh/2 ..
#pragma unroll 1
    for (int q = 0; q < HALF / 16; ++q) {
      float x0[16], x1[16];
      tmem_ld16(acc + (uint32_t)(hb + 16 * q), x0);
      tmem_ld16(acc + (uint32_t)(hb + HALF + 16 * q), x1);
      if (hb + DH >= BN && q == HALF / 16 - 1) release_acc<PAIR>(tempty, lane);
      if (!live) continue;
      const int ca = c0 + 16 * q, cb = c0 + HALF + 16 * q;
      if (e.n_lora) {
        lora_add(e, m, ca, x0);
        lora_add(e, m, cb, x1);
      }
      if (R.bias) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          x0[i] += R.bias[ca + i];
          x1[i] += R.bias[cb + i];
        }
      }
      if (rot) {   // y0 = x0 cos - x1 sin, y1 = x0 sin + x1 cos
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 c = crow[16 * q + i];
          const float a0 = x0[i], a1 = x1[i];
          x0[i] = a0 * c.x - a1 * c.y;
          x1[i] = a0 * c.y + a1 * c.x;
        }
      }
      store_split16(oh + dst + 16 * q, ol + dst + 16 * q, x0);
      store_split16(oh + dst + HALF + 16 * q, ol + dst + HALF + 16 * q, x1);
    }
  }
}

// kEpiSwiGLU for one tile row of a tile with paired B rows: columns [0, BN/2)
// are gate features n0/2 .., [BN/2, BN) the same up features; 16 of each at a time.
template <int BN, bool PAIR>
__device__ __forceinline__ void epi_swiglu(const Epilogue& e, int m, int n0, bool row_ok, uint32_t acc,
                                           uint64_t* tempty, int lane) {
  const int ff = e.pair_off, f0 = n0 / 2;
#pragma unroll 1
  for (int k = 0; k < BN / 32; ++k) {
    float g[16], u[16];
    tmem_ld16(acc + (uint32_t)(16 * k), g);
    tmem_ld16(acc + (uint32_t)(BN / 2 + 16 * k), u);
    if (k == BN / 32 - 1) release_acc<PAIR>(tempty, lane);
    const int fc = f0 + 16 * k;
    if (!row_ok || fc >= ff) continue;
    if (e.n_lora) {
      lora_add(e, m, fc, g);        // gate columns [0, ff)
      lora_add(e, m, ff + fc, u);   // up columns [ff, 2 ff)
    }
    float* orow = e.out + (long long)m * e.m_s0;
    float4* og = reinterpret_cast<float4*>(orow + fc);
    float4* ou = reinterpret_cast<float4*>(orow + ff + fc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      og[i] = make_float4(g[4 * i], g[4 * i + 1], g[4 * i + 2], g[4 * i + 3]);
      ou[i] = make_float4(u[4 * i], u[4 * i + 1], u[4 * i + 2], u[4 * i + 3]);
    }
    // silu with the hardware exp2 / reciprocal approximations (~1e-7 relative)
#pragma unroll
    for (int i = 0; i < 16; ++i) g[i] = __fdividef(g[i], 1.0f + __expf(-g[i])) * u[i];
    store_split16(e.out_hi + (long long)m * ff + fc, e.out_lo + (long long)m * ff + fc, g);
  }
}

// FUSED instantiations carry the fused epilogues (LoRA addends, RoPE / SwiGLU
// modes); the others leave that code out so they keep their register budget.
template <int BN, bool SPLIT, bool Q8, bool FUSED, bool PAIR>
__global__ void __launch_bounds__(threads_of<BN, Q8, FUSED>(), 1)
    gemm_split_bf16_kernel(const __grid_constant__ CUtensorMap map_a_hi, const __grid_constant__ CUtensorMap map_a_lo,
                           const __grid_constant__ CUtensorMap map_b_hi, const __grid_constant__ CUtensorMap map_b_lo,
                           const KArgs args) {
  static_assert(!Q8 || SPLIT, "a Q8_0 operand is always dequantised into split planes");
  static_assert(!PAIR || (SPLIT && (BN == 128 || BN == 256)), "CTA pairs run split planes, 128 / 256-wide tiles");
  using St = Stages<BN, SPLIT, Q8, PAIR>;
  constexpr int STAGES = St::kStages;
  constexpr int kTileA = Cfg<BN, PAIR>::kTileA;
  constexpr int kTileB = Cfg<BN, PAIR>::kTileB;
  constexpr int RB = Cfg<BN, PAIR>::kRowsB;   // B rows (output columns) held by this CTA
  constexpr int BMT = PAIR ? 2 * BM : BM;     // output rows of a unit
  constexpr int kStageBytes = St::kStageBytes;
  constexpr int kTxBytes = St::kTxBytes;
  constexpr uint32_t kAccCols = Cfg<BN>::kAccCols;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2] accumulator ready for the epilogue
  uint64_t* tempty = tfull + 2;       // [2] accumulator drained by the epilogue
  uint64_t* conv = tempty + 2;        // [STAGES] Q8_0: B tiles dequantised
  uint64_t* qfull = conv + (Q8 ? STAGES : 0);   // [STAGES] Q8_0: this CTA's quant tile landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qfull + (Q8 ? STAGES : 0));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  // CTA pair: both CTAs walk the same units; rank 0 issues the MMAs and owns
  // the full / conv / tempty barriers the pair shares (the peer reaches them
  // through cluster addresses)
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int walker = PAIR ? (int)(blockIdx.x / 2) : (int)blockIdx.x;
  const int walkers = PAIR ? (int)(gridDim.x / 2) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      if (Q8) mbar_init(&conv[s], (PAIR ? 2 : 1) * kConvWarps);
      if (Q8) mbar_init(&qfull[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], (PAIR ? 2 : 1) * epi_warps<BN, Q8, FUSED>());
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg<BN>::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg<BN>::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();   // the peer's barriers are initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Barrier set-up and the TMEM allocation above overlap the previous kernel's
  // tail; nothing in global memory is touched before this point.
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&map_a_hi);
      tma_prefetch_desc(&map_b_hi);
      const uint64_t keep_pol = args.b_keep ? l2_policy_evict_last() : 0ull;
      uint32_t it = 0;
      bool ok = true;
      for (int u = walker; u < args.units && ok; u += walkers) {
        const Unit w = decode<BN, BMT>(args, u);
        if (w.skip) continue;
        const int za = args.gtab ? 0 : batch_index(w.z, args.a_bdiv1, args.a_bmul1, args.a_bdiv2, args.a_bmul2);
        const int zb = batch_index(w.z, args.b_bdiv1, args.b_bmul1, args.b_bdiv2, args.b_bmul2);
        const int m0 = w.m0 + (int)rank * BM;   // this CTA's A rows
        const int nb = w.n0 + (int)rank * RB;   // this CTA's B rows (unpaired)
        // paired gate / up rows: one CTA of a pair loads the gate rows, the other the up rows
        const int pr = (int)rank == 0 ? w.n0 / 2 : args.epi.pair_off + w.n0 / 2;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, args.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          // A (and B) plane tiles of both CTAs count on rank 0's full barrier
          const uint32_t fc = PAIR ? cluster_addr(&full[s], 0) : 0u;
          auto ld = [&](void* dst, const CUtensorMap* map, int c0, int c1, int c2) {
            if constexpr (PAIR) tma_load_3d_pair(dst, map, fc, c0, c1, c2);
            else tma_load_3d(dst, map, &full[s], c0, c1, c2);
          };
          // B plane tiles of an operand kept resident in the L2 (args.b_keep):
          // loaded with the evict-last policy, so reading them does not demote them
          auto ldb = [&](void* dst, const CUtensorMap* map, int c0, int c1, int c2) {
            if (!args.b_keep) {
              ld(dst, map, c0, c1, c2);
            } else if constexpr (PAIR) {
              tma_load_3d_pair_hint(dst, map, fc, c0, c1, c2, keep_pol);
            } else {
              tma_load_3d_hint(dst, map, &full[s], c0, c1, c2, keep_pol);
            }
          };
          if (!PAIR || rank == 0) mbar_arrive_expect_tx(&full[s], kTxBytes);
          if (Q8) mbar_arrive_expect_tx(&qfull[s], St::kQBytes);
          uint8_t* st = smem + s * kStageBytes;
          uint8_t* a_hi = st;
          uint8_t* b_hi = st + kTileA;
          uint8_t* a_lo = st + kTileA + kTileB;
          uint8_t* b_lo = a_lo + kTileA;
          const int k0 = kb * BK;
          if (!args.a_mn) {
            ld(a_hi, &map_a_hi, k0, m0, za);
            if (SPLIT) ld(a_lo, &map_a_lo, k0, m0, za);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) {
              ld(a_hi + j * 64 * 128, &map_a_hi, m0 + 64 * j, k0, za);
              if (SPLIT) ld(a_lo + j * 64 * 128, &map_a_lo, m0 + 64 * j, k0, za);
            }
          }
          if (Q8) {
            // int8 quants; map_b_hi is the quant map (box {64 bytes, rows}),
            // counted on this CTA's qfull: its own converters read them
            uint8_t* qd = st + 2 * (kTileA + kTileB);
            uint64_t* qb = &qfull[s];
            if (args.epi.pair_off) {
              if (PAIR) {
                tma_load_3d(qd, &map_b_hi, qb, k0, pr, zb);
              } else {   // gate rows, then the matching up rows
                tma_load_3d(qd, &map_b_hi, qb, k0, w.n0 / 2, zb);
                tma_load_3d(qd + (BN / 2) * 64, &map_b_hi, qb, k0, args.epi.pair_off + w.n0 / 2, zb);
              }
            } else if (!args.b_mn) {
              tma_load_3d(qd, &map_b_hi, qb, k0, nb, zb);
            } else {
#pragma unroll
              for (int j = 0; j < RB / 64; ++j) tma_load_3d(qd + j * 64 * 64, &map_b_hi, qb, nb + 64 * j, k0, zb);
            }
          } else if (args.epi.pair_off) {
            if (PAIR) {
              ldb(b_hi, &map_b_hi, k0, pr, zb);
              ldb(b_lo, &map_b_lo, k0, pr, zb);
            } else {   // gate rows, then the matching up rows
              const int r0 = w.n0 / 2, r1 = args.epi.pair_off + w.n0 / 2;
              ldb(b_hi, &map_b_hi, k0, r0, zb);
              ldb(b_hi + (BN / 2) * 128, &map_b_hi, k0, r1, zb);
              if (SPLIT) {
                ldb(b_lo, &map_b_lo, k0, r0, zb);
                ldb(b_lo + (BN / 2) * 128, &map_b_lo, k0, r1, zb);
              }
            }
          } else if (!args.b_mn) {
            ldb(b_hi, &map_b_hi, k0, nb, zb);
            if (SPLIT) ldb(b_lo, &map_b_lo, k0, nb, zb);
          } else {
#pragma unroll
            for (int j = 0; j < RB / 64; ++j) {
              ldb(b_hi + j * 64 * 128, &map_b_hi, nb + 64 * j, k0, zb);
              if (SPLIT) ldb(b_lo + j * 64 * 128, &map_b_lo, nb + 64 * j, k0, zb);
            }
          }
        }
      }
      // A pair member exits only after the MMAs have released every stage it
      // filled (their commits arrive on this CTA's empty barriers).
      if (PAIR && ok) {
        for (int j = 0; j < STAGES; ++j, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, args.err, kErrWaitEmpty)) break;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && (!PAIR || rank == 0)) {
      const uint32_t idesc = make_idesc_f16(BMT, BN, args.f16 == 0, args.a_mn != 0, args.b_mn != 0);
      // K-major: advance 32 B per 16-element k-step inside the swizzle atom.
      // MN-major: advance 16 rows of 128 B; MN atoms are 64 rows (8 KB) apart.
      const uint32_t a_kstep = args.a_mn ? 2048u : 32u;
      const uint32_t b_kstep = args.b_mn ? 2048u : 32u;
      const uint32_t a_lbo = args.a_mn ? 8192u : 16u;
      const uint32_t b_lbo = args.b_mn ? 8192u : 16u;
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int u = walker; u < args.units && ok; u += walkers) {
        const Unit w = decode<BN, BMT>(args, u);
        if (w.skip) continue;
        const uint32_t b = local & 1, tph = (local >> 1) & 1;
        ok = PAIR ? mbar_wait_cluster(&tempty[b], tph ^ 1, args.err, kErrWaitAccum)
                  : mbar_wait(&tempty[b], tph ^ 1, args.err, kErrWaitAccum);
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc_tmem = tmem_base + b * kAccCols;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          ok = mbar_wait(&full[s], ph, args.err, kErrWaitFull);
          if (Q8) {
            ok = ok && (PAIR ? mbar_wait_cluster(&conv[s], ph, args.err, kErrWaitFull)
                             : mbar_wait(&conv[s], ph, args.err, kErrWaitFull));
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * kStageBytes);
          const uint32_t a_hi = st, b_hi = st + kTileA, a_lo = st + kTileA + kTileB, b_lo = a_lo + kTileA;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            const uint64_t dah = make_sdesc_sw128(a_hi + ks * a_kstep, a_lbo, 1024);
            const uint64_t dbh = make_sdesc_sw128(b_hi + ks * b_kstep, b_lbo, 1024);
            const uint32_t acc = (kb > w.kb0 || ks > 0) ? 1u : 0u;
            if constexpr (PAIR) {
              const uint64_t dal = make_sdesc_sw128(a_lo + ks * a_kstep, a_lbo, 1024);
              const uint64_t dbl = make_sdesc_sw128(b_lo + ks * b_kstep, b_lbo, 1024);
              umma_f16_pair(acc_tmem, dah, dbh, idesc, acc);
              umma_f16_pair(acc_tmem, dal, dbh, idesc, 1u);
              umma_f16_pair(acc_tmem, dah, dbl, idesc, 1u);
            } else {
              umma_f16(acc_tmem, dah, dbh, idesc, acc);
              if (SPLIT) {
                const uint64_t dal = make_sdesc_sw128(a_lo + ks * a_kstep, a_lbo, 1024);
                const uint64_t dbl = make_sdesc_sw128(b_lo + ks * b_kstep, b_lbo, 1024);
                umma_f16(acc_tmem, dal, dbh, idesc, 1u);
                umma_f16(acc_tmem, dah, dbl, idesc, 1u);
              }
            }
          }
          if constexpr (PAIR) {   // free the stage in both CTAs
            umma_commit_pair(cluster_addr(&empty[s], 0));
            umma_commit_pair(cluster_addr(&empty[s], 1));
          } else {
            umma_commit(&empty[s]);
          }
        }
        if constexpr (PAIR) {
          umma_commit_pair(cluster_addr(&tfull[b], 0));
          umma_commit_pair(cluster_addr(&tfull[b], 1));
        } else {
          umma_commit(&tfull[b]);
        }
        ++local;
      }
    }
  } else if (warp >= 2 + epi_warps<BN, Q8, FUSED>()) {
    // ------------------------------------------------ Q8_0 dequantisation
    // Each item is one Q8_0 block (32 quants of a stored row, one scale): value
    // = scale * q, split into hi / lo bf16 and written to the B plane tiles in
    // the swizzled layout the UMMA descriptors expect -- the same bits a TMA
    // load of planes would give.
    if constexpr (Q8) {
      const int ct = threadIdx.x - kThreads;
      const int sblk = args.q8_cols / 32;
      // one Q8_0 block (item) per converter thread and k-block: tile row r,
      // half c32 of the 64 columns and, MN-major, 64-column tile tj
      static_assert(RB * 2 <= 32 * kConvWarps, "one item per converter thread");
      const bool has_item = ct < RB * 2;
      const int c32 = ct & 1;
      const int r = args.b_mn ? (ct >> 1) & 63 : ct >> 1;
      const int tj = args.b_mn ? ct >> 7 : 0;
      uint32_t it = 0;
      bool ok = true;
      for (int u = walker; u < args.units && ok; u += walkers) {
        const Unit w = decode<BN, BMT>(args, u);
        if (w.skip) continue;
        const int nb = w.n0 + (int)rank * RB;
        const int zq = batch_index(w.z, args.b_bdiv1, args.b_bmul1, args.b_bdiv2, args.b_bmul2);   // B batch
        // this item's scale for k-block kb (a global load, issued ahead of
        // the stage wait so its latency overlaps the wait and the conversion)
        auto scale_of = [&](int kb) -> float {
          const int k0 = kb * BK;
          int srow, sb;
          if (!args.b_mn) {
            if (!args.epi.pair_off) srow = nb + r;
            else if (PAIR) srow = ((int)rank == 0 ? w.n0 / 2 : args.epi.pair_off + w.n0 / 2) + r;
            else srow = r < BN / 2 ? w.n0 / 2 + r : args.epi.pair_off + w.n0 / 2 + r - BN / 2;
            sb = (k0 >> 5) + c32;
          } else {
            srow = k0 + r;
            sb = ((nb + 64 * tj) >> 5) + c32;
          }
          return (has_item && srow < args.q8_rows && sb < sblk)
                     ? __half2float(__ushort_as_half(args.q8_scale[((long long)zq * args.q8_rows + srow) * sblk + sb]))
                     : 0.f;
        };
        float sc_next = scale_of(w.kb0);
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const float sc = sc_next;
          if (kb + 1 < w.kb1) sc_next = scale_of(kb + 1);
          ok = warp_wait(&qfull[s], ph, args.err, kErrWaitFull);
          if (!ok) break;
          uint8_t* st = smem + s * kStageBytes;
          uint8_t* b_hi = st + kTileA;
          uint8_t* b_lo = st + 2 * kTileA + kTileB;
          const uint8_t* qs = st + 2 * (kTileA + kTileB);
          if (has_item) {
            // item = one Q8_0 block: 32 quants of tile row r, columns c32 * 32 .. +31 of this tile's 64
            const uint8_t* src = !args.b_mn ? qs + r * 64 + c32 * 32 : qs + tj * 4096 + r * 64 + c32 * 32;
            const uint32_t tile = !args.b_mn ? 0u : (uint32_t)tj * 8192u;
            // the two 16-byte halves in a lane-dependent order: each 8-lane
            // phase of a shared load then touches 8 distinct bank groups
            const int sw = (lane >> 2) & 1;
            const uint4 ra = reinterpret_cast<const uint4*>(src)[sw];
            const uint4 rb = reinterpret_cast<const uint4*>(src)[sw ^ 1];
            const uint4 raw0 = sw ? rb : ra, raw1 = sw ? ra : rb;
            const uint32_t words[8] = {raw0.x, raw0.y, raw0.z, raw0.w, raw1.x, raw1.y, raw1.z, raw1.w};
            const uint64_t scp = pack_f2(sc, sc);
#pragma unroll
            for (int u = 0; u < 4; ++u) {   // 16-byte chunk c32 * 4 + u of each plane
              uint32_t hv[4], lv[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                // q + 128 as the low mantissa byte of 2^23: exact int8 -> f32 (a pair at a time)
                const uint32_t wv = words[2 * u + (e >> 1)] ^ 0x80808080u;
                const int b0 = (e & 1) * 2;
                const uint64_t m = ((uint64_t)__byte_perm(wv, 0x4B000000u, 0x7540u | (b0 + 1)) << 32) |
                                   __byte_perm(wv, 0x4B000000u, 0x7540u | b0);
                split_pair2(f2_mul(f2_add(m, kMagicPair), scp), hv[e], lv[e]);
              }
              const uint32_t o = tile + sw_off(r, c32 * 4 + u);
              *reinterpret_cast<uint4*>(b_hi + o) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
              *reinterpret_cast<uint4*>(b_lo + o) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) mbar_arrive_cluster(cluster_addr(&conv[s], 0));
            else mbar_arrive(&conv[s]);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // warp w reads TMEM lanes 32 (w % 4) ..; with 8 epilogue warps, warps 2..5
    // take the tile's first half of 32-column chunks and warps 6..9 the second
    constexpr int EW = epi_warps<BN, Q8, FUSED>();
    constexpr int kCh = BN / 32 / (EW / 4);   // chunks per warp
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int c_begin = EW == 8 ? ((warp - 2) >> 2) * kCh : 0, c_end = c_begin + kCh;
    const Epilogue& e = args.epi;
    uint32_t local = 0;
    for (int u = walker; u < args.units; u += walkers) {
      const Unit w = decode<BN, BMT>(args, u);
      if (w.skip) continue;
      const uint32_t b = local & 1, tph = (local >> 1) & 1;
      ++local;
      const int m = w.m0 + (int)rank * BM + row;
      const bool row_in = m < w.m1;
      const bool direct = args.splits == 1;
      // output offset of this row (without the column part); the residual /
      // accumulate addend of the first chunk is loaded before the accumulator
      // is ready, the next chunk's while the current one is stored
      const long long rowoff = row_in && direct ? epi_offset(e, w.z, m, 0) : 0;
      float4 pre[2][8];
      const int n_first = w.n0 + c_begin * 32;
      if (row_in && direct && n_first < args.N)
        epi_prefetch(e, args.N, rowoff + (n_first / e.n_div) * e.n_s1 + (n_first % e.n_div), n_first, pre[0]);
      const bool ok = mbar_wait(&tfull[b], tph, args.err, kErrWaitAccum);
      tc_fence_after();
      const bool row_ok = ok && row_in;
      const uint32_t acc_tmem = tmem_base + b * kAccCols + ((uint32_t)(q * 32) << 16);
      if constexpr (FUSED) {
        if (e.mode == kEpiRopeQKV) {   // whole heads of 64 or 128 columns per tile
          if (e.rope.dh == 64) {
            epi_rope<BN, 2, PAIR>(e, m, w.n0, row_ok, args.N, acc_tmem, &tempty[b], lane);
          } else if constexpr (BN % 128 == 0) {
            epi_rope<BN, 4, PAIR>(e, m, w.n0, row_ok, args.N, acc_tmem, &tempty[b], lane);
          }
          continue;
        }
        if (e.mode == kEpiSwiGLU) {
          if constexpr (BN == 128 || BN == 256) epi_swiglu<BN, PAIR>(e, m, w.n0, row_ok, acc_tmem, &tempty[b], lane);
          continue;
        }
      }
      // split-K partial of split s: plain row-major [M][N] slab s of the workspace
      float* part = args.ws + (long long)(u % args.splits) * args.M * args.N + (long long)m * args.N;
      float lse_m = -INFINITY, lse_s = 0.f;   // kEpiStoreLse: running pair of the current 64-column group
      // one 32-column chunk: drain TMEM, store (or write the partial); the
      // addend of the following chunk is prefetched into `next`
      auto chunk = [&](int c, const float4 (&cur)[8], float4 (&next)[8]) {
        float v[32];
        tmem_ld32(acc_tmem + (uint32_t)(c * 32), v);
        if (c == c_end - 1) release_acc<PAIR>(&tempty[b], lane);   // accumulator read: back to the MMA issuer
        const int nc = w.n0 + c * 32;
        if (!row_ok || nc >= args.N) return;
        if constexpr (!Q8) {   // (the LM head's operands are planes; Q8_0 kernels keep their registers)
          if (e.mode == kEpiStoreLse) {
            // (max, sum exp) of this row's valid columns in the chunk, merged
            // with the other chunk of its 64-column group; written once per group
            float cm = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (nc + i < args.N) cm = fmaxf(cm, v[i]);
            // hardware exp2-based exponential (~2 ulp): these sums only set the
            // normaliser, far inside the loss tolerance, and the four epilogue
            // warps must keep pace with the main loop
            float cs = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (nc + i < args.N) cs += __expf(v[i] - cm);
            if ((c & 1) == 0) {
              lse_m = cm;
              lse_s = cs;
            } else {
              const float mm = fmaxf(lse_m, cm);
              lse_s = lse_s * __expf(lse_m - mm) + cs * __expf(cm - mm);
              lse_m = mm;
            }
            if ((c & 1) == 1 || nc + 32 >= args.N)
              e.lse_part[(long long)(nc >> 6) * args.M + m] = make_float2(lse_m, lse_s);
          }
        }
        if (!direct) {
          if (nc + 32 <= args.N && (args.N & 3) == 0) {   // float4 stores need 16-byte aligned rows
            float4* p4 = reinterpret_cast<float4*>(part + nc);
#pragma unroll
            for (int i = 0; i < 8; ++i) p4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (nc + i < args.N) part[nc + i] = v[i];
          }
        } else {
          if (c + 1 < c_end && nc + 32 < args.N)
            epi_prefetch(e, args.N, rowoff + ((nc + 32) / e.n_div) * e.n_s1 + ((nc + 32) % e.n_div), nc + 32, next);
          if constexpr (FUSED) {
            if (e.n_lora) lora_add(e, m, nc, v);
          }
          epi_store(e, args.N, rowoff + (nc / e.n_div) * e.n_s1 + (nc % e.n_div), nc, v, cur);
        }
      };
#pragma unroll 1
      for (int c = c_begin; c < c_end; c += 2) {   // (a warp's chunk count is odd for 192-wide tiles)
        chunk(c, pre[0], pre[1]);
        if (c + 1 < c_end) chunk(c + 1, pre[1], pre[0]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // a pair frees its TMEM together, after both CTAs are done with each
  // other's barriers and accumulators
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, Cfg<BN>::kTmemCols);
    else tmem_dealloc(tmem_base, Cfg<BN>::kTmemCols);
  }
}

// Split-K reduction: out(m, n) = epilogue(sum over s in order of ws[s][m][n]).
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N, Epilogue e) {
  griddep_wait();
  const long long n32 = (long long)M * ((N + 31) / 32);
  const long long slab = (long long)M * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n32; i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / ((N + 31) / 32));
    const int nc = (int)(i % ((N + 31) / 32)) * 32;
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = 0.f;
    const float* p = ws + (long long)m * N + nc;
    if (nc + 32 <= N && (N % 4) == 0) {
      for (int s = 0; s < splits; ++s) {
        const float4* p4 = reinterpret_cast<const float4*>(p + s * slab);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 x = __ldcs(p4 + k);
          v[4 * k] += x.x; v[4 * k + 1] += x.y; v[4 * k + 2] += x.z; v[4 * k + 3] += x.w;
        }
      }
    } else {
      for (int s = 0; s < splits; ++s)
        for (int k = 0; k < 32; ++k)
          if (nc + k < N) v[k] += p[s * slab + k];
    }
    float4 pre[8];
    const long long off = epi_offset(e, 0, m, nc);
    epi_prefetch(e, N, off, nc, pre);
    epi_store(e, N, off, nc, v, pre);
  }
}

// ------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor map over one bf16 plane: dims {cols, rows, nbatch}, box {64, box_rows, 1}, 128B swizzle.
int make_map(CUtensorMap* map, const __nv_bfloat16* base, const Operand& o, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return -10;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return -11;
  if ((o.ld * 2) % 16 != 0 || (o.batch_stride * 2) % 16 != 0) return -12;
  cuuint64_t dims[3] = {(cuuint64_t)o.cols, (cuuint64_t)o.rows, (cuuint64_t)(o.nbatch > 0 ? o.nbatch : 1)};
  cuuint64_t strides[2] = {(cuuint64_t)(o.ld * 2), (cuuint64_t)(o.batch_stride > 0 ? o.batch_stride * 2 : o.ld * 2 * o.rows)};
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -13;
}

// Tensor map over the int8 quants of a Q8_0 operand: dims {cols, rows, 1},
// row stride ld bytes, box {64 bytes, box_rows, 1}, no swizzle (the converters
// read it row by row). Rows / columns past the matrix read as zero.
int make_q8_map(CUtensorMap* map, const Operand& o, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return -10;
  if (reinterpret_cast<uintptr_t>(o.q8) % 16 != 0 || o.ld % 16 != 0) return -11;
  cuuint64_t dims[3] = {(cuuint64_t)o.cols, (cuuint64_t)o.rows, (cuuint64_t)(o.nbatch > 0 ? o.nbatch : 1)};
  cuuint64_t strides[2] = {(cuuint64_t)o.ld, (cuuint64_t)o.ld * o.rows};   // batches (experts) back to back
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(o.q8), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -13;
}

// Launch plan: tile width BN and number of K splits, chosen by a cost model
// (a pure function of the shape, so the choice -- and with it the summation
// order -- is the same on every run and every rank). Calibrated on this
// kernel's measured behaviour on B200: the main loop sustains ~1310 TFLOP/s
// of executed MMA work over 148 SMs; a CTA switching tiles costs ~0.5 us;
// filling the pipeline ~1.2 us; the last tile's epilogue drains its output at
// the CTA's share of HBM bandwidth; K splits add a reduction kernel that
// streams the partial slabs once. A k-block also cannot finish faster than
// its operand tiles arrive: ~82 GB/s per SM from L2 (~12 TB/s over the chip),
// which is what makes narrow tiles slow.
//
// These constants price a GEMM that shares the GPU with the weight-gradient
// stream of a full fine-tune's backward: the 96-CTA tiles they prefer for
// N = 576 leave SMs to that stream. A GEMM that has the GPU to itself (the
// forward, the backward of an adapter recipe: GemmDesc::alone) is priced with
// constants fitted to in-graph times of each of the step's shapes alone (M =
// 4096 tokens; forward, dX and dW products of the SmolLM2 projections; every
// tile width x K splits 1..8): ~8 us before the first k-block, up to ~1880
// TFLOP/s executed, ~121 GB/s of operand tiles per SM (MN-major ~12 %
// cheaper), 0.12 us per tile switch, an epilogue drain of ~44 GB/s per CTA
// (~4.3 TB/s over the chip), K-split reductions at ~2.7 TB/s + 0.5 us. Their
// picks are 4.5 % faster than these constants' on those shapes timed alone,
// but the full fine-tune's two-stream backward ran 0.7 % slower with them.
struct CostModel {
  double sm_flops_per_us, operand_bytes_per_us, mn_major_bytes, fill_us, switch_us, drain_cta, drain_total,
      split_bw, split_us;
};
constexpr CostModel kShared = {1310.0e6 / kNumSMs, 82.0e3, 1.0, 1.2, 0.5, 100.0e3, 6.5e6, 5.0e6, 2.5};
constexpr CostModel kAlone = {1880.0e6 / kNumSMs, 121.0e3, 0.88, 8.2, 0.12, 44.0e3, 4.25e6, 2.7e6, 0.5};

// Q8_0 B operand: elements the 8 converter warps dequantise and split per us
constexpr double kConvElemsPerUs = 6000.0;

double estimate_us(const GemmDesc& d, int bn, int s, bool pair, bool q8) {
  const CostModel& cm = d.alone ? kAlone : kShared;
  const int bmt = pair ? 2 * BM : BM;            // output rows of a unit
  const double slots = pair ? kNumSMs / 2 : kNumSMs;   // units in flight
  const int rb = pair ? bn / 2 : bn;              // B rows per CTA
  const int tm = (d.M + bmt - 1) / bmt, tn = (d.N + bn - 1) / bn;
  double tiles = (double)d.batch * tm * tn;
  int kb = (d.K + BK - 1) / BK;
  if (d.causal == 1) tiles *= (double)(tm + 1) / (2.0 * tm);   // tiles above the diagonal are skipped
  if (d.causal == 2) kb = kb / 2 + 1;                          // K clamped at the diagonal, on average
  const double units = tiles * s;
  const double per_cta = std::ceil(units / slots);
  const bool reads_out = d.epi.mode == kEpiAccumF32 || d.epi.mode == kEpiResidF32;
  // bytes the epilogue moves per output element: they share the SM's path to
  // L2 with the operand tiles of the next unit's main loop
  double out_b = (s == 1 && reads_out) ? 8.0 : 4.0;
  if (d.epi.mode == kEpiStoreBoth) out_b = 8.0;
  if (d.epi.mode == kEpiSwiGLU) out_b = 6.0;   // gate|up f32 + half of a feature's planes
  const double tile_bytes = (double)BM * bn * out_b;
  const double kb_unit = std::ceil((double)kb / s);
  const double planes = d.split ? 2.0 : 1.0;
  const double t_mma = (d.split ? 3.0 : 1.0) * 2.0 * BM * bn * BK / cm.sm_flops_per_us;
  const double b_bytes = (q8 ? (double)rb * BK : planes * rb * BK * 2.0) * (d.b.mn_major ? cm.mn_major_bytes : 1.0);
  const double a_bytes = planes * BM * BK * 2.0 * (d.a.mn_major ? cm.mn_major_bytes : 1.0);
  const double t_feed = (a_bytes + b_bytes + tile_bytes / kb_unit) / cm.operand_bytes_per_us;
  const double t_conv = q8 ? (double)rb * BK / kConvElemsPerUs : 0.0;
  const double t_kb = std::max(t_mma, std::max(t_feed, t_conv));
  const double active = (units < slots ? units : slots) * (pair ? 2 : 1);
  const double drain_bw = std::min(cm.drain_cta, cm.drain_total / active);   // bytes per us per CTA
  double t = cm.fill_us + per_cta * (kb_unit * t_kb + cm.switch_us) + tile_bytes / drain_bw;
  if (s > 1) t += ((s + 1.0) * d.M * d.N * 4.0 + (reads_out ? d.M * d.N * 4.0 : 0.0)) / cm.split_bw + cm.split_us;
  return t;
}

struct Plan {
  int bn = 128, splits = 1;
  bool pair = false;
};

// CTA pairs: -1 by shape (below), 0 never, 1 wherever the shape allows
int g_pair_mode = -1;
// output tile width: 0 by the cost model, else 64 / 128 / 192 / 256 wherever the shape allows it
int g_tile_bn = 0;

// Measured on B200 (SmolLM2 step shapes, M = 4096 tokens): a pair beats two
// single CTAs when both operands are K-major and N is wide -- the LM head
// (N = 49152: 746 -> 625 us), gate|up (N = 3072; Q8_0 with a plain store:
// 100 -> 75 us, the converter work per MMA halves). With N = 576 .. 960 the
// 256-row units leave half the pairs idle, with an MN-major B (dX products)
// the pair's cross-CTA stage hand-off costs more than it saves, and the Q8_0
// gate|up with its SwiGLU epilogue measured slower in the step (91 -> 103 us).
bool pair_wins(const GemmDesc& d) {
  return !d.a.mn_major && !d.b.mn_major && d.N >= 2048 && d.M >= 1024 && d.epi.mode != kEpiSwiGLU;
}

Plan choose_plan(const GemmDesc& d, long long ws_floats, bool q8) {
  static const int kBn[] = {64, 128, 192, 256};
  const int kb = (d.K + BK - 1) / BK;
  // fused epilogues act on whole output rows of a tile: no K splits
  const bool fused = d.epi.mode == kEpiRopeQKV || d.epi.mode == kEpiSwiGLU || d.epi.n_lora > 0;
  // the logsumexp epilogue reduces whole tile rows: no K splits either
  const bool can_split =
      !d.causal && d.batch == 1 && ws_floats > 0 && !fused && d.epi.mode != kEpiStoreLse && !d.group_tiles;
  const bool pair_ok = g_pair_mode != 0 && d.split && !d.causal && !d.group_tiles && (g_pair_mode == 1 || pair_wins(d));
  Plan best;
  double best_t = 1e30;
  auto search = [&](int force_bn) {
  for (int pr = 0; pr < 2; ++pr) {
    const bool pair = pr == 1;
    if (pair && !pair_ok) continue;
    if (!pair && pair_ok) continue;   // a shape that qualifies runs on pairs
    for (int bn : kBn) {
      if (force_bn && bn != force_bn) continue;
      if (pair && bn != 128 && bn != 256) continue;
      if (q8 && !pair && bn > 128) break;
      if (bn > 64 && bn - 64 >= d.N && !(pair && bn == 128)) break;   // a narrower tile already covers N
      if (d.epi.mode == kEpiSwiGLU && bn != 128 && bn != 256) continue;   // BN/2 gate + BN/2 up columns
      if (d.epi.mode == kEpiSwiGLU && q8 && !pair && bn != 128) continue;
      if (d.epi.mode == kEpiRopeQKV && bn % d.epi.rope.dh) continue;       // whole heads per tile
      // the logsumexp pairs 32-column chunks into 64-column groups: a 192-wide
      // tile's 8 epilogue warps would split a group between two warps
      if (d.epi.mode == kEpiStoreLse && bn == 192) continue;
      int s_lo = 1, s_hi = 1;
      if (d.splits > 0 && !fused && d.epi.mode != kEpiStoreLse && !d.group_tiles) {
        s_lo = s_hi = d.splits;
      } else if (can_split && kb >= 8) {
        s_hi = std::min(16, kb / 2);
      }
      for (int s = s_lo; s <= s_hi; ++s) {
        if (s > 1 && (long long)s * d.M * d.N > ws_floats) break;
        const double t = estimate_us(d, bn, s, pair, q8);
        if (t < best_t - 1e-9) {
          best_t = t;
          best.bn = bn;
          best.splits = s;
          best.pair = pair;
        }
      }
    }
  }
  };
  search(d.tile_bn ? d.tile_bn : g_tile_bn);
  if (best_t >= 1e30) search(0);   // the forced width does not fit this shape
  return best;
}

template <int BN, bool SPLIT, bool Q8 = false, bool FUSED = false, bool PAIR = false>
int launch_bn(const GemmDesc& d, const GemmScratch& sc, int* dev_err, cudaStream_t stream, int splits) {
  using S = Stages<BN, SPLIT, Q8, PAIR>;
  auto* kern = gemm_split_bf16_kernel<BN, SPLIT, Q8, FUSED, PAIR>;
  static DeviceOnce setup;
  static int max_pairs_of[64] = {};   // co-resident CTA pairs (clusters of 2) per GPU
  int dev_rc = setup.ensure([&](int dev) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes) != cudaSuccess)
      return -20;
    if (PAIR) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * kNumSMs);
      cfg.blockDim = dim3(threads_of<BN, Q8, FUSED>());
      cfg.dynamicSmemBytes = S::kSmemBytes;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int mp = 0;
      if (cudaOccupancyMaxActiveClusters(&mp, kern, &cfg) != cudaSuccess || mp < 1) return -22;
      max_pairs_of[dev] = mp;
    }
    return 0;
  });
  if (dev_rc) return dev_rc;
  int cur_dev = 0;
  cudaGetDevice(&cur_dev);
  const int max_pairs = max_pairs_of[cur_dev];
  CUtensorMap ma_hi, ma_lo, mb_hi, mb_lo;
  const int a_box = d.a.mn_major ? 64 : BM;
  // B box rows: a pair holds half of B's rows per CTA, paired gate|up rows are
  // fetched as two half-width boxes
  const int b_box = d.epi.pair_off ? BN / 2 : (d.b.mn_major ? 64 : Cfg<BN, PAIR>::kRowsB);
  int rc;
  if ((rc = make_map(&ma_hi, d.a.hi, d.a, a_box))) return rc;
  if (Q8) {
    if ((rc = make_q8_map(&mb_hi, d.b, b_box))) return rc;
  } else if ((rc = make_map(&mb_hi, d.b.hi, d.b, b_box))) {
    return rc;
  }
  if (SPLIT) {
    if ((rc = make_map(&ma_lo, d.a.lo, d.a, a_box))) return rc;
    if (Q8) mb_lo = mb_hi;
    else if ((rc = make_map(&mb_lo, d.b.lo, d.b, b_box))) return rc;
  } else {
    ma_lo = ma_hi;
    mb_lo = mb_hi;
  }
  KArgs k;
  k.M = d.M; k.N = d.N; k.K = d.K; k.batch = d.batch;
  k.a_mn = d.a.mn_major; k.b_mn = d.b.mn_major;
  k.a_bdiv1 = d.a.bdiv1; k.a_bmul1 = d.a.bmul1; k.a_bdiv2 = d.a.bdiv2; k.a_bmul2 = d.a.bmul2;
  k.b_bdiv1 = d.b.bdiv1; k.b_bmul1 = d.b.bmul1; k.b_bdiv2 = d.b.bdiv2; k.b_bmul2 = d.b.bmul2;
  k.tiles_m = d.group_tiles ? d.group_mtiles : (d.M + (PAIR ? 2 : 1) * BM - 1) / ((PAIR ? 2 : 1) * BM);
  k.gtab = d.group_tiles;
  k.tiles_n = (d.N + BN - 1) / BN;
  k.kb_total = (d.K + BK - 1) / BK;
  k.causal = d.causal;
  k.f16 = d.f16 ? 1 : 0;
  const long long tiles = (long long)d.batch * k.tiles_m * k.tiles_n;
  if (splits < 1 || d.epi.mode == kEpiStoreLse || d.group_tiles) splits = 1;
  if (splits > k.kb_total) splits = k.kb_total;
  if (splits > 1 && (d.causal || d.batch != 1 || !sc.ws || (long long)splits * d.M * d.N > sc.ws_floats))
    splits = 1;
  if (tiles * splits > (1LL << 31) - 1) return -5;
  k.splits = splits;
  k.units = (int)(tiles * splits);
  k.epi = d.epi;
  k.ws = sc.ws;
  k.b_keep = d.b.l2_keep && !Q8;
  k.err = dev_err;
  k.q8_scale = d.b.q8_scale;
  k.q8_rows = d.b.rows;
  k.q8_cols = d.b.cols;
  if constexpr (PAIR) {
    int pairs = k.units < max_pairs ? k.units : max_pairs;
    if (d.max_ctas >= 2 && pairs > d.max_ctas / 2) pairs = d.max_ctas / 2;
    if (launch_pdl_cluster(kern, dim3(2 * pairs), dim3(threads_of<BN, Q8, FUSED>()), S::kSmemBytes, stream, 2, ma_hi,
                           ma_lo, mb_hi, mb_lo, k) != 0)
      return -21;
  } else {
    int grid = k.units < kNumSMs ? k.units : kNumSMs;
    if (d.max_ctas > 0 && grid > d.max_ctas) grid = d.max_ctas;
    if (launch_pdl(kern, dim3(grid), dim3(threads_of<BN, Q8, FUSED>()), S::kSmemBytes, stream, ma_hi, ma_lo, mb_hi, mb_lo,
                   k) != 0)
      return -21;
  }
  t_last_launches = 1;
  if (splits > 1) {
    const long long work = (long long)d.M * ((d.N + 31) / 32);
    long long blocks = (work + 127) / 128;
    if (blocks > 8 * kNumSMs) blocks = 8 * kNumSMs;
    if (launch_pdl(splitk_reduce_kernel, dim3((int)blocks), dim3(128), 0, stream, sc.ws, splits, d.M, d.N, d.epi) != 0)
      return -21;
    t_last_launches = 2;
  }
  return 0;
}

}  // namespace

int gemm_set_pair_mode(int mode) {
  if (mode < -1 || mode > 1) return -1;
  g_pair_mode = mode;
  return 0;
}

int gemm_set_tile_width(int bn) {
  if (bn != 0 && bn != 64 && bn != 128 && bn != 192 && bn != 256) return -1;
  const int prev = g_tile_bn;
  g_tile_bn = bn;
  return prev;
}

int make_plane_map(CUtensorMap* map, const __nv_bfloat16* base, const Operand& o, int box_rows) {
  return make_map(map, base, o, box_rows);
}

int gemm_effective_splits(const GemmDesc& d, int ksplits) {
  const Epilogue& e = d.epi;
  const bool fused = e.mode == kEpiRopeQKV || e.mode == kEpiSwiGLU || e.n_lora > 0;
  if (ksplits <= 1 || d.causal || d.batch != 1 || fused || e.mode == kEpiStoreLse) return 1;
  const int kb = (d.K + BK - 1) / BK;
  return ksplits < kb ? ksplits : kb;
}

int gemm_last_launches() { return t_last_launches; }

int gemm_launch(const GemmDesc& d, const GemmScratch& sc, int* dev_err, cudaStream_t stream) {
  t_last_launches = 0;
  if (d.M <= 0 || d.N <= 0 || d.K <= 0 || d.batch <= 0) return -1;
  if (d.causal < 0 || d.causal > 2) return -1;
  if (d.group_tiles && (d.group_mtiles < 1 || d.causal || d.batch != 1 || d.a.mn_major)) return -1;
  if (!d.group_tiles && d.group_mtiles) return -1;
  // Epilogue vector stores need 16-byte aligned rows.
  const Epilogue& e = d.epi;
  const int al = (e.mode == kEpiStoreSplit || e.mode == kEpiStoreBoth) ? 8 : 4;
  if ((e.m_s0 % al) || (e.m_s1 % al) || (e.n_s1 % al) || (e.bstride % al) || (e.z_s1 % al) || (e.n_div % 32))
    return -3;
  if (e.n_lora < 0 || e.n_lora > kMaxLoraAddends || (e.n_lora && e.alpha != 1.0f)) return -3;
  // the device factor scales the plain stores only
  if (e.alpha_dev && (e.n_lora || e.mode == kEpiRopeQKV || e.mode == kEpiSwiGLU || e.mode == kEpiStoreLse)) return -3;
  // fp16 operands: one pass over plain (non-Q8_0) single planes
  if (d.f16 && (d.split || d.b.q8)) return -4;
  for (int i = 0; i < e.n_lora; ++i) {
    const LoraAddend& L = e.lora[i];
    if (!L.u || !L.bt || L.r < 1 || L.c0 % 32 || L.width % 32 || L.c0 + L.width > d.N ||
        (reinterpret_cast<uintptr_t>(L.bt) & 15))
      return -3;
  }
  if (e.mode == kEpiRopeQKV) {
    const RopeOut& R = e.rope;
    if ((R.dh != 64 && R.dh != 128) || d.N != (R.H + 2 * R.KV) * R.dh || d.M % R.T || !R.pos || !R.cs ||
        !R.q_hi || !R.q_lo || !R.k_hi || !R.k_lo || !R.v_hi || !R.v_lo || d.batch != 1)
      return -3;
  }
  if (e.mode == kEpiSwiGLU) {
    if (e.pair_off <= 0 || d.N != 2 * e.pair_off || e.pair_off % 64 || d.b.mn_major || d.batch != 1 || !e.out ||
        !e.out_hi || !e.out_lo || e.m_s0 != 2LL * e.pair_off)
      return -3;
  } else if (e.pair_off) {
    return -3;
  }
  if (e.mode == kEpiStoreLse && (!e.lse_part || e.alpha != 1.0f || d.batch != 1 || e.m_div != (1 << 30) ||
                                 e.n_div != (1 << 30) || d.b.q8))
    return -3;
  const bool fused = e.mode == kEpiRopeQKV || e.mode == kEpiSwiGLU || e.n_lora > 0;
  if (fused && !d.split) return -3;
  const Plan pl = choose_plan(d, sc.ws ? sc.ws_floats : 0, d.b.q8 != nullptr);
  if (d.b.q8 && (!d.split || d.batch != 1 || !d.b.q8_scale || d.b.cols % 32 || !d.a.hi || !d.a.lo)) return -4;
  if (!d.b.q8 && (!d.a.hi || !d.b.hi || (d.split && (!d.a.lo || !d.b.lo)))) return -4;
  if (pl.pair) {   // CTA pairs: 256-row units, 128 / 256-wide tiles, split planes
    const int sp = pl.splits;
    const bool w = pl.bn == 256;
    if (d.b.q8) {
      if (fused) return w ? launch_bn<256, true, true, true, true>(d, sc, dev_err, stream, sp)
                          : launch_bn<128, true, true, true, true>(d, sc, dev_err, stream, sp);
      return w ? launch_bn<256, true, true, false, true>(d, sc, dev_err, stream, sp)
               : launch_bn<128, true, true, false, true>(d, sc, dev_err, stream, sp);
    }
    if (fused) return w ? launch_bn<256, true, false, true, true>(d, sc, dev_err, stream, sp)
                        : launch_bn<128, true, false, true, true>(d, sc, dev_err, stream, sp);
    return w ? launch_bn<256, true, false, false, true>(d, sc, dev_err, stream, sp)
             : launch_bn<128, true, false, false, true>(d, sc, dev_err, stream, sp);
  }
  if (d.b.q8) {
    // Q8_0 B: dequantised in shared memory into split planes; 64 / 128-wide tiles
    // keep three stages of A planes + B planes + quants within shared memory
    if (fused)
      return pl.bn <= 64 ? launch_bn<64, true, true, true>(d, sc, dev_err, stream, pl.splits)
                         : launch_bn<128, true, true, true>(d, sc, dev_err, stream, pl.splits);
    return pl.bn <= 64 ? launch_bn<64, true, true>(d, sc, dev_err, stream, pl.splits)
                       : launch_bn<128, true, true>(d, sc, dev_err, stream, pl.splits);
  }
  const int sp = pl.splits;
  if (fused) {
    switch (pl.bn) {
      case 64: return launch_bn<64, true, false, true>(d, sc, dev_err, stream, sp);
      case 128: return launch_bn<128, true, false, true>(d, sc, dev_err, stream, sp);
      case 192: return launch_bn<192, true, false, true>(d, sc, dev_err, stream, sp);
      default: return launch_bn<256, true, false, true>(d, sc, dev_err, stream, sp);
    }
  }
  switch (pl.bn) {
    case 64:
      return d.split ? launch_bn<64, true>(d, sc, dev_err, stream, sp) : launch_bn<64, false>(d, sc, dev_err, stream, sp);
    case 128:
      return d.split ? launch_bn<128, true>(d, sc, dev_err, stream, sp)
                     : launch_bn<128, false>(d, sc, dev_err, stream, sp);
    case 192:
      return d.split ? launch_bn<192, true>(d, sc, dev_err, stream, sp)
                     : launch_bn<192, false>(d, sc, dev_err, stream, sp);
    default:
      return d.split ? launch_bn<256, true>(d, sc, dev_err, stream, sp)
                     : launch_bn<256, false>(d, sc, dev_err, stream, sp);
  }
}

}  // namespace tb2
