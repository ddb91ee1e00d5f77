// Fused causal attention forward and backward on tcgen05 (sm_100a).
//
// Every product runs on split-bf16 operands with three UMMAs per k-step
// (hi*hi + lo*hi + hi*lo, f32 accumulate in TMEM), like the GEMM in gemm.cu.
// At head width 64, tiles are 128 rows x 64 head columns (head width 128:
// see the second half of this file); one [128 x 64] bf16 plane tile is a
// 16 KB block in the TMA 128-byte swizzle layout (row r at r * 128 bytes, its
// 16-byte chunk c stored at chunk c ^ (r % 8)). The same tile serves as a
// K-major operand (rows = M or N, head columns = K) and as an MN-major operand
// (rows = K, head columns = N), so Q, K, V and dO are loaded once per use.
//
// CTA = 10 warps: warp 0 issues TMA loads, warp 1 allocates TMEM and issues
// the UMMAs, warps 2..9 do the softmax arithmetic. A warp may only touch the
// 32 TMEM lanes of its quarter (warp % 4), so each quarter -- 32 query rows in
// the forward, 32 key rows in the backward -- is served by two warps, one per
// 64-column half of the 128-column score tile. Probability / score-gradient
// tiles go from registers to shared memory in the swizzled layout and feed the
// next UMMA directly; nothing of size T x T reaches HBM.
//
// Forward (per sequence, head, query tile of 128): one pass over the key tiles
// 0..qi with a running row maximum m. For each tile the softmax warps take the
// tile's row maxima (the two warps of a row quarter exchange theirs), and once
// the previous O += P V has completed they scale their O columns in TMEM by
// exp(m_old - m_new) when the maximum grew, write P = exp(S - m) to shared
// memory and add it to the running row sums (scaled alike); the MMA issuer
// then accumulates O += P V. The epilogue divides O by the sum. The scores of
// the next key tile are computed while the softmax warps work on the current
// one (two TMEM score buffers).
//
// Backward (per sequence, query head, key tile j of 128), over the query tiles
// i = j .. : dP^T = V dO^T and S^T = K Q^T in TMEM; the softmax warps write
// P^T to shared memory and park dS^T = P^T (dP^T - D) * scale in the S^T
// columns; dV += P^T dO; then dS^T moves to the same shared buffer, dK += dS^T Q
// and dQ_i = dS K (the dS^T tile read MN-major).
// dQ_i leaves through one of two TMEM buffers as this key tile's partial; dK
// and dV leave at the end as this query head's partial. The RoPE backward
// kernel sums the partials in a fixed order, so the result is deterministic.
#include "flash_attn.cuh"

#include "gemm.cuh"
#include "pdl.cuh"
#include "runtime.cuh"
#include "tc_common.cuh"

#include <cmath>

namespace tb2 {

namespace {

constexpr int kTile = 128;                 // query / key rows per tile
constexpr int kDh = 64;                    // head width
constexpr int kPlane = kTile * kDh * 2;    // one [128 x 64] bf16 plane tile: 16 KB
constexpr int kSoftWarps = 8;              // two per TMEM lane quarter, one per 64-column half
constexpr int kThreads = 32 * (2 + kSoftWarps);
constexpr int kRing = 3;                   // forward key/value stages

// forward: Q, ring, P, then the row max / row sum exchange between column halves
constexpr int kFwdSmem = (2 + 2 * kRing + 4) * kPlane + 6 * kTile * 4 + 1024 + 256;
// backward: K, V, Q, dO, P^T / dS^T, then per-warp lse2 / D staging
constexpr int kBwdSmem = (8 + 4) * kPlane + kSoftWarps * 2 * 64 * 4 + 1024 + 256;

struct FwdArgs {
  int B, T, H, KV, G, nq;
  float scale_log2;
  bf16* o_hi;
  bf16* o_lo;
  __half* o16;      // optional fp16 copy of O (same offsets)
  long long o_ld;   // token-major O row pitch
  float* lse2;
  int* err;
};

struct BwdArgs {
  int B, T, H, KV, G, nq;
  float scale_log2, scale;
  const float* lse2;
  const float* Dv;
  float* dq_part;
  float* dk_part;
  float* dv_part;
  int* err;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void split8(const float (&v)[32], int u, uint4& h, uint4& l) {
  split_pair(v[8 * u], v[8 * u + 1], h.x, l.x);
  split_pair(v[8 * u + 2], v[8 * u + 3], h.y, l.y);
  split_pair(v[8 * u + 4], v[8 * u + 5], h.z, l.z);
  split_pair(v[8 * u + 6], v[8 * u + 7], h.w, l.w);
}

// Store 32 values as columns c*32 .. c*32+31 (c = 0, 1) of row `row` of one
// swizzled [128 x 64] tile per plane (hi tile th, lo tile tl).
__device__ __forceinline__ void store_row32(uint8_t* th, uint8_t* tl, int row, int c, const float (&v)[32]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint4 h, l;
    split8(v, u, h, l);
    const uint32_t off = sw_off(row, c * 4 + u);
    *reinterpret_cast<uint4*>(th + off) = h;
    *reinterpret_cast<uint4*>(tl + off) = l;
  }
}

// 32 values as planes at 16-byte aligned global addresses.
__device__ __forceinline__ void store_planes32(bf16* hi, bf16* lo, const float (&v)[32]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint4 h, l;
    split8(v, u, h, l);
    reinterpret_cast<uint4*>(hi)[u] = h;
    reinterpret_cast<uint4*>(lo)[u] = l;
  }
}

// 32 values as fp16 (saturated to +-65504) at a 16-byte aligned address.
__device__ __forceinline__ void store_f16x32(__half* dst, const float (&v)[32]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    __align__(16) __half q[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float x = v[8 * u + k];
      q[k] = __float2half_rn(x > 65504.f ? 65504.f : (x < -65504.f ? -65504.f : x));
    }
    reinterpret_cast<uint4*>(dst)[u] = *reinterpret_cast<const uint4*>(q);
  }
}

__device__ __forceinline__ void store_f32x32(float* dst, const float (&v)[32]) {
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int u = 0; u < 8; ++u) d4[u] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
}

// acc (+)= A * B^T over K = 16 * nsteps with split operands (three UMMAs per
// k-step). A K-major operand spans K in 64-column tiles `a_tile` / `b_tile`
// bytes apart (the tile's rows x 128 bytes); an MN-major operand holds K as
// rows of 128 bytes, with MN atoms `lbo` bytes apart.
__device__ __forceinline__ void mma_split_t(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t a_lbo, bool a_mn,
                                            uint32_t a_tile, uint32_t b_hi, uint32_t b_lo, uint32_t b_lbo, bool b_mn,
                                            uint32_t b_tile, uint32_t idesc, int nsteps, bool accumulate) {
#pragma unroll 1
  for (int ks = 0; ks < nsteps; ++ks) {
    // K-major: 32 B per 16 columns inside a tile, next tile every 4 steps.
    // MN-major: 16 rows of 128 B per step.
    const uint32_t ao = a_mn ? (uint32_t)ks * 2048u : (uint32_t)(ks >> 2) * a_tile + (uint32_t)(ks & 3) * 32u;
    const uint32_t bo = b_mn ? (uint32_t)ks * 2048u : (uint32_t)(ks >> 2) * b_tile + (uint32_t)(ks & 3) * 32u;
    const uint64_t dah = make_sdesc_sw128(a_hi + ao, a_lbo, 1024), dal = make_sdesc_sw128(a_lo + ao, a_lbo, 1024);
    const uint64_t dbh = make_sdesc_sw128(b_hi + bo, b_lbo, 1024), dbl = make_sdesc_sw128(b_lo + bo, b_lbo, 1024);
    umma_f16(d, dah, dbh, idesc, (accumulate || ks > 0) ? 1u : 0u);
    umma_f16(d, dal, dbh, idesc, 1u);
    umma_f16(d, dah, dbl, idesc, 1u);
  }
}

// mma_split_t on [128 x 64] K-major tiles.
__device__ __forceinline__ void mma_split(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t a_lbo, bool a_mn,
                                          uint32_t b_hi, uint32_t b_lo, uint32_t b_lbo, bool b_mn, uint32_t idesc,
                                          int nsteps, bool accumulate) {
  mma_split_t(d, a_hi, a_lo, a_lbo, a_mn, kPlane, b_hi, b_lo, b_lbo, b_mn, kPlane, idesc, nsteps, accumulate);
}

// ------------------------------------------------------------------ forward
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap mq_hi, const __grid_constant__ CUtensorMap mq_lo,
                     const __grid_constant__ CUtensorMap mk_hi, const __grid_constant__ CUtensorMap mk_lo,
                     const __grid_constant__ CUtensorMap mv_hi, const __grid_constant__ CUtensorMap mv_lo,
                     const FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem;                          // Q hi, Q lo
  uint8_t* sRing = sQ + 2 * kPlane;            // kRing x (hi, lo) key or value tiles
  uint8_t* sP = sRing + 2 * kRing * kPlane;    // P hi (2 tiles), P lo (2 tiles)
  float* xmax = reinterpret_cast<float*>(sP + 4 * kPlane);   // [tile parity][column half][128] tile maxima
  float* xsum = xmax + 4 * kTile;                             // [2][128]
  uint64_t* bar = reinterpret_cast<uint64_t*>(xsum + 2 * kTile);
  uint64_t* q_full = bar;
  uint64_t* r_full = bar + 1;
  uint64_t* r_empty = r_full + kRing;
  uint64_t* s_full = r_empty + kRing;   // [2]
  uint64_t* s_empty = s_full + 2;       // [2]
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 1;
  uint64_t* o_full = p_empty + 1;
  uint64_t* sum_done = o_full + 1;   // both halves' row sums written
  uint64_t* mx_q = o_full + 2;       // [4] per row quarter: both halves' tile maxima written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 6);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int BH = a.B * a.H;
  const int bh = blockIdx.x % BH;
  const int qi = a.nq - 1 - blockIdx.x / BH;   // longest query tiles first
  const int b = bh / a.H, h = bh % a.H;
  const int bkv = b * a.KV + h / a.G;
  const int n = qi + 1;                        // key tiles 0 .. qi

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], kSoftWarps);
    }
    mbar_init(p_full, kSoftWarps);
    mbar_init(p_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(sum_done, kSoftWarps);
    for (int q = 0; q < 4; ++q) mbar_init(&mx_q[q], 2);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;   // S buffers at columns 0 and 128, O at 256
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Ring order: K_0 and, for each j, K_{j+1} (if any) followed by V_j --
    // the order the MMA issuer consumes.
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * kPlane);
      tma_load_3d(sQ, &mq_hi, q_full, 0, qi * kTile, bh);
      tma_load_3d(sQ + kPlane, &mq_lo, q_full, 0, qi * kTile, bh);
      uint32_t it = 0;
      auto push = [&](const CUtensorMap* mh, const CUtensorMap* ml, int j) -> bool {
        const int s = it % kRing;
        const uint32_t ph = (it / kRing) & 1;
        ++it;
        if (!mbar_wait(&r_empty[s], ph ^ 1, a.err, kErrWaitEmpty)) return false;
        uint8_t* dst = sRing + s * 2 * kPlane;
        mbar_arrive_expect_tx(&r_full[s], 2 * kPlane);
        tma_load_3d(dst, mh, &r_full[s], 0, j * kTile, bkv);
        tma_load_3d(dst + kPlane, ml, &r_full[s], 0, j * kTile, bkv);
        return true;
      };
      bool ok = push(&mk_hi, &mk_lo, 0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) ok = push(&mk_hi, &mk_lo, j + 1);
        if (ok) ok = push(&mv_hi, &mv_lo, j);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_s = make_idesc_f16(kTile, kTile, true, false, false);
      const uint32_t id_o = make_idesc_f16(kTile, kDh, true, false, true);
      const uint32_t q_hi = smem_u32(sQ), q_lo = q_hi + kPlane;
      const uint32_t p_hi = smem_u32(sP), p_lo = p_hi + 2 * kPlane;
      uint32_t it = 0, sc = 0;
      bool ok = mbar_wait(q_full, 0, a.err, kErrWaitFull);
      tc_fence_after();
      // S = Q K^T for the next ring item, into score buffer sc % 2
      auto issue_s = [&]() -> bool {
        const int s = it % kRing;
        const uint32_t ph = (it / kRing) & 1;
        ++it;
        const uint32_t sb = sc & 1, sph = (sc >> 1) & 1;
        ++sc;
        if (!mbar_wait(&s_empty[sb], sph ^ 1, a.err, kErrWaitAccum)) return false;
        if (!mbar_wait(&r_full[s], ph, a.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t k_hi = smem_u32(sRing + s * 2 * kPlane), k_lo = k_hi + kPlane;
        mma_split(tmem + sb * kTile, q_hi, q_lo, 16, false, k_hi, k_lo, 16, false, id_s, kDh / 16, false);
        umma_commit(&r_empty[s]);
        umma_commit(&s_full[sb]);
        return true;
      };
      if (ok) ok = issue_s();   // key tile 0
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) ok = issue_s();
        if (!ok) break;
        // O += P_j V_j: P K-major over the 128 keys, V MN-major (keys = K rows)
        const int s = it % kRing;
        const uint32_t ph = (it / kRing) & 1;
        ++it;
        ok = mbar_wait(&r_full[s], ph, a.err, kErrWaitFull) && mbar_wait(p_full, j & 1, a.err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        const uint32_t v_hi = smem_u32(sRing + s * 2 * kPlane), v_lo = v_hi + kPlane;
        mma_split(tmem + 2 * kTile, p_hi, p_lo, 16, false, v_hi, v_lo, 2 * kPlane, true, id_o, kTile / 16, j > 0);
        umma_commit(&r_empty[s]);
        umma_commit(p_empty);
      }
      if (ok) umma_commit(o_full);
    }
  } else {
    // -------------------------------------------------------- softmax warps
    const int sw = warp - 2;
    const int qw = warp & 3;     // TMEM lane quarter this warp may access
    const int half = sw >> 2;    // score columns half * 64 .. half * 64 + 63
    const int row = qw * 32 + lane;
    const int qrow = qi * kTile + row;
    const uint32_t lanes = (uint32_t)(qw * 32) << 16;
    uint32_t sc = 0;
    bool ok = true;
    float m = -INFINITY;   // the raw-score maximum every P of this row is relative to
    float l = 0.f;         // this half's sum of P
    uint8_t* th = sP + half * kPlane;
    uint8_t* tl = sP + (2 + half) * kPlane;
    // Every tile is walked even after a failed wait, so both warps of a quarter
    // arrive on its exchange barrier the same number of times.
    for (int j = 0; j < n; ++j, ++sc) {
      const uint32_t sb = sc & 1, sph = (sc >> 1) & 1;
      ok = ok && warp_wait(&s_full[sb], sph, a.err, kErrWaitAccum);
      tc_fence_after();
      // this half's 64 raw scores and their maximum over the live keys (k <= q,
      // k < T); only the diagonal tile (also a ragged last tile) needs the mask
      const bool mask = j == qi;
      float v[2][32];
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (ok) tmem_ld32(tmem + lanes + sb * kTile + half * 64 + c * 32, v[c]);
        const int k0 = j * kTile + half * 64 + c * 32;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const bool live = !mask || (k0 + e <= qrow && k0 + e < a.T);
          if (!ok) v[c][e] = 0.f;
          if (live) mt = fmaxf(mt, v[c][e]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&s_empty[sb]);   // the scores are in registers
      // the row's tile maximum over both halves
      float* xm = xmax + (j & 1) * 2 * kTile;
      xm[half * kTile + row] = mt;
      __syncwarp();
      if (lane == 0) mbar_arrive(&mx_q[qw]);
      ok = ok && warp_wait(&mx_q[qw], j & 1, a.err, kErrWaitAccum);
      const float m_new = fmaxf(m, fmaxf(mt, xm[(half ^ 1) * kTile + row]));
      const bool grow = j > 0 && m_new > m;
      const float alpha = grow ? ex2((m - m_new) * a.scale_log2) : 1.f;
      m = m_new;
      const float mb = m * a.scale_log2;   // p = exp2(S * scale_log2 - mb); scale_log2 > 0
      // the P buffer is free and O final for tiles < j once O += P_{j-1} V_{j-1} completed
      ok = ok && warp_wait(p_empty, (j & 1) ^ 1, a.err, kErrWaitAccum);
      tc_fence_after();
      if (ok && __any_sync(0xffffffffu, grow)) {   // O *= alpha on this warp's 32 rows x 32 columns
        float o[32];
        tmem_ld32(tmem + lanes + 2 * kTile + half * 32, o);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= alpha;
        tmem_st32(tmem + lanes + 2 * kTile + half * 32, o);
        tmem_wait_st();
      }
      l *= alpha;
      if (ok) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int k0 = j * kTile + half * 64 + c * 32;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float p = ex2(fmaf(v[c][e], a.scale_log2, -mb));
            if (mask && !(k0 + e <= qrow && k0 + e < a.T)) p = 0.f;
            v[c][e] = p;
            l += p;
          }
          store_row32(th, tl, row, c, v[c]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(p_full);
    }
    const float mb = m * a.scale_log2;
    xsum[half * kTile + row] = l;
    __syncwarp();
    if (lane == 0) mbar_arrive(sum_done);
    ok = ok && warp_wait(sum_done, 0, a.err, kErrWaitAccum) && warp_wait(o_full, 0, a.err, kErrWaitAccum);
    tc_fence_after();
    if (ok) {
      // this half's 32 of the 64 output columns, divided by the row sum
      const float lt = xsum[row] + xsum[kTile + row];
      const float inv = lt > 0.f ? 1.0f / lt : 0.f;
      float o[32];
      tmem_ld32(tmem + lanes + 2 * kTile + half * 32, o);
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] *= inv;
      if (qrow < a.T) {
        const long long off = (long long)(b * a.T + qrow) * a.o_ld + h * kDh + half * 32;
        store_planes32(a.o_hi + off, a.o_lo + off, o);
        if (a.o16) store_f16x32(a.o16 + off, o);
        if (half == 0) a.lse2[(long long)bh * a.T + qrow] = mb + log2f(lt);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ backward
__global__ void __launch_bounds__(kThreads, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap mq_hi, const __grid_constant__ CUtensorMap mq_lo,
                     const __grid_constant__ CUtensorMap mk_hi, const __grid_constant__ CUtensorMap mk_lo,
                     const __grid_constant__ CUtensorMap mv_hi, const __grid_constant__ CUtensorMap mv_lo,
                     const __grid_constant__ CUtensorMap mo_hi, const __grid_constant__ CUtensorMap mo_lo,
                     const BwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sK = smem;                  // K hi, lo
  uint8_t* sV = sK + 2 * kPlane;       // V hi, lo
  uint8_t* sQ = sV + 2 * kPlane;       // Q_i hi, lo
  uint8_t* sO = sQ + 2 * kPlane;       // dO_i hi, lo
  uint8_t* sP = sO + 2 * kPlane;       // P^T then dS^T: hi (2 tiles), lo (2 tiles)
  float* s_vec = reinterpret_cast<float*>(sP + 4 * kPlane);   // per softmax warp: lse2[64], D[64]
  uint64_t* bar = reinterpret_cast<uint64_t*>(s_vec + kSoftWarps * 2 * 64);
  uint64_t* kv_full = bar;
  uint64_t* q_full = bar + 1;
  uint64_t* q_empty = bar + 2;
  uint64_t* o_full = bar + 3;
  uint64_t* o_empty = bar + 4;
  uint64_t* sdp_full = bar + 5;
  uint64_t* sdp_empty = bar + 6;
  uint64_t* p_full = bar + 7;
  uint64_t* p_used = bar + 8;
  uint64_t* ds_full = bar + 9;
  uint64_t* ds_used = bar + 10;
  uint64_t* dq_full = bar + 11;    // [2]
  uint64_t* dq_empty = bar + 13;   // [2]
  uint64_t* acc_full = bar + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 16);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int BH = a.B * a.H;
  const int bh = blockIdx.x % BH;
  const int j = blockIdx.x / BH;       // key tile; j = 0 has the most query tiles
  const int b = bh / a.H, h = bh % a.H;
  const int bkv = b * a.KV + h / a.G;
  const int n_it = a.nq - j;           // query tiles i = j .. nq - 1

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 1);
    mbar_init(sdp_full, 1);
    mbar_init(sdp_empty, kSoftWarps);
    mbar_init(p_full, kSoftWarps);
    mbar_init(p_used, 1);
    mbar_init(ds_full, kSoftWarps);
    mbar_init(ds_used, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&dq_full[s], 1);
      mbar_init(&dq_empty[s], kSoftWarps);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // TMEM columns: S^T 0, dP^T 128, dV 256, dK 320, dQ buffers 384 and 448
  const uint32_t tmem = *tmem_slot;
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 4 * kPlane);
      tma_load_3d(sK, &mk_hi, kv_full, 0, j * kTile, bkv);
      tma_load_3d(sK + kPlane, &mk_lo, kv_full, 0, j * kTile, bkv);
      tma_load_3d(sV, &mv_hi, kv_full, 0, j * kTile, bkv);
      tma_load_3d(sV + kPlane, &mv_lo, kv_full, 0, j * kTile, bkv);
      for (int it = 0; it < n_it; ++it) {
        const int i = j + it;
        const uint32_t ph = (it & 1) ^ 1;
        if (!mbar_wait(q_empty, ph, a.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(q_full, 2 * kPlane);
        tma_load_3d(sQ, &mq_hi, q_full, 0, i * kTile, bh);
        tma_load_3d(sQ + kPlane, &mq_lo, q_full, 0, i * kTile, bh);
        if (!mbar_wait(o_empty, ph, a.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(o_full, 2 * kPlane);
        tma_load_3d(sO, &mo_hi, o_full, 0, i * kTile, bh);
        tma_load_3d(sO + kPlane, &mo_lo, o_full, 0, i * kTile, bh);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_s = make_idesc_f16(kTile, kTile, true, false, false);
      const uint32_t id_kv = make_idesc_f16(kTile, kDh, true, false, true);   // dV, dK: B (dO, Q) MN-major
      const uint32_t id_q = make_idesc_f16(kTile, kDh, true, true, true);     // dQ: A (dS) and B (K) MN-major
      const uint32_t k_hi = smem_u32(sK), k_lo = k_hi + kPlane;
      const uint32_t v_hi = smem_u32(sV), v_lo = v_hi + kPlane;
      const uint32_t q_hi = smem_u32(sQ), q_lo = q_hi + kPlane;
      const uint32_t o_hi = smem_u32(sO), o_lo = o_hi + kPlane;
      const uint32_t p_hi = smem_u32(sP), p_lo = p_hi + 2 * kPlane;
      bool ok = mbar_wait(kv_full, 0, a.err, kErrWaitFull);
      for (int it = 0; it < n_it && ok; ++it) {
        const uint32_t ph = it & 1;
        // dO_i arrives first (its slot frees after dV), so dP^T goes before S^T
        ok = mbar_wait(o_full, ph, a.err, kErrWaitFull) && mbar_wait(sdp_empty, ph ^ 1, a.err, kErrWaitAccum);
        if (!ok) break;
        tc_fence_after();
        mma_split(tmem + kTile, v_hi, v_lo, 16, false, o_hi, o_lo, 16, false, id_s, kDh / 16, false);   // dP^T
        ok = mbar_wait(q_full, ph, a.err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        mma_split(tmem, k_hi, k_lo, 16, false, q_hi, q_lo, 16, false, id_s, kDh / 16, false);           // S^T
        umma_commit(sdp_full);
        ok = mbar_wait(p_full, ph, a.err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        // dV += P^T dO   (K = the 128 queries)
        mma_split(tmem + 2 * kTile, p_hi, p_lo, 16, false, o_hi, o_lo, 2 * kPlane, true, id_kv, kTile / 16,
                  it > 0);
        umma_commit(p_used);
        umma_commit(o_empty);
        ok = mbar_wait(ds_full, ph, a.err, kErrWaitFull) &&
             mbar_wait(&dq_empty[it & 1], ((it >> 1) & 1) ^ 1, a.err, kErrWaitAccum);
        if (!ok) break;
        tc_fence_after();
        // dK += dS^T Q; the Q slot then takes the next query tile during dQ
        mma_split(tmem + 2 * kTile + kDh, p_hi, p_lo, 16, false, q_hi, q_lo, 2 * kPlane, true, id_kv, kTile / 16,
                  it > 0);
        umma_commit(q_empty);
        // dQ_i = dS K: dS^T read MN-major (query atoms 64 wide, one tile apart), K MN-major
        mma_split(tmem + 2 * kTile + 2 * kDh + (it & 1) * kDh, p_hi, p_lo, kPlane, true, k_hi, k_lo, 2 * kPlane,
                  true, id_q, kTile / 16, false);
        umma_commit(ds_used);
        umma_commit(&dq_full[it & 1]);
      }
      if (ok) umma_commit(acc_full);
    }
  } else {
    // -------------------------------------------------------- softmax warps
    const int sw = warp - 2;
    const int qw = warp & 3;     // TMEM lane quarter
    const int half = sw >> 2;    // query columns half * 64 .. half * 64 + 63 of the tile
    const int row = qw * 32 + lane;
    const int key = j * kTile + row;
    const uint32_t lanes = (uint32_t)(qw * 32) << 16;
    float* vec = s_vec + sw * 128;   // this warp's lse2[64] and D[64]
    uint8_t* th = sP + half * kPlane;
    uint8_t* tl = sP + (2 + half) * kPlane;
    bool ok = true;
    // dQ partial of iteration it: TMEM rows are the queries of tile j + it
    auto dq_out = [&](int it) {
      ok = ok && warp_wait(&dq_full[it & 1], (it >> 1) & 1, a.err, kErrWaitAccum);
      tc_fence_after();
      if (!ok) return;
      float v[32];
      tmem_ld32(tmem + lanes + 2 * kTile + 2 * kDh + (it & 1) * kDh + half * 32, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_empty[it & 1]);
      const int q = (j + it) * kTile + row;
      if (q < a.T) store_f32x32(a.dq_part + (((long long)j * a.B * a.H + bh) * a.T + q) * kDh + half * 32, v);
    };
    for (int it = 0; it < n_it && ok; ++it) {
      const int i = j + it;
      const uint32_t ph = it & 1;
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = lane + 32 * u, q = i * kTile + half * 64 + c;
        vec[c] = q < a.T ? a.lse2[(long long)bh * a.T + q] : INFINITY;
        vec[64 + c] = q < a.T ? a.Dv[(long long)bh * a.T + q] : 0.f;
      }
      __syncwarp();
      ok = warp_wait(sdp_full, ph, a.err, kErrWaitAccum) && warp_wait(ds_used, ph ^ 1, a.err, kErrWaitAccum);
      tc_fence_after();
      if (ok) {
        // P^T[key, q] = exp2(S^T * scale_log2 - lse2[q]) for live q >= key, and
        // dS^T = P^T (dP^T - D[q]) * scale parked in the S^T columns
        const bool mask = i == j || (i + 1) * kTile > a.T;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float sv[32], dp[32];
          const uint32_t col = half * 64 + c * 32;
          tmem_ld32(tmem + lanes + col, sv);
          tmem_ld32(tmem + lanes + kTile + col, dp);
          const float4* l4 = reinterpret_cast<const float4*>(vec + c * 32);
          const float4* d4 = reinterpret_cast<const float4*>(vec + 64 + c * 32);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float4 L = l4[u], D = d4[u];
            const float lv[4] = {L.x, L.y, L.z, L.w}, dv[4] = {D.x, D.y, D.z, D.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int e = 4 * u + k;
              float p = ex2(fmaf(sv[e], a.scale_log2, -lv[k]));
              if (mask) {
                const int q = i * kTile + (int)col + e;
                if (!(q >= key && q < a.T)) p = 0.f;
              }
              dp[e] = p * (dp[e] - dv[k]) * a.scale;
              sv[e] = p;
            }
          }
          store_row32(th, tl, row, c, sv);
          tmem_st32(tmem + lanes + col, dp);
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (it > 0) dq_out(it - 1);   // overlaps the dV UMMAs
      ok = ok && warp_wait(p_used, ph, a.err, kErrWaitAccum);
      tc_fence_after();
      if (ok) {
        // the P^T buffer is free: dS^T into it
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_ld32(tmem + lanes + half * 64 + c * 32, v);
          store_row32(th, tl, row, c, v);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(sdp_empty);
        mbar_arrive(ds_full);
      }
    }
    if (ok && n_it > 0) dq_out(n_it - 1);
    ok = ok && warp_wait(acc_full, 0, a.err, kErrWaitAccum);
    tc_fence_after();
    if (ok) {
      const int g = h % a.G;
      const long long off = (((long long)g * a.B * a.KV + bkv) * a.T + key) * kDh + half * 32;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {   // 0: dV, 1: dK
        float v[32];
        tmem_ld32(tmem + lanes + 2 * kTile + which * kDh + half * 32, v);
        if (key < a.T) store_f32x32((which ? a.dk_part : a.dv_part) + off, v);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================ head width 128
//
// The same algorithms at dh = 128, with tiles sized so that the split-plane
// operands fit one CTA's shared memory. A [rows x 128] operand tile is two
// [rows x 64] swizzled sub-tiles per plane (head columns 0..63 and 64..127),
// hi sub-tiles first.
// Forward: 128 query rows x 64 keys per score tile (Q 64 KB, three 32 KB key /
// value stages, P 32 KB); scores in TMEM columns 0 and 64, O [128 x 128] f32 in
// columns 128..255. The two softmax warps of a lane quarter take 32 key
// columns each, and 64 of O's columns each for the rescale and the epilogue.
// Backward: 128 keys x 64 queries per step (K and V 64 KB each, Q_i, dO_i and
// P^T / dS^T 32 KB each). dQ leaves transposed, dQ_i^T = K^T dS^T, so that
// every product has 128 TMEM lanes (the head columns, for dQ^T); TMEM: S^T 0,
// dP^T 64, dV 128, dK 256, dQ^T buffers 384 and 448.

constexpr int kDh2 = 128;
constexpr int kKt2 = 64;                 // forward key tile, backward query tile
constexpr int kSub = kKt2 * 128;         // one [64 x 64] bf16 sub-tile: 8 KB
constexpr int kQ2 = 4 * kPlane;          // [128 x 128] in both planes: 64 KB
constexpr int kItem2 = 4 * kSub;         // [64 x 128] in both planes: 32 KB
constexpr int kRing2 = 3;
constexpr int kO2 = 2 * kKt2;            // forward: O's first TMEM column
constexpr int kFwd2Smem = kQ2 + kRing2 * kItem2 + 2 * kPlane + 6 * kTile * 4 + 1024 + 256;
constexpr int kBwd2Smem = 2 * kQ2 + 2 * kItem2 + 2 * kPlane + 1024 + 256;
static_assert(kFwd2Smem <= 232448 && kBwd2Smem <= 232448, "shared memory of one CTA");

// TMA loads of the [rows x 128] tile at (row0, z) in both planes: hi head
// columns 0..63, hi 64..127, lo 0..63, lo 64..127, `sub` bytes apart.
__device__ __forceinline__ void tma_tile128(uint8_t* dst, const CUtensorMap* mh, const CUtensorMap* ml, uint64_t* bar,
                                            int row0, int z, uint32_t sub) {
  tma_load_3d(dst, mh, bar, 0, row0, z);
  tma_load_3d(dst + sub, mh, bar, 64, row0, z);
  tma_load_3d(dst + 2 * sub, ml, bar, 0, row0, z);
  tma_load_3d(dst + 3 * sub, ml, bar, 64, row0, z);
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_d128_kernel(const __grid_constant__ CUtensorMap mq_hi, const __grid_constant__ CUtensorMap mq_lo,
                          const __grid_constant__ CUtensorMap mk_hi, const __grid_constant__ CUtensorMap mk_lo,
                          const __grid_constant__ CUtensorMap mv_hi, const __grid_constant__ CUtensorMap mv_lo,
                          const FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem;                          // Q [128 x 128]: hi, lo
  uint8_t* sRing = sQ + kQ2;                   // kRing2 key or value items [64 x 128]
  uint8_t* sP = sRing + kRing2 * kItem2;       // P [128 x 64]: hi, lo
  float* xmax = reinterpret_cast<float*>(sP + 2 * kPlane);   // [tile parity][column half][128] tile maxima
  float* xsum = xmax + 4 * kTile;                             // [2][128]
  uint64_t* bar = reinterpret_cast<uint64_t*>(xsum + 2 * kTile);
  uint64_t* q_full = bar;
  uint64_t* r_full = bar + 1;
  uint64_t* r_empty = r_full + kRing2;
  uint64_t* s_full = r_empty + kRing2;   // [2]
  uint64_t* s_empty = s_full + 2;        // [2]
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 1;
  uint64_t* o_full = p_empty + 1;
  uint64_t* sum_done = o_full + 1;
  uint64_t* mx_q = o_full + 2;           // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 6);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int BH = a.B * a.H;
  const int bh = blockIdx.x % BH;
  const int qi = a.nq - 1 - blockIdx.x / BH;   // longest query tiles first
  const int b = bh / a.H, h = bh % a.H;
  const int bkv = b * a.KV + h / a.G;
  const int nk = (a.T + kKt2 - 1) / kKt2;
  const int n = 2 * (qi + 1) < nk ? 2 * (qi + 1) : nk;   // 64-key tiles 0 .. n - 1

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kRing2; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], kSoftWarps);
    }
    mbar_init(p_full, kSoftWarps);
    mbar_init(p_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(sum_done, kSoftWarps);
    for (int q = 0; q < 4; ++q) mbar_init(&mx_q[q], 2);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;   // S buffers at columns 0 and 64, O at 128
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Ring order: K_0 and, for each j, K_{j+1} (if any) followed by V_j.
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kQ2);
      tma_tile128(sQ, &mq_hi, &mq_lo, q_full, qi * kTile, bh, kPlane);
      uint32_t it = 0;
      auto push = [&](const CUtensorMap* mh, const CUtensorMap* ml, int j) -> bool {
        const int s = it % kRing2;
        const uint32_t ph = (it / kRing2) & 1;
        ++it;
        if (!mbar_wait(&r_empty[s], ph ^ 1, a.err, kErrWaitEmpty)) return false;
        mbar_arrive_expect_tx(&r_full[s], kItem2);
        tma_tile128(sRing + s * kItem2, mh, ml, &r_full[s], j * kKt2, bkv, kSub);
        return true;
      };
      bool ok = push(&mk_hi, &mk_lo, 0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) ok = push(&mk_hi, &mk_lo, j + 1);
        if (ok) ok = push(&mv_hi, &mv_lo, j);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_s = make_idesc_f16(kTile, kKt2, true, false, false);
      const uint32_t id_o = make_idesc_f16(kTile, kDh2, true, false, true);
      const uint32_t q_hi = smem_u32(sQ), q_lo = q_hi + 2 * kPlane;
      const uint32_t p_hi = smem_u32(sP), p_lo = p_hi + kPlane;
      uint32_t it = 0, sc = 0;
      bool ok = mbar_wait(q_full, 0, a.err, kErrWaitFull);
      tc_fence_after();
      // S = Q K^T (K = the 128 head columns) for the next ring item, into score buffer sc % 2
      auto issue_s = [&]() -> bool {
        const int s = it % kRing2;
        const uint32_t ph = (it / kRing2) & 1;
        ++it;
        const uint32_t sb = sc & 1, sph = (sc >> 1) & 1;
        ++sc;
        if (!mbar_wait(&s_empty[sb], sph ^ 1, a.err, kErrWaitAccum)) return false;
        if (!mbar_wait(&r_full[s], ph, a.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t k_hi = smem_u32(sRing + s * kItem2), k_lo = k_hi + 2 * kSub;
        mma_split_t(tmem + sb * kKt2, q_hi, q_lo, 16, false, kPlane, k_hi, k_lo, 16, false, kSub, id_s, kDh2 / 16,
                    false);
        umma_commit(&r_empty[s]);
        umma_commit(&s_full[sb]);
        return true;
      };
      if (ok) ok = issue_s();   // key tile 0
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) ok = issue_s();
        if (!ok) break;
        // O += P_j V_j: P K-major over the 64 keys, V MN-major (keys = K rows,
        // head-column atoms one sub-tile apart)
        const int s = it % kRing2;
        const uint32_t ph = (it / kRing2) & 1;
        ++it;
        ok = mbar_wait(&r_full[s], ph, a.err, kErrWaitFull) && mbar_wait(p_full, j & 1, a.err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        const uint32_t v_hi = smem_u32(sRing + s * kItem2), v_lo = v_hi + 2 * kSub;
        mma_split_t(tmem + kO2, p_hi, p_lo, 16, false, kPlane, v_hi, v_lo, kSub, true, 0, id_o, kKt2 / 16, j > 0);
        umma_commit(&r_empty[s]);
        umma_commit(p_empty);
      }
      if (ok) umma_commit(o_full);
    }
  } else {
    // -------------------------------------------------------- softmax warps
    const int sw = warp - 2;
    const int qw = warp & 3;     // TMEM lane quarter
    const int half = sw >> 2;    // key columns half * 32 .. + 31; O columns half * 64 .. + 63
    const int row = qw * 32 + lane;
    const int qrow = qi * kTile + row;
    const uint32_t lanes = (uint32_t)(qw * 32) << 16;
    uint32_t sc = 0;
    bool ok = true;
    float m = -INFINITY;
    float l = 0.f;
    for (int j = 0; j < n; ++j, ++sc) {
      const uint32_t sb = sc & 1, sph = (sc >> 1) & 1;
      ok = ok && warp_wait(&s_full[sb], sph, a.err, kErrWaitAccum);
      tc_fence_after();
      // key tiles from 2 qi on reach the diagonal (or the ragged end)
      const bool mask = j >= 2 * qi;
      const int k0 = j * kKt2 + half * 32;
      float v[32];
      float mt = -INFINITY;
      if (ok) tmem_ld32(tmem + lanes + sb * kKt2 + half * 32, v);
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const bool live = !mask || (k0 + e <= qrow && k0 + e < a.T);
        if (!ok) v[e] = 0.f;
        if (live) mt = fmaxf(mt, v[e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&s_empty[sb]);
      float* xm = xmax + (j & 1) * 2 * kTile;
      xm[half * kTile + row] = mt;
      __syncwarp();
      if (lane == 0) mbar_arrive(&mx_q[qw]);
      ok = ok && warp_wait(&mx_q[qw], j & 1, a.err, kErrWaitAccum);
      const float m_new = fmaxf(m, fmaxf(mt, xm[(half ^ 1) * kTile + row]));
      const bool grow = j > 0 && m_new > m;
      const float alpha = grow ? ex2((m - m_new) * a.scale_log2) : 1.f;
      m = m_new;
      const float mb = m * a.scale_log2;
      ok = ok && warp_wait(p_empty, (j & 1) ^ 1, a.err, kErrWaitAccum);
      tc_fence_after();
      if (ok && __any_sync(0xffffffffu, grow)) {   // O *= alpha on this warp's 32 rows x 64 columns
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float o[32];
          tmem_ld32(tmem + lanes + kO2 + half * 64 + c * 32, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= alpha;
          tmem_st32(tmem + lanes + kO2 + half * 64 + c * 32, o);
        }
        tmem_wait_st();
      }
      l *= alpha;
      if (ok) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          float p = ex2(fmaf(v[e], a.scale_log2, -mb));
          if (mask && !(k0 + e <= qrow && k0 + e < a.T)) p = 0.f;
          v[e] = p;
          l += p;
        }
        store_row32(sP, sP + kPlane, row, half, v);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(p_full);
    }
    const float mb = m * a.scale_log2;
    xsum[half * kTile + row] = l;
    __syncwarp();
    if (lane == 0) mbar_arrive(sum_done);
    ok = ok && warp_wait(sum_done, 0, a.err, kErrWaitAccum) && warp_wait(o_full, 0, a.err, kErrWaitAccum);
    tc_fence_after();
    if (ok) {
      // this half's 64 of the 128 output columns, divided by the row sum
      const float lt = xsum[row] + xsum[kTile + row];
      const float inv = lt > 0.f ? 1.0f / lt : 0.f;
      const long long off = (long long)(b * a.T + qrow) * a.o_ld + h * kDh2 + half * 64;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float o[32];
        tmem_ld32(tmem + lanes + kO2 + half * 64 + c * 32, o);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= inv;
        if (qrow < a.T) {
          store_planes32(a.o_hi + off + c * 32, a.o_lo + off + c * 32, o);
          if (a.o16) store_f16x32(a.o16 + off + c * 32, o);
        }
      }
      if (qrow < a.T && half == 0) a.lse2[(long long)bh * a.T + qrow] = mb + log2f(lt);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_bwd_d128_kernel(const __grid_constant__ CUtensorMap mq_hi, const __grid_constant__ CUtensorMap mq_lo,
                          const __grid_constant__ CUtensorMap mk_hi, const __grid_constant__ CUtensorMap mk_lo,
                          const __grid_constant__ CUtensorMap mv_hi, const __grid_constant__ CUtensorMap mv_lo,
                          const __grid_constant__ CUtensorMap mo_hi, const __grid_constant__ CUtensorMap mo_lo,
                          const BwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sK = smem;              // K [128 x 128]: hi, lo
  uint8_t* sV = sK + kQ2;          // V [128 x 128]
  uint8_t* sQ = sV + kQ2;          // Q_i [64 x 128]
  uint8_t* sO = sQ + kItem2;       // dO_i [64 x 128]
  uint8_t* sP = sO + kItem2;       // P^T then dS^T [128 keys x 64 queries]: hi, lo
  uint64_t* bar = reinterpret_cast<uint64_t*>(sP + 2 * kPlane);
  uint64_t* kv_full = bar;
  uint64_t* q_full = bar + 1;
  uint64_t* q_empty = bar + 2;
  uint64_t* o_full = bar + 3;
  uint64_t* o_empty = bar + 4;
  uint64_t* sdp_full = bar + 5;
  uint64_t* sdp_empty = bar + 6;
  uint64_t* p_full = bar + 7;
  uint64_t* p_used = bar + 8;
  uint64_t* ds_full = bar + 9;
  uint64_t* ds_used = bar + 10;
  uint64_t* dq_full = bar + 11;    // [2]
  uint64_t* dq_empty = bar + 13;   // [2]
  uint64_t* acc_full = bar + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 16);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int BH = a.B * a.H;
  const int bh = blockIdx.x % BH;
  const int j = blockIdx.x / BH;       // key tile of 128; j = 0 has the most query tiles
  const int b = bh / a.H, h = bh % a.H;
  const int bkv = b * a.KV + h / a.G;
  const int i0 = 2 * j;                // first 64-query tile that sees a key of tile j
  const int n_it = (a.T + kKt2 - 1) / kKt2 - i0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 1);
    mbar_init(sdp_full, 1);
    mbar_init(sdp_empty, kSoftWarps);
    mbar_init(p_full, kSoftWarps);
    mbar_init(p_used, 1);
    mbar_init(ds_full, kSoftWarps);
    mbar_init(ds_used, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&dq_full[s], 1);
      mbar_init(&dq_empty[s], kSoftWarps);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // TMEM columns: S^T 0, dP^T 64, dV 128, dK 256, dQ^T buffers 384 and 448
  const uint32_t tmem = *tmem_slot;
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * kQ2);
      tma_tile128(sK, &mk_hi, &mk_lo, kv_full, j * kTile, bkv, kPlane);
      tma_tile128(sV, &mv_hi, &mv_lo, kv_full, j * kTile, bkv, kPlane);
      for (int it = 0; it < n_it; ++it) {
        const int i = i0 + it;
        const uint32_t ph = (it & 1) ^ 1;
        if (!mbar_wait(q_empty, ph, a.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(q_full, kItem2);
        tma_tile128(sQ, &mq_hi, &mq_lo, q_full, i * kKt2, bh, kSub);
        if (!mbar_wait(o_empty, ph, a.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(o_full, kItem2);
        tma_tile128(sO, &mo_hi, &mo_lo, o_full, i * kKt2, bh, kSub);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_s = make_idesc_f16(kTile, kKt2, true, false, false);    // [128 keys x 64 queries]
      const uint32_t id_kv = make_idesc_f16(kTile, kDh2, true, false, true);    // dV, dK: B (dO, Q) MN-major
      const uint32_t id_q = make_idesc_f16(kTile, kKt2, true, true, true);      // dQ^T: A (K) and B (dS^T) MN-major
      const uint32_t k_hi = smem_u32(sK), k_lo = k_hi + 2 * kPlane;
      const uint32_t v_hi = smem_u32(sV), v_lo = v_hi + 2 * kPlane;
      const uint32_t q_hi = smem_u32(sQ), q_lo = q_hi + 2 * kSub;
      const uint32_t o_hi = smem_u32(sO), o_lo = o_hi + 2 * kSub;
      const uint32_t p_hi = smem_u32(sP), p_lo = p_hi + kPlane;
      bool ok = mbar_wait(kv_full, 0, a.err, kErrWaitFull);
      for (int it = 0; it < n_it && ok; ++it) {
        const uint32_t ph = it & 1;
        ok = mbar_wait(o_full, ph, a.err, kErrWaitFull) && mbar_wait(sdp_empty, ph ^ 1, a.err, kErrWaitAccum);
        if (!ok) break;
        tc_fence_after();
        // dP^T = V dO^T and S^T = K Q^T (K = the 128 head columns)
        mma_split_t(tmem + kKt2, v_hi, v_lo, 16, false, kPlane, o_hi, o_lo, 16, false, kSub, id_s, kDh2 / 16, false);
        ok = mbar_wait(q_full, ph, a.err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        mma_split_t(tmem, k_hi, k_lo, 16, false, kPlane, q_hi, q_lo, 16, false, kSub, id_s, kDh2 / 16, false);
        umma_commit(sdp_full);
        ok = mbar_wait(p_full, ph, a.err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        // dV += P^T dO   (K = the 64 queries; dO's head-column atoms one sub-tile apart)
        mma_split_t(tmem + 2 * kKt2, p_hi, p_lo, 16, false, kPlane, o_hi, o_lo, kSub, true, 0, id_kv, kKt2 / 16,
                    it > 0);
        umma_commit(p_used);
        umma_commit(o_empty);
        ok = mbar_wait(ds_full, ph, a.err, kErrWaitFull) &&
             mbar_wait(&dq_empty[it & 1], ((it >> 1) & 1) ^ 1, a.err, kErrWaitAccum);
        if (!ok) break;
        tc_fence_after();
        // dK += dS^T Q; the Q slot then takes the next query tile during dQ^T
        mma_split_t(tmem + 2 * kKt2 + kDh2, p_hi, p_lo, 16, false, kPlane, q_hi, q_lo, kSub, true, 0, id_kv,
                    kKt2 / 16, it > 0);
        umma_commit(q_empty);
        // dQ_i^T = K^T dS^T (K = the 128 keys): K read MN-major (head-column
        // atoms one [128 x 64] sub-tile apart), dS^T MN-major (one query atom)
        mma_split_t(tmem + 2 * kKt2 + 2 * kDh2 + (it & 1) * kKt2, k_hi, k_lo, kPlane, true, 0, p_hi, p_lo, kPlane,
                    true, 0, id_q, kTile / 16, false);
        umma_commit(ds_used);
        umma_commit(&dq_full[it & 1]);
      }
      if (ok) umma_commit(acc_full);
    }
  } else {
    // -------------------------------------------------------- softmax warps
    const int sw = warp - 2;
    const int qw = warp & 3;     // TMEM lane quarter
    const int half = sw >> 2;    // query columns half * 32 .. + 31 of the step
    const int row = qw * 32 + lane;
    const int key = j * kTile + row;
    const uint32_t lanes = (uint32_t)(qw * 32) << 16;
    bool ok = true;
    // dQ partial of step it: TMEM lane = head column `row`, columns = queries
    auto dq_out = [&](int it) {
      ok = ok && warp_wait(&dq_full[it & 1], (it >> 1) & 1, a.err, kErrWaitAccum);
      tc_fence_after();
      if (!ok) return;
      float v[32];
      tmem_ld32(tmem + lanes + 2 * kKt2 + 2 * kDh2 + (it & 1) * kKt2 + half * 32, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_empty[it & 1]);
      const int q0 = (i0 + it) * kKt2 + half * 32;
      float* dst = a.dq_part + ((long long)j * a.B * a.H + bh) * a.T * kDh2 + row;
#pragma unroll
      for (int e = 0; e < 32; ++e)   // a warp stores 32 consecutive head columns of query q0 + e
        if (q0 + e < a.T) dst[(long long)(q0 + e) * kDh2] = v[e];
    };
    for (int it = 0; it < n_it && ok; ++it) {
      const int i = i0 + it;
      const uint32_t ph = it & 1;
      const int q0 = i * kKt2 + half * 32;
      // lane e holds lse2 and D of query q0 + e
      const float lse_l = q0 + lane < a.T ? a.lse2[(long long)bh * a.T + q0 + lane] : INFINITY;
      const float d_l = q0 + lane < a.T ? a.Dv[(long long)bh * a.T + q0 + lane] : 0.f;
      ok = warp_wait(sdp_full, ph, a.err, kErrWaitAccum) && warp_wait(ds_used, ph ^ 1, a.err, kErrWaitAccum);
      tc_fence_after();
      if (ok) {
        // P^T[key, q] = exp2(S^T * scale_log2 - lse2[q]) for live q >= key, and
        // dS^T = P^T (dP^T - D[q]) * scale parked in the S^T columns
        const bool mask = i <= i0 + 1 || (i + 1) * kKt2 > a.T;
        float sv[32], dp[32];
        tmem_ld32(tmem + lanes + half * 32, sv);
        tmem_ld32(tmem + lanes + kKt2 + half * 32, dp);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float L = __shfl_sync(0xffffffffu, lse_l, e);
          const float D = __shfl_sync(0xffffffffu, d_l, e);
          float p = ex2(fmaf(sv[e], a.scale_log2, -L));
          if (mask && !(q0 + e >= key && q0 + e < a.T)) p = 0.f;
          dp[e] = p * (dp[e] - D) * a.scale;
          sv[e] = p;
        }
        store_row32(sP, sP + kPlane, row, half, sv);
        tmem_st32(tmem + lanes + half * 32, dp);
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (it > 0) dq_out(it - 1);   // overlaps the dV UMMAs
      ok = ok && warp_wait(p_used, ph, a.err, kErrWaitAccum);
      tc_fence_after();
      if (ok) {   // the P^T buffer is free: dS^T into it
        float v[32];
        tmem_ld32(tmem + lanes + half * 32, v);
        store_row32(sP, sP + kPlane, row, half, v);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(sdp_empty);
        mbar_arrive(ds_full);
      }
    }
    if (ok && n_it > 0) dq_out(n_it - 1);
    ok = ok && warp_wait(acc_full, 0, a.err, kErrWaitAccum);
    tc_fence_after();
    if (ok) {
      const int g = h % a.G;
      const long long off = (((long long)g * a.B * a.KV + bkv) * a.T + key) * kDh2 + half * 64;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {   // 0: dV, 1: dK
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_ld32(tmem + lanes + 2 * kKt2 + which * kDh2 + half * 64 + c * 32, v);
          if (key < a.T) store_f32x32((which ? a.dk_part : a.dv_part) + off + c * 32, v);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dO planes (head-major) and D = rowsum(dO * O). Half a warp per (b, h, t)
// row of DH values, DH / 16 per lane in float4 groups 64 columns apart; the
// lanes' partial sums are reduced in a fixed butterfly order.
template <int DH>
__global__ void __launch_bounds__(256) flash_bwd_prep_kernel(const float* __restrict__ dO32, Planes O, Planes dO,
                                                             float* __restrict__ Dv, int B, int T, int H,
                                                             long long o_ld) {
  constexpr int kG = DH / 64;   // float4 groups per lane
  griddep_wait();
  const int lane = threadIdx.x % 32, hl = lane % 16;
  const long long rows = (long long)B * H * T;
  const long long span = (rows + 1) / 2 * 2;   // both half-warps stay in the shuffles
  for (long long r0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) / 16; r0 < span;
       r0 += (long long)gridDim.x * blockDim.x / 16) {
    const long long r = r0 < rows ? r0 : rows - 1;
    const int t = (int)(r % T);
    const long long bh = r / T;
    const int b = (int)(bh / H), h = (int)(bh % H);
    float4 g[kG];
    float d = 0.f;
#pragma unroll
    for (int u = 0; u < kG; ++u) {
      const int c = 4 * hl + 64 * u;
      g[u] = reinterpret_cast<const float4*>(dO32 + r * DH + c)[0];
      const long long oo = (long long)(b * T + t) * o_ld + h * DH + c;
      const uint2 oh = *reinterpret_cast<const uint2*>(O.hi + oo);
      const uint2 ol = *reinterpret_cast<const uint2*>(O.lo + oo);
      const float o0 = __uint_as_float(oh.x << 16) + __uint_as_float(ol.x << 16);
      const float o1 = __uint_as_float(oh.x & 0xffff0000u) + __uint_as_float(ol.x & 0xffff0000u);
      const float o2 = __uint_as_float(oh.y << 16) + __uint_as_float(ol.y << 16);
      const float o3 = __uint_as_float(oh.y & 0xffff0000u) + __uint_as_float(ol.y & 0xffff0000u);
      const float du = g[u].x * o0 + g[u].y * o1 + g[u].z * o2 + g[u].w * o3;
      d = u == 0 ? du : d + du;
    }
#pragma unroll
    for (int s = 8; s; s >>= 1) d += __shfl_xor_sync(0xffffffffu, d, s);
    if (r0 >= rows) continue;
#pragma unroll
    for (int u = 0; u < kG; ++u) {
      const int c = 4 * hl + 64 * u;
      uint32_t hv[2], lv[2];
      split_pair(g[u].x, g[u].y, hv[0], lv[0]);
      split_pair(g[u].z, g[u].w, hv[1], lv[1]);
      *reinterpret_cast<uint2*>(dO.hi + r * DH + c) = make_uint2(hv[0], hv[1]);
      *reinterpret_cast<uint2*>(dO.lo + r * DH + c) = make_uint2(lv[0], lv[1]);
    }
    if (hl == 0) Dv[r] = d;
  }
}

Operand head_operand(const bf16* hi, const bf16* lo, int T, int nbatch, int dh) {
  Operand o;
  o.hi = hi; o.lo = lo; o.mn_major = 0; o.ld = dh; o.rows = T; o.cols = dh;
  o.batch_stride = (long long)T * dh; o.nbatch = nbatch;
  return o;
}

// hi and lo tensor maps of head-major planes with [box_rows x 64] boxes
int maps_for(CUtensorMap* m, Planes p, int T, int nbatch, int dh, int box_rows) {
  const Operand o = head_operand(p.hi, p.lo, T, nbatch, dh);
  int rc = make_plane_map(&m[0], p.hi, o, box_rows);
  if (!rc) rc = make_plane_map(&m[1], p.lo, o, box_rows);
  return rc;
}

bool shape_ok(int B, int T, int H, int KV, int dh) {
  return B > 0 && T > 0 && H > 0 && KV > 0 && H % KV == 0 && (dh == kDh || dh == kDh2);
}

template <typename K>
int smem_attr(K kern, int bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess ? 0 : -20;
}

}  // namespace

bool flash_supported(int dh) { return dh == kDh || dh == kDh2; }

int launch_flash_fwd(Planes Q, Planes K, Planes V, Planes O, float* lse2, int B, int T, int H, int KV, int dh,
                     float scale, int* err, cudaStream_t st, long long o_ld) {
  if (o_ld == 0) o_ld = (long long)H * dh;
  if (!shape_ok(B, T, H, KV, dh) || o_ld < (long long)H * dh || o_ld % 8) return -1;
  const bool wide = dh == kDh2;
  static DeviceOnce setup;
  if (int rc0 = setup.ensure([](int) {
        int rc = smem_attr(flash_fwd_kernel, kFwdSmem);
        return rc ? rc : smem_attr(flash_fwd_d128_kernel, kFwd2Smem);
      }))
    return rc0;
  // key / value boxes: 128 rows at dh 64, 64 rows at dh 128
  CUtensorMap mq[2], mk[2], mv[2];
  const int kv_rows = wide ? kKt2 : kTile;
  int rc;
  if ((rc = maps_for(mq, Q, T, B * H, dh, kTile)) || (rc = maps_for(mk, K, T, B * KV, dh, kv_rows)) ||
      (rc = maps_for(mv, V, T, B * KV, dh, kv_rows)))
    return rc;
  FwdArgs a;
  a.B = B; a.T = T; a.H = H; a.KV = KV; a.G = H / KV; a.nq = (T + kTile - 1) / kTile;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.o_hi = O.hi; a.o_lo = O.lo; a.o16 = O.f16; a.o_ld = o_ld; a.lse2 = lse2; a.err = err;
  const long long grid = (long long)a.nq * B * H;
  if (grid > 0x7fffffffLL) return -5;
  if (wide)
    return launch_pdl(flash_fwd_d128_kernel, dim3((unsigned)grid), dim3(kThreads), kFwd2Smem, st, mq[0], mq[1], mk[0],
                      mk[1], mv[0], mv[1], a) ? -21 : 0;
  return launch_pdl(flash_fwd_kernel, dim3((unsigned)grid), dim3(kThreads), kFwdSmem, st, mq[0], mq[1], mk[0], mk[1],
                    mv[0], mv[1], a) ? -21 : 0;
}

int launch_flash_bwd_prep(const float* dO32, Planes O, Planes dO, float* Dvec, int B, int T, int H, int dh,
                          cudaStream_t st, long long o_ld) {
  if (o_ld == 0) o_ld = (long long)H * dh;
  if ((dh != kDh && dh != kDh2) || o_ld < (long long)H * dh || o_ld % 4) return -1;
  const long long rows = (long long)B * H * T;
  long long blocks = (rows + 15) / 16;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (dh == kDh2)
    return launch_pdl(flash_bwd_prep_kernel<kDh2>, dim3((unsigned)blocks), dim3(256), 0, st, dO32, O, dO, Dvec, B, T,
                      H, o_ld) ? -21 : 0;
  return launch_pdl(flash_bwd_prep_kernel<kDh>, dim3((unsigned)blocks), dim3(256), 0, st, dO32, O, dO, Dvec, B, T, H,
                    o_ld) ? -21 : 0;
}

long long flash_bwd_ws_floats(int B, int T, int H, int KV, int dh) {
  const long long nq = (T + kTile - 1) / kTile;
  const long long G = KV > 0 ? H / KV : 0;
  return nq * B * H * T * dh + 2 * G * B * KV * T * dh;
}

int launch_flash_bwd(Planes Q, Planes K, Planes V, Planes dO, const float* lse2, const float* Dvec, float* ws, int B,
                     int T, int H, int KV, int dh, float scale, int* err, cudaStream_t st) {
  if (!shape_ok(B, T, H, KV, dh)) return -1;
  const bool wide = dh == kDh2;
  static DeviceOnce setup;
  if (int rc0 = setup.ensure([](int) {
        int rc = smem_attr(flash_bwd_kernel, kBwdSmem);
        return rc ? rc : smem_attr(flash_bwd_d128_kernel, kBwd2Smem);
      }))
    return rc0;
  // query / dO boxes: 128 rows at dh 64, 64 rows at dh 128
  CUtensorMap mq[2], mk[2], mv[2], mo[2];
  const int q_rows = wide ? kKt2 : kTile;
  int rc;
  if ((rc = maps_for(mq, Q, T, B * H, dh, q_rows)) || (rc = maps_for(mk, K, T, B * KV, dh, kTile)) ||
      (rc = maps_for(mv, V, T, B * KV, dh, kTile)) || (rc = maps_for(mo, dO, T, B * H, dh, q_rows)))
    return rc;
  BwdArgs a;
  a.B = B; a.T = T; a.H = H; a.KV = KV; a.G = H / KV; a.nq = (T + kTile - 1) / kTile;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.scale = scale;
  a.lse2 = lse2; a.Dv = Dvec;
  a.dq_part = ws;
  a.dk_part = ws + (long long)a.nq * B * H * T * dh;
  a.dv_part = a.dk_part + (long long)a.G * B * KV * T * dh;
  a.err = err;
  const long long grid = (long long)a.nq * B * H;
  if (grid > 0x7fffffffLL) return -5;
  if (wide)
    return launch_pdl(flash_bwd_d128_kernel, dim3((unsigned)grid), dim3(kThreads), kBwd2Smem, st, mq[0], mq[1], mk[0],
                      mk[1], mv[0], mv[1], mo[0], mo[1], a) ? -21 : 0;
  return launch_pdl(flash_bwd_kernel, dim3((unsigned)grid), dim3(kThreads), kBwdSmem, st, mq[0], mq[1], mk[0], mk[1],
                    mv[0], mv[1], mo[0], mo[1], a) ? -21 : 0;
}

int launch_flash_rope_bwd(const float* ws, const int* pos, const float* cs_tab, int tab_rows, Planes dqkv,
                          float* dqkv_f32, int B, int T, int H, int KV, int dh, cudaStream_t st,
                          long long ld_dqkv) {
  if (!shape_ok(B, T, H, KV, dh)) return -1;
  const long long nq = (T + kTile - 1) / kTile;
  const long long qs = (long long)B * H * T * dh, kvs = (long long)B * KV * T * dh;
  const int G = H / KV;
  const float* dk = ws + nq * qs;
  const float* dv = dk + G * kvs;
  return launch_rope_qkv_bwd_sum(ws, qs, kTile, dk, dv, kvs, G, pos, cs_tab, tab_rows, dqkv, dqkv_f32, B, T, H, KV, dh,
                                 st, ld_dqkv);
}

}  // namespace tb2
