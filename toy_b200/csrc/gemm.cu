// Split-bf16 tensor-core GEMM for sm_100a: TMA-fed shared-memory pipeline,
// single-thread tcgen05.mma issue into a TMEM accumulator, 4-warp epilogue.
//
// CTA = 6 warps:  warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2..5 epilogue (warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31).
// One 128 x BN output tile per CTA; K is walked in 64-element blocks through a
// STAGES-deep ring of shared-memory buffers guarded by full/empty mbarriers.
#include "gemm.cuh"
#include "tc_common.cuh"

#include <cudaTypedefs.h>
#include <cstdio>
#include <mutex>

namespace tb2 {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;          // one 128-byte swizzle atom of bf16 along K
constexpr int kThreads = 192;
constexpr int kSmemBudget = 200 * 1024;

struct KArgs {
  int M, N, K, batch;
  int a_mn, b_mn;
  int a_bdiv1, a_bmul1, a_bdiv2, a_bmul2;
  int b_bdiv1, b_bmul1, b_bdiv2, b_bmul2;
  Epilogue epi;
  int* err;
};

__device__ __forceinline__ int batch_index(int z, int d1, int m1, int d2, int m2) {
  return (z / d1) * m1 + ((z % d1) / d2) * m2;
}

template <int BN>
struct Cfg {
  static constexpr int kTileA = BM * BK * 2;  // bytes per plane
  static constexpr int kTileB = BN * BK * 2;
  static constexpr int kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
};

template <int BN, bool SPLIT>
struct Stages {
  static constexpr int kStageBytes = (SPLIT ? 2 : 1) * (Cfg<BN>::kTileA + Cfg<BN>::kTileB);
  static constexpr int kStages = (kSmemBudget / kStageBytes) > 6 ? 6 : (kSmemBudget / kStageBytes);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align slack*/ + 256 /*barriers*/;
};

template <int BN, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_split_bf16_kernel(const __grid_constant__ CUtensorMap map_a_hi, const __grid_constant__ CUtensorMap map_a_lo,
                           const __grid_constant__ CUtensorMap map_b_hi, const __grid_constant__ CUtensorMap map_b_lo,
                           const KArgs args) {
  constexpr int STAGES = Stages<BN, SPLIT>::kStages;
  constexpr int kTileA = Cfg<BN>::kTileA;
  constexpr int kTileB = Cfg<BN>::kTileB;
  constexpr int kStageBytes = Stages<BN, SPLIT>::kStageBytes;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* accum_full = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_full + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * BM;
  const int z = blockIdx.z;
  const int num_kb = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg<BN>::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&map_a_hi);
      tma_prefetch_desc(&map_b_hi);
      const int za = batch_index(z, args.a_bdiv1, args.a_bmul1, args.a_bdiv2, args.a_bmul2);
      const int zb = batch_index(z, args.b_bdiv1, args.b_bmul1, args.b_bdiv2, args.b_bmul2);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, args.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        uint8_t* st = smem + s * kStageBytes;
        uint8_t* a_hi = st;
        uint8_t* b_hi = st + kTileA;
        uint8_t* a_lo = st + kTileA + kTileB;
        uint8_t* b_lo = a_lo + kTileA;
        const int k0 = kb * BK;
        if (!args.a_mn) {
          tma_load_3d(a_hi, &map_a_hi, &full[s], k0, m0, za);
          if (SPLIT) tma_load_3d(a_lo, &map_a_lo, &full[s], k0, m0, za);
        } else {
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) {
            tma_load_3d(a_hi + j * 64 * 128, &map_a_hi, &full[s], m0 + 64 * j, k0, za);
            if (SPLIT) tma_load_3d(a_lo + j * 64 * 128, &map_a_lo, &full[s], m0 + 64 * j, k0, za);
          }
        }
        if (!args.b_mn) {
          tma_load_3d(b_hi, &map_b_hi, &full[s], k0, n0, zb);
          if (SPLIT) tma_load_3d(b_lo, &map_b_lo, &full[s], k0, n0, zb);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) {
            tma_load_3d(b_hi + j * 64 * 128, &map_b_hi, &full[s], n0 + 64 * j, k0, zb);
            if (SPLIT) tma_load_3d(b_lo + j * 64 * 128, &map_b_lo, &full[s], n0 + 64 * j, k0, zb);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(BM, BN, true, args.a_mn != 0, args.b_mn != 0);
      // K-major: advance 32 B per 16-element k-step inside the swizzle atom.
      // MN-major: advance 16 rows of 128 B; MN atoms are 64 rows (8 KB) apart.
      const uint32_t a_kstep = args.a_mn ? 2048u : 32u;
      const uint32_t b_kstep = args.b_mn ? 2048u : 32u;
      const uint32_t a_lbo = args.a_mn ? 8192u : 16u;
      const uint32_t b_lbo = args.b_mn ? 8192u : 16u;
      bool ok = true;
      for (int kb = 0; kb < num_kb && ok; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        ok = mbar_wait(&full[s], ph, args.err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * kStageBytes);
        const uint32_t a_hi = st, b_hi = st + kTileA, a_lo = st + kTileA + kTileB, b_lo = a_lo + kTileA;
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks) {
          const uint64_t dah = make_sdesc_sw128(a_hi + ks * a_kstep, a_lbo, 1024);
          const uint64_t dbh = make_sdesc_sw128(b_hi + ks * b_kstep, b_lbo, 1024);
          const uint32_t acc = (kb > 0 || ks > 0) ? 1u : 0u;
          umma_f16(tmem_base, dah, dbh, idesc, acc);
          if (SPLIT) {
            const uint64_t dal = make_sdesc_sw128(a_lo + ks * a_kstep, a_lbo, 1024);
            const uint64_t dbl = make_sdesc_sw128(b_lo + ks * b_kstep, b_lbo, 1024);
            umma_f16(tmem_base, dal, dbh, idesc, 1u);
            umma_f16(tmem_base, dah, dbl, idesc, 1u);
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int m = m0 + row;
    const bool ok = mbar_wait(accum_full, 0, args.err, kErrWaitAccum);
    tc_fence_after();
    const Epilogue& e = args.epi;
    const bool row_ok = ok && m < args.M;
    long long row_off = 0;
    if (row_ok)
      row_off = (long long)(z / e.z_div) * e.z_s1 + (long long)(z % e.z_div) * e.bstride +
                (long long)(m / e.m_div) * e.m_s1 + (long long)(m % e.m_div) * e.m_s0;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
      const int nc = n0 + c * 32;
      if (!row_ok || nc >= args.N) continue;
      const long long off = row_off + (long long)(nc / e.n_div) * e.n_s1 + (nc % e.n_div);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= e.alpha;
      const bool full_chunk = nc + 32 <= args.N;
      if (e.mode == kEpiStoreF32 || e.mode == kEpiAccumF32 || e.mode == kEpiResidF32 || e.mode == kEpiStoreBoth) {
        float* dst = e.out + off;
        if (full_chunk) {
          float4* d4 = reinterpret_cast<float4*>(dst);
          if (e.mode == kEpiAccumF32) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float4 o = d4[i];
              o.x += v[4 * i]; o.y += v[4 * i + 1]; o.z += v[4 * i + 2]; o.w += v[4 * i + 3];
              d4[i] = o;
            }
          } else if (e.mode == kEpiResidF32) {
            const float4* r4 = reinterpret_cast<const float4*>(e.res + off);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float4 r = r4[i];
              d4[i] = make_float4(r.x + v[4 * i], r.y + v[4 * i + 1], r.z + v[4 * i + 2], r.w + v[4 * i + 3]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
        } else {
          for (int i = 0; i < 32 && nc + i < args.N; ++i) {
            if (e.mode == kEpiAccumF32) dst[i] += v[i];
            else if (e.mode == kEpiResidF32) dst[i] = e.res[off + i] + v[i];
            else dst[i] = v[i];
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
          for (int i = 0; i < 32 && nc + i < args.N; ++i) {
            const __nv_bfloat16 h0 = __float2bfloat16_rn(v[i]);
            dh[i] = h0;
            dl[i] = __float2bfloat16_rn(v[i] - __bfloat162float(h0));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg<BN>::kTmemCols);
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

template <int BN, bool SPLIT>
int launch_bn(const GemmDesc& d, int* dev_err, cudaStream_t stream) {
  using S = Stages<BN, SPLIT>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(gemm_split_bf16_kernel<BN, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             S::kSmemBytes) != cudaSuccess)
      return -20;
    attr_set = true;
  }
  CUtensorMap ma_hi, ma_lo, mb_hi, mb_lo;
  const int a_box = d.a.mn_major ? 64 : BM;
  const int b_box = d.b.mn_major ? 64 : BN;
  int rc;
  if ((rc = make_map(&ma_hi, d.a.hi, d.a, a_box))) return rc;
  if ((rc = make_map(&mb_hi, d.b.hi, d.b, b_box))) return rc;
  if (SPLIT) {
    if ((rc = make_map(&ma_lo, d.a.lo, d.a, a_box))) return rc;
    if ((rc = make_map(&mb_lo, d.b.lo, d.b, b_box))) return rc;
  } else {
    ma_lo = ma_hi;
    mb_lo = mb_hi;
  }
  KArgs k;
  k.M = d.M; k.N = d.N; k.K = d.K; k.batch = d.batch;
  k.a_mn = d.a.mn_major; k.b_mn = d.b.mn_major;
  k.a_bdiv1 = d.a.bdiv1; k.a_bmul1 = d.a.bmul1; k.a_bdiv2 = d.a.bdiv2; k.a_bmul2 = d.a.bmul2;
  k.b_bdiv1 = d.b.bdiv1; k.b_bmul1 = d.b.bmul1; k.b_bdiv2 = d.b.bdiv2; k.b_bmul2 = d.b.bmul2;
  k.epi = d.epi;
  k.err = dev_err;
  dim3 grid((d.N + BN - 1) / BN, (d.M + BM - 1) / BM, d.batch);
  gemm_split_bf16_kernel<BN, SPLIT><<<grid, kThreads, S::kSmemBytes, stream>>>(ma_hi, ma_lo, mb_hi, mb_lo, k);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -21;
}

int pick_bn(int N) {
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  const int t256 = (N + 255) / 256 * 256, t192 = (N + 191) / 192 * 192;
  return t192 < t256 ? 192 : 256;
}

}  // namespace

int gemm_launch(const GemmDesc& d, int* dev_err, cudaStream_t stream) {
  if (d.M <= 0 || d.N <= 0 || d.K <= 0 || d.batch <= 0) return -1;
  if (d.batch > 65535) return -2;
  // Epilogue vector stores need 16-byte aligned rows.
  const Epilogue& e = d.epi;
  const int al = (e.mode == kEpiStoreSplit || e.mode == kEpiStoreBoth) ? 8 : 4;
  if ((e.m_s0 % al) || (e.m_s1 % al) || (e.n_s1 % al) || (e.bstride % al) || (e.z_s1 % al) || (e.n_div % 32))
    return -3;
  if (!d.a.hi || !d.b.hi || (d.split && (!d.a.lo || !d.b.lo))) return -4;
  switch (pick_bn(d.N)) {
    case 64: return d.split ? launch_bn<64, true>(d, dev_err, stream) : launch_bn<64, false>(d, dev_err, stream);
    case 128: return d.split ? launch_bn<128, true>(d, dev_err, stream) : launch_bn<128, false>(d, dev_err, stream);
    case 192: return d.split ? launch_bn<192, true>(d, dev_err, stream) : launch_bn<192, false>(d, dev_err, stream);
    default: return d.split ? launch_bn<256, true>(d, dev_err, stream) : launch_bn<256, false>(d, dev_err, stream);
  }
}

}  // namespace tb2
