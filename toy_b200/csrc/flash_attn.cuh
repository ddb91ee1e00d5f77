// Fused causal attention on tcgen05 tiles (sm_100a): the scores and the
// probabilities never reach HBM.
//
// Layouts (split-bf16 planes, see gemm.cuh):
//   Q  [B][H][T][dh], K and V [B][KV][T][dh]   (head-major, written by RoPE)
//   O  [B*T][H*dh]                              (token-major, read by the Wo GEMM)
//   lse2 [B][H][T]  log2-domain softmax normaliser of the scaled scores:
//                   P[q, k] = exp2(S[q, k] * scale * log2(e) - lse2[q])
// Query head h reads key/value head h / (H / KV) (grouped-query attention).
// Supported head widths: dh = 64 and 128.
#pragma once
#include "kernels.cuh"

namespace tb2 {

bool flash_supported(int dh);

// O = softmax(scale * Q K^T + causal mask) V, and lse2. O is token-major,
// rows o_ld apart (0: H dh); O.f16, when set, also gets an fp16 copy (no
// scale) at the same offsets.
int launch_flash_fwd(Planes Q, Planes K, Planes V, Planes O, float* lse2, int B, int T, int H, int KV, int dh,
                     float scale, int* err, cudaStream_t st, long long o_ld = 0);

// Backward preparation: dO (f32, head-major [B][H][T][dh]) as planes, and
// D[b, h, t] = sum_c dO[b, h, t, c] * O[b, t, h, c].
int launch_flash_bwd_prep(const float* dO32, Planes O, Planes dO, float* Dvec, int B, int T, int H, int dh,
                          cudaStream_t st, long long o_ld = 0);   // O rows o_ld apart (0: H dh)

// Floats of the partial-gradient workspace launch_flash_bwd writes.
long long flash_bwd_ws_floats(int B, int T, int H, int KV, int dh);

// Backward. One CTA per (sequence, query head, key tile of 128) writes
//   dq_part[j][b][h][t][dh]   (key tile j's share of dQ, j <= t / 128)
//   dk_part[g][b][kv][t][dh], dv_part[g][b][kv][t][dh]   (query head g of the group's share)
// into ws (dq_part first, then dk_part, then dv_part); launch_flash_rope_bwd
// sums them in a fixed order.
int launch_flash_bwd(Planes Q, Planes K, Planes V, Planes dO, const float* lse2, const float* Dvec, float* ws, int B,
                     int T, int H, int KV, int dh, float scale, int* err, cudaStream_t st);

// RoPE backward over the flash backward's partials: dQ = sum over key tiles
// j <= t / 128, dK and dV = sum over the group's query heads; writes the
// token-major dqkv planes, rows ld_dqkv apart (0: (H + 2 KV) dh), and the f32
// copy when dqkv_f32 is set.
int launch_flash_rope_bwd(const float* ws, const int* pos, const float* cs_tab, int tab_rows, Planes dqkv,
                          float* dqkv_f32, int B, int T, int H, int KV, int dh, cudaStream_t st,
                          long long ld_dqkv = 0);

}  // namespace tb2
