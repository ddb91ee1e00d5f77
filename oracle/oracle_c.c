/* Oracle (test infrastructure only): byte- and integer-exact restatements of
 * the reference's host-side streams and of the Q8_0 block format.
 *
 * Nothing in the product links this file; it is compiled into
 * oracle/_build/liboracle.so and loaded by the tests, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg, as the checker.
 *
 * Build with -ffp-contract=off (no FMA contraction) so float arithmetic
 * matches the reference's strict IEEE evaluation.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* One step of the reference's 31-bit LCG.
 * lib/toy/llm/engine/llama_seq_engine.rb:1409-1414 (lcg_uniform!):
 *   s = (s * 1103515245 + 12345) & 0x7FFFFFFF ;  u = (s + 1.0) / 2147483648.0 */
int64_t toy_lcg_next(int64_t s) {
  return (int64_t)(((uint64_t)s * 1103515245ULL + 12345ULL) & 0x7FFFFFFFULL);
}

static double lcg_uniform(int64_t *s) {
  *s = toy_lcg_next(*s);
  return ((double)*s + 1.0) / 2147483648.0;
}

/* llama_seq_engine.rb:1416-1428 (lcg_seed_state): multiply-fold of the seed
 * mod 2^31-1 (Ruby integer arithmetic, non-negative remainder), fall back to
 * seed + 104729 when the fold is <= 0, then 8 warm-up draws. */
int64_t toy_lcg_seed_state(int64_t seed) {
  __int128 v = ((__int128)seed + 104729) * (__int128)2654435761LL;
  __int128 m = v % 2147483647;
  if (m < 0) m += 2147483647;
  int64_t s = (int64_t)m;
  if (s <= 0) s = seed + 104729;
  for (int w = 0; w < 8; ++w) lcg_uniform(&s);
  return s;
}

/* llama_seq_engine.rb:1383-1407 (upload_gaussian): Box-Muller over pairs of
 * LCG uniforms, emitting the cos branch then the saved sin branch; the pair
 * state restarts with every call (an odd n drops the last sin value). Values
 * are f64 and narrowed to f32 by the upload (tinynn_ggml.c upload_from_float_array).
 * Returns the advanced LCG state. */
int64_t toy_gaussian_fill(int64_t state, float *out, int64_t n, double std) {
  int pair = 0;
  double saved = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    if (pair == 0) {
      double u1 = lcg_uniform(&state);
      double u2 = lcg_uniform(&state);
      if (u1 < 1.0e-300) u1 = 1.0e-300;
      double r = sqrt(-2.0 * log(u1));
      double theta = 2.0 * M_PI * u2;
      double z0 = r * cos(theta) * std;
      double z1 = r * sin(theta) * std;
      out[i] = (float)z0;
      saved = z1;
      pair = 1;
    } else {
      out[i] = (float)saved;
      pair = 0;
    }
  }
  return state;
}

/* llama_seq_engine.rb:2545-2575 (upload_lora_q_init!): raw-seed LCG (no
 * fold, no warm-up), two draws per element, cos branch only. */
int64_t toy_lora_a_fill(int64_t s, float *out, int64_t n, double init_scale) {
  for (int64_t i = 0; i < n; ++i) {
    s = toy_lcg_next(s);
    double u1 = ((double)s + 1.0) / 2147483648.0;
    s = toy_lcg_next(s);
    double u2 = ((double)s + 1.0) / 2147483648.0;
    out[i] = (float)(init_scale * sqrt(-2.0 * log(u1)) * cos(2.0 * M_PI * u2));
  }
  return s;
}

/* IEEE binary16 from binary32, round to nearest even (the conversion ggml's
 * GGML_FP32_TO_FP16 and numpy's astype(float16) perform). */
uint16_t toy_fp32_to_fp16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    int shift = 14 - e;
    uint32_t h = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

float toy_fp16_to_fp32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t x;
  if (exp == 0) {
    if (man == 0) {
      x = sign;
    } else {
      int e = -1;
      do { e++; man <<= 1; } while (!(man & 0x400u));
      x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 0x1Fu) {
    x = sign | 0x7F800000u | (man << 13);
  } else {
    x = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/* Q8_0: blocks of 32 values -> 34 bytes {fp16 d; int8 q[32]} with
 * d = amax / 127 and q = round-half-away(x * (1/d)), all in f32
 * (ggml quantize_row_q8_0_ref; gguf-py gguf/quants.py class Q8_0, which the
 * reference converter prep/convert_smollm2_to_gguf.py uses for --quantize q8_0). */
void toy_q8_0_quantize(const float *x, int64_t n, uint8_t *out) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const float *xb = x + b * 32;
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      float a = fabsf(xb[j]);
      if (a > amax) amax = a;
    }
    volatile float d = amax / 127.0f;
    volatile float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = toy_fp32_to_fp16(d);
    uint8_t *ob = out + b * 34;
    ob[0] = (uint8_t)(dh & 0xFF);
    ob[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 32; ++j) {
      volatile float v = xb[j] * id;
      ob[2 + j] = (uint8_t)(int8_t)roundf(v);
    }
  }
}

void toy_q8_0_dequantize(const uint8_t *in, int64_t n, float *out) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const uint8_t *ib = in + b * 34;
    float d = toy_fp16_to_fp32((uint16_t)(ib[0] | (ib[1] << 8)));
    for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)ib[2 + j] * d;
  }
}

/* Advance an LCG state by k steps (used by tests that check jump-ahead). */
int64_t toy_lcg_skip(int64_t s, int64_t k) {
  for (int64_t i = 0; i < k; ++i) s = toy_lcg_next(s);
  return s;
}
