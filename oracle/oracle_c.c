/*
 * CPU restatement of the reference's weighted unpermute arithmetic.
 * TEST INFRASTRUCTURE ONLY: this is the checker for the CUDA path, never part
 * of the product; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline may load it.
 *
 * The reference's unpermute (smxx/permute/moe_permute.cu:182-246) accumulates
 * `accum += w * float(x)` in slot order, which nvcc contracts to one fused
 * multiply-add per slot; glibc's fmaf is correctly rounded, so this loop
 * yields the same fp32 bits as that kernel.  Compiled with -mfma (one
 * instruction per fmaf instead of glibc's software path) and
 * -ffp-contract=off so no other expression is fused.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Round-to-nearest-even fp32 -> bf16 (quiet NaN kept quiet). */
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t b) {
  _Float16 h;
  memcpy(&h, &b, 2);
  return (float)h;
}

static inline uint16_t f32_to_f16(float f) {
  _Float16 h = (_Float16)f;
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}

/* out[t, h] = round16(fma chain over k of w[t,k] * in[s2d[t,k], h]).
 * is_fp16 selects the 16-bit format of `in` and `out` (0 = bf16).  The loop
 * runs k outside h with one fp32 accumulator per h, so every element still
 * sees its slots in order k = 0..K-1. */
void oracle_unpermute_sum(const uint16_t* in, const float* w, const int32_t* s2d, int64_t T,
                          int32_t K, int64_t H, int32_t is_fp16, uint16_t* out) {
  float* acc = (float*)malloc(sizeof(float) * (size_t)(H > 0 ? H : 1));
  if (acc == NULL) return;
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t h = 0; h < H; ++h) acc[h] = 0.0f;
    for (int32_t k = 0; k < K; ++k) {
      const float wk = w[t * K + k];
      const uint16_t* row = in + (int64_t)s2d[t * K + k] * H;
      if (is_fp16) {
        for (int64_t h = 0; h < H; ++h) acc[h] = fmaf(wk, f16_to_f32(row[h]), acc[h]);
      } else {
        for (int64_t h = 0; h < H; ++h) acc[h] = fmaf(wk, bf16_to_f32(row[h]), acc[h]);
      }
    }
    for (int64_t h = 0; h < H; ++h) out[t * H + h] = is_fp16 ? f32_to_f16(acc[h]) : f32_to_bf16(acc[h]);
  }
  free(acc);
}
