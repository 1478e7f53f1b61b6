/* math_sweep.h -- the input points of the pinned-function sweep (test
 * infrastructure).  The families and counts follow the reference's sweep
 * generator (code/cis2-fp/src/bin/math_dump.rs:67-180): 20 edge bit
 * patterns; exp clamp and reduction boundaries with both float neighbours;
 * k*pi/4 .. k*pi for |k| <= 64 with neighbours; powers of two and
 * 2^e*sqrt(1/2) for |e| <= 30 with neighbours; four theta values; the
 * SmolLM2 RoPE angles pos*inv_freq; then 4 x 60,000 points from the 64-bit
 * MMIX LCG (math_dump.rs:53-65): raw bit patterns, [-100, 100],
 * [-9000, 9000] and positive values with exponents in [-60, 60).  The last
 * family is built from exponent and mantissa bits (no pow), so this file
 * needs no libm.  242,428 points in all.
 *
 * ln_fn / exp_fn are the pinned ln and exp (the RoPE family depends on
 * them); the oracle passes its own, the reference driver the reference's.
 * Header-only so that both the oracle library and oracle/refmath.cpp use
 * the same generator. */
#ifndef CIS2_MATH_SWEEP_H
#define CIS2_MATH_SWEEP_H
#include <stddef.h>
#include <stdint.h>
#include <string.h>

static inline float msw_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t msw_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline int msw_isnan(float x) { return x != x; }

static inline float msw_next_up(float x) {
  if (msw_isnan(x) || msw_bits(x) == 0x7F800000u) return x;
  if (x == 0.0f) return msw_from_bits(1u);
  uint32_t b = msw_bits(x);
  return x > 0.0f ? msw_from_bits(b + 1) : msw_from_bits(b - 1);
}
static inline float msw_next_down(float x) {
  if (msw_isnan(x) || msw_bits(x) == 0xFF800000u) return x;
  if (x == 0.0f) return msw_from_bits(0x80000001u);
  uint32_t b = msw_bits(x);
  return x > 0.0f ? msw_from_bits(b - 1) : msw_from_bits(b + 1);
}

typedef struct { float *out; size_t n; } msw_sink;
static inline void msw_put(msw_sink *s, float x) {
  if (s->out) s->out[s->n] = x;
  s->n++;
}
static inline void msw_put3(msw_sink *s, float x) {
  msw_put(s, x);
  msw_put(s, msw_next_up(x));
  msw_put(s, msw_next_down(x));
}

static inline uint64_t msw_lcg(uint64_t *st) {
  *st = *st * 6364136223846793005ull + 1442695040888963407ull;
  return *st;
}
/* (word >> 11) / 2^53, in [0, 1) */
static inline double msw_unit(uint64_t *st) { return (double)(msw_lcg(st) >> 11) * (1.0 / 9007199254740992.0); }

/* Writes the points to out (when non-NULL) and returns their number. */
static inline size_t cis2_math_sweep_inputs(float *out, float (*ln_fn)(float), float (*exp_fn)(float)) {
  msw_sink s = {out, 0};
  static const uint32_t edge[20] = {0x00000000u, 0x80000000u, 0x00000001u, 0x80000001u, 0x007FFFFFu,
                                    0x807FFFFFu, 0x00800000u, 0x80800000u, 0x3F800000u, 0xBF800000u,
                                    0x3F000000u, 0xBF000000u, 0x7F7FFFFFu, 0xFF7FFFFFu, 0x7F800000u,
                                    0xFF800000u, 0x7FC00000u, 0x34000000u, 0x4B000000u, 0x5F000000u};
  for (int i = 0; i < 20; ++i) msw_put(&s, msw_from_bits(edge[i]));
  static const float expb[14] = {-88.0f, -87.99999f, -88.00001f, 88.0f, 87.99999f, 88.00001f, -0.0f,
                                 1e-10f, -1e-10f, 0.6931472f, -0.6931472f, 0.3465736f, 1e10f, -1e10f};
  for (int i = 0; i < 14; ++i) msw_put3(&s, expb[i]);
  const double pi_2 = 1.5707963267948966;
  static const double fr[4] = {0.5, 1.0, 1.5, 2.0};
  for (int k = -64; k <= 64; ++k)
    for (int j = 0; j < 4; ++j) msw_put3(&s, (float)((double)k * pi_2 * fr[j]));
  for (int e = -30; e <= 30; ++e) {
    double p = 1.0;
    for (int i = 0; i < (e < 0 ? -e : e); ++i) p = e < 0 ? p * 0.5 : p * 2.0;  /* exact 2^e */
    msw_put3(&s, (float)p);
    msw_put3(&s, (float)(p * 0.7071067811865475));
  }
  static const float th[4] = {100000.0f, 1000000.0f, 10000.0f, 500000.0f};
  for (int i = 0; i < 4; ++i) msw_put(&s, th[i]);
  const float ln_theta = ln_fn(100000.0f);
  static const int pos[14] = {0, 1, 2, 3, 4, 7, 15, 16, 63, 127, 255, 1023, 4095, 8191};
  for (int i = 0; i < 32; ++i) {
    const float frac = (float)(2 * i) / 64.0f;
    const float a = frac * ln_theta;
    const float inv_freq = exp_fn(-a);
    for (int j = 0; j < 14; ++j) msw_put(&s, (float)pos[j] * inv_freq);
  }
  uint64_t st = 0x0123456789ABCDEFull;
  for (int i = 0; i < 60000; ++i) msw_put(&s, msw_from_bits((uint32_t)msw_lcg(&st)));
  for (int i = 0; i < 60000; ++i) msw_put(&s, (float)(msw_unit(&st) * 200.0 - 100.0));
  for (int i = 0; i < 60000; ++i) msw_put(&s, (float)(msw_unit(&st) * 18000.0 - 9000.0));
  for (int i = 0; i < 60000; ++i) {
    const uint64_t w = msw_lcg(&st);
    const uint32_t e = (uint32_t)((w >> 40) % 120u);   /* exponent -60 .. 59 */
    const uint32_t man = (uint32_t)(w >> 9) & 0x7FFFFFu;
    msw_put(&s, msw_from_bits(((e + 127u - 60u) << 23) | man));
  }
  return s.n;
}

#endif
