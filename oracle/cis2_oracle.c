/* oracle/cis2_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker; never shipped
 * in, linked into, or called by the product path).
 *
 * Plain-C11 restatement of the CIS-2 deterministic fp32 decode path, written
 * from the reference's specification and code behaviour:
 *   pinned math      code/cis2-fp/gpu/cis2_math.h:84-467  (src/math.rs:29-544)
 *   constants        code/cis2-fp/gpu/cis2_consts.inc:4-32 (bit patterns below)
 *   forward pass     code/cis2-fp/gpu/cis2_model.h:503-760 (src/main.rs:355-529)
 *   Qwen3 QK-norm    labs/w1x-qwen3/scripts/qwen3-port.diff:66-80
 *   decode + witness code/cis2-fp/gpu/cis2_host.cpp:179-218 (src/main.rs:1084-1226)
 *   E23 sampler      code/patches/cis2-fp__cm_e23-pinned-sampling.patch:592-725
 *
 * Build (oracle/Makefile): -O2 -ffp-contract=off -fno-fast-math -msse2
 * -mfpmath=sse, so every fp32 operation below is one separately rounded SSE
 * scalar instruction.  FTZ|DAZ (spec §1.3, cis2_fpenv.h:62-135) is pinned in
 * MXCSR on entry to every exported function and restored on exit, so the
 * library is safe to call from many threads at once.
 */
#include "cis2_oracle.h"
#include "math_sweep.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <xmmintrin.h>

/* ------------------------------------------------------------ FP environment */

typedef struct { unsigned saved; } fpenv_guard;
static fpenv_guard fp_enter(void) {
  fpenv_guard g;
  g.saved = _mm_getcsr();
  _mm_setcsr(g.saved | (1u << 15) | (1u << 6)); /* FTZ | DAZ (cis2_fpenv.h:71-76) */
  return g;
}
static void fp_leave(fpenv_guard g) { _mm_setcsr(g.saved); }

/* ------------------------------------------------------------ bits */

static inline uint32_t fbits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float ffrom(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }
static inline uint64_t dbits(double x) { uint64_t u; memcpy(&u, &x, 8); return u; }
static inline double dfrom(uint64_t u) { double x; memcpy(&x, &u, 8); return x; }
static inline float widen(uint16_t b) { return ffrom((uint32_t)b << 16); } /* cis2_math.h:181-183 */

/* Pinned constants: the CIS-2 v0.3b coefficient table, as exact bit patterns
 * (cis2_consts.inc:4-32).  Same values, same declared order as the table
 * digest (cis2_model.h:428-448). */
#define K_EXP_LOG2E 0x3fb8aa3bu
#define K_EXP_C1    0x3f318000u
#define K_EXP_C2    0xb95e8083u
static const uint32_t K_EXP_P[6] = {0x39506967u, 0x3ab743ceu, 0x3c088908u,
                                    0x3d2aa9c1u, 0x3e2aaaaau, 0x3f000000u};
static const uint32_t K_SIN[3] = {0xbe2aaaa3u, 0x3c08839eu, 0xb94ca1f9u};
static const uint32_t K_COS[3] = {0x3d2aaaa5u, 0xbab6061au, 0x37ccf5ceu};
#define K_LOG_SQRTHF 0x3f3504f3u
#define K_LOG_Q1     0xb95e8083u
#define K_LOG_Q2     0x3f318000u
static const uint32_t K_LOG_P[9] = {0x3d9021bbu, 0xbdebd1b8u, 0x3def251bu, 0xbdfe5d4fu,
                                    0x3e11e9bfu, 0xbe2aae50u, 0x3e4cceadu, 0xbe7ffffcu,
                                    0x3eaaaaaau};
#define K_PI_2_F64 0x3ff921fb54442d18ull

/* ------------------------------------------------------------ SHA-256 (FIPS 180-4) */

typedef struct { uint32_t h[8]; uint64_t len; uint8_t buf[64]; uint32_t n; } sha_t;

static const uint32_t SHA_K[64] = {
  0x428a2f98u,0x71374491u,0xb5c0fbcfu,0xe9b5dba5u,0x3956c25bu,0x59f111f1u,0x923f82a4u,0xab1c5ed5u,
  0xd807aa98u,0x12835b01u,0x243185beu,0x550c7dc3u,0x72be5d74u,0x80deb1feu,0x9bdc06a7u,0xc19bf174u,
  0xe49b69c1u,0xefbe4786u,0x0fc19dc6u,0x240ca1ccu,0x2de92c6fu,0x4a7484aau,0x5cb0a9dcu,0x76f988dau,
  0x983e5152u,0xa831c66du,0xb00327c8u,0xbf597fc7u,0xc6e00bf3u,0xd5a79147u,0x06ca6351u,0x14292967u,
  0x27b70a85u,0x2e1b2138u,0x4d2c6dfcu,0x53380d13u,0x650a7354u,0x766a0abbu,0x81c2c92eu,0x92722c85u,
  0xa2bfe8a1u,0xa81a664bu,0xc24b8b70u,0xc76c51a3u,0xd192e819u,0xd6990624u,0xf40e3585u,0x106aa070u,
  0x19a4c116u,0x1e376c08u,0x2748774cu,0x34b0bcb5u,0x391c0cb3u,0x4ed8aa4au,0x5b9cca4fu,0x682e6ff3u,
  0x748f82eeu,0x78a5636fu,0x84c87814u,0x8cc70208u,0x90befffau,0xa4506cebu,0xbef9a3f7u,0xc67178f2u};

static inline uint32_t ror(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static void sha_init(sha_t *s) {
  static const uint32_t iv[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                 0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
  memcpy(s->h, iv, sizeof iv);
  s->len = 0;
  s->n = 0;
}
static void sha_block(uint32_t h[8], const uint8_t *p) {
  uint32_t w[64];
  for (int i = 0; i < 16; ++i)
    w[i] = ((uint32_t)p[4 * i] << 24) | ((uint32_t)p[4 * i + 1] << 16) |
           ((uint32_t)p[4 * i + 2] << 8) | (uint32_t)p[4 * i + 3];
  for (int i = 16; i < 64; ++i) {
    uint32_t s0 = ror(w[i - 15], 7) ^ ror(w[i - 15], 18) ^ (w[i - 15] >> 3);
    uint32_t s1 = ror(w[i - 2], 17) ^ ror(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
  for (int i = 0; i < 64; ++i) {
    uint32_t t1 = hh + (ror(e, 6) ^ ror(e, 11) ^ ror(e, 25)) + ((e & f) ^ (~e & g)) + SHA_K[i] + w[i];
    uint32_t t2 = (ror(a, 2) ^ ror(a, 13) ^ ror(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
    hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}
static void sha_update(sha_t *s, const void *data, size_t n) {
  const uint8_t *p = (const uint8_t *)data;
  s->len += n;
  if (s->n) {
    size_t take = 64 - s->n;
    if (take > n) take = n;
    memcpy(s->buf + s->n, p, take);
    s->n += (uint32_t)take; p += take; n -= take;
    if (s->n == 64) { sha_block(s->h, s->buf); s->n = 0; }
  }
  while (n >= 64) { sha_block(s->h, p); p += 64; n -= 64; }
  if (n) { memcpy(s->buf, p, n); s->n = (uint32_t)n; }
}
static void sha_u32le(sha_t *s, uint32_t v) {
  uint8_t b[4] = {(uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24)};
  sha_update(s, b, 4);
}
static void sha_final(const sha_t *s0, uint8_t out[32]) {
  sha_t s = *s0; /* finalising a copy leaves the running state usable */
  uint64_t bits = s.len * 8;
  uint8_t pad[72];
  size_t padn = (s.n < 56) ? (56 - s.n) : (120 - s.n);
  memset(pad, 0, sizeof pad);
  pad[0] = 0x80;
  for (int i = 0; i < 8; ++i) pad[padn + i] = (uint8_t)(bits >> (56 - 8 * i));
  sha_update(&s, pad, padn + 8);
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (uint8_t)(s.h[i] >> 24); out[4 * i + 1] = (uint8_t)(s.h[i] >> 16);
    out[4 * i + 2] = (uint8_t)(s.h[i] >> 8); out[4 * i + 3] = (uint8_t)s.h[i];
  }
}

/* ------------------------------------------------------------ pinned math */

/* Saturating casts and libm-free rounding (cis2_math.h:112-157). */
static inline int32_t f32_to_i32_sat(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return (int32_t)x;
}
static inline int64_t f64_to_i64_sat(double x) {
  if (x != x) return 0;
  if (x >= 9223372036854775808.0) return INT64_MAX;
  if (x <= -9223372036854775808.0) return INT64_MIN;
  return (int64_t)x;
}
static inline float floor_f32(float x) {
  float a = x < 0.0f ? -x : x;
  if (!(a < 8388608.0f)) return x;
  float t = (float)(int32_t)x;
  if (x < t) t = t - 1.0f;
  return t;
}
static inline double round_f64_away(double x) {
  double a = x < 0.0 ? -x : x;
  if (!(a < 4503599627370496.0)) return x;
  double t = (double)(int64_t)a;
  double frac = a - t;
  if (frac >= 0.5) t = t + 1.0;
  return dfrom((dbits(t) & 0x7FFFFFFFFFFFFFFFull) | (dbits(x) & 0x8000000000000000ull));
}
static inline float sqrt_cr(float x) { return _mm_cvtss_f32(_mm_sqrt_ss(_mm_set_ss(x))); }

/* ldexp by exponent-field arithmetic; underflow returns +0 (cis2_math.h:275-285). */
static inline float ldexp_exact(float x, int32_t k) {
  if (x == 0.0f) return x;
  uint32_t b = fbits(x);
  int32_t e = (int32_t)((b >> 23) & 0xFFu) + k;
  if (e <= 0) return 0.0f;
  if (e >= 0xFF) return (b >> 31) ? ffrom(0xFF800000u) : ffrom(0x7F800000u);
  return ffrom((b & ~(0xFFu << 23)) | ((uint32_t)e << 23));
}

/* exp route (b): Cephes-pattern split reduction + Horner (cis2_math.h:287-313). */
static float p_exp(float x) {
  if (x != x) return ffrom(0x7FC00000u);
  if (x > 88.0f) return ffrom(0x7F800000u);
  if (x < -88.0f) return 0.0f;
  float t = x * ffrom(K_EXP_LOG2E);
  float z0 = t + 0.5f;
  float k = floor_f32(z0);
  float kc1 = k * ffrom(K_EXP_C1);
  float r0 = x - kc1;
  float kc2 = k * ffrom(K_EXP_C2);
  float r = r0 - kc2;
  float r2 = r * r;
  float poly = ffrom(K_EXP_P[0]);
  for (int i = 1; i < 6; ++i) {
    float m = poly * r;
    poly = m + ffrom(K_EXP_P[i]);
  }
  float m1 = poly * r2;
  float poly2 = m1 + r;
  float result = poly2 + 1.0f;
  return ldexp_exact(result, f32_to_i32_sat(k));
}

/* f64-staged pi/2 reduction, one f32 narrowing (cis2_math.h:320-327). */
static void reduce_pi_2(float x, float *r, int64_t *k) {
  double xd = (double)x;
  double kf = round_f64_away(xd / dfrom(K_PI_2_F64));
  double khi = kf * dfrom(K_PI_2_F64);
  double r64 = xd - khi;
  *r = (float)r64;
  *k = f64_to_i64_sat(kf);
}
static float sin_poly(float r) { /* cis2_math.h:330-340 */
  float r2 = r * r;
  float in = ffrom(K_SIN[2]);
  float m0 = in * r2; in = m0 + ffrom(K_SIN[1]);
  float m1 = in * r2; in = m1 + ffrom(K_SIN[0]);
  float r3 = r2 * r;
  float term = in * r3;
  return r + term;
}
static float cos_poly(float r) { /* cis2_math.h:343-355 */
  float r2 = r * r;
  float in = ffrom(K_COS[2]);
  float m0 = in * r2; in = m0 + ffrom(K_COS[1]);
  float m1 = in * r2; in = m1 + ffrom(K_COS[0]);
  float r4 = r2 * r2;
  float term = in * r4;
  float half_r2 = 0.5f * r2;
  float s1 = 1.0f - half_r2;
  return s1 + term;
}
static float p_sin(float x) { /* cis2_math.h:361-372 */
  float r; int64_t k;
  reduce_pi_2(x, &r, &k);
  float sr = sin_poly(r), cr = cos_poly(r);
  switch ((int)(((k % 4) + 4) % 4)) {
    case 0: return sr;
    case 1: return cr;
    case 2: return -sr;
    default: return -cr;
  }
}
static float p_cos(float x) { /* cis2_math.h:374-385 */
  float r; int64_t k;
  reduce_pi_2(x, &r, &k);
  float sr = sin_poly(r), cr = cos_poly(r);
  switch ((int)(((k % 4) + 4) % 4)) {
    case 0: return cr;
    case 1: return -sr;
    case 2: return -cr;
    default: return sr;
  }
}
/* ln route (b) (cis2_math.h:391-429). */
static float p_ln(float x) {
  if (x != x || x < 0.0f) return ffrom(0x7FC00000u);
  if (x == 0.0f) return ffrom(0xFF800000u);
  uint32_t b = fbits(x);
  int32_t e = (int32_t)((b >> 23) & 0xFFu) - 126;
  float m = ffrom((b & 0x807FFFFFu) | (126u << 23));
  if (m < ffrom(K_LOG_SQRTHF)) {
    e -= 1;
    float mm = m + m;
    m = mm - 1.0f;
  } else {
    m = m - 1.0f;
  }
  float z = m * m;
  float poly = ffrom(K_LOG_P[0]);
  for (int i = 1; i < 9; ++i) {
    float t = poly * m;
    poly = t + ffrom(K_LOG_P[i]);
  }
  float y = poly * m;
  y = y * z;
  float fe = (float)e;
  float t1 = fe * ffrom(K_LOG_Q1);
  y = y + t1;
  float half_z = 0.5f * z;
  y = y - half_z;
  float res = m + y;
  float t2 = fe * ffrom(K_LOG_Q2);
  return res + t2;
}
static float p_silu(float x) { /* cis2_math.h:432-437 */
  float e = p_exp(-x);
  float d = 1.0f + e;
  return x / d;
}
static float p_rsqrt(float x) { return 1.0f / sqrt_cr(x); } /* cis2_math.h:268 */

/* ------------------------------------------------------------ reductions */

/* §5.1 strict left-to-right; acc starts at +0 (cis2_math.h:186-200). */
static float dot_seq(const float *a, const float *b, int n) {
  float acc = 0.0f;
  for (int i = 0; i < n; ++i) { float p = a[i] * b[i]; acc = acc + p; }
  return acc;
}
static float sum_seq(const float *a, int n) {
  float acc = 0.0f;
  for (int i = 0; i < n; ++i) acc = acc + a[i];
  return acc;
}
/* v0.4 tree: 32 zero-padded leaves, five pairwise rounds, block partials
 * folded left to right from +0 (cis2_math.h:212-265). */
static float tree32(float *leaf) {
  for (int w = 32; w > 1; w >>= 1)
    for (int i = 0; i < w / 2; ++i) leaf[i] = leaf[2 * i] + leaf[2 * i + 1];
  return leaf[0];
}
static float tree_dot(const float *a, const float *b, int n) {
  float acc = 0.0f;
  for (int s = 0; s < n; s += 32) {
    float leaf[32];
    for (int i = 0; i < 32; ++i) leaf[i] = (s + i < n) ? a[s + i] * b[s + i] : 0.0f;
    float part = tree32(leaf);
    acc = acc + part;
  }
  return acc;
}
static float tree_sum(const float *a, int n) {
  float acc = 0.0f;
  for (int s = 0; s < n; s += 32) {
    float leaf[32];
    for (int i = 0; i < 32; ++i) leaf[i] = (s + i < n) ? a[s + i] : 0.0f;
    float part = tree32(leaf);
    acc = acc + part;
  }
  return acc;
}
static float dot_mode(const float *a, const float *b, int n, int tree) {
  return tree ? tree_dot(a, b, n) : dot_seq(a, b, n);
}
static float sum_mode(const float *a, int n, int tree) {
  return tree ? tree_sum(a, n) : sum_seq(a, n);
}
/* Row dot against a bf16 weight row (widened exactly, then the same fold). */
static float dot_row_bf16(const uint16_t *w, const float *x, int n, int tree) {
  if (!tree) {
    float acc = 0.0f;
    for (int i = 0; i < n; ++i) { float p = widen(w[i]) * x[i]; acc = acc + p; }
    return acc;
  }
  float acc = 0.0f;
  for (int s = 0; s < n; s += 32) {
    float leaf[32];
    for (int i = 0; i < 32; ++i) leaf[i] = (s + i < n) ? widen(w[s + i]) * x[s + i] : 0.0f;
    float part = tree32(leaf);
    acc = acc + part;
  }
  return acc;
}

/* §10 softmax in place (cis2_math.h:442-467): strict '>' max scan, pinned exp,
 * mode-selected denominator, elementwise divide. */
static void softmax_mode(float *v, int n, int tree) {
  if (n == 0) return;
  float mx = v[0];
  for (int i = 1; i < n; ++i) if (v[i] > mx) mx = v[i];
  for (int i = 0; i < n; ++i) v[i] = p_exp(v[i] - mx);
  float den = sum_mode(v, n, tree);
  for (int i = 0; i < n; ++i) v[i] = v[i] / den;
}

static uint32_t argmax_first(const float *v, int n) { /* cis2_model.h:764-774 */
  int best = 0;
  float bv = v[0];
  for (int i = 0; i < n; ++i) if (v[i] > bv) { bv = v[i]; best = i; }
  return (uint32_t)best;
}

/* ------------------------------------------------------------ E23 sampler */

static uint64_t sm64(uint64_t x) { /* splitmix64 round, e23 patch :617-623 */
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
uint64_t cis2o_rng_word(uint64_t seed, uint64_t position) { return sm64(seed ^ sm64(position)); }

typedef struct { float p; uint32_t i; } pi_t;
static int cmp_pi(const void *a, const void *b) {
  const pi_t *x = (const pi_t *)a, *y = (const pi_t *)b;
  if (x->p != y->p) return (x->p > y->p) ? -1 : 1;   /* probability descending */
  return (x->i < y->i) ? -1 : (x->i > y->i);          /* index ascending */
}
/* e23 patch :650-725. */
static uint32_t sample_e23(const float *logits, int n, float temperature, float top_p,
                           uint64_t seed, uint64_t position, float *scratch, pi_t *order) {
  for (int i = 0; i < n; ++i) scratch[i] = logits[i] / temperature;
  float mx = scratch[0];
  for (int i = 1; i < n; ++i) if (scratch[i] > mx) mx = scratch[i];
  for (int i = 0; i < n; ++i) scratch[i] = p_exp(scratch[i] - mx);
  float den = sum_seq(scratch, n);
  for (int i = 0; i < n; ++i) scratch[i] = scratch[i] / den;
  for (int i = 0; i < n; ++i) { order[i].p = scratch[i]; order[i].i = (uint32_t)i; }
  qsort(order, (size_t)n, sizeof(pi_t), cmp_pi);
  float cum = 0.0f;
  int nuc = n;
  for (int i = 0; i < n; ++i) {
    cum = cum + order[i].p;
    if (cum >= top_p) { nuc = i + 1; break; }
  }
  float total = 0.0f;
  for (int i = 0; i < nuc; ++i) total = total + order[i].p;
  double u = (double)(cis2o_rng_word(seed, position) >> 11) * (1.0 / 9007199254740992.0);
  float cdf = 0.0f;
  for (int i = 0; i < nuc; ++i) {
    float p = order[i].p / total;
    cdf = cdf + p;
    if ((double)cdf > u) return order[i].i;
  }
  return order[nuc - 1].i;
}

/* -------------------------------------------- seeded Gumbel-max sampler
 * The "CIS2-SAMPLE-1" clause (code/patches/cis2-spec__seeded-sampling.patch
 * :81-145).  Its one new primitive is MurmurHash3_x86_32 (Austin Appleby,
 * public domain), restated here from the published algorithm; the clause
 * pins it with the hash seed 0x43495332 over a 16-byte key. */

static uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

uint32_t cis2o_murmur3_32(const uint8_t *key, size_t len, uint32_t seed) {
  const uint32_t c1 = 0xcc9e2d51u, c2 = 0x1b873593u;
  uint32_t h = seed;
  const size_t nb = len / 4;
  for (size_t b = 0; b < nb; ++b) {
    uint32_t k = (uint32_t)key[4 * b] | (uint32_t)key[4 * b + 1] << 8 | (uint32_t)key[4 * b + 2] << 16 |
                 (uint32_t)key[4 * b + 3] << 24;
    k *= c1;
    k = rotl32(k, 15);
    k *= c2;
    h ^= k;
    h = rotl32(h, 13);
    h = h * 5u + 0xe6546b64u;
  }
  const uint8_t *tail = key + 4 * nb;
  uint32_t k = 0;
  switch (len & 3) {
    case 3: k ^= (uint32_t)tail[2] << 16; /* fall through */
    case 2: k ^= (uint32_t)tail[1] << 8;  /* fall through */
    case 1:
      k ^= tail[0];
      k *= c1;
      k = rotl32(k, 15);
      k *= c2;
      h ^= k;
  }
  h ^= (uint32_t)len;
  h ^= h >> 16;
  h *= 0x85ebca6bu;
  h ^= h >> 13;
  h *= 0xc2b2ae35u;
  h ^= h >> 16;
  return h;
}

/* 14.2: key = seed (u64 LE) || step (u32 LE) || index (u32 LE);
 * u = f32((h >> 9) * 2 + 1) * 2^-24 (exact); g = 0 - ln(0 - ln(u)). */
static float gumbel_noise(uint64_t seed, uint32_t step, uint32_t index, uint32_t *h_out, float *u_out) {
  uint8_t key[16];
  for (int i = 0; i < 8; ++i) key[i] = (uint8_t)(seed >> (8 * i));
  for (int i = 0; i < 4; ++i) key[8 + i] = (uint8_t)(step >> (8 * i));
  for (int i = 0; i < 4; ++i) key[12 + i] = (uint8_t)(index >> (8 * i));
  const uint32_t h = cis2o_murmur3_32(key, 16, 0x43495332u);
  const uint32_t m = (h >> 9) * 2u + 1u;
  const float u = (float)m * 0x1p-24f;
  if (h_out) *h_out = h;
  if (u_out) *u_out = u;
  return 0.0f - p_ln(0.0f - p_ln(u));
}

void cis2o_gumbel_noise(uint64_t seed, uint32_t step, uint32_t index, uint32_t *hash, float *u, float *g) {
  fpenv_guard fg = fp_enter();
  *g = gumbel_noise(seed, step, index, hash, u);
  fp_leave(fg);
}

typedef struct { float s; uint32_t i; } si_t;
static int cmp_rank(const void *a, const void *b) { /* 14.3 step 2: s descending, index ascending */
  const si_t *x = (const si_t *)a, *y = (const si_t *)b;
  if (x->s > y->s) return -1;
  if (y->s > x->s) return 1;
  return (x->i < y->i) ? -1 : (x->i > y->i);
}

/* 14.3-14.4.  z_out (optional, [n]) receives z (-inf where masked). */
static uint32_t sample_gumbel(const float *logits, int n, float temperature, uint32_t top_k, float top_p,
                              uint64_t seed, uint32_t step, si_t *order, float *z_out) {
  for (int i = 0; i < n; ++i) { order[i].s = logits[i] / temperature; order[i].i = (uint32_t)i; }
  qsort(order, (size_t)n, sizeof(si_t), cmp_rank);
  const int K = (top_k > 0 && top_k < (uint32_t)n) ? (int)top_k : n;
  int P = K;
  if (top_p < 1.0f) {
    const float m = order[0].s;
    float den = 0.0f;
    for (int r = 0; r < K; ++r) den = den + p_exp(order[r].s - m);
    float c = 0.0f;
    for (int r = 0; r < K; ++r) {
      if (r > 0 && !(c < top_p)) { P = r; break; }
      c = c + p_exp(order[r].s - m) / den;
    }
  }
  if (z_out)
    for (int i = 0; i < n; ++i) z_out[i] = ffrom(0xff800000u);
  uint32_t best_i = 0;
  float best_z = ffrom(0xff800000u);
  int have = 0;
  for (int r = 0; r < P; ++r) {
    const uint32_t i = order[r].i;
    const float z = order[r].s + gumbel_noise(seed, step, i, NULL, NULL);
    if (z_out) z_out[i] = z;
    if (!have || z > best_z || (z == best_z && i < best_i)) { best_z = z; best_i = i; have = 1; }
  }
  return best_i;
}

uint32_t cis2o_sample_gumbel(const float *logits, int32_t n, float temperature, uint32_t top_k, float top_p,
                             uint64_t seed, uint32_t step, float *z_out) {
  fpenv_guard fg = fp_enter();
  si_t *order = (si_t *)malloc(sizeof(si_t) * (size_t)n);
  const uint32_t r = sample_gumbel(logits, n, temperature, top_k, top_p, seed, step, order, z_out);
  free(order);
  fp_leave(fg);
  return r;
}

/* ------------------------------------------------------------ model */

typedef struct {
  cis2o_config c;
  const uint16_t *embed, *final_norm, *lm_head;
  const uint16_t **L; /* [n_layers][CIS2O_LAYER_SLOTS] */
  float *inv_freq;    /* [head_dim/2] */
  uint8_t inv_freq_digest[32];
  uint8_t table_digest[32];
} model_t;

static void table_digest(uint8_t out[32]) { /* cis2_model.h:414-450 */
  sha_t s;
  sha_init(&s);
  sha_u32le(&s, K_EXP_LOG2E); sha_u32le(&s, K_EXP_C1); sha_u32le(&s, K_EXP_C2);
  for (int i = 0; i < 6; ++i) sha_u32le(&s, K_EXP_P[i]);
  uint64_t pb = K_PI_2_F64;
  uint8_t le[8];
  for (int i = 0; i < 8; ++i) le[i] = (uint8_t)(pb >> (8 * i));
  sha_update(&s, le, 8);
  for (int i = 0; i < 3; ++i) sha_u32le(&s, K_SIN[i]);
  for (int i = 0; i < 3; ++i) sha_u32le(&s, K_COS[i]);
  sha_u32le(&s, K_LOG_SQRTHF); sha_u32le(&s, K_LOG_Q1); sha_u32le(&s, K_LOG_Q2);
  for (int i = 0; i < 9; ++i) sha_u32le(&s, K_LOG_P[i]);
  sha_final(&s, out);
}

void cis2o_table_digest(uint8_t out[32]) {
  fpenv_guard g = fp_enter();
  table_digest(out);
  fp_leave(g);
}

void *cis2o_model_new(const cis2o_config *cfg, const uint16_t *embed, const uint16_t *final_norm,
                      const uint16_t *lm_head, const uint16_t *const *layer_tensors) {
  fpenv_guard g = fp_enter();
  model_t *m = (model_t *)calloc(1, sizeof(model_t));
  m->c = *cfg;
  m->embed = embed;
  m->final_norm = final_norm;
  m->lm_head = cfg->tied ? embed : lm_head;
  size_t nl = (size_t)cfg->n_layers * CIS2O_LAYER_SLOTS;
  m->L = (const uint16_t **)malloc(nl * sizeof(uint16_t *));
  for (size_t i = 0; i < nl; ++i) m->L[i] = layer_tensors[i];
  /* §7.2 inv_freq (cis2_model.h:456-476): ln of the f64 theta narrowed once. */
  int half = cfg->head_dim / 2;
  m->inv_freq = (float *)malloc(sizeof(float) * (size_t)(half > 0 ? half : 1));
  float ln_theta = p_ln((float)cfg->rope_theta);
  sha_t s;
  sha_init(&s);
  for (int i = 0; i < half; ++i) {
    float frac = (float)(2 * i) / (float)cfg->head_dim;
    float a = frac * ln_theta;
    m->inv_freq[i] = p_exp(-a);
    sha_u32le(&s, fbits(m->inv_freq[i]));
  }
  sha_final(&s, m->inv_freq_digest);
  table_digest(m->table_digest);
  fp_leave(g);
  return m;
}

void cis2o_model_free(void *mp) {
  model_t *m = (model_t *)mp;
  if (!m) return;
  free(m->L);
  free(m->inv_freq);
  free(m);
}

void cis2o_inv_freq(const void *mp, float *out_half, uint8_t out_digest[32]) {
  const model_t *m = (const model_t *)mp;
  if (out_half) memcpy(out_half, m->inv_freq, sizeof(float) * (size_t)(m->c.head_dim / 2));
  if (out_digest) memcpy(out_digest, m->inv_freq_digest, 32);
}

typedef struct {
  float *h, *h2, *ln, *q, *k, *v, *att, *o, *gate, *up, *hid, *down, *hn, *logits, *scores;
  float *kc, *vc; /* [n_layers][max_pos][kv_dim] */
  int max_pos;
} ws_t;

static int ws_alloc(ws_t *w, const model_t *m, int max_pos) {
  const cis2o_config *c = &m->c;
  size_t H = (size_t)c->hidden, I = (size_t)c->inter, QD = (size_t)c->n_heads * (size_t)c->head_dim;
  size_t KV = (size_t)c->n_kv_heads * (size_t)c->head_dim;
  memset(w, 0, sizeof *w);
  w->max_pos = max_pos;
  w->h = malloc(H * 4); w->h2 = malloc(H * 4); w->ln = malloc(H * 4);
  w->q = malloc(QD * 4); w->k = malloc(KV * 4); w->v = malloc(KV * 4);
  w->att = malloc(QD * 4); w->o = malloc(H * 4);
  w->gate = malloc(I * 4); w->up = malloc(I * 4); w->hid = malloc(I * 4); w->down = malloc(H * 4);
  w->hn = malloc(H * 4); w->logits = malloc((size_t)c->vocab * 4);
  w->scores = malloc((size_t)c->n_heads * (size_t)max_pos * 4);
  w->kc = malloc((size_t)c->n_layers * (size_t)max_pos * KV * 4);
  w->vc = malloc((size_t)c->n_layers * (size_t)max_pos * KV * 4);
  return (w->kc && w->vc && w->logits) ? 0 : -1;
}
static void ws_free(ws_t *w) {
  float *ps[] = {w->h, w->h2, w->ln, w->q, w->k, w->v, w->att, w->o, w->gate, w->up,
                 w->hid, w->down, w->hn, w->logits, w->scores, w->kc, w->vc};
  for (size_t i = 0; i < sizeof ps / sizeof ps[0]; ++i) free(ps[i]);
}

/* Trace lines in the reference's --trace format (cis2_model.h:482-496). */
static void trace_emit(FILE *fp, int pos, int layer, const char *op, const float *x, size_t n) {
  if (!fp) return;
  sha_t s;
  sha_init(&s);
  for (size_t i = 0; i < n; ++i) sha_u32le(&s, fbits(x[i]));
  uint8_t d[32];
  sha_final(&s, d);
  fprintf(fp, "pos=%d layer=%d op=%s sha256=", pos, layer, op);
  for (int i = 0; i < 32; ++i) fprintf(fp, "%02x", d[i]);
  fputc('\n', fp);
}

/* RMSNorm (cis2_model.h:511-523): sq = x*x; ss = fold(sq); mean = ss/n;
 * inv = 1/sqrt(mean+eps); out = (x*inv)*w.  In-place safe. */
static void rmsnorm(const float *x, const uint16_t *w, float eps, int n, int tree, float *sq,
                    float *out) {
  for (int i = 0; i < n; ++i) sq[i] = x[i] * x[i];
  float ss = sum_mode(sq, n, tree);
  float mean = ss / (float)n;
  float inv = p_rsqrt(mean + eps);
  for (int i = 0; i < n; ++i) { float s = x[i] * inv; out[i] = s * widen(w[i]); }
}

static void matvec(const uint16_t *W, const float *x, int out_f, int in_f, int tree, float *y) {
  for (int o = 0; o < out_f; ++o) y[o] = dot_row_bf16(W + (size_t)o * (size_t)in_f, x, in_f, tree);
}
static void add_bias(float *x, const uint16_t *b, int n) {
  if (!b) return;
  for (int i = 0; i < n; ++i) x[i] = x[i] + widen(b[i]);
}

/* RoPE rotate-half (cis2_model.h:547-568). */
static void rope(float *x, int n_heads, int hd, int pos, const float *inv_freq) {
  int half = hd / 2;
  for (int h = 0; h < n_heads; ++h) {
    float *head = x + (size_t)h * (size_t)hd;
    for (int i = 0; i < half; ++i) {
      float angle = (float)pos * inv_freq[i];
      float c = p_cos(angle), s = p_sin(angle);
      float x1 = head[i], x2 = head[i + half];
      float t1 = x1 * c;
      float t2 = (-x2) * s;
      float o1 = t1 + t2;
      float t3 = x2 * c;
      float t4 = x1 * s;
      float o2 = t3 + t4;
      head[i] = o1;
      head[i + half] = o2;
    }
  }
}

/* One token through the model (cis2_model.h:685-760 + qwen3-port.diff). */
static void forward_token(const model_t *m, ws_t *w, int pos, uint32_t tok, int want_logits,
                          FILE *tr) {
  const cis2o_config *c = &m->c;
  const int H = c->hidden, I = c->inter, hd = c->head_dim, nh = c->n_heads, nkv = c->n_kv_heads;
  const int QD = nh * hd, KV = nkv * hd, group = nh / nkv, tree = c->tree;
  const float scale = p_rsqrt((float)hd);
  float *sqv = (float *)malloc(sizeof(float) * (size_t)(H > hd ? H : hd)); /* squares scratch */

  const uint16_t *row = m->embed + (size_t)tok * (size_t)H;
  for (int i = 0; i < H; ++i) w->h[i] = widen(row[i]);
  trace_emit(tr, pos, -1, "embedding", w->h, (size_t)H);

  for (int li = 0; li < c->n_layers; ++li) {
    const uint16_t *const *L = m->L + (size_t)li * CIS2O_LAYER_SLOTS;
    float *kc = w->kc + ((size_t)li * (size_t)w->max_pos) * (size_t)KV;
    float *vc = w->vc + ((size_t)li * (size_t)w->max_pos) * (size_t)KV;

    rmsnorm(w->h, L[CIS2O_IN_NORM], c->eps, H, tree, sqv, w->ln);
    trace_emit(tr, pos, li, "norm1", w->ln, (size_t)H);
    matvec(L[CIS2O_Q], w->ln, QD, H, tree, w->q);
    add_bias(w->q, L[CIS2O_Q_BIAS], QD);
    trace_emit(tr, pos, li, "q", w->q, (size_t)QD);
    matvec(L[CIS2O_K], w->ln, KV, H, tree, w->k);
    add_bias(w->k, L[CIS2O_K_BIAS], KV);
    trace_emit(tr, pos, li, "k", w->k, (size_t)KV);
    matvec(L[CIS2O_V], w->ln, KV, H, tree, w->v);
    add_bias(w->v, L[CIS2O_V_BIAS], KV);
    trace_emit(tr, pos, li, "v", w->v, (size_t)KV);
    if (L[CIS2O_Q_NORM]) {
      for (int h = 0; h < nh; ++h)
        rmsnorm(w->q + (size_t)h * hd, L[CIS2O_Q_NORM], c->eps, hd, tree, sqv, w->q + (size_t)h * hd);
      trace_emit(tr, pos, li, "q_norm", w->q, (size_t)QD);
    }
    if (L[CIS2O_K_NORM]) {
      for (int h = 0; h < nkv; ++h)
        rmsnorm(w->k + (size_t)h * hd, L[CIS2O_K_NORM], c->eps, hd, tree, sqv, w->k + (size_t)h * hd);
      trace_emit(tr, pos, li, "k_norm", w->k, (size_t)KV);
    }
    rope(w->q, nh, hd, pos, m->inv_freq);
    trace_emit(tr, pos, li, "rope_q", w->q, (size_t)QD);
    rope(w->k, nkv, hd, pos, m->inv_freq);
    trace_emit(tr, pos, li, "rope_k", w->k, (size_t)KV);
    memcpy(kc + (size_t)pos * KV, w->k, sizeof(float) * (size_t)KV);
    memcpy(vc + (size_t)pos * KV, w->v, sizeof(float) * (size_t)KV);

    const int len = pos + 1;
    for (int qh = 0; qh < nh; ++qh) {
      const float *qv = w->q + (size_t)qh * hd;
      int kvh = qh / group;
      for (int j = 0; j < len; ++j) {
        float d = dot_mode(qv, kc + (size_t)j * KV + (size_t)kvh * hd, hd, tree);
        w->scores[(size_t)qh * len + j] = d * scale;
      }
    }
    trace_emit(tr, pos, li, "scores", w->scores, (size_t)nh * (size_t)len);
    for (int qh = 0; qh < nh; ++qh) softmax_mode(w->scores + (size_t)qh * len, len, tree);
    trace_emit(tr, pos, li, "softmax", w->scores, (size_t)nh * (size_t)len);
    for (int qh = 0; qh < nh; ++qh) {
      int kvh = qh / group;
      const float *sc = w->scores + (size_t)qh * len;
      for (int d = 0; d < hd; ++d) {
        float acc = 0.0f;
        for (int j = 0; j < len; ++j) {
          float p = sc[j] * vc[(size_t)j * KV + (size_t)kvh * hd + d];
          acc = acc + p;
        }
        w->att[(size_t)qh * hd + d] = acc;
      }
    }
    trace_emit(tr, pos, li, "attn_out", w->att, (size_t)QD);
    matvec(L[CIS2O_O], w->att, H, QD, tree, w->o);
    trace_emit(tr, pos, li, "o_proj", w->o, (size_t)H);
    for (int i = 0; i < H; ++i) w->h2[i] = w->h[i] + w->o[i];
    { float *t = w->h; w->h = w->h2; w->h2 = t; }
    trace_emit(tr, pos, li, "resid1", w->h, (size_t)H);

    rmsnorm(w->h, L[CIS2O_POST_NORM], c->eps, H, tree, sqv, w->ln);
    trace_emit(tr, pos, li, "norm2", w->ln, (size_t)H);
    matvec(L[CIS2O_GATE], w->ln, I, H, tree, w->gate);
    trace_emit(tr, pos, li, "gate", w->gate, (size_t)I);
    matvec(L[CIS2O_UP], w->ln, I, H, tree, w->up);
    trace_emit(tr, pos, li, "up", w->up, (size_t)I);
    for (int i = 0; i < I; ++i) { float s = p_silu(w->gate[i]); w->hid[i] = s * w->up[i]; }
    trace_emit(tr, pos, li, "silu_mul", w->hid, (size_t)I);
    matvec(L[CIS2O_DOWN], w->hid, H, I, tree, w->down);
    trace_emit(tr, pos, li, "down", w->down, (size_t)H);
    for (int i = 0; i < H; ++i) w->h2[i] = w->h[i] + w->down[i];
    { float *t = w->h; w->h = w->h2; w->h2 = t; }
    trace_emit(tr, pos, li, "resid2", w->h, (size_t)H);
  }
  free(sqv);
  if (want_logits || tr) {
    rmsnorm(w->h, m->final_norm, c->eps, H, tree, w->down, w->hn);
    trace_emit(tr, pos, -1, "final_norm", w->hn, (size_t)H);
    matvec(m->lm_head, w->hn, c->vocab, H, tree, w->logits);
    trace_emit(tr, pos, -1, "logits", w->logits, (size_t)c->vocab);
  }
}

int cis2o_generate(const void *mp, const uint32_t *prompt_ids, const uint32_t *prompt_lens,
                   uint32_t n_seq, uint32_t gen, const cis2o_sample *sample, const uint8_t hdr[96],
                   uint32_t *out_tokens, uint8_t *out_step_digests, uint8_t *out_witness,
                   uint8_t *out_argmax, const char *trace_path) {
  const model_t *m = (const model_t *)mp;
  const cis2o_config *c = &m->c;
  fpenv_guard g = fp_enter();
  uint32_t max_prompt = 0;
  for (uint32_t s = 0; s < n_seq; ++s) if (prompt_lens[s] > max_prompt) max_prompt = prompt_lens[s];
  ws_t w;
  if (ws_alloc(&w, m, (int)(max_prompt + gen)) != 0) { fp_leave(g); return -1; }
  const int scheme = sample ? sample->enabled : 0;  /* 0 greedy, 1 E23, 2 CIS2-SAMPLE-1 */
  const int sampled = scheme == 1;
  float *scratch = sampled ? (float *)malloc(sizeof(float) * (size_t)c->vocab) : NULL;
  pi_t *order = sampled ? (pi_t *)malloc(sizeof(pi_t) * (size_t)c->vocab) : NULL;
  si_t *gorder = scheme == 2 ? (si_t *)malloc(sizeof(si_t) * (size_t)c->vocab) : NULL;
  FILE *tr = trace_path ? fopen(trace_path, "w") : NULL;
  size_t off = 0;
  for (uint32_t s = 0; s < n_seq; ++s) {
    const uint32_t *ids = prompt_ids + off;
    uint32_t np = prompt_lens[s];
    off += np;
    FILE *trs = (s == 0) ? tr : NULL;
    sha_t wit, ah;
    sha_init(&wit);
    sha_init(&ah);
    if (sampled) { /* e23 patch :617-624 */
      sha_update(&wit, "CIS2_SAMPLE_V1", 14);
      uint8_t le[8];
      for (int i = 0; i < 8; ++i) le[i] = (uint8_t)(sample->seed >> (8 * i));
      sha_update(&wit, le, 8);
      sha_u32le(&wit, fbits(sample->temperature));
      sha_u32le(&wit, fbits(sample->top_p));
    }
    sha_update(&wit, hdr, 96);
    sha_update(&wit, m->table_digest, 32);
    sha_update(&wit, m->inv_freq_digest, 32);
    for (uint32_t i = 0; i < np; ++i) { sha_u32le(&wit, ids[i]); sha_u32le(&ah, ids[i]); }
    if (scheme == 2) { /* seeded-sampling patch :128-134: after the prompt ids */
      sha_update(&wit, "CIS2-SAMPLE-1", 13);
      uint8_t le[8];
      for (int i = 0; i < 8; ++i) le[i] = (uint8_t)(sample->seed >> (8 * i));
      sha_update(&wit, le, 8);
      sha_u32le(&wit, fbits(sample->temperature));
      sha_u32le(&wit, sample->top_k);
      sha_u32le(&wit, fbits(sample->top_p));
    }
    for (uint32_t p = 0; p < np; ++p)
      forward_token(m, &w, (int)p, ids[p], p + 1 == np, trs);
    for (uint32_t t = 0; t < gen; ++t) {
      uint32_t next = sampled
          ? sample_e23(w.logits, c->vocab, sample->temperature, sample->top_p, sample->seed,
                       (uint64_t)np + t, scratch, order)
          : scheme == 2 ? sample_gumbel(w.logits, c->vocab, sample->temperature, sample->top_k, sample->top_p,
                                        sample->seed, t, gorder, NULL)
                        : argmax_first(w.logits, c->vocab);
      for (int i = 0; i < c->vocab; ++i) sha_u32le(&wit, fbits(w.logits[i]));
      sha_u32le(&wit, next);
      sha_u32le(&ah, next);
      out_tokens[(size_t)s * gen + t] = next;
      if (out_step_digests) sha_final(&wit, out_step_digests + ((size_t)s * gen + t) * 32);
      if (t + 1 < gen) forward_token(m, &w, (int)(np + t), next, 1, trs);
    }
    sha_final(&wit, out_witness + (size_t)s * 32);
    sha_final(&ah, out_argmax + (size_t)s * 32);
  }
  if (tr) fclose(tr);
  free(scratch);
  free(order);
  free(gorder);
  ws_free(&w);
  fp_leave(g);
  return 0;
}

int cis2o_logits(const void *mp, const uint32_t *ids, uint32_t n_prompt, uint32_t n_rows,
                 float *out_logits) {
  const model_t *m = (const model_t *)mp;
  fpenv_guard g = fp_enter();
  ws_t w;
  if (ws_alloc(&w, m, (int)(n_prompt + n_rows)) != 0) { fp_leave(g); return -1; }
  uint32_t total = n_prompt + n_rows - 1;
  for (uint32_t p = 0; p < total; ++p) {
    int want = p + 1 >= n_prompt;
    forward_token(m, &w, (int)p, ids[p], want, NULL);
    if (want)
      memcpy(out_logits + (size_t)(p + 1 - n_prompt) * (size_t)m->c.vocab, w.logits,
             sizeof(float) * (size_t)m->c.vocab);
  }
  ws_free(&w);
  fp_leave(g);
  return 0;
}

/* ------------------------------------------------------------ exported scalars */

#define WRAP1(name, fn)                         \
  float name(float x) {                         \
    fpenv_guard g = fp_enter();                 \
    float r = fn(x);                            \
    fp_leave(g);                                \
    return r;                                   \
  }
WRAP1(cis2o_exp, p_exp)
WRAP1(cis2o_sin, p_sin)
WRAP1(cis2o_cos, p_cos)
WRAP1(cis2o_ln, p_ln)
WRAP1(cis2o_silu, p_silu)
WRAP1(cis2o_rsqrt, p_rsqrt)

void cis2o_map(int32_t f, const float *x, float *y, size_t n) {
  fpenv_guard g = fp_enter();
  for (size_t i = 0; i < n; ++i) {
    switch (f) {
      case 0: y[i] = p_exp(x[i]); break;
      case 1: y[i] = p_sin(x[i]); break;
      case 2: y[i] = p_cos(x[i]); break;
      case 3: y[i] = p_ln(x[i]); break;
      case 4: y[i] = p_silu(x[i]); break;
      default: y[i] = p_rsqrt(x[i]); break;
    }
  }
  fp_leave(g);
}

float cis2o_dot(const float *a, const float *b, int32_t n, int32_t tree) {
  fpenv_guard g = fp_enter();
  float r = dot_mode(a, b, n, tree);
  fp_leave(g);
  return r;
}
float cis2o_sum(const float *a, int32_t n, int32_t tree) {
  fpenv_guard g = fp_enter();
  float r = sum_mode(a, n, tree);
  fp_leave(g);
  return r;
}
void cis2o_matmul_bf16(const uint16_t *W, const float *X, int32_t rows, int32_t n_out, int32_t k,
                       int32_t tree, float *Y) {
  fpenv_guard g = fp_enter();
  for (int32_t r = 0; r < rows; ++r)
    matvec(W, X + (size_t)r * (size_t)k, n_out, k, tree, Y + (size_t)r * (size_t)n_out);
  fp_leave(g);
}
void cis2o_softmax(float *v, int32_t n, int32_t tree) {
  fpenv_guard g = fp_enter();
  softmax_mode(v, n, tree);
  fp_leave(g);
}
uint32_t cis2o_argmax(const float *v, int32_t n) { return argmax_first(v, n); }
uint32_t cis2o_sample_pinned(const float *logits, int32_t n, float temperature, float top_p,
                             uint64_t seed, uint64_t position) {
  fpenv_guard g = fp_enter();
  float *sc = (float *)malloc(sizeof(float) * (size_t)n);
  pi_t *ord = (pi_t *)malloc(sizeof(pi_t) * (size_t)n);
  uint32_t r = sample_e23(logits, n, temperature, top_p, seed, position, sc, ord);
  free(sc);
  free(ord);
  fp_leave(g);
  return r;
}
void cis2o_sha256(const uint8_t *data, size_t n, uint8_t out[32]) {
  sha_t s;
  sha_init(&s);
  sha_update(&s, data, n);
  sha_final(&s, out);
}

/* Points of the pinned-function sweep (math_sweep.h), with this port's
 * ln and exp for the RoPE family; out may be NULL to count. */
static float sweep_ln(float x) { return p_ln(x); }
static float sweep_exp(float x) { return p_exp(x); }
size_t cis2o_math_sweep(float *out) {
  fpenv_guard g = fp_enter();
  const size_t n = cis2_math_sweep_inputs(out, sweep_ln, sweep_exp);
  fp_leave(g);
  return n;
}
