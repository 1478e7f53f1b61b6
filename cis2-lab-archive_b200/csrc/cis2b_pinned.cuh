// cis2b_pinned.cuh -- CIS-2 pinned fp32 arithmetic on sm_100a.
//
// Every fp32 operation on the decode path goes through the wrappers below,
// which are single PTX instructions with an explicit round-to-nearest
// modifier and .ftz:
//   * an explicit .rn on mul/add forbids the optimiser from contracting the
//     pair into an FMA (PTX ISA, "add"/"mul" floating-point notes), which is
//     the device form of the reference's -ffp-contract=off / -fmad=false
//     (code/cis2-fp/gpu/Makefile:66-88);
//   * .ftz flushes subnormal inputs and results to sign-preserving zero, the
//     device form of the reference's MXCSR FTZ|DAZ pin (cis2_fpenv.h:62-135,
//     spec §1.3).
// Division and square root are the correctly rounded div.rn / sqrt.rn
// instructions (spec §6.1: IEEE-754 pins their result).
//
// The pinned transcendentals restate the reference's published algorithms
// (code/cis2-fp/gpu/cis2_math.h:270-437; src/math.rs:153-419) with the
// reference's coefficient table (cis2_consts.inc:4-32).  The table is an
// interface of the spec and is reproduced value for value.
#pragma once
#include <stdint.h>

namespace cis2b {

// ------------------------------------------------------------------ constants
// Bit patterns of the CIS-2 v0.3b coefficient table, in the table-digest order.
constexpr uint32_t EXP_LOG2E = 0x3fb8aa3bu, EXP_C1 = 0x3f318000u, EXP_C2 = 0xb95e8083u;
constexpr uint32_t EXP_P0 = 0x39506967u, EXP_P1 = 0x3ab743ceu, EXP_P2 = 0x3c088908u,
                   EXP_P3 = 0x3d2aa9c1u, EXP_P4 = 0x3e2aaaaau, EXP_P5 = 0x3f000000u;
constexpr uint64_t PI_2_F64 = 0x3ff921fb54442d18ull;
constexpr uint32_t SIN_C0 = 0xbe2aaaa3u, SIN_C1 = 0x3c08839eu, SIN_C2 = 0xb94ca1f9u;
constexpr uint32_t COS_C0 = 0x3d2aaaa5u, COS_C1 = 0xbab6061au, COS_C2 = 0x37ccf5ceu;
constexpr uint32_t LOG_SQRTHF = 0x3f3504f3u, LOG_Q1 = 0xb95e8083u, LOG_Q2 = 0x3f318000u;
constexpr uint32_t LOG_P0 = 0x3d9021bbu, LOG_P1 = 0xbdebd1b8u, LOG_P2 = 0x3def251bu,
                   LOG_P3 = 0xbdfe5d4fu, LOG_P4 = 0x3e11e9bfu, LOG_P5 = 0xbe2aae50u,
                   LOG_P6 = 0x3e4cceadu, LOG_P7 = 0xbe7ffffcu, LOG_P8 = 0x3eaaaaaau;

#if defined(__CUDACC__)
#define CIS2B_D __device__ __forceinline__

CIS2B_D float bitsf(uint32_t u) { return __uint_as_float(u); }
CIS2B_D uint32_t fbits(float x) { return __float_as_uint(x); }

// ------------------------------------------------------------------ IEEE ops
CIS2B_D float fadd(float a, float b) {
  float r; asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b)); return r;
}
CIS2B_D float fsub(float a, float b) {
  float r; asm("sub.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b)); return r;
}
CIS2B_D float fmul(float a, float b) {
  float r; asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b)); return r;
}
CIS2B_D float fdiv(float a, float b) {
  float r; asm("div.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b)); return r;
}
CIS2B_D float fsqrt(float a) {
  float r; asm("sqrt.rn.ftz.f32 %0, %1;" : "=f"(r) : "f"(a)); return r;
}
CIS2B_D float fneg(float a) { return __uint_as_float(__float_as_uint(a) ^ 0x80000000u); }
// f32 -> f64 widening and the single f64 -> f32 narrowing of reduce_pi_2,
// with the same subnormal flushing the pinned host environment applies.
CIS2B_D double f2d(float a) {
  double r; asm("cvt.ftz.f64.f32 %0, %1;" : "=d"(r) : "f"(a)); return r;
}
CIS2B_D float d2f(double a) {
  float r; asm("cvt.rn.ftz.f32.f64 %0, %1;" : "=f"(r) : "d"(a)); return r;
}
// Packed pair forms (sm_100): two independent, separately rounded lanes.
CIS2B_D float2 fmul2(float2 a, float2 b) {
  uint64_t ra, rb, rr;
  ra = ((uint64_t)__float_as_uint(a.y) << 32) | __float_as_uint(a.x);
  rb = ((uint64_t)__float_as_uint(b.y) << 32) | __float_as_uint(b.x);
  asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(rr) : "l"(ra), "l"(rb));
  return make_float2(__uint_as_float((uint32_t)rr), __uint_as_float((uint32_t)(rr >> 32)));
}
CIS2B_D float2 fadd2(float2 a, float2 b) {
  uint64_t ra, rb, rr;
  ra = ((uint64_t)__float_as_uint(a.y) << 32) | __float_as_uint(a.x);
  rb = ((uint64_t)__float_as_uint(b.y) << 32) | __float_as_uint(b.x);
  asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(rr) : "l"(ra), "l"(rb));
  return make_float2(__uint_as_float((uint32_t)rr), __uint_as_float((uint32_t)(rr >> 32)));
}

CIS2B_D float widen_bf16(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
CIS2B_D bool is_nan(float x) { return (__float_as_uint(x) & 0x7fffffffu) > 0x7f800000u; }

// ------------------------------------------------------------------ helpers
// Rust-style saturating casts, floor and ties-away round without libm
// (cis2_math.h:112-157).
CIS2B_D int32_t f32_to_i32_sat(float x) {
  if (is_nan(x)) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return __float2int_rz(x);
}
CIS2B_D int64_t f64_to_i64_sat(double x) {
  if (x != x) return 0;
  if (x >= 9223372036854775808.0) return INT64_MAX;
  if (x <= -9223372036854775808.0) return INT64_MIN;
  return __double2ll_rz(x);
}
CIS2B_D float floor_f32(float x) {
  float a = fabsf(x);
  if (!(a < 8388608.0f)) return x;
  float t = __int2float_rn(__float2int_rz(x));
  if (x < t) t = fsub(t, 1.0f);
  return t;
}
CIS2B_D double round_f64_away(double x) {
  double a = fabs(x);
  if (!(a < 4503599627370496.0)) return x;
  double t = __ll2double_rn(__double2ll_rz(a));
  double frac = __dsub_rn(a, t);
  if (frac >= 0.5) t = __dadd_rn(t, 1.0);
  uint64_t tb = (uint64_t)__double_as_longlong(t) & 0x7FFFFFFFFFFFFFFFull;
  uint64_t sb = (uint64_t)__double_as_longlong(x) & 0x8000000000000000ull;
  return __longlong_as_double((long long)(tb | sb));
}
// Exponent-field scaling; underflow gives +0, overflow +-inf (cis2_math.h:275-285).
CIS2B_D float ldexp_exact(float x, int32_t k) {
  if (x == 0.0f) return x;
  uint32_t b = __float_as_uint(x);
  int32_t e = (int32_t)((b >> 23) & 0xFFu) + k;
  if (e <= 0) return 0.0f;
  if (e >= 0xFF) return (b >> 31) ? bitsf(0xFF800000u) : bitsf(0x7F800000u);
  return __uint_as_float((b & ~(0xFFu << 23)) | ((uint32_t)e << 23));
}

// ------------------------------------------------------------------ pinned functions
CIS2B_D float exp_pinned(float x) {
  if (is_nan(x)) return bitsf(0x7FC00000u);
  if (x > 88.0f) return bitsf(0x7F800000u);
  if (x < -88.0f) return 0.0f;
  float t = fmul(x, bitsf(EXP_LOG2E));
  float z0 = fadd(t, 0.5f);
  float k = floor_f32(z0);
  float r0 = fsub(x, fmul(k, bitsf(EXP_C1)));
  float r = fsub(r0, fmul(k, bitsf(EXP_C2)));
  float r2 = fmul(r, r);
  float poly = bitsf(EXP_P0);
  poly = fadd(fmul(poly, r), bitsf(EXP_P1));
  poly = fadd(fmul(poly, r), bitsf(EXP_P2));
  poly = fadd(fmul(poly, r), bitsf(EXP_P3));
  poly = fadd(fmul(poly, r), bitsf(EXP_P4));
  poly = fadd(fmul(poly, r), bitsf(EXP_P5));
  float poly2 = fadd(fmul(poly, r2), r);
  float result = fadd(poly2, 1.0f);
  return ldexp_exact(result, f32_to_i32_sat(k));
}

CIS2B_D void reduce_pi_2(float x, float &r, int64_t &k) {
  double xd = f2d(x);
  double pi2 = __longlong_as_double((long long)PI_2_F64);
  double kf = round_f64_away(__ddiv_rn(xd, pi2));
  double khi = __dmul_rn(kf, pi2);
  double r64 = __dsub_rn(xd, khi);
  r = d2f(r64);
  k = f64_to_i64_sat(kf);
}
CIS2B_D float sin_poly(float r) {
  float r2 = fmul(r, r);
  float in = bitsf(SIN_C2);
  in = fadd(fmul(in, r2), bitsf(SIN_C1));
  in = fadd(fmul(in, r2), bitsf(SIN_C0));
  float r3 = fmul(r2, r);
  return fadd(r, fmul(in, r3));
}
CIS2B_D float cos_poly(float r) {
  float r2 = fmul(r, r);
  float in = bitsf(COS_C2);
  in = fadd(fmul(in, r2), bitsf(COS_C1));
  in = fadd(fmul(in, r2), bitsf(COS_C0));
  float r4 = fmul(r2, r2);
  float term = fmul(in, r4);
  float step1 = fsub(1.0f, fmul(0.5f, r2));
  return fadd(step1, term);
}
CIS2B_D int quadrant(int64_t k) { return (int)(((k % 4) + 4) % 4); }
CIS2B_D float sin_pinned(float x) {
  float r; int64_t k;
  reduce_pi_2(x, r, k);
  float sr = sin_poly(r), cr = cos_poly(r);
  switch (quadrant(k)) {
    case 0: return sr;
    case 1: return cr;
    case 2: return fneg(sr);
    default: return fneg(cr);
  }
}
CIS2B_D float cos_pinned(float x) {
  float r; int64_t k;
  reduce_pi_2(x, r, k);
  float sr = sin_poly(r), cr = cos_poly(r);
  switch (quadrant(k)) {
    case 0: return cr;
    case 1: return fneg(sr);
    case 2: return fneg(cr);
    default: return sr;
  }
}
CIS2B_D float ln_pinned(float x) {
  if (is_nan(x) || x < 0.0f) return bitsf(0x7FC00000u);
  if (x == 0.0f) return bitsf(0xFF800000u);
  uint32_t b = __float_as_uint(x);
  int32_t e = (int32_t)((b >> 23) & 0xFFu) - 126;
  float m = __uint_as_float((b & 0x807FFFFFu) | (126u << 23));
  if (m < bitsf(LOG_SQRTHF)) {
    e -= 1;
    m = fsub(fadd(m, m), 1.0f);
  } else {
    m = fsub(m, 1.0f);
  }
  float z = fmul(m, m);
  float poly = bitsf(LOG_P0);
  poly = fadd(fmul(poly, m), bitsf(LOG_P1));
  poly = fadd(fmul(poly, m), bitsf(LOG_P2));
  poly = fadd(fmul(poly, m), bitsf(LOG_P3));
  poly = fadd(fmul(poly, m), bitsf(LOG_P4));
  poly = fadd(fmul(poly, m), bitsf(LOG_P5));
  poly = fadd(fmul(poly, m), bitsf(LOG_P6));
  poly = fadd(fmul(poly, m), bitsf(LOG_P7));
  poly = fadd(fmul(poly, m), bitsf(LOG_P8));
  float y = fmul(poly, m);
  y = fmul(y, z);
  float fe = __int2float_rn(e);
  y = fadd(y, fmul(fe, bitsf(LOG_Q1)));
  y = fsub(y, fmul(0.5f, z));
  float res = fadd(m, y);
  return fadd(res, fmul(fe, bitsf(LOG_Q2)));
}
CIS2B_D float silu_pinned(float x) {
  float e = exp_pinned(fneg(x));
  return fdiv(x, fadd(1.0f, e));
}
CIS2B_D float rsqrt_cr(float x) { return fdiv(1.0f, fsqrt(x)); }

#endif  // __CUDACC__
}  // namespace cis2b
