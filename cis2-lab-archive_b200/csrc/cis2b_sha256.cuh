// cis2b_sha256.cuh -- SHA-256 (FIPS 180-4) for the CIS-2 witness on sm_100a.
//
// The witness (spec §12, code/cis2-fp/gpu/cis2_host.cpp:179-218) is one
// running SHA-256 per sequence over
//   [E23 prefix "CIS2_SAMPLE_V1"||seed||T||top_p]  (sampled mode only)
//   weights_sha || tokenizer_sha || config_sha || table_digest || inv_freq_digest
//   prompt ids (u32 LE)
//   per step: V logits as u32 LE bit patterns, then the chosen id (u32 LE).
// A Merkle-Damgard chain cannot be split, so the compression runs in ONE
// thread per sequence (32 sequences share a warp's instruction stream).  To
// keep that thread's issue slots for the 64 rounds only, the message
// schedule W[0..63] + K[t] of every block of a step is expanded ahead of
// time by many threads (sha_prep kernel); the compression thread streams
// the expanded words (16 x 16-byte loads per block) and runs the rounds.
#pragma once
#include <stdint.h>

namespace cis2b {

#if defined(__CUDACC__)
__device__ __constant__ uint32_t kShaK[64] = {
  0x428a2f98u,0x71374491u,0xb5c0fbcfu,0xe9b5dba5u,0x3956c25bu,0x59f111f1u,0x923f82a4u,0xab1c5ed5u,
  0xd807aa98u,0x12835b01u,0x243185beu,0x550c7dc3u,0x72be5d74u,0x80deb1feu,0x9bdc06a7u,0xc19bf174u,
  0xe49b69c1u,0xefbe4786u,0x0fc19dc6u,0x240ca1ccu,0x2de92c6fu,0x4a7484aau,0x5cb0a9dcu,0x76f988dau,
  0x983e5152u,0xa831c66du,0xb00327c8u,0xbf597fc7u,0xc6e00bf3u,0xd5a79147u,0x06ca6351u,0x14292967u,
  0x27b70a85u,0x2e1b2138u,0x4d2c6dfcu,0x53380d13u,0x650a7354u,0x766a0abbu,0x81c2c92eu,0x92722c85u,
  0xa2bfe8a1u,0xa81a664bu,0xc24b8b70u,0xc76c51a3u,0xd192e819u,0xd6990624u,0xf40e3585u,0x106aa070u,
  0x19a4c116u,0x1e376c08u,0x2748774cu,0x34b0bcb5u,0x391c0cb3u,0x4ed8aa4au,0x5b9cca4fu,0x682e6ff3u,
  0x748f82eeu,0x78a5636fu,0x84c87814u,0x8cc70208u,0x90befffau,0xa4506cebu,0xbef9a3f7u,0xc67178f2u};

// Per-sequence running state, kept in device memory between steps.
struct ShaState {
  uint32_t h[8];
  uint64_t len;          // bytes absorbed so far (including carry)
  uint32_t carry_n;      // bytes pending in `carry` (0..63)
  uint32_t pad_;
  uint8_t carry[64];     // pending partial block, stream order
};

__device__ __forceinline__ uint32_t rotr(uint32_t x, uint32_t n) { return __funnelshift_r(x, x, n); }

__device__ __forceinline__ void sha_init(uint32_t h[8]) {
  h[0] = 0x6a09e667u; h[1] = 0xbb67ae85u; h[2] = 0x3c6ef372u; h[3] = 0xa54ff53au;
  h[4] = 0x510e527fu; h[5] = 0x9b05688cu; h[6] = 0x1f83d9abu; h[7] = 0x5be0cd19u;
}

// Expand 16 big-endian message words into W[t] + K[t], t = 0..63.
__device__ __forceinline__ void sha_expand_wk(const uint32_t m[16], uint32_t wk[64]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) { w[i] = m[i]; wk[i] = m[i] + kShaK[i]; }
#pragma unroll
  for (int i = 16; i < 64; ++i) {
    uint32_t x15 = w[(i - 15) & 15], x2 = w[(i - 2) & 15];
    uint32_t s0 = rotr(x15, 7) ^ rotr(x15, 18) ^ (x15 >> 3);
    uint32_t s1 = rotr(x2, 17) ^ rotr(x2, 19) ^ (x2 >> 10);
    uint32_t v = w[i & 15] + s0 + w[(i - 7) & 15] + s1;
    w[i & 15] = v;
    wk[i] = v + kShaK[i];
  }
}

// One round with the pre-added W+K word, arranged so that both recurrences
// are three dependent instructions deep:
//   e' = (d + h + WK) + S1(e) + Ch(e,f,g)      -- d, h are 3 rounds old
//   a' = (h + WK) + S1(e) + Ch(e,f,g) + S0(a) + Maj(a,b,c)
// (FIPS 180-4 §6.2.2 step 3, regrouped; integer addition is associative
// mod 2^32, so the result is the same word.)
#define CIS2B_SHA_ROUND(a, b, c, d, e, f, g, h, wkv)                                 \
  do {                                                                               \
    const uint32_t hk_ = (h) + (wkv);                                                \
    const uint32_t x_ = hk_ + (d);                                                   \
    const uint32_t s1_ = rotr((e), 6) ^ rotr((e), 11) ^ rotr((e), 25);               \
    const uint32_t ch_ = ((e) & (f)) ^ (~(e) & (g));                                 \
    const uint32_t s0_ = rotr((a), 2) ^ rotr((a), 13) ^ rotr((a), 22);               \
    const uint32_t mj_ = ((a) & (b)) ^ ((a) & (c)) ^ ((b) & (c));                    \
    const uint32_t t1_ = hk_ + s1_ + ch_;                                            \
    (d) = x_ + s1_ + ch_;                                                            \
    (h) = t1_ + s0_ + mj_;                                                           \
  } while (0)

// The same round balanced across the two issue pipes a lone warp can use.
// Rotations and the bitwise functions (six funnel shifts, four 3-input
// logic ops) need the integer pipe, which accepts one warp instruction per
// two cycles; additions can instead be issued as multiply-adds by a
// runtime `one` on the multiply-add pipe, which runs beside it at the same
// rate.  The round is written as
//   x  = (h + WK) + d                   -- off both recurrences
//   e' = (x + Ch(e,f,g)) + S1(e)        -- = d + T1
//   a' = e' + S0(a) + (Maj(a,b,c) - d)  -- = T1 + T2
// (FIPS 180-4 §6.2.2 step 3, regrouped; integer arithmetic is mod 2^32),
// with five multiply-adds and one 3-input add beside the ten logic ops.
// Measured on B200 with one chain per lane: 24.8 cycles per round against
// 28.2 for the form with three 3-input adds.
__device__ __forceinline__ uint32_t sha_madd(uint32_t x, uint32_t one, uint32_t y) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(one), "r"(y));
  return r;
}
#define CIS2B_SHA_ROUND_M(a, b, c, d, e, f, g, h, wkv, one, neg)                     \
  do {                                                                               \
    const uint32_t x_ = sha_madd(sha_madd((h), (one), (wkv)), (one), (d));           \
    const uint32_t s1_ = rotr((e), 6) ^ rotr((e), 11) ^ rotr((e), 25);               \
    const uint32_t ch_ = ((e) & (f)) ^ (~(e) & (g));                                 \
    const uint32_t s0_ = rotr((a), 2) ^ rotr((a), 13) ^ rotr((a), 22);               \
    const uint32_t mj_ = ((a) & (b)) ^ ((a) & (c)) ^ ((b) & (c));                    \
    const uint32_t md_ = sha_madd((d), (neg), mj_);                                  \
    (d) = sha_madd(s1_, (one), sha_madd(ch_, (one), x_));                            \
    (h) = (d) + s0_ + md_;                                                           \
  } while (0)

// Compress one block given its 64 W+K words; `one` must be 1 (a kernel
// argument, so the compiler cannot fold the multiply-adds into additions).
__device__ __forceinline__ void sha_compress_wk_m(uint32_t st[8], const uint32_t wk[64], uint32_t one) {
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
  const uint32_t neg = 0u - one;
#pragma unroll
  for (int i = 0; i < 64; i += 8) {
    CIS2B_SHA_ROUND_M(a, b, c, d, e, f, g, h, wk[i + 0], one, neg);
    CIS2B_SHA_ROUND_M(h, a, b, c, d, e, f, g, wk[i + 1], one, neg);
    CIS2B_SHA_ROUND_M(g, h, a, b, c, d, e, f, wk[i + 2], one, neg);
    CIS2B_SHA_ROUND_M(f, g, h, a, b, c, d, e, wk[i + 3], one, neg);
    CIS2B_SHA_ROUND_M(e, f, g, h, a, b, c, d, wk[i + 4], one, neg);
    CIS2B_SHA_ROUND_M(d, e, f, g, h, a, b, c, wk[i + 5], one, neg);
    CIS2B_SHA_ROUND_M(c, d, e, f, g, h, a, b, wk[i + 6], one, neg);
    CIS2B_SHA_ROUND_M(b, c, d, e, f, g, h, a, wk[i + 7], one, neg);
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d; st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

// Compress one block given its 64 W+K words (fully unrolled, register-renamed).
__device__ __forceinline__ void sha_compress_wk(uint32_t st[8], const uint32_t wk[64]) {
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll
  for (int i = 0; i < 64; i += 8) {
    CIS2B_SHA_ROUND(a, b, c, d, e, f, g, h, wk[i + 0]);
    CIS2B_SHA_ROUND(h, a, b, c, d, e, f, g, wk[i + 1]);
    CIS2B_SHA_ROUND(g, h, a, b, c, d, e, f, wk[i + 2]);
    CIS2B_SHA_ROUND(f, g, h, a, b, c, d, e, wk[i + 3]);
    CIS2B_SHA_ROUND(e, f, g, h, a, b, c, d, wk[i + 4]);
    CIS2B_SHA_ROUND(d, e, f, g, h, a, b, c, wk[i + 5]);
    CIS2B_SHA_ROUND(c, d, e, f, g, h, a, b, wk[i + 6]);
    CIS2B_SHA_ROUND(b, c, d, e, f, g, h, a, wk[i + 7]);
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d; st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

__device__ __forceinline__ void sha_compress_words(uint32_t st[8], const uint32_t m[16]) {
  uint32_t wk[64];
  sha_expand_wk(m, wk);
  sha_compress_wk(st, wk);
}

// Slow byte-serial absorb, for short inputs (headers, id lists, padding).
// `buf`/`bn` is the caller's pending partial block.
__device__ __forceinline__ void sha_absorb_byte(uint32_t st[8], uint8_t buf[64], uint32_t &bn,
                                                uint8_t byte) {
  buf[bn++] = byte;
  if (bn == 64) {
    uint32_t m[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      m[i] = ((uint32_t)buf[4 * i] << 24) | ((uint32_t)buf[4 * i + 1] << 16) |
             ((uint32_t)buf[4 * i + 2] << 8) | (uint32_t)buf[4 * i + 3];
    sha_compress_words(st, m);
    bn = 0;
  }
}

// Digest of the state WITHOUT modifying it (finalise a copy).
__device__ __forceinline__ void sha_final_copy(const uint32_t h_in[8], uint64_t len,
                                               const uint8_t carry[64], uint32_t carry_n,
                                               uint8_t out[32]) {
  uint32_t st[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) st[i] = h_in[i];
  uint8_t buf[64];
  uint32_t bn = 0;
  for (uint32_t i = 0; i < carry_n; ++i) buf[bn++] = carry[i];
  uint64_t bits = len * 8ull;
  sha_absorb_byte(st, buf, bn, 0x80);
  while (bn != 56) sha_absorb_byte(st, buf, bn, 0);
  for (int i = 0; i < 8; ++i) sha_absorb_byte(st, buf, bn, (uint8_t)(bits >> (56 - 8 * i)));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (uint8_t)(st[i] >> 24); out[4 * i + 1] = (uint8_t)(st[i] >> 16);
    out[4 * i + 2] = (uint8_t)(st[i] >> 8); out[4 * i + 3] = (uint8_t)st[i];
  }
}
#endif  // __CUDACC__

}  // namespace cis2b
