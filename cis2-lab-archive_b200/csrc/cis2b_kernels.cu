// cis2b_kernels.cu -- sm_100a kernels of the CIS-2 deterministic decode path.
//
// Arithmetic contract (what makes every output bit-identical to the
// reference CPU path, code/cis2-fp/gpu/cis2_model.h:503-760):
//   * one output element is produced by ONE thread walking its reduction in
//     the pinned order -- sequential (spec §5.1/§5.3) or the v0.4 32-leaf
//     tree (cis2_math.h:212-265) -- and no reduction is ever split across
//     threads except as the tree prescribes (warp butterflies reproduce the
//     pairwise rounds exactly because IEEE addition is commutative);
//   * every multiply and add is a separately rounded .rn.ftz instruction
//     (cis2b_pinned.cuh);
//   * order-free steps (max, argmax with lowest-index ties, element-wise
//     maps) use parallel reductions with the reference's tie and NaN rules.
// No tensor cores: their fp32 accumulation order is unspecified.
#include "../../include/cis2b.h"
#include "cis2b_kernels.h"
#include "cis2b_pinned.cuh"
#include "cis2b_sha256.cuh"

#include <stdio.h>

#include <mutex>

namespace cis2b {

static constexpr unsigned FULL = 0xffffffffu;

// A kernel's dynamic shared-memory limit.  cudaFuncSetAttribute acts on the
// current device only, and one process may drive several devices (one model
// handle each, possibly from several threads), so each launcher keeps one of
// these per kernel and raises the limit once per device, never lowering it.
struct SmemLimit {
  static constexpr int kMaxDevices = 64;
  std::mutex mu;
  size_t bytes[kMaxDevices] = {};
  template <class F>
  void ensure(F fn, size_t need) {
    int d = -1;
    cudaGetDevice(&d);
    std::lock_guard<std::mutex> lk(mu);
    if (d >= 0 && d < kMaxDevices) {
      if (bytes[d] >= need) return;
      bytes[d] = need;
    }
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need);
  }
};

// ============================================================ reductions

// Pairwise 32-leaf tree across a warp: after round s every lane holds the
// sum of its aligned 2^(s+1)-lane group, built exactly as
// leaf[i] = leaf[2i] + leaf[2i+1] (cis2_math.h:218-228).
__device__ __forceinline__ float warp_tree32(float v) {
#pragma unroll
  for (int s = 1; s < 32; s <<= 1) v = fadd(v, __shfl_xor_sync(FULL, v, s));
  return v;
}

// Asynchronous 16-byte global -> shared copies (sm_80+ cp.async).
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Thread-local pinned dot of two smem/global vectors.
__device__ __forceinline__ float dot_seq(const float *a, const float *b, int n) {
  float acc = 0.0f;
  for (int i = 0; i < n; ++i) acc = fadd(acc, fmul(a[i], b[i]));
  return acc;
}
__device__ __forceinline__ float tree32_local(float *leaf) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) leaf[i] = fadd(leaf[2 * i], leaf[2 * i + 1]);
  return leaf[0];
}
__device__ __forceinline__ float dot_tree(const float *a, const float *b, int n) {
  float acc = 0.0f;
  for (int s = 0; s < n; s += 32) {
    float leaf[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) leaf[i] = (s + i < n) ? fmul(a[s + i], b[s + i]) : 0.0f;
    acc = fadd(acc, tree32_local(leaf));
  }
  return acc;
}

// Strict left-to-right sum of a[0..n) from +0 by ONE thread.  Operands
// are fetched 32 at a time ahead of the dependent adds, so the chain runs
// near add latency (4 cycles) rather than load latency (~34 for shared).
__device__ __forceinline__ float serial_sum(const float *a, int n) {
  float acc = 0.0f;
  int i = 0;
  for (; i + 32 <= n; i += 32) {
    float v[32];
#pragma unroll
    for (int u = 0; u < 32; ++u) v[u] = a[i + u];
#pragma unroll
    for (int u = 0; u < 32; ++u) acc = fadd(acc, v[u]);
  }
  for (; i < n; ++i) acc = fadd(acc, a[i]);
  return acc;
}

// serial_sum for a 16-byte aligned array: the same adds, four operands per load.
__device__ __forceinline__ float serial_sum4(const float *a, int n) {
  const float4 *a4 = reinterpret_cast<const float4 *>(a);
  float acc = 0.0f;
  int q = 0;
  for (; q + 8 <= n / 4; q += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = a4[q + u];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      acc = fadd(acc, v[u].x);
      acc = fadd(acc, v[u].y);
      acc = fadd(acc, v[u].z);
      acc = fadd(acc, v[u].w);
    }
  }
  for (int i = 4 * q; i < n; ++i) acc = fadd(acc, a[i]);
  return acc;
}

// RMSNorm of one row by one warp (cis2_model.h:511-523):
// sq = x*x; ss = fold(sq); mean = ss/n; inv = 1/sqrt(mean+eps); out = (x*inv)*w.
// `sq` is warp-private shared scratch of 2n floats (squares, then a copy of
// x, so the row is read from global memory once).  out (element stride os)
// may alias x.
__device__ __forceinline__ void warp_rmsnorm(const float *x, const uint16_t *w, float eps, int n,
                                             bool tree, float *sq, float *out, int os = 1) {
  const int lane = threadIdx.x & 31;
  float *xc = sq + n;
  for (int i = lane; i < n; i += 32) xc[i] = x[i];
  __syncwarp();
  x = xc;
  float ss;
  if (!tree) {
    for (int i = lane; i < n; i += 32) sq[i] = fmul(x[i], x[i]);
    __syncwarp();
    float acc = 0.0f;
    if (lane == 0) acc = serial_sum(sq, n);
    ss = __shfl_sync(FULL, acc, 0);
  } else {
    float acc = 0.0f;
    for (int s = 0; s < n; s += 32) {
      float v = (s + lane < n) ? fmul(x[s + lane], x[s + lane]) : 0.0f;
      acc = fadd(acc, warp_tree32(v));
    }
    ss = acc;
  }
  float mean = fdiv(ss, __int2float_rn(n));
  float inv = rsqrt_cr(fadd(mean, eps));
  __syncwarp();
  for (int i = lane; i < n; i += 32) out[(size_t)i * os] = fmul(fmul(x[i], inv), widen_bf16(w[i]));
  __syncwarp();
}

// ============================================================ tables

__global__ void k_inv_freq(float theta, int hd, float *out) {
  int i = threadIdx.x + blockIdx.x * blockDim.x;
  if (i >= hd / 2) return;
  // cis2_model.h:456-465: ln of theta narrowed once; frac = (2i)/hd.
  float ln_theta = ln_pinned(theta);
  float frac = fdiv(__int2float_rn(2 * i), __int2float_rn(hd));
  float a = fmul(frac, ln_theta);
  out[i] = exp_pinned(fneg(a));
}

__global__ void k_rope_table(const float *inv_freq, int half, int max_pos, float *cos_t, float *sin_t) {
  size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)half * (size_t)max_pos) return;
  int pos = (int)(idx / half), i = (int)(idx % half);
  // angle = (f32)pos * inv_freq[i] (cis2_model.h:554); cos/sin pinned.
  float angle = fmul(__int2float_rn(pos), inv_freq[i]);
  cos_t[idx] = cos_pinned(angle);
  sin_t[idx] = sin_pinned(angle);
}

void launch_inv_freq(float theta, int hd, float *inv_freq, cudaStream_t s) {
  k_inv_freq<<<1, 256, 0, s>>>(theta, hd, inv_freq);
}
void launch_rope_table(const float *inv_freq, int half, int max_pos, float *cos_t, float *sin_t,
                       cudaStream_t s) {
  size_t n = (size_t)half * (size_t)max_pos;
  k_rope_table<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(inv_freq, half, max_pos, cos_t, sin_t);
}

// ============================================================ embed / norm / elementwise

__global__ void k_embed(const uint16_t *E, int H, const uint32_t *tokens, int rows, float *h) {
  int r = blockIdx.x;
  const uint16_t *src = E + (size_t)tokens[r] * (size_t)H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) h[(size_t)r * H + i] = widen_bf16(src[i]);
}
void launch_embed(const uint16_t *E, int H, const uint32_t *tokens, int rows, float *h,
                  cudaStream_t s) {
  if (rows <= 0) return;
  k_embed<<<rows, 256, 0, s>>>(E, H, tokens, rows, h);
}

__global__ void k_rmsnorm(const float *x, int ldx, const uint16_t *w, float eps, int n, int rows,
                          int tree, float *out, int ors, int ocs) {
  extern __shared__ float sm[];
  int warp = threadIdx.x >> 5;
  int r = blockIdx.x * (blockDim.x >> 5) + warp;
  if (r >= rows) return;
  warp_rmsnorm(x + (size_t)r * ldx, w, eps, n, tree != 0, sm + (size_t)warp * 2 * n,
               out + (size_t)r * ors, ocs);
}
// Sequential-mode RMSNorm of up to 32 rows per block: the block stages its
// rows in shared memory (row pitch n+4 floats, so the 16-byte loads of the
// lanes below hit distinct banks), lane r of warp 0 then runs row r's
// dependent sum of squares -- rb chains side by side, four squares per
// load -- and every thread writes the scaled rows with coalesced stores.
// rb (rows per block, a power of two) is chosen per launch: the chain is the
// same length whatever rb is, so few rows go one or two per block over many
// SMs (decode steps), many rows 32 per block.
constexpr int RMS_ROWS = 32, RMS_THREADS = 256;
__global__ void __launch_bounds__(RMS_THREADS, 1)
k_rmsnorm_rows(const float *__restrict__ x, int ldx, const uint16_t *__restrict__ w, float eps, int n, int rows,
               int rb, float *__restrict__ out, int ors, int ocs) {
  extern __shared__ __align__(16) float sm[];  // [rb][n + 4], then [RMS_ROWS] inv
  const int P = n + 4, nq = n / 4;
  float *inv_s = sm + rb * P;
  const int r0 = blockIdx.x * rb;
  const int nr = min(rb, rows - r0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = RMS_THREADS / 32;
  const uint32_t sb = (uint32_t)__cvta_generic_to_shared(sm);
  for (int i = threadIdx.x; i < nr * nq; i += RMS_THREADS) {
    const int r = i / nq, q = i - r * nq;
    cp_async16(sb + (uint32_t)((r * P + 4 * q) * 4), x + (size_t)(r0 + r) * ldx + 4 * q);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  if (threadIdx.x < nr) {
    const float4 *row = reinterpret_cast<const float4 *>(sm + threadIdx.x * P);
    float acc = 0.0f;
    int q = 0;
    for (; q + 8 <= nq; q += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = row[q + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc = fadd(acc, fmul(v[u].x, v[u].x));
        acc = fadd(acc, fmul(v[u].y, v[u].y));
        acc = fadd(acc, fmul(v[u].z, v[u].z));
        acc = fadd(acc, fmul(v[u].w, v[u].w));
      }
    }
    for (; q < nq; ++q) {
      const float4 v = row[q];
      acc = fadd(acc, fmul(v.x, v.x));
      acc = fadd(acc, fmul(v.y, v.y));
      acc = fadd(acc, fmul(v.z, v.z));
      acc = fadd(acc, fmul(v.w, v.w));
    }
    const float mean = fdiv(acc, __int2float_rn(n));
    inv_s[threadIdx.x] = rsqrt_cr(fadd(mean, eps));
  }
  __syncthreads();
  if (ocs == 1) {  // row-major out: a warp per row, lanes along k
    for (int r = warp; r < nr; r += nw) {
      const float inv = inv_s[r];
      float *o = out + (size_t)(r0 + r) * ors;
      for (int k = lane; k < n; k += 32) o[k] = fmul(fmul(sm[r * P + k], inv), widen_bf16(w[k]));
    }
  } else {  // k-major out: a warp covers rb rows (lanes along rows first) x 32 / rb k
    const int r = lane % rb, kw = 32 / rb;
    if (r < nr) {
      const float inv = inv_s[r];
      for (int k = warp * kw + lane / rb; k < n; k += nw * kw)
        out[(size_t)(r0 + r) * ors + (size_t)k * ocs] = fmul(fmul(sm[r * P + k], inv), widen_bf16(w[k]));
    }
  }
}

void launch_rmsnorm(const float *x, int ldx, const uint16_t *w, float eps, int n, int rows, bool tree,
                    float *out, int ors, int ocs, cudaStream_t s) {
  if (rows <= 0) return;
  // Rows per block: a power of two, so that all 148 SMs get a block before a
  // block takes more rows (at most 32).
  int rb = 1;
  while (rb < RMS_ROWS && rb * 148 < rows) rb *= 2;
  const size_t rsm = ((size_t)rb * (n + 4) + RMS_ROWS) * sizeof(float);
  if (!tree && n % 4 == 0 && ldx % 4 == 0 && ((uintptr_t)x & 15) == 0 && rsm <= 227 * 1024) {
    static SmemLimit lim;
    lim.ensure(k_rmsnorm_rows, 227 * 1024);
    k_rmsnorm_rows<<<(rows + rb - 1) / rb, RMS_THREADS, rsm, s>>>(x, ldx, w, eps, n, rows, rb, out, ors, ocs);
    return;
  }
  const int wpb = 4;
  k_rmsnorm<<<(rows + wpb - 1) / wpb, 32 * wpb, (size_t)wpb * 2 * n * sizeof(float), s>>>(
      x, ldx, w, eps, n, rows, tree ? 1 : 0, out, ors, ocs);
}

// gu rows hold gate and up interleaved: gate i at 2i, up i at 2i + 1 (the
// gate/up panels are laid out that way, see launch_panelize).
__global__ void k_silu_mul(const float *gu, int I, int rows, float *hid, int hrs, int hcs) {
  size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)rows * I) return;
  size_t r = idx / I, i = idx % I;
  const float2 gv = reinterpret_cast<const float2 *>(gu + r * 2 * (size_t)I)[i];
  hid[r * hrs + i * hcs] = fmul(silu_pinned(gv.x), gv.y);  // silu(g)*up (cis2_model.h:619-623)
}
void launch_silu_mul(const float *gu, int I, int rows, float *hid, int hrs, int hcs, cudaStream_t s) {
  size_t n = (size_t)rows * I;
  if (!n) return;
  k_silu_mul<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(gu, I, rows, hid, hrs, hcs);
}

__global__ void k_add_bias(float *x, int ld, int rows, const uint16_t *b, int n) {
  size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)rows * n) return;
  size_t r = idx / n, i = idx % n;
  float *p = x + r * ld + i;
  *p = fadd(*p, widen_bf16(b[i]));  // cis2_model.h:535-538
}
void launch_add_bias(float *x, int ld, int rows, const uint16_t *b, int n, cudaStream_t s) {
  size_t tot = (size_t)rows * n;
  if (!b || !tot) return;
  k_add_bias<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(x, ld, rows, b, n);
}

__global__ void k_pinned_map(int fn, const float *x, float *y, size_t n) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = x[i], r;
  switch (fn) {
    case 0: r = exp_pinned(v); break;
    case 1: r = sin_pinned(v); break;
    case 2: r = cos_pinned(v); break;
    case 3: r = ln_pinned(v); break;
    case 4: r = silu_pinned(v); break;
    default: r = rsqrt_cr(v); break;
  }
  y[i] = r;
}
void launch_pinned_map(int fn, const float *x, float *y, size_t n, cudaStream_t s) {
  if (!n) return;
  k_pinned_map<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(fn, x, y, n);
}

// ============================================================ GEMM
//
// Y[m][n] = dot(W[n][:], X[m][:]) for M activation rows and N outputs.
// One thread owns a TM x TN tile of outputs and walks k = 0..K-1 in order
// for all of them: register tiling shares shared-memory loads between
// outputs without ever splitting a dot product.
//
// Operand layouts (chosen so every tile is a run of 16-byte chunks that
// cp.async can move without a register round trip):
//   X^T  [K][ldm] fp32   activations k-major (the producing kernels write it)
//   Wp   [N8][K][8] bf16 weights in 8-row k-major panels, re-laid once at
//                        load from the checkpoint's [N][K] (same bf16 bits)
// STAGES k-tiles of 32 are in flight; the widen bits<<16 happens as a
// thread reads its weights.  Padding past K or N is zero-filled by cp.async:
// a +0 product leaves a sequential accumulator unchanged (it starts at +0
// and can never become -0) and is the spec's own zero leaf in tree mode.
constexpr int GEMM_KT = 32;
constexpr int GEMM_STAGES = 4;

__device__ __forceinline__ void cp_async16_zfill(uint32_t saddr, const void *g, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(sz) : "memory");
}

template <int BM, int BP, int TM, int TN, bool TREE>
__global__ void __launch_bounds__((BM / TM) * (8 * BP / TN), 1)
k_gemm_t(const float *__restrict__ XT, int ldm, const uint16_t *__restrict__ Wp, int K, int N, int M,
         float *__restrict__ Y, int ldy, const float *__restrict__ R, int ldr, const int32_t *y_slot,
         size_t y_slot_stride) {
  constexpr int BN = 8 * BP;
  constexpr int NT = (BM / TM) * (BN / TN);
  constexpr int XF = GEMM_KT * BM;            // floats per X stage
  constexpr int WH = GEMM_KT * BN;            // bf16 per W stage
  constexpr int XCH = GEMM_KT * BM / 4;       // 16-byte chunks per X stage
  constexpr int WCH = GEMM_KT * BP;           // 16-byte chunks per W stage
  extern __shared__ __align__(16) float smem[];
  float *Xs = smem;                                                  // [S][KT][BM]
  uint16_t *Ws = reinterpret_cast<uint16_t *>(smem + GEMM_STAGES * XF);  // [S][KT][BP][8]
  const int tid = threadIdx.x;
  const int tn = tid % (BN / TN), tm = tid / (BN / TN);
  const int n8_0 = blockIdx.x * BP, m0 = blockIdx.y * BM;
  const int N8 = (N + 7) / 8;
  const uint32_t xs_base = (uint32_t)__cvta_generic_to_shared(Xs);
  const uint32_t ws_base = (uint32_t)__cvta_generic_to_shared(Ws);

  auto issue = [&](int kt) {
    const int slot = kt % GEMM_STAGES, k0 = kt * GEMM_KT;
    for (int c = tid; c < XCH; c += NT) {
      const int k = c / (BM / 4), q = c % (BM / 4);
      const bool ok = (k0 + k < K) && (m0 + 4 * q < ldm);
      const float *src = ok ? XT + (size_t)(k0 + k) * ldm + m0 + 4 * q : XT;
      cp_async16_zfill(xs_base + (uint32_t)((slot * XF + k * BM + 4 * q) * 4), src, ok);
    }
    for (int c = tid; c < WCH; c += NT) {
      const int k = c / BP, p = c % BP;
      const bool ok = (k0 + k < K) && (n8_0 + p < N8);
      const uint16_t *src = ok ? Wp + ((size_t)(n8_0 + p) * K + k0 + k) * 8 : Wp;
      cp_async16_zfill(ws_base + (uint32_t)((slot * WH + (k * BP + p) * 8) * 2), src, ok);
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  const int nk = (K + GEMM_KT - 1) / GEMM_KT;
#pragma unroll
  for (int s = 0; s < GEMM_STAGES - 1; ++s) {
    if (s < nk) issue(s);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  const int nl0 = tn * TN;                     // first output column of this thread (within BN)
  const int wp = nl0 / 8, wj = nl0 % 8;        // panel and lane within the panel
  for (int kt = 0; kt < nk; ++kt) {
    asm volatile("cp.async.wait_group %0;" ::"n"(GEMM_STAGES - 2) : "memory");
    __syncthreads();
    if (kt + GEMM_STAGES - 1 < nk) issue(kt + GEMM_STAGES - 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const int slot = kt % GEMM_STAGES;
    const float *xs = Xs + slot * XF + tm * TM;
    const uint16_t *ws = Ws + slot * WH + wp * 8 + wj;
    if (!TREE) {
      // Operands of GRP k-steps are fetched into registers one group ahead
      // of the multiply-adds that use them, so the ~34-cycle shared-memory
      // latency overlaps the dependent-add chain instead of adding to it.
      constexpr int GRP = (TM + TN <= 4) ? 8 : 4;
      constexpr int NG = GEMM_KT / GRP;
      float xr[2][GRP][TM], wr[2][GRP][TN];
      auto fetch = [&](int buf, int g) {
#pragma unroll
        for (int u = 0; u < GRP; ++u) {
          const int kk = g * GRP + u;
#pragma unroll
          for (int i = 0; i < TM; ++i) xr[buf][u][i] = xs[kk * BM + i];
#pragma unroll
          for (int j = 0; j < TN; ++j) wr[buf][u][j] = widen_bf16(ws[kk * BN + j]);
        }
      };
      fetch(0, 0);
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        if (g + 1 < NG) fetch((g + 1) & 1, g + 1);
#pragma unroll
        for (int u = 0; u < GRP; ++u)
#pragma unroll
          for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j)
              acc[i][j] = fadd(acc[i][j], fmul(wr[g & 1][u][j], xr[g & 1][u][i]));
      }
    } else {
      // Streaming pairwise tree over the 32 leaves of this k tile: level L
      // holds the pending left operand; leaf kk closes as many levels as kk
      // has trailing one bits.  Same adds, same operands as tree32.
      float lv[5][TM][TN];
#pragma unroll
      for (int kk = 0; kk < GEMM_KT; ++kk) {
        float x[TM], w[TN];
#pragma unroll
        for (int i = 0; i < TM; ++i) x[i] = xs[kk * BM + i];
#pragma unroll
        for (int j = 0; j < TN; ++j) w[j] = widen_bf16(ws[kk * BN + j]);
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            float v = fmul(w[j], x[i]);
            int t = kk, lvl = 0;
#pragma unroll
            for (int q = 0; q < 5; ++q) {
              if (t & 1) { v = fadd(lv[lvl][i][j], v); t >>= 1; ++lvl; }
              else break;
            }
            if (lvl < 5) lv[lvl][i][j] = v;
            else acc[i][j] = fadd(acc[i][j], v);
          }
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");

  float *Yb = Y + (y_slot ? (size_t)(*y_slot) * y_slot_stride : 0);
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + tm * TM + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n8_0 * 8 + nl0 + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (R) v = fadd(R[(size_t)m * ldr + n], v);  // residual h + o (cis2_model.h:540-542)
      Yb[(size_t)m * ldy + n] = v;
    }
  }
}

template <int BM, int BP, int TM, int TN, bool TREE>
static void run_gemm_t(const float *XT, int ldm, const uint16_t *Wp, int K, int N, int M, float *Y, int ldy,
                       const float *R, int ldr, const int32_t *y_slot, size_t y_slot_stride, cudaStream_t s) {
  constexpr int NT = (BM / TM) * (8 * BP / TN);
  const size_t smem = (size_t)GEMM_STAGES * (GEMM_KT * BM * 4 + GEMM_KT * 8 * BP * 2);
  static SmemLimit lim;
  lim.ensure(k_gemm_t<BM, BP, TM, TN, TREE>, smem);
  dim3 grid((N + 8 * BP - 1) / (8 * BP), (M + BM - 1) / BM);
  k_gemm_t<BM, BP, TM, TN, TREE><<<grid, NT, smem, s>>>(XT, ldm, Wp, K, N, M, Y, ldy, R, ldr, y_slot,
                                                          y_slot_stride);
}

// Tile choice.  No dot product may be split, so a GEMM of M rows and N
// outputs has exactly M*N serial chains to spread over 148 SMs x 4
// schedulers.  Each candidate is scored by the issue cycles of the busiest
// SM (its CTAs' multiply-adds over the fraction of issue slots that are
// FP32 work, spread over the schedulers its warps occupy), floored by the
// dependent-add latency of one chain.
struct TileCfg { int bm, bp, tm, tn; };
static const TileCfg kTiles[] = {{64, 4, 4, 4}, {64, 2, 4, 2}, {32, 1, 2, 1}, {16, 2, 2, 1}, {4, 4, 1, 1},
                                 {32, 2, 2, 2}, {32, 4, 2, 4}};
constexpr int kNumTiles = 7;

static double tile_cost(const TileCfg &c, int M, int N, int K) {
  const int bn = 8 * c.bp;
  const long ctas = (long)((N + bn - 1) / bn) * ((M + c.bm - 1) / c.bm);
  const int threads = (c.bm / c.tm) * (bn / c.tn);
  const long per_sm = (ctas + 147) / 148;
  const double fp = 2.0 * c.tm * c.tn;
  const double other = (c.tm + 3) / 4 + 1 + c.tn;   // x loads, w load, widens
  const double eff = fp / (fp + other);
  const double warps = (double)per_sm * threads / 32.0;
  const double sched = warps < 4.0 ? warps : 4.0;
  const double issue = (double)per_sm * c.bm * bn * K * 2.0 / eff / (32.0 * sched);
  const double chain = 4.0 * K;
  return issue > chain ? issue : chain;
}

int gemm_tile_choice(int M, int N, int K, bool tree) {
  int best = -1;
  double best_cost = 0;
  for (int i = 0; i < kNumTiles; ++i) {
    const TileCfg &c = kTiles[i];
    if (tree && c.tm * c.tn > 8) continue;       // tree mode keeps 5 pending levels per output
    if (c.bm > 4 && M < c.bm / 2) continue;      // at most half a row tile wasted
    const double cost = tile_cost(c, M, N, K);
    if (best < 0 || cost < best_cost * 0.97) { best = i; best_cost = cost; }
  }
  return best;
}

// ---- many rows (the prompt pass, lm_head over 64 rows or more, and decode
// steps with many rows), sequential order: a block tile of up to 128 x 64
// outputs over up to 256 threads, up to 8 x 4 per thread.  Per k a thread
// reads its activations as broadcast 16-byte loads and its weights as 8- or
// 16-byte loads (the activation tile is [k][m], the weight tile [k][n], both
// conflict-free), then does its multiply-adds; each output still walks
// k = 0..K-1 in order.  Products are rounded singly and added as pairs of
// independent accumulators with add.rn.ftz.f32x2, which halves the issue
// slots the adds take.  The weights come from fp32 panels (the checkpoint's
// bf16 widened once at load, which is exact), so the inner loop spends no
// issue slots on widening: measured on B200, 4-20 % faster than widening
// bf16 panels per thread and per k, from 256 x 576 x 576 to 4,096 x 3,072
// x 576.  Operands arrive through an ST-deep cp.async ring of KT-deep k
// stages (ST and KT per tile: the few-warp tiles of decode steps gain from
// 32-deep stages, measured 5-15 % over 16).
// Two independent, separately rounded products (lanes of one packed op).
__device__ __forceinline__ float2 fmul_pair(float a0, float a1, float b0, float b1) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rr;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.ftz.f32x2 rr, ra, rb;\n\tmov.b64 {%0, %1}, rr;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
  return r;
}

__device__ __forceinline__ float2 fadd_pair(float2 a, float b0, float b1) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rr;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.ftz.f32x2 rr, ra, rb;\n\tmov.b64 {%0, %1}, rr;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b0), "f"(b1));
  return r;
}

// tree_group (below) on two independent chains at once (packed adds).
__device__ __forceinline__ void tree_group2(float2 &acc, float2 &t3, float2 &t4, float2 &t5, float2 c, int g) {
  if ((g & 1) == 0) { t3 = c; return; }
  const float2 l3 = fadd_pair(t3, c.x, c.y);
  if ((g & 2) == 0) { t4 = l3; return; }
  const float2 l4 = fadd_pair(t4, l3.x, l3.y);
  if ((g & 4) == 0) { t5 = l4; return; }
  const float2 b = fadd_pair(t5, l4.x, l4.y);
  acc = fadd_pair(acc, b.x, b.y);
}

// Block tile BM x BN over TY x TX threads; a thread owns TMR rows x TNC
// columns (TMR * TNC output chains).  Rows come in blocks of RW = min(TMR,
// 4) consecutive rows, RW * TY apart; columns in blocks of CW = min(TNC, 4),
// CW * TX apart, and columns (n, n + 1) share one packed accumulator.
// Per k a thread reads its rows' activations (one 8- or 16-byte load per
// row block) and its columns' weights (one 8- or 16-byte load per column
// block), forms its products singly and adds them as packed pairs of
// independent accumulators (add.f32x2): every output still walks
// k = 0..K-1 in order.  The products stay scalar: with packed products
// (mul.f32x2) feeding the packed adds, B200 results no longer matched the
// pinned order bit for bit (measured: most outputs of every tile shape
// differed), so that pairing is never formed here.
// Wpf: fp32 panels [N8][K][8] (launch_panelize into float).
// TREE: the v0.4 tree order (K % 32 == 0; a KT = 32 stage is one block):
// the products of four consecutive k form ((p0 + p1) + (p2 + p3)) per
// chain, and the eight group sums of the block join in three more pairwise
// levels (tree_group2) before the block sum is added to the chain.
// Output element (m, n) goes to Y[m * ysm + n * ysn] (row-major: ysm = ldy,
// ysn = 1; k-major for the next product: ysm = 1, ysn = ldm).  glu: W is a
// gate/up pair panelised with its rows interleaved (gate i, up i at rows 2i,
// 2i + 1), so a column pair (n, n + 1) is (gate i, up i) and the epilogue
// writes silu(gate) * up as output column i = n / 2 (cis2_model.h:619-623).
template <int TY, int TX, int TMR, int TNC, int ST, int KT, bool TREE>
__global__ void __launch_bounds__(TY * TX, 1)
k_gemm_big(const float *__restrict__ XT, int ldm, const float *__restrict__ Wpf, int K, int N, int M,
           float *__restrict__ Y, int ysm, int ysn, const float *__restrict__ R, int ldr, const int32_t *y_slot,
           size_t y_slot_stride, int glu) {
  constexpr int RW = TMR < 4 ? TMR : 4, RB = TMR / RW;
  constexpr int CW = TNC < 4 ? TNC : 4, CB = TNC / CW;
  constexpr int NT = TY * TX, BM = RW * TY * RB, BN = CW * TX * CB;
  constexpr int XF = KT * BM;      // floats per X stage
  constexpr int WF = KT * BN;      // floats per W stage
  constexpr int TNP = TNC / 2;     // column pairs per thread
  constexpr int XCH = XF / 4;      // 16-byte X chunks per stage
  constexpr int WCH = WF / 4;      // 16-byte W chunks per stage
  constexpr int PF = TMR * TNC >= 16 ? 2 : 4;  // register prefetch distance, k-steps
  static_assert((RW == 2 || RW == 4) && (CW == 2 || CW == 4) && BM % 4 == 0 && BN % 8 == 0, "tile shape");
  static_assert(ST >= 2 && KT % 4 == 0 && (!TREE || KT == 32), "pipeline shape");
  extern __shared__ __align__(16) float smem[];
  float *Xs = smem;            // [ST][KT][BM]
  float *Ws = smem + ST * XF;  // [ST][KT][BN]
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN, n8_0 = n0 / 8;
  const int N8 = (N + 7) / 8;
  const uint32_t xs_b = (uint32_t)__cvta_generic_to_shared(Xs), ws_b = (uint32_t)__cvta_generic_to_shared(Ws);
  auto issue = [&](int kt) {
    const int slot = kt % ST, k0 = kt * KT;
#pragma unroll
    for (int r = 0; r < (XCH + NT - 1) / NT; ++r) {  // X: KT rows of BM floats
      const int c = tid + r * NT, k = c / (BM / 4), q = c % (BM / 4);
      if (c < XCH) {
        const bool ok = (k0 + k < K) && (m0 + 4 * q < ldm);
        const float *src = ok ? XT + (size_t)(k0 + k) * ldm + m0 + 4 * q : XT;
        cp_async16_zfill(xs_b + (uint32_t)((slot * XF + k * BM + 4 * q) * 4), src, ok);
      }
    }
#pragma unroll
    for (int r = 0; r < (WCH + NT - 1) / NT; ++r) {  // W: KT x BN/4 halves of 8-column panels, to [k][n]
      const int c = tid + r * NT, k = c / (BN / 4), h = c % (BN / 4), pnl = h / 2;
      if (c < WCH) {
        const bool ok = (k0 + k < K) && (n8_0 + pnl < N8);
        const float *src = ok ? Wpf + ((size_t)(n8_0 + pnl) * K + k0 + k) * 8 + (h & 1) * 4 : Wpf;
        cp_async16_zfill(ws_b + (uint32_t)((slot * WF + k * BN + 4 * h) * 4), src, ok);
      }
    }
  };
  float2 acc[TMR][TNP];
  // Tree order only (unused, so not allocated, otherwise): the pending
  // pairwise sums of the current 32-k block.
  float2 l1[TMR][TNP], l1b[TMR][TNP], t3[TMR][TNP], t4[TMR][TNP], t5[TMR][TNP];
#pragma unroll
  for (int i = 0; i < TMR; ++i)
#pragma unroll
    for (int j = 0; j < TNP; ++j) acc[i][j] = make_float2(0.0f, 0.0f);
  const int nk = (K + KT - 1) / KT;
#pragma unroll
  for (int st = 0; st < ST - 1; ++st) {
    if (st < nk) issue(st);
    cp_async_commit();
  }
  for (int kt = 0; kt < nk; ++kt) {
    cp_async_wait<ST - 2>();
    __syncthreads();
    if (kt + ST - 1 < nk) issue(kt + ST - 1);
    cp_async_commit();
    const int slot = kt % ST;
    const float *xs = Xs + slot * XF + ty * RW;
    const float *ws = Ws + slot * WF + tx * CW;
    // The operands of the next PF k-steps are loaded into registers ahead of
    // the products that use them: with few warps per scheduler (the decode
    // steps) nothing else hides the shared-memory latency.
    float xb[PF][TMR], wb[PF][TNC];
    auto ld = [&](int b, int k) {
#pragma unroll
      for (int g = 0; g < RB; ++g) {
        if (RW == 4) {
          const float4 xv = *reinterpret_cast<const float4 *>(xs + k * BM + g * RW * TY);
          xb[b][4 * g] = xv.x; xb[b][4 * g + 1] = xv.y; xb[b][4 * g + 2] = xv.z; xb[b][4 * g + 3] = xv.w;
        } else {
          const float2 xv = *reinterpret_cast<const float2 *>(xs + k * BM + g * RW * TY);
          xb[b][2 * g] = xv.x; xb[b][2 * g + 1] = xv.y;
        }
      }
#pragma unroll
      for (int h = 0; h < CB; ++h) {
        if (CW == 4) {
          const float4 wv = *reinterpret_cast<const float4 *>(ws + k * BN + CW * TX * h);
          wb[b][4 * h] = wv.x; wb[b][4 * h + 1] = wv.y; wb[b][4 * h + 2] = wv.z; wb[b][4 * h + 3] = wv.w;
        } else {
          const float2 wv = *reinterpret_cast<const float2 *>(ws + k * BN + CW * TX * h);
          wb[b][2 * h] = wv.x; wb[b][2 * h + 1] = wv.y;
        }
      }
    };
#pragma unroll
    for (int q = 0; q < PF; ++q) ld(q, q);
#pragma unroll
    for (int k = 0; k < KT; ++k) {
      const int b = k % PF;
      float x[TMR], w[TNC];
#pragma unroll
      for (int i = 0; i < TMR; ++i) x[i] = xb[b][i];
#pragma unroll
      for (int j = 0; j < TNC; ++j) w[j] = wb[b][j];
      if (k + PF < KT) ld(b, k + PF);
      if (TREE) {
        const int km = k & 3;
#pragma unroll
        for (int i = 0; i < TMR; ++i)
#pragma unroll
          for (int j = 0; j < TNP; ++j) {
            const float2 pp = make_float2(fmul(w[2 * j], x[i]), fmul(w[2 * j + 1], x[i]));
            if (km == 0) {
              l1[i][j] = pp;
            } else if (km == 1) {
              l1[i][j] = fadd_pair(l1[i][j], pp.x, pp.y);
            } else if (km == 2) {
              l1b[i][j] = pp;
            } else {
              const float2 l2b = fadd_pair(l1b[i][j], pp.x, pp.y);
              const float2 c = fadd_pair(l1[i][j], l2b.x, l2b.y);
              tree_group2(acc[i][j], t3[i][j], t4[i][j], t5[i][j], c, (k >> 2) & 7);
            }
          }
      } else {
#pragma unroll
        for (int i = 0; i < TMR; ++i)
#pragma unroll
          for (int j = 0; j < TNP; ++j)
            acc[i][j] = fadd_pair(acc[i][j], fmul(w[2 * j], x[i]), fmul(w[2 * j + 1], x[i]));
      }
    }
  }
  cp_async_wait<0>();
  float *Yb = Y + (y_slot ? (size_t)(*y_slot) * y_slot_stride : 0);
#pragma unroll
  for (int i = 0; i < TMR; ++i) {
    const int m = m0 + (i / RW) * RW * TY + ty * RW + (i % RW);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TNP; ++j) {
      const int n = n0 + (2 * j / CW) * CW * TX + tx * CW + (2 * j) % CW;
      float2 v = acc[i][j];
      if (glu) {
        if (n < N) Yb[(size_t)m * ysm + (size_t)(n / 2) * ysn] = fmul(silu_pinned(v.x), v.y);
        continue;
      }
      if (R) {  // residual h + o (cis2_model.h:540-542)
        if (n < N) v.x = fadd(R[(size_t)m * ldr + n], v.x);
        if (n + 1 < N) v.y = fadd(R[(size_t)m * ldr + n + 1], v.y);
      }
      if (n < N) Yb[(size_t)m * ysm + (size_t)n * ysn] = v.x;
      if (n + 1 < N) Yb[(size_t)m * ysm + (size_t)(n + 1) * ysn] = v.y;
    }
  }
}

template <int TY, int TX, int TMR, int TNC, int ST, int KT, bool TREE>
static void run_gemm_big(const float *XT, int ldm, const float *Wpf, int K, int N, int M, float *Y, int ysm, int ysn,
                         const float *R, int ldr, const int32_t *y_slot, size_t y_slot_stride, int glu,
                         cudaStream_t s) {
  constexpr int BM = TMR * TY, BN = TNC * TX;
  const size_t smem = (size_t)ST * KT * (BM + BN) * 4;
  static SmemLimit lim;
  lim.ensure(k_gemm_big<TY, TX, TMR, TNC, ST, KT, TREE>, smem);
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  k_gemm_big<TY, TX, TMR, TNC, ST, KT, TREE><<<grid, TY * TX, smem, s>>>(XT, ldm, Wpf, K, N, M, Y, ysm, ysn, R,
                                                                          ldr, y_slot, y_slot_stride, glu);
}

// Block tile choice for the sequential product from 64 rows on (the prompt
// pass, lm_head, and decode steps with many rows).  No dot product may be
// split, so M x N chains are all the parallelism there is; a tile trades
// chains per thread (fewer loads per product, fewer issue slots) against
// warps (every scheduler of every SM needs work).  Cost = the largest
// per-SM share of the outputs over the fraction of its FP32 pipe the SM's
// warps can keep busy: one warp per scheduler suffices from 8 chains per
// thread on, two from 4, and issue efficiency falls a little with the
// chains per thread.  Measured on B200 with the tiles below: 0.73-0.80 of
// the FP32 pipe on lm_head (256-300 rows) and the prompt-pass projections
// (4,096 rows); 0.37-0.64 on the decode-step projections of 256-300 rows,
// where 300 x 768 outputs are under one warp per scheduler.
struct BigCfg { int ty, tx, tmr, tnc; };
static const BigCfg kBigTiles[] = {{16, 16, 8, 4}, {16, 16, 4, 4}, {16, 8, 4, 4}, {16, 8, 4, 2}, {8, 16, 2, 2}};
constexpr int kNumBigTiles = 5;

bool gemm_big_ok(int K, bool tree) { return !tree || K % 32 == 0; }

int gemm_big_choice(int M, int N, bool tree) {
  int best = -1;
  double best_cost = 0;
  for (int i = 0; i < kNumBigTiles; ++i) {
    const BigCfg &c = kBigTiles[i];
    const int bm = c.tmr * c.ty, bn = c.tnc * c.tx, nt = c.ty * c.tx, chains = c.tmr * c.tnc;
    if (tree && chains > 16) continue;               // the tree's pending sums take 6 registers per chain pair
    if (best >= 0 && M < bm / 2) continue;           // at most half a row tile wasted
    const long blocks = (long)((M + bm - 1) / bm) * ((N + bn - 1) / bn);
    const long per_sm = (blocks + 147) / 148;
    const double warps = (double)per_sm * nt / 32.0;
    const double need = chains >= 8 ? 4.0 : 8.0;
    const double busy = warps < need ? warps / need : 1.0;
    const double eff = chains >= 32 ? 1.0 : chains >= 16 ? 0.95 : chains >= 8 ? 0.9 : 0.8;
    const double cost = (double)per_sm * bm * bn / (busy * eff);
    if (best < 0 || cost < best_cost * 0.97) { best = i; best_cost = cost; }
  }
  return best;
}

void launch_gemm_big(const float *XT, int ldm, const float *Wpf, int K, int N, int M, float *Y, int ysm, int ysn,
                     const float *resid, int ldr, const int32_t *y_slot, size_t y_slot_stride, int glu,
                     cudaStream_t s, bool tree) {
  if (M <= 0 || N <= 0) return;
#define CIS2B_BIG2(TY_, TX_, TMR_, TNC_, ST_, KT_, TREE_)                                                    \
  run_gemm_big<TY_, TX_, TMR_, TNC_, ST_, KT_, TREE_>(XT, ldm, Wpf, K, N, M, Y, ysm, ysn, resid, ldr, y_slot, \
                                                      y_slot_stride, glu, s)
#define CIS2B_BIG(TY_, TX_, TMR_, TNC_, ST_, KT_)                 \
  do {                                                           \
    if (tree) CIS2B_BIG2(TY_, TX_, TMR_, TNC_, ST_, KT_, true);  \
    else CIS2B_BIG2(TY_, TX_, TMR_, TNC_, ST_, KT_, false);      \
  } while (0)
  // Stage depth and k per stage per tile, measured on B200 (fp32 panels).
  switch (gemm_big_choice(M, N, tree)) {
    case 0:
      if (!tree) { CIS2B_BIG2(16, 16, 8, 4, 3, 32, false); break; }  // (not chosen in tree order)
      [[fallthrough]];
    case 1: CIS2B_BIG(16, 16, 4, 4, 4, 32); break;
    case 2: CIS2B_BIG(16, 8, 4, 4, 6, 32); break;
    case 3: CIS2B_BIG(16, 8, 4, 2, 4, 32); break;
    default: CIS2B_BIG(8, 16, 2, 2, 4, 32); break;
  }
#undef CIS2B_BIG
#undef CIS2B_BIG2
}

void launch_gemm(const float *XT, int ldm, const uint16_t *Wp, const float *Wpf, int K, int N, int M, float *Y,
                 int ldy, const float *resid, int ldr, bool tree, const int32_t *y_slot, size_t y_slot_stride,
                 cudaStream_t s) {
  if (M <= 0 || N <= 0) return;
  if (M >= 64 && gemm_big_ok(K, tree)) {
    launch_gemm_big(XT, ldm, Wpf, K, N, M, Y, ldy, 1, resid, ldr, y_slot, y_slot_stride, 0, s, tree);
    return;
  }
  // Fewer rows, or tree mode: SIMT register tiles (tree mode with the
  // streaming 32-leaf tree per k tile).
#define CIS2B_GEMM(BM_, BP_, TM_, TN_)                                                           \
  do {                                                                                           \
    if (tree)                                                                                    \
      run_gemm_t<BM_, BP_, TM_, TN_, true>(XT, ldm, Wp, K, N, M, Y, ldy, resid, ldr, y_slot,      \
                                           y_slot_stride, s);                                   \
    else                                                                                         \
      run_gemm_t<BM_, BP_, TM_, TN_, false>(XT, ldm, Wp, K, N, M, Y, ldy, resid, ldr, y_slot,     \
                                            y_slot_stride, s);                                  \
    return;                                                                                      \
  } while (0)
  switch (gemm_tile_choice(M, N, K, tree)) {
    case 0: if (!tree) CIS2B_GEMM(64, 4, 4, 4); break;
    case 1: CIS2B_GEMM(64, 2, 4, 2);
    case 2: CIS2B_GEMM(32, 1, 2, 1);
    case 3: CIS2B_GEMM(16, 2, 2, 1);
    case 5: CIS2B_GEMM(32, 2, 2, 2);
    case 6: CIS2B_GEMM(32, 4, 2, 4);
    default: break;
  }
  CIS2B_GEMM(4, 4, 1, 1);
#undef CIS2B_GEMM
}

// Wp[n8][k][j] = W[src(8*n8 + j)][k] (zero rows past N): the panel layout
// above, src(n) = n, or for a gate/up pair (il_half = I, N = 2I) the rows
// interleaved, src(2i) = i (gate), src(2i + 1) = I + i (up).
// T = float: the same panels widened to fp32 (exact: bits << 16).
__device__ __forceinline__ void panel_put(uint16_t *d, uint16_t v) { *d = v; }
__device__ __forceinline__ void panel_put(float *d, uint16_t v) { *d = widen_bf16(v); }
template <class T>
__global__ void k_panelize(const uint16_t *W, int N, int K, T *Wp, int il_half) {
  const size_t N8 = (size_t)(N + 7) / 8;
  const size_t total = N8 * (size_t)K * 8;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const size_t j = idx % 8, k = (idx / 8) % K, n8 = idx / (8 * (size_t)K);
    const size_t n = n8 * 8 + j;
    const size_t src = il_half ? ((n & 1) ? (size_t)il_half + n / 2 : n / 2) : n;
    panel_put(Wp + idx, n < (size_t)N ? W[src * K + k] : (uint16_t)0);
  }
}
void launch_panelize(const uint16_t *W, int N, int K, uint16_t *Wp, cudaStream_t s, int il_half) {
  k_panelize<uint16_t><<<1184, 256, 0, s>>>(W, N, K, Wp, il_half);
}
void launch_panelize(const uint16_t *W, int N, int K, float *Wp, cudaStream_t s, int il_half) {
  k_panelize<float><<<1184, 256, 0, s>>>(W, N, K, Wp, il_half);
}
size_t panel_elems(int N, int K) { return (size_t)((N + 7) / 8) * 8 * (size_t)K; }

// ============================================================ decode GEMM
//
// Few activation rows (one per sequence at a decode step) against a large
// weight matrix.  Lanes own output COLUMNS: lane j of a warp produces
// column 32*tile + j for TM rows, walking k = 0..K-1 in order for each.
// Per four k a lane reads its column's four weights with one 8-byte shared
// load and each row's four activations with one broadcast 16-byte load, so
// every shared load feeds at least four multiply-adds.  Rows are split over
// the RW warps of a block; all RW*TM rows of the block sit in shared memory
// for the whole K, weights stream through a STAGES-deep cp.async ring.
//
// Operand layouts:
//   X   [M][ldx] fp32  row-major activations (ldx % 4 == 0)
//   Wt  [N32][K/4][32][4] bf16  32-column tiles, four consecutive k of a
//       column contiguous (same bf16 bits as the checkpoint's [N][K]);
//       K % 4 == 0, zero columns past N.
// The products of four k are formed as two packed pairs (mul.f32x2: two
// independent, separately rounded products) and added to the accumulator
// one at a time, k ascending, exactly as dot_seq does.
constexpr int DEC_KC = 64;      // k per weight stage
constexpr int DEC_STAGES = 6;

__host__ __device__ size_t tile32_elems(int N, int K) { return (size_t)((N + 31) / 32) * 32 * (size_t)K; }

// Wt[n32][kq][j][q] = W[src(n32, j)][4*kq + q] with src = 32*n32 + j, or,
// for a gate/up pair (glu_half = I, N = 2I), gate row 16*n32 + j in lanes
// 0..15 and up row I + 16*n32 + j - 16 in lanes 16..31.
__global__ void k_tile32(const uint16_t *W, int N, int K, uint16_t *Wt, int glu_half) {
  const size_t total = tile32_elems(N, K);
  const size_t KQ = (size_t)K / 4;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const size_t q = idx % 4, j = (idx / 4) % 32, kq = (idx / 128) % KQ, n32 = idx / 128 / KQ;
    const size_t n = glu_half ? (j < 16 ? n32 * 16 + j : (size_t)glu_half + n32 * 16 + j - 16) : n32 * 32 + j;
    Wt[idx] = n < (size_t)N ? W[n * K + kq * 4 + q] : (uint16_t)0;
  }
}
void launch_tile32(const uint16_t *W, int N, int K, uint16_t *Wt, cudaStream_t s, int glu_half) {
  k_tile32<<<1184, 256, 0, s>>>(W, N, K, Wt, glu_half);
}

// One group of four products (c = ((p0 + p1) + (p2 + p3)), group g = 0..7
// of a 32-product block) into the block's pairwise tree: levels 3, 4 and 5
// join group sums (g0 + g1), ((g0 + g1) + (g2 + g3)), ...; the finished
// block sum is added to acc (cis2_math.h:212-265).
__device__ __forceinline__ void tree_group(float &acc, float &t3, float &t4, float &t5, float c, int g) {
  if ((g & 1) == 0) { t3 = c; return; }
  const float l3 = fadd(t3, c);
  if ((g & 2) == 0) { t4 = l3; return; }
  const float l4 = fadd(t4, l3);
  if ((g & 4) == 0) { t5 = l4; return; }
  acc = fadd(acc, fadd(t5, l4));
}

__device__ __forceinline__ float4 widen4(uint2 u) {
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

// XS = false: the block's activation rows stay resident in shared memory
// for the whole K (one copy up front).  XS = true: they stream through the
// same ring as the weights, DEC_KC columns per stage, which keeps shared
// memory small when ROWS x K is large (several blocks per SM instead of one).
// TREE: the v0.4 tree order (K % 32 == 0): each block of 32 products is
// summed as the balanced pairwise tree of cis2_math.h:212-265, its sum
// added to the running total from +0.  A lane builds the tree of its column
// from groups of four products, ((p0 + p1) + (p2 + p3)), joining the eight
// group sums of a block in three more levels as they complete.
template <int TM, int RW, bool XS, bool TREE = false>
__global__ void __launch_bounds__(32 * RW, 1)
k_gemm_dec(const float *__restrict__ X, int ldx, const uint16_t *__restrict__ Wt, int K, int N, int M,
           float *__restrict__ Y, int ldy, const float *__restrict__ R, int ldr, const int32_t *y_slot,
           size_t y_slot_stride, int glu) {
  constexpr int ROWS = TM * RW, NT = 32 * RW;
  constexpr int WST = DEC_KC * 32;  // bf16 per weight stage
  constexpr int XST = ROWS * DEC_KC;  // floats per streamed activation stage
  constexpr int PF = 2;             // register prefetch distance in groups of four k
  extern __shared__ __align__(16) float smem[];
  // XS: [STAGES][ROWS][KC] floats, then the weight ring; else [ROWS][K].
  float *Xs = smem;
  uint16_t *Ws = reinterpret_cast<uint16_t *>(smem + (XS ? (size_t)DEC_STAGES * XST : (size_t)ROWS * K));
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int n32 = blockIdx.x, m0 = blockIdx.y * ROWS;
  const uint16_t *Wtile = Wt + (size_t)n32 * K * 32;
  const uint32_t xs_b = (uint32_t)__cvta_generic_to_shared(Xs);
  const uint32_t ws_b = (uint32_t)__cvta_generic_to_shared(Ws);
  const int nc = (K + DEC_KC - 1) / DEC_KC;
  const int KQ = K / 4;

  if (!XS) {
    // The block's rows, whole K (rows past M are zero-filled), in group 0.
    for (int i = tid; i < ROWS * KQ; i += NT) {
      const int r = i / KQ, q = i - r * KQ;
      const bool ok = m0 + r < M;
      cp_async16_zfill(xs_b + (uint32_t)((r * K + 4 * q) * 4), ok ? X + (size_t)(m0 + r) * ldx + 4 * q : X, ok);
    }
  }
  auto issue_w = [&](int c) {
    const int slot = c % DEC_STAGES, k0 = c * DEC_KC;
    const int kn = min(DEC_KC, K - k0);
    const int nchunk = kn * 4;  // 16-byte pieces: kn * 32 bf16 * 2 B / 16
    for (int i = tid; i < nchunk; i += NT)
      cp_async16(ws_b + (uint32_t)(slot * WST * 2 + i * 16), Wtile + (size_t)k0 * 32 + (size_t)i * 8);
    if (XS) {  // the rows' k0 .. k0 + kn columns, row stride DEC_KC in the stage
      const int nq = kn / 4;
      for (int i = tid; i < ROWS * nq; i += NT) {
        const int r = i / nq, q = i - r * nq;
        const bool ok = m0 + r < M;
        cp_async16_zfill(xs_b + (uint32_t)((slot * XST + r * DEC_KC + 4 * q) * 4),
                         ok ? X + (size_t)(m0 + r) * ldx + k0 + 4 * q : X, ok);
      }
    }
  };
#pragma unroll
  for (int s = 0; s < DEC_STAGES - 1; ++s) {
    if (s < nc) issue_w(s);
    cp_async_commit();
  }

  float acc[TM], t3[TM], t4[TM], t5[TM];  // t3..t5: pending tree levels (TREE)
#pragma unroll
  for (int i = 0; i < TM; ++i) acc[i] = t3[i] = t4[i] = t5[i] = 0.0f;
  const int xstride = XS ? DEC_KC : K;  // row stride of the activations read below
  for (int c = 0; c < nc; ++c) {
    cp_async_wait<DEC_STAGES - 2>();
    __syncthreads();
    if (c + DEC_STAGES - 1 < nc) issue_w(c + DEC_STAGES - 1);
    cp_async_commit();
    const uint2 *wsl = reinterpret_cast<const uint2 *>(Ws + (c % DEC_STAGES) * WST) + lane;
    const float *xc = XS ? Xs + (size_t)(c % DEC_STAGES) * XST + (size_t)(w * TM) * DEC_KC
                         : Xs + (size_t)(w * TM) * K + c * DEC_KC;
    const int kn = min(DEC_KC, K - c * DEC_KC);
    if (kn == DEC_KC) {
      constexpr int NQ = DEC_KC / 4;
      float4 xb[PF][TM], wb[PF];
      auto ld = [&](int sl, int kq) {
        wb[sl] = widen4(wsl[kq * 32]);
#pragma unroll
        for (int i = 0; i < TM; ++i) xb[sl][i] = *reinterpret_cast<const float4 *>(xc + (size_t)i * xstride + 4 * kq);
      };
#pragma unroll
      for (int q = 0; q < PF; ++q) ld(q, q);
#pragma unroll
      for (int kq = 0; kq < NQ; ++kq) {
        const int sl = kq % PF;
        const float4 wv = wb[sl];
        float4 xv[TM];
#pragma unroll
        for (int i = 0; i < TM; ++i) xv[i] = xb[sl][i];
        if (kq + PF < NQ) ld(sl, kq + PF);
        float2 p01[TM], p23[TM];
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          p01[i] = fmul_pair(wv.x, wv.y, xv[i].x, xv[i].y);
          p23[i] = fmul_pair(wv.z, wv.w, xv[i].z, xv[i].w);
        }
        if (TREE) {
#pragma unroll
          for (int i = 0; i < TM; ++i)
            tree_group(acc[i], t3[i], t4[i], t5[i], fadd(fadd(p01[i].x, p01[i].y), fadd(p23[i].x, p23[i].y)), kq & 7);
        } else {
#pragma unroll
          for (int i = 0; i < TM; ++i) acc[i] = fadd(acc[i], p01[i].x);
#pragma unroll
          for (int i = 0; i < TM; ++i) acc[i] = fadd(acc[i], p01[i].y);
#pragma unroll
          for (int i = 0; i < TM; ++i) acc[i] = fadd(acc[i], p23[i].x);
#pragma unroll
          for (int i = 0; i < TM; ++i) acc[i] = fadd(acc[i], p23[i].y);
        }
      }
    } else {
      for (int kq = 0; kq < kn / 4; ++kq) {
        const float4 wv = widen4(wsl[kq * 32]);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const float4 xv = *reinterpret_cast<const float4 *>(xc + (size_t)i * xstride + 4 * kq);
          if (TREE) {
            const float c = fadd(fadd(fmul(wv.x, xv.x), fmul(wv.y, xv.y)), fadd(fmul(wv.z, xv.z), fmul(wv.w, xv.w)));
            tree_group(acc[i], t3[i], t4[i], t5[i], c, kq & 7);
          } else {
            acc[i] = fadd(acc[i], fmul(wv.x, xv.x));
            acc[i] = fadd(acc[i], fmul(wv.y, xv.y));
            acc[i] = fadd(acc[i], fmul(wv.z, xv.z));
            acc[i] = fadd(acc[i], fmul(wv.w, xv.w));
          }
        }
      }
    }
  }
  cp_async_wait<0>();

  if (glu) {
    // Gate/up tile: lane j < 16 holds gate 16*n32 + j, lane j + 16 its up.
    const int col = n32 * 16 + lane;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int m = m0 + w * TM + i;
      if (m >= M) break;
      const float up = __shfl_down_sync(FULL, acc[i], 16);
      if (lane < 16 && col < glu) Y[(size_t)m * ldy + col] = fmul(silu_pinned(acc[i]), up);  // cis2_model.h:619-623
    }
    return;
  }
  const int n = n32 * 32 + lane;
  if (n >= N) return;
  float *Yb = Y + (y_slot ? (size_t)(*y_slot) * y_slot_stride : 0);
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + w * TM + i;
    if (m >= M) break;
    float v = acc[i];
    if (R) v = fadd(R[(size_t)m * ldr + n], v);  // residual h + o (cis2_model.h:540-542)
    Yb[(size_t)m * ldy + n] = v;
  }
}

template <int TM, int RW, bool XS, bool TREE>
static void run_gemm_dec(const float *X, int ldx, const uint16_t *Wt, int K, int N, int M, float *Y, int ldy,
                         const float *R, int ldr, const int32_t *y_slot, size_t y_slot_stride, int glu,
                         cudaStream_t s) {
  constexpr int ROWS = TM * RW;
  const size_t smem = (XS ? (size_t)DEC_STAGES * ROWS * DEC_KC * 4 : (size_t)ROWS * K * 4) +
                      (size_t)DEC_STAGES * DEC_KC * 32 * 2;
  static SmemLimit lim;
  lim.ensure(k_gemm_dec<TM, RW, XS, TREE>, 227 * 1024);
  dim3 grid((N + 31) / 32, (M + ROWS - 1) / ROWS);
  k_gemm_dec<TM, RW, XS, TREE><<<grid, 32 * RW, smem, s>>>(X, ldx, Wt, K, N, M, Y, ldy, R, ldr, y_slot,
                                                            y_slot_stride, glu);
}

// Rows per block: the largest candidate that still gives at least two
// blocks per SM and whose rows fit shared memory next to the weight ring.
struct DecCfg { int tm, rw; };
static const DecCfg kDecTiles[] = {{8, 4}, {4, 4}, {2, 4}, {2, 2}};
constexpr int kNumDecTiles = 4;
// Resident activation rows above this many bytes stream instead.  Measured
// on B200: 300 x 768 x 3,072 takes 102 us streamed against 143 us with
// 16 x 3,072 rows resident (one block per SM), and 32 x 6,144 x 1,024 takes
// 31.7 against 35.7 us; at 48 KB and below, resident rows are as fast or
// faster (4 x 3,072 rows: 30.7 us resident, 34.9 streamed).
constexpr size_t DEC_RESIDENT_MAX = 48 * 1024;

bool gemm_dec_ok(int K, bool tree) { return K > 0 && K % (tree ? 32 : 4) == 0; }

int gemm_dec_choice(int M, int N, int K) {
  const long n32 = (N + 31) / 32;
  int pick = -1;
  for (int i = 0; i < kNumDecTiles; ++i) {
    const int rows = kDecTiles[i].tm * kDecTiles[i].rw;
    // Eight rows per lane pay off only on very wide products (lm_head):
    // measured on B200, 4 x 4 is faster for the layer projections at 64 and 300 rows.
    if (kDecTiles[i].tm == 8 && N < 16384) continue;
    pick = i;
    if (n32 * ((M + rows - 1) / rows) >= 2 * 148) break;
  }
  return pick;
}

void launch_gemm_dec(const float *X, int ldx, const uint16_t *Wt, int K, int N, int M, float *Y, int ldy,
                     const float *resid, int ldr, const int32_t *y_slot, size_t y_slot_stride, cudaStream_t s,
                     int glu, bool tree) {
  if (M <= 0 || N <= 0) return;
  const int pick = gemm_dec_choice(M, N, K);
  const bool xs = (size_t)kDecTiles[pick].tm * kDecTiles[pick].rw * K * 4 > DEC_RESIDENT_MAX;
#define CIS2B_DEC2(TM_, RW_, TREE_)                                                                              \
  do {                                                                                                          \
    if (xs) run_gemm_dec<TM_, RW_, true, TREE_>(X, ldx, Wt, K, N, M, Y, ldy, resid, ldr, y_slot, y_slot_stride, \
                                                glu, s);                                                        \
    else run_gemm_dec<TM_, RW_, false, TREE_>(X, ldx, Wt, K, N, M, Y, ldy, resid, ldr, y_slot, y_slot_stride,  \
                                              glu, s);                                                          \
  } while (0)
#define CIS2B_DEC(TM_, RW_)                    \
  do {                                        \
    if (tree) CIS2B_DEC2(TM_, RW_, true);     \
    else CIS2B_DEC2(TM_, RW_, false);         \
  } while (0)
  switch (pick) {
    case 0: CIS2B_DEC(8, 4); break;
    case 1: CIS2B_DEC(4, 4); break;
    case 2: CIS2B_DEC(2, 4); break;
    default: CIS2B_DEC(2, 2); break;
  }
#undef CIS2B_DEC
#undef CIS2B_DEC2
}

// ============================================================ attention

// Per row: optional per-head q/k RMSNorm (qwen3-port.diff:66-80), RoPE of
// every q and k head from the pinned cos/sin table (cis2_model.h:547-568),
// then the KV-cache append of post-RoPE k and raw v (cis2_model.h:718-721).
__global__ void k_qkv_post(float *qkv, int ld, const int32_t *rseq, const int32_t *rpos, int nh,
                           int nkv, int hd, const uint16_t *qn, const uint16_t *kn, float eps,
                           int tree, const float *cos_t, const float *sin_t, float *kc, float *vc,
                           int max_pos) {
  extern __shared__ float sm[];
  const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  float *row = qkv + (size_t)r * ld;
  const int seq = rseq[r], pos = rpos[r];
  const int half = hd / 2, QD = nh * hd, KV = nkv * hd;
  const float *ct = cos_t + (size_t)pos * half;
  const float *st = sin_t + (size_t)pos * half;
  float *sq = sm + (size_t)warp * 2 * hd;
  for (int h = warp; h < nh + nkv; h += nw) {
    const bool is_k = h >= nh;
    float *x = is_k ? row + QD + (size_t)(h - nh) * hd : row + (size_t)h * hd;
    const uint16_t *nwt = is_k ? kn : qn;
    if (nwt) warp_rmsnorm(x, nwt, eps, hd, tree != 0, sq, x);
    for (int i = lane; i < half; i += 32) {
      float x1 = x[i], x2 = x[i + half], c = ct[i], s = st[i];
      float o1 = fadd(fmul(x1, c), fmul(fneg(x2), s));
      float o2 = fadd(fmul(x2, c), fmul(x1, s));
      x[i] = o1;
      x[i + half] = o2;
    }
    __syncwarp();
    if (is_k) {
      float *dst = kc + ((size_t)seq * max_pos + pos) * KV + (size_t)(h - nh) * hd;
      for (int i = lane; i < hd; i += 32) dst[i] = x[i];
    }
  }
  float *vdst = vc + ((size_t)seq * max_pos + pos) * KV;
  for (int i = threadIdx.x; i < KV; i += blockDim.x) vdst[i] = row[QD + KV + i];
}

void launch_qkv_post(float *qkv, int ld, int rows, RowMap rm, int n_heads, int n_kv, int hd,
                     const uint16_t *q_norm, const uint16_t *k_norm, float eps, bool tree,
                     const float *cos_t, const float *sin_t, float *kcache, float *vcache,
                     int max_pos, cudaStream_t s) {
  if (rows <= 0) return;
  const int threads = 128;
  k_qkv_post<<<rows, threads, (size_t)(threads / 32) * 2 * hd * sizeof(float), s>>>(
      qkv, ld, rm.seq, rm.pos, n_heads, n_kv, hd, q_norm, k_norm, eps, tree ? 1 : 0, cos_t, sin_t,
      kcache, vcache, max_pos);
}

// NaN-aware max combine reproducing the serial "if (v > max) max = v" scan
// started at element 0: NaNs after element 0 are never selected.
__device__ __forceinline__ float max_comb(float a, float b) {
  if (is_nan(a)) return b;
  if (is_nan(b)) return a;
  return (b > a) ? b : a;
}

// One CTA per (row, KV head), covering the G = n_heads / n_kv query heads
// that share it (GQA), so each key/value row crosses HBM once per row:
//   scores  q_g . k_j * scale          (cis2_model.h:571-585; scale after the dot)
//   softmax strict-'>' max, pinned exp, pinned-order denominator, divide
//                                      (cis2_math.h:442-467)
//   V-mix   acc = acc + p_j * v_j[d], j ascending, both modes
//                                      (cis2_model.h:599-617)
// K and V stream through shared memory in chunks of ATT_JC positions
// (coalesced loads); one thread owns each (head, position) dot product and
// each (head, d) V-mix chain.
constexpr int ATT_JC = 64;
// K/V ring depth of the decode-step attention (k_attention_dec).  Measured
// on B200 (C5 shape, 256 rows at position ~1,535): 2 slots 155 us, 3 slots
// 169 us, 4 slots 174 us: a deeper ring costs CTAs per SM (shared memory),
// and the kernel is bound by its serial chains and their waits, not by HBM
// (the same launch with every K/V chunk served from L2 takes as long).  A
// ring filled by per-position bulk copies (cp.async.bulk + mbarrier) took
// 274 us.  With the current form, 3 slots made the whole C5 decode step 11 %
// slower (9.2 against 8.3 ms).
constexpr int ATT_DEC_STAGES = 2;

size_t attention_smem_floats(int G, int hd, int max_len) {
  const size_t scs = ((size_t)max_len + 3) & ~(size_t)3;  // score rows start 16-byte aligned
  size_t f = (size_t)G * hd + (size_t)G * scs + (size_t)G * (max_len / 32 + 1) + 64;
  f = (f + 3) & ~(size_t)3;                              // tiles start 16-byte aligned
  return f + (size_t)2 * ATT_JC * (hd + 4);
}

bool launch_attention_dec(float *qkv, int ld, int rows, RowMap rm, int n_heads, int n_kv, int hd, float *kcache,
                          float *vcache, int max_pos, float *att, int ars, int acs, int max_len,
                          const uint16_t *q_norm, const uint16_t *k_norm, float eps, const float *cos_t,
                          const float *sin_t, bool tree, cudaStream_t s);

__global__ void k_attention(float *qkv, int ld, const int32_t *rseq, const int32_t *rpos,
                            int nh, int nkv, int hd, float *kc, float *vc, int max_pos,
                            int tree, float *att, int ars, int acs, int max_len, int fuse_post,
                            const uint16_t *qn, const uint16_t *kn, float eps, const float *cos_t,
                            const float *sin_t, float *dbg) {
  extern __shared__ __align__(16) float sm[];
  const int r = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x, nt = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
  const int G = nh / nkv, KV = nkv * hd;
  const int seq = rseq[r], pos = rpos[r], len = pos + 1;
  const int nb = (len + 31) / 32;
  const int scs = (max_len + 3) & ~3;         // score row stride (16-byte aligned rows)
  float *q = sm;                              // [G][hd]
  float *sc = q + G * hd;                     // [G][scs]
  float *part = sc + (size_t)G * scs;         // [G][max_len/32 + 1]
  float *red = part + (size_t)G * (max_len / 32 + 1);  // [64]
  size_t toff = (size_t)(red + 64 - sm);
  toff = (toff + 3) & ~(size_t)3;
  float *tiles = sm + toff;                   // [2][ATT_JC][hd + 4], K then V chunks
  const int ts = hd + 4;
  if (fuse_post) {
    // Decode rows only (each CTA's row is its sequence's newest position):
    // the work of k_qkv_post for this KV head's q heads, k head and v head,
    // done here so the new key/value reach the cache without another launch.
    float *row = qkv + (size_t)r * ld;
    const int QD = nh * hd, half = hd / 2;
    const float *ct = cos_t + (size_t)pos * half, *st = sin_t + (size_t)pos * half;
    for (int hh = warp; hh <= G; hh += nw) {
      const bool is_k = hh == G;
      float *x = is_k ? row + QD + (size_t)kvh * hd : row + ((size_t)kvh * G + hh) * hd;
      const uint16_t *nwt = is_k ? kn : qn;
      if (nwt) warp_rmsnorm(x, nwt, eps, hd, tree != 0, tiles + (size_t)warp * 2 * hd, x);
      for (int i = lane; i < half; i += 32) {
        float x1 = x[i], x2 = x[i + half], c = ct[i], sn = st[i];
        float o1 = fadd(fmul(x1, c), fmul(fneg(x2), sn));
        float o2 = fadd(fmul(x2, c), fmul(x1, sn));
        x[i] = o1;
        x[i + half] = o2;
      }
      __syncwarp();
      if (is_k) {
        float *dst = kc + ((size_t)seq * max_pos + pos) * KV + (size_t)kvh * hd;
        for (int i = lane; i < hd; i += 32) dst[i] = x[i];
      }
    }
    const float *vsrc = row + QD + KV + (size_t)kvh * hd;
    float *vdst = vc + ((size_t)seq * max_pos + pos) * KV + (size_t)kvh * hd;
    for (int i = tid; i < hd; i += nt) vdst[i] = vsrc[i];
    __syncthreads();
  }
  for (int i = tid; i < G * hd; i += nt) q[i] = qkv[(size_t)r * ld + (size_t)kvh * G * hd + i];
  const float scale = rsqrt_cr(__int2float_rn(hd));
  const float *kbase = kc + (size_t)seq * max_pos * KV + (size_t)kvh * hd;
  const float *vbase = vc + (size_t)seq * max_pos * KV + (size_t)kvh * hd;
  const int nch = (len + ATT_JC - 1) / ATT_JC;
  const uint32_t tbase = (uint32_t)__cvta_generic_to_shared(tiles);
  // K or V rows [j0, j0+ATT_JC) of this KV head -> tile buffer `buf`, async.
  auto stage = [&](const float *base, int c, int buf) {
    const int j0 = c * ATT_JC, jc = min(ATT_JC, len - j0), nq = hd / 4;
    for (int i = tid; i < jc * nq; i += nt) {
      const int jj = i / nq, q4 = i - jj * nq;
      cp_async16(tbase + (uint32_t)(((buf * ATT_JC + jj) * ts + 4 * q4) * 4), base + (size_t)(j0 + jj) * KV + 4 * q4);
    }
    cp_async_commit();
  };

  // ---- scores, K streamed through two tile buffers
  stage(kbase, 0, 0);
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) stage(kbase, c + 1, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int j0 = c * ATT_JC, jc = min(ATT_JC, len - j0);
    const float *tile = tiles + (size_t)(c & 1) * ATT_JC * ts;
    for (int pr = tid; pr < G * jc; pr += nt) {
      const int g = pr / jc, jj = pr - g * jc;
      const float *qg = q + g * hd, *kj = tile + jj * ts;
      float d;
      if (!tree) {
        // 16-byte loads (hd % 4 == 0; the key rows' pitch hd+4 keeps the 32
        // lanes' rows on distinct banks), four k per load, k ascending.
        const float4 *q4 = reinterpret_cast<const float4 *>(qg), *k4 = reinterpret_cast<const float4 *>(kj);
        d = 0.0f;
        int i = 0;
        for (; i + 4 <= hd / 4; i += 4) {
          float4 a[4], b[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) { a[u] = q4[i + u]; b[u] = k4[i + u]; }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            d = fadd(d, fmul(a[u].x, b[u].x));
            d = fadd(d, fmul(a[u].y, b[u].y));
            d = fadd(d, fmul(a[u].z, b[u].z));
            d = fadd(d, fmul(a[u].w, b[u].w));
          }
        }
        for (; i < hd / 4; ++i) {
          const float4 a = q4[i], b = k4[i];
          d = fadd(d, fmul(a.x, b.x));
          d = fadd(d, fmul(a.y, b.y));
          d = fadd(d, fmul(a.z, b.z));
          d = fadd(d, fmul(a.w, b.w));
        }
      } else {
        d = dot_tree(qg, kj, hd);
      }
      sc[(size_t)g * scs + j0 + jj] = fmul(d, scale);  // scale after the dot (gpu/README.md §4)
    }
    __syncthreads();
  }
  // Trace mode (one row): the scaled scores of this KV head's q heads,
  // [n_heads][len] at dbg.
  if (dbg)
    for (int i = tid; i < G * len; i += nt)
      dbg[((size_t)kvh * G + i / len) * len + i % len] = sc[(size_t)(i / len) * scs + i % len];
  // V chunk 0 loads while the softmax runs.
  stage(vbase, 0, 0);
  // ---- max per head (serial-scan semantics, see max_comb)
  for (int g = warp; g < G; g += nw) {
    const float *sg = sc + (size_t)g * scs;
    float m = bitsf(0x7fc00000u);
    for (int j = lane; j < len; j += 32) m = max_comb(m, sg[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max_comb(m, __shfl_xor_sync(FULL, m, o));
    if (lane == 0) red[g] = is_nan(sg[0]) ? sg[0] : m;
  }
  __syncthreads();
  for (int g = 0; g < G; ++g) {
    float *sg = sc + (size_t)g * scs;
    const float mg = red[g];
    for (int j = tid; j < len; j += nt) sg[j] = exp_pinned(fsub(sg[j], mg));
  }
  __syncthreads();
  // ---- denominators
  if (tree) {
    for (int pb = warp; pb < G * nb; pb += nw) {
      const int g = pb / nb, b = pb - g * nb, j = b * 32 + lane;
      float v = warp_tree32(j < len ? sc[(size_t)g * scs + j] : 0.0f);
      if (lane == 0) part[(size_t)g * (max_len / 32 + 1) + b] = v;
    }
    __syncthreads();
  }
  for (int g = warp; g < G; g += nw) {
    if (lane == 0) {
      float acc;
      if (!tree) acc = serial_sum4(sc + (size_t)g * scs, len);
      else acc = serial_sum(part + (size_t)g * (max_len / 32 + 1), nb);
      red[32 + g] = acc;
    }
  }
  __syncthreads();
  for (int g = 0; g < G; ++g) {
    float *sg = sc + (size_t)g * scs;
    const float den = red[32 + g];
    for (int j = tid; j < len; j += nt) sg[j] = fdiv(sg[j], den);
  }
  if (dbg) {  // trace mode: the softmax weights, [n_heads][len] after the scores
    __syncthreads();
    for (int i = tid; i < G * len; i += nt)
      dbg[((size_t)nh + kvh * G + i / len) * len + i % len] = sc[(size_t)(i / len) * scs + i % len];
  }
  // ---- V-mix, V streamed through the two tile buffers.  Thread t owns the
  // chain (g, d) = (t / hd, t % hd): the block's G*hd threads all work on
  // every chunk, the lanes of a warp read consecutive d of one V row
  // (conflict-free) and share the weights of one head (four positions per
  // broadcast load).
  const int g = tid / hd, d = tid - (tid / hd) * hd;
  const bool owns = tid < G * hd;
  float acc = 0.0f;
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) stage(vbase, c + 1, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int j0 = c * ATT_JC, jc = min(ATT_JC, len - j0);
    const float *tile = tiles + (size_t)(c & 1) * ATT_JC * ts + d;
    if (owns) {
      const float *pg = sc + (size_t)g * scs + j0;  // j0 % 4 == 0: 16-byte aligned
      int jj = 0;
      for (; jj + 4 <= jc; jj += 4) {
        const float4 pw = *reinterpret_cast<const float4 *>(pg + jj);
        const float v0 = tile[jj * ts], v1 = tile[(jj + 1) * ts], v2 = tile[(jj + 2) * ts], v3 = tile[(jj + 3) * ts];
        acc = fadd(acc, fmul(pw.x, v0));
        acc = fadd(acc, fmul(pw.y, v1));
        acc = fadd(acc, fmul(pw.z, v2));
        acc = fadd(acc, fmul(pw.w, v3));
      }
      for (; jj < jc; ++jj) acc = fadd(acc, fmul(pg[jj], tile[jj * ts]));
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  if (owns) att[(size_t)r * ars + ((size_t)kvh * G + g) * hd * acs + (size_t)d * acs] = acc;
}

void launch_attention(float *qkv, int ld, int rows, RowMap rm, int n_heads, int n_kv, int hd,
                      float *kcache, float *vcache, int max_pos, bool tree, float *att,
                      int ars, int acs, int max_len, bool fuse_post, const uint16_t *q_norm,
                      const uint16_t *k_norm, float eps, const float *cos_t, const float *sin_t,
                      cudaStream_t s, float *dbg) {
  if (rows <= 0) return;
  if (fuse_post && !dbg &&
      launch_attention_dec(qkv, ld, rows, rm, n_heads, n_kv, hd, kcache, vcache, max_pos, att, ars, acs, max_len,
                           q_norm, k_norm, eps, cos_t, sin_t, tree, s))
    return;
  const int G = n_heads / n_kv;
  int nt = ((G * hd + 31) / 32) * 32;
  if (nt < 128) nt = 128;
  size_t smem = attention_smem_floats(G, hd, max_len) * sizeof(float);
  static SmemLimit lim;
  if (smem > 48 * 1024) lim.ensure(k_attention, smem);
  dim3 grid(rows, n_kv);
  k_attention<<<grid, nt, smem, s>>>(qkv, ld, rm.seq, rm.pos, n_heads, n_kv, hd, kcache, vcache, max_pos,
                                     tree ? 1 : 0, att, ars, acs, max_len, fuse_post ? 1 : 0, q_norm,
                                     k_norm, eps, cos_t, sin_t, dbg);
}

// ---- Decode-step attention in sequential mode, specialised on the head
// size HD and the group G = n_heads / n_kv.  Same CTA grid, same
// arithmetic in the same order as k_attention (scaled dots, serial-scan
// max, pinned exp, serial denominator, division, V-mix chains over j
// ascending), with the index arithmetic resolved at compile time and the
// K/V chunks streamed through an ST-deep cp.async ring (ST - 1 chunks in
// flight while one is consumed).  Measured on B200, the generic kernel's
// integer index arithmetic (divisions by the head size and chunk length per
// copy and per dot) made the integer pipe its busiest unit, ahead of memory.
// Beyond that: each thread keeps a running max of the scores it writes
// (combined per head afterwards, the same NaN-aware combine), the
// denominators run in one warp, each thread stages fixed rows of every
// chunk, and a V-mix thread owns two adjacent d (two independent chains, one
// packed add per position).  Measured at the C5 shape (256 rows, position
// ~1,535): 78 M to 62 M instructions, 157 to 149 us; the rest is the wait
// on each chunk and the per-chunk barrier.
template <int HD, int G>
struct AttDec {
  static constexpr int NT = G * HD < 128 ? 128 : G * HD;  // threads: one V-mix chain per (g, d)
  static constexpr int JC = 64;                           // positions per chunk
  static constexpr int TS = HD + 4;                       // tile row pitch (floats)
  static constexpr int NQ = HD / 4;                       // 16-byte pieces per row
  static constexpr int DPT = (G * JC + NT - 1) / NT;      // dots per thread per chunk

};

// Score row pitch: max_len rounded to 4, plus 4 so that the G rows start on
// different banks (the denominator lanes read them side by side).
__host__ __device__ inline int att_dec_scs(int max_len) { return ((max_len + 3) & ~3) + 4; }
size_t attention_dec_smem_floats(int G, int hd, int max_len, int stages) {
  return (size_t)G * hd + (size_t)G * att_dec_scs(max_len) + 64 + (size_t)stages * 64 * (hd + 4);
}

// TREE: the v0.4 tree order for the two reductions it covers (the dots over
// HD in 32-product pairwise trees, the denominator in 32-leaf blocks);
// max, exp, division and the V-mix chains are the same as in sequential
// order (cis2_math.h:212-265, 442-467).
template <int HD, int G, int ST, bool TREE>
__global__ void __launch_bounds__(AttDec<HD, G>::NT, 1)
k_attention_dec(float *qkv, int ld, const int32_t *rseq, const int32_t *rpos, int nkv, float *kc, float *vc,
                int max_pos, float *att, int ars, int acs, int max_len, const uint16_t *qn, const uint16_t *kn,
                float eps, const float *cos_t, const float *sin_t) {
  using C = AttDec<HD, G>;
  constexpr int NT = C::NT, JC = C::JC, TS = C::TS, NQ = C::NQ, NW = NT / 32;
  static_assert(C::DPT == 1 && JC % 32 == 0 && NT % NQ == 0 && G * JC <= NT, "one dot per thread per chunk");
  static_assert(NW <= 32 && G <= 16 && HD % 2 == 0, "red[] layout");
  extern __shared__ __align__(16) float sm[];
  const int r = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int KV = nkv * HD;
  const int seq = rseq[r], pos = rpos[r], len = pos + 1;
  const int scs = att_dec_scs(max_len);
  float *q = sm;                       // [G][HD]
  float *sc = q + G * HD;              // [G][scs]
  float *red = sc + (size_t)G * scs;   // [64]: per-warp maxima, denominators at 32, maxima at 48
  float *tiles = red + 64;             // [ST][JC][TS]; offset is a multiple of 4 floats
  {
    // The row's q/k norm, RoPE and cache append for this KV head (the work
    // of k_qkv_post; each CTA's row is its sequence's newest position).
    float *row = qkv + (size_t)r * ld;
    const int QD = nkv * G * HD, half = HD / 2;
    const float *ct = cos_t + (size_t)pos * half, *st = sin_t + (size_t)pos * half;
    for (int hh = warp; hh <= G; hh += NW) {
      const bool is_k = hh == G;
      float *x = is_k ? row + QD + (size_t)kvh * HD : row + ((size_t)kvh * G + hh) * HD;
      const uint16_t *nwt = is_k ? kn : qn;
      if (nwt) warp_rmsnorm(x, nwt, eps, HD, TREE, tiles + (size_t)warp * 2 * HD, x);
      for (int i = lane; i < half; i += 32) {
        float x1 = x[i], x2 = x[i + half], c = ct[i], sn = st[i];
        float o1 = fadd(fmul(x1, c), fmul(fneg(x2), sn));
        float o2 = fadd(fmul(x2, c), fmul(x1, sn));
        x[i] = o1;
        x[i + half] = o2;
      }
      __syncwarp();
      if (is_k) {
        float *dst = kc + ((size_t)seq * max_pos + pos) * KV + (size_t)kvh * HD;
        for (int i = lane; i < HD; i += 32) dst[i] = x[i];
      }
    }
    const float *vsrc = row + QD + KV + (size_t)kvh * HD;
    float *vdst = vc + ((size_t)seq * max_pos + pos) * KV + (size_t)kvh * HD;
    for (int i = tid; i < HD; i += NT) vdst[i] = vsrc[i];
    __syncthreads();
  }
  for (int i = tid; i < G * HD; i += NT) q[i] = qkv[(size_t)r * ld + (size_t)kvh * G * HD + i];
  const float scale = rsqrt_cr(__int2float_rn(HD));
  const float *kbase = kc + (size_t)seq * max_pos * KV + (size_t)kvh * HD;
  const float *vbase = vc + (size_t)seq * max_pos * KV + (size_t)kvh * HD;
  const int nch = (len + JC - 1) / JC;
  const uint32_t tbase = (uint32_t)__cvta_generic_to_shared(tiles);
  // Staging: thread t copies 16-byte piece t % NQ of rows t / NQ, + RP, ...
  constexpr int RP = NT / NQ;
  const int sq = tid % NQ, sr = tid / NQ;
  auto stage = [&](const float *base, int c) {  // rows [c*JC, c*JC + JC) -> ring slot c % ST
    if (c < nch) {
      const int j0 = c * JC, jc = min(JC, len - j0), buf = c % ST;
      const float *src = base + (size_t)(j0 + sr) * KV + 4 * sq;
      uint32_t dst = tbase + (uint32_t)(((buf * JC + sr) * TS + 4 * sq) * 4);
      for (int jj = sr; jj < jc; jj += RP) {
        cp_async16(dst, src);
        src += (size_t)RP * KV;
        dst += (uint32_t)(RP * TS * 4);
      }
    }
    cp_async_commit();  // empty groups keep the count uniform
  };
  // Waits until chunk c sits in its slot (every thread's copies), then a barrier.
  auto land = [&](int) {
    cp_async_wait<ST - 2>();
    __syncthreads();
  };
#pragma unroll
  for (int c = 0; c < ST - 1; ++c) stage(kbase, c);
  __syncthreads();  // q visible

  // ---- scores: thread (g, jj) = (tid / JC, tid % JC) of each chunk; q from
  // shared memory (a broadcast load: all lanes of a warp share g).  The
  // thread's running max uses the combine of the serial-scan max.
  const int sg = tid / JC, sj = tid % JC;
  float mloc = bitsf(0x7fc00000u);
  for (int c = 0; c < nch; ++c) {
    land(c);
    stage(kbase, c + ST - 1);  // its slot was last read in chunk c - 1
    const int j0 = c * JC, jc = min(JC, len - j0);
    const float *tile = tiles + (size_t)(c % ST) * JC * TS;
    if (sg < G && sj < jc) {
      const float4 *k4 = reinterpret_cast<const float4 *>(tile + sj * TS);
      const float4 *q4 = reinterpret_cast<const float4 *>(q + sg * HD);
      float d = 0.0f, t3 = 0.0f, t4 = 0.0f, t5 = 0.0f;
#pragma unroll
      for (int i = 0; i < NQ; ++i) {
        const float4 b = k4[i];
        const float4 a = q4[i];
        if (TREE) {
          tree_group(d, t3, t4, t5, fadd(fadd(fmul(a.x, b.x), fmul(a.y, b.y)), fadd(fmul(a.z, b.z), fmul(a.w, b.w))),
                     i & 7);
        } else {
          d = fadd(d, fmul(a.x, b.x));
          d = fadd(d, fmul(a.y, b.y));
          d = fadd(d, fmul(a.z, b.z));
          d = fadd(d, fmul(a.w, b.w));
        }
      }
      const float sv = fmul(d, scale);  // scale after the dot (gpu/README.md §4)
      sc[(size_t)sg * scs + j0 + sj] = sv;
      mloc = max_comb(mloc, sv);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mloc = max_comb(mloc, __shfl_xor_sync(FULL, mloc, o));
  if (lane == 0) red[warp] = mloc;  // warp w's scores all belong to head 32 w / JC
  __syncthreads();  // every ring slot is free again; the warp maxima are visible
#pragma unroll
  for (int c = 0; c < ST - 1; ++c) stage(vbase, c);  // V chunks load while the softmax runs

  // ---- softmax (serial-scan max, pinned exp, serial denominator, divide)
  if (tid < G) {
    constexpr int WPH = JC / 32;  // warps per head
    const float *s0 = sc + (size_t)tid * scs;
    float m = red[tid * WPH];
#pragma unroll
    for (int w = 1; w < WPH; ++w) m = max_comb(m, red[tid * WPH + w]);
    red[48 + tid] = is_nan(s0[0]) ? s0[0] : m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float *srow = sc + (size_t)g * scs;
    const float mg = red[48 + g];
    for (int j = tid; j < len; j += NT) srow[j] = exp_pinned(fsub(srow[j], mg));
  }
  __syncthreads();
  if (TREE) {  // head g's 32-leaf blocks (zero-padded) in warp g, block sums added in order
    if (warp < G) {
      const float *srow = sc + (size_t)warp * scs;
      float acc = 0.0f;
      for (int j0 = 0; j0 < len; j0 += 32) {
        const float t = warp_tree32(j0 + lane < len ? srow[j0 + lane] : 0.0f);
        acc = fadd(acc, t);
      }
      if (lane == 0) red[32 + warp] = acc;
    }
  } else if (tid < G) {
    red[32 + tid] = serial_sum4(sc + (size_t)tid * scs, len);
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float *srow = sc + (size_t)g * scs;
    const float den = red[32 + g];
    for (int j = tid; j < len; j += NT) srow[j] = fdiv(srow[j], den);
  }

  // ---- V-mix: thread (g, d, d + 1) = (tid / (HD/2), 2 (tid % (HD/2))), two
  // independent chains, j ascending, one packed add per position
  constexpr int DPW = HD / 2;
  const int g = tid / DPW, d = 2 * (tid % DPW);
  const bool owns = tid < G * DPW;
  float2 acc = make_float2(0.0f, 0.0f);
  for (int c = 0; c < nch; ++c) {
    land(c);
    stage(vbase, c + ST - 1);
    const int j0 = c * JC, jc = min(JC, len - j0);
    const float *tile = tiles + (size_t)(c % ST) * JC * TS + d;
    if (owns) {
      const float *pg = sc + (size_t)g * scs + j0;  // j0 % 4 == 0: 16-byte aligned
      if (jc == JC) {
        // Full chunk: the weights and values of the next two groups of four
        // positions are loaded while the chains consume the current group.
        float4 pw[2];
        float2 vv[2][4];
        auto ld = [&](int b, int jj) {
          pw[b] = *reinterpret_cast<const float4 *>(pg + jj);
#pragma unroll
          for (int u = 0; u < 4; ++u) vv[b][u] = *reinterpret_cast<const float2 *>(tile + (jj + u) * TS);
        };
        ld(0, 0);
        ld(1, 4);
#pragma unroll
        for (int qd = 0; qd < JC / 4; ++qd) {
          const int b = qd & 1;
          const float4 w = pw[b];
          const float2 v0 = vv[b][0], v1 = vv[b][1], v2 = vv[b][2], v3 = vv[b][3];
          if (qd + 2 < JC / 4) ld(b, 4 * (qd + 2));
          acc = fadd_pair(acc, fmul(w.x, v0.x), fmul(w.x, v0.y));
          acc = fadd_pair(acc, fmul(w.y, v1.x), fmul(w.y, v1.y));
          acc = fadd_pair(acc, fmul(w.z, v2.x), fmul(w.z, v2.y));
          acc = fadd_pair(acc, fmul(w.w, v3.x), fmul(w.w, v3.y));
        }
      } else {
        for (int jj = 0; jj < jc; ++jj) {
          const float p = pg[jj];
          const float2 v = *reinterpret_cast<const float2 *>(tile + jj * TS);
          acc = fadd_pair(acc, fmul(p, v.x), fmul(p, v.y));
        }
      }
    }
  }
  cp_async_wait<0>();
  if (owns) {
    float *o = att + (size_t)r * ars + ((size_t)kvh * G + g) * HD * acs + (size_t)d * acs;
    o[0] = acc.x;
    o[acs] = acc.y;
  }
}

template <int HD, int G, int ST, bool TREE>
static void run_attention_dec(float *qkv, int ld, int rows, RowMap rm, int n_kv, float *kc, float *vc, int max_pos,
                              float *att, int ars, int acs, int max_len, const uint16_t *qn, const uint16_t *kn,
                              float eps, const float *cos_t, const float *sin_t, cudaStream_t s) {
  const size_t smem = attention_dec_smem_floats(G, HD, max_len, ST) * sizeof(float);
  static SmemLimit lim;
  lim.ensure(k_attention_dec<HD, G, ST, TREE>, smem);
  k_attention_dec<HD, G, ST, TREE><<<dim3(rows, n_kv), AttDec<HD, G>::NT, smem, s>>>(
      qkv, ld, rm.seq, rm.pos, n_kv, kc, vc, max_pos, att, ars, acs, max_len, qn, kn, eps, cos_t, sin_t);
}

// Decode-step attention through the specialised kernel when it covers the
// shape ((head size, group) of the configurations built here); returns
// false if the caller must use the generic kernel.
bool launch_attention_dec(float *qkv, int ld, int rows, RowMap rm, int n_heads, int n_kv, int hd, float *kcache,
                          float *vcache, int max_pos, float *att, int ars, int acs, int max_len,
                          const uint16_t *q_norm, const uint16_t *k_norm, float eps, const float *cos_t,
                          const float *sin_t, bool tree, cudaStream_t s) {
  if (rows <= 0) return true;
  const int G = n_heads / n_kv;
  constexpr int ST = ATT_DEC_STAGES;
#define CIS2B_ATTD(HD_, G_)                                                                                   \
  if (hd == HD_ && G == G_ && attention_dec_smem_floats(G_, HD_, max_len, ST) * 4 <= 227 * 1024) {            \
    if (tree)                                                                                                 \
      run_attention_dec<HD_, G_, ST, true>(qkv, ld, rows, rm, n_kv, kcache, vcache, max_pos, att, ars, acs,   \
                                           max_len, q_norm, k_norm, eps, cos_t, sin_t, s);                    \
    else                                                                                                      \
      run_attention_dec<HD_, G_, ST, false>(qkv, ld, rows, rm, n_kv, kcache, vcache, max_pos, att, ars, acs,  \
                                            max_len, q_norm, k_norm, eps, cos_t, sin_t, s);                   \
    return true;                                                                                              \
  }
  CIS2B_ATTD(64, 3)
  CIS2B_ATTD(64, 1)
  CIS2B_ATTD(128, 2)
#undef CIS2B_ATTD
  return false;
}

// Trace mode: the per-head q/k RMSNorm alone (qwen3-port.diff:66-80), in
// place on one qkv row, with the same warp routine k_qkv_post applies before
// its RoPE; launch_qkv_post then runs without norm weights.
__global__ void k_qk_norm_row(float *row, int nh, int nkv, int hd, const uint16_t *qn, const uint16_t *kn,
                              float eps, int tree) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int h = warp; h < nh + nkv; h += nw) {
    const bool is_k = h >= nh;
    const uint16_t *w = is_k ? kn : qn;
    float *x = is_k ? row + (size_t)nh * hd + (size_t)(h - nh) * hd : row + (size_t)h * hd;
    if (w) warp_rmsnorm(x, w, eps, hd, tree != 0, sm + (size_t)warp * 2 * hd, x);
  }
}
void launch_qk_norm_row(float *row, int n_heads, int n_kv, int hd, const uint16_t *q_norm, const uint16_t *k_norm,
                        float eps, bool tree, cudaStream_t s) {
  k_qk_norm_row<<<1, 128, (size_t)4 * 2 * hd * sizeof(float), s>>>(row, n_heads, n_kv, hd, q_norm, k_norm, eps,
                                                                     tree ? 1 : 0);
}

// ---- Prompt-pass attention, several rows per CTA.  In the prompt pass the
// rows of one sequence are consecutive positions, and row p reads keys and
// values 0..p, so one CTA takes a tile of up to `rt` such rows for one KV
// head and streams each K/V chunk through shared memory once for all of
// them (the one-row kernel above waits for each chunk once per row).  Per
// (row, head) the arithmetic is the one-row kernel's, in the same order: the
// scaled dot of every key, the serial-scan max, pinned exp, the pinned-order
// denominator (one thread per (row, head) chain, or the 32-leaf blocks in
// tree mode), the division, and the V-mix chain per (row, head, d) over keys
// ascending.  tiles[t] = (first row, rows) of the pass's row list.
constexpr int ATTR_NT = 256;
constexpr int ATTR_CHAINS = 16;  // V-mix chains per thread at most

int attention_rows_rt(int G, int hd, int max_len) {
  const size_t row_bytes = (size_t)G * (((size_t)max_len + 3) / 4 * 4 + 4) * 4;  // one row's scores
  int rt = (int)((64 * 1024) / row_bytes);
  const int by_chains = ATTR_CHAINS * (ATTR_NT / hd) / G;
  if (rt > by_chains) rt = by_chains;
  if (rt > 16) rt = 16;
  return rt < 1 ? 1 : rt;
}
size_t attention_rows_smem_floats(int rt, int G, int hd, int max_len) {
  const size_t scs = (((size_t)max_len + 3) & ~(size_t)3) + 4;  // +4: rows start on different banks
  const size_t P = (size_t)rt * G;
  size_t f = P * hd + P * scs + P * ((size_t)max_len / 32 + 1) + 3 * P + 8;
  f = (f + 3) & ~(size_t)3;
  return f + (size_t)2 * ATT_JC * (hd + 4);
}

__global__ void __launch_bounds__(ATTR_NT)
k_attention_rows(const float *qkv, int ld, const int2 *tiles, const int32_t *rseq, const int32_t *rpos, int rt,
                 int nh, int nkv, int hd, const float *kc, const float *vc, int max_pos, int tree, float *att,
                 int ars, int acs, int max_len) {
  extern __shared__ __align__(16) float sm[];
  const int kvh = blockIdx.y, tid = threadIdx.x, nt = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
  const int G = nh / nkv, KV = nkv * hd;
  const int2 tl = tiles[blockIdx.x];
  const int r0 = tl.x, nr = tl.y, P = nr * G;
  const int seq = rseq[r0], p0 = rpos[r0];
  const int lenmax = p0 + nr;                        // keys 0 .. p0 + nr - 1
  const int scs = ((max_len + 3) & ~3) + 4;
  const int npb = max_len / 32 + 1;
  const int PR = rt * G;                             // pair slots the layout reserves
  float *q = sm;                                     // [pair][hd], pair = i * G + g
  float *sc = q + (size_t)PR * hd;                   // [pair][scs]
  float *part = sc + (size_t)PR * scs;               // [pair][npb] (tree mode)
  float *red = part + (size_t)PR * npb;              // [2][pair]: max, denominator
  int *lim = reinterpret_cast<int *>(red + 2 * PR);  // [pair]: last key position the row reads
  size_t toff = (size_t)(red + 3 * PR + 8 - sm);
  toff = (toff + 3) & ~(size_t)3;
  float *tiles_s = sm + toff;                        // [2][ATT_JC][hd + 4]
  const int ts = hd + 4;
  for (int x = tid; x < P * hd; x += nt) {
    const int pr = x / hd, d = x - pr * hd, i = pr / G, g = pr - i * G;
    q[x] = qkv[(size_t)(r0 + i) * ld + ((size_t)kvh * G + g) * hd + d];
  }
  for (int pr = tid; pr < P; pr += nt) lim[pr] = p0 + pr / G;
  const float scale = rsqrt_cr(__int2float_rn(hd));
  const float *kbase = kc + (size_t)seq * max_pos * KV + (size_t)kvh * hd;
  const float *vbase = vc + (size_t)seq * max_pos * KV + (size_t)kvh * hd;
  const int nch = (lenmax + ATT_JC - 1) / ATT_JC;
  const uint32_t tbase = (uint32_t)__cvta_generic_to_shared(tiles_s);
  auto stage = [&](const float *base, int c, int buf) {
    const int j0 = c * ATT_JC, jc = min(ATT_JC, lenmax - j0), nq = hd / 4;
    for (int x = tid; x < jc * nq; x += nt) {
      const int jj = x / nq, q4 = x - jj * nq;
      cp_async16(tbase + (uint32_t)(((buf * ATT_JC + jj) * ts + 4 * q4) * 4), base + (size_t)(j0 + jj) * KV + 4 * q4);
    }
    cp_async_commit();
  };

  // ---- scores
  stage(kbase, 0, 0);
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) stage(kbase, c + 1, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int j0 = c * ATT_JC;
    const float *tile = tiles_s + (size_t)(c & 1) * ATT_JC * ts;
    for (int x = tid; x < P * ATT_JC; x += nt) {
      const int pr = x / ATT_JC, jj = x % ATT_JC;
      if (j0 + jj > lim[pr]) continue;  // past this row's position (and past the chunk)
      const float *qg = q + (size_t)pr * hd, *kj = tile + jj * ts;
      float d;
      if (!tree) {
        const float4 *q4 = reinterpret_cast<const float4 *>(qg), *k4 = reinterpret_cast<const float4 *>(kj);
        d = 0.0f;
        for (int u = 0; u < hd / 4; ++u) {
          const float4 a = q4[u], b = k4[u];
          d = fadd(d, fmul(a.x, b.x));
          d = fadd(d, fmul(a.y, b.y));
          d = fadd(d, fmul(a.z, b.z));
          d = fadd(d, fmul(a.w, b.w));
        }
      } else {
        d = dot_tree(qg, kj, hd);
      }
      sc[(size_t)pr * scs + j0 + jj] = fmul(d, scale);
    }
    __syncthreads();
  }
  stage(vbase, 0, 0);  // V chunk 0 loads while the softmax runs
  // ---- max per (row, head), serial-scan semantics
  for (int pr = warp; pr < P; pr += nw) {
    const float *sg = sc + (size_t)pr * scs;
    const int len = lim[pr] + 1;
    float mx = bitsf(0x7fc00000u);
    for (int j = lane; j < len; j += 32) mx = max_comb(mx, sg[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max_comb(mx, __shfl_xor_sync(FULL, mx, o));
    if (lane == 0) red[pr] = is_nan(sg[0]) ? sg[0] : mx;
  }
  __syncthreads();
  for (int pr = 0; pr < P; ++pr) {
    float *sg = sc + (size_t)pr * scs;
    const int len = lim[pr] + 1;
    const float mg = red[pr];
    for (int j = tid; j < len; j += nt) sg[j] = exp_pinned(fsub(sg[j], mg));
  }
  __syncthreads();
  // ---- denominators: one thread per (row, head) chain
  if (tree) {
    for (int pr = 0; pr < P; ++pr) {
      const int len = lim[pr] + 1, nb = (len + 31) / 32;
      for (int b = warp; b < nb; b += nw) {
        const int j = b * 32 + lane;
        const float v = warp_tree32(j < len ? sc[(size_t)pr * scs + j] : 0.0f);
        if (lane == 0) part[(size_t)pr * npb + b] = v;
      }
    }
    __syncthreads();
  }
  for (int pr = tid; pr < P; pr += nt) {
    const int len = lim[pr] + 1;
    red[PR + pr] = tree ? serial_sum(part + (size_t)pr * npb, (len + 31) / 32) : serial_sum4(sc + (size_t)pr * scs, len);
  }
  __syncthreads();
  for (int pr = 0; pr < P; ++pr) {
    float *sg = sc + (size_t)pr * scs;
    const int len = lim[pr] + 1;
    const float den = red[PR + pr];
    for (int j = tid; j < len; j += nt) sg[j] = fdiv(sg[j], den);
  }
  // ---- V-mix: thread owns d = tid % hd of pairs tid / hd + k * (nt / hd)
  const int d = tid % hd, slot0 = tid / hd, slots = nt / hd;
  float acc[ATTR_CHAINS];
#pragma unroll
  for (int k = 0; k < ATTR_CHAINS; ++k) acc[k] = 0.0f;
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) stage(vbase, c + 1, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int j0 = c * ATT_JC;
    const float *tile = tiles_s + (size_t)(c & 1) * ATT_JC * ts + d;
    if (slot0 < slots) {
#pragma unroll
      for (int k = 0; k < ATTR_CHAINS; ++k) {
        const int pr = slot0 + k * slots;
        if (pr < P) {
          const int je = min(ATT_JC, lim[pr] + 1 - j0);  // keys of this chunk the row reads
          const float *pg = sc + (size_t)pr * scs + j0;
          float a = acc[k];
          for (int jj = 0; jj < je; ++jj) a = fadd(a, fmul(pg[jj], tile[jj * ts]));
          acc[k] = a;
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  if (slot0 < slots) {
#pragma unroll
    for (int k = 0; k < ATTR_CHAINS; ++k) {
      const int pr = slot0 + k * slots;
      if (pr < P) {
        const int i = pr / G, g = pr - i * G;
        att[(size_t)(r0 + i) * ars + (((size_t)kvh * G + g) * hd + d) * acs] = acc[k];
      }
    }
  }
}

// Sequential-mode prompt-pass attention specialised on the head size HD and
// the group G (the same arithmetic as k_attention_rows, in the same order).
// Per chunk of ATT_JC keys, a thread computes the dots of one row of the
// tile with one key for all G heads of the group: each 16-byte key load
// feeds G independent chains (the scores were bound by shared-memory
// bandwidth when every (head, key) dot loaded its key), the q loads are
// broadcasts, and a warp's 32 key rows are consecutive (the TS pitch keeps
// those loads conflict-free).  In the V-mix a thread owns two
// adjacent d of up to PPT pairs: per key one 8-byte value load serves all
// its pairs, the weights of four keys come in one 16-byte load per pair,
// and each pair's two chains take one packed add per key.
// TREE: the tree order for the dots (32-product pairwise trees over HD)
// and the denominators (32-leaf blocks, block sums in order); the V-mix
// chains are the same in both orders.
template <int HD, int G, bool TREE>
__global__ void __launch_bounds__(ATTR_NT, 2)
k_attention_rows_s(const float *qkv, int ld, const int2 *tiles, const int32_t *rseq, const int32_t *rpos, int nkv,
                   const float *kc, const float *vc, int max_pos, float *att, int ars, int acs, int max_len) {
  constexpr int NT = ATTR_NT, JC = ATT_JC, TS = HD + 4, NQ = HD / 4;
  constexpr int S = NT / (HD / 2);           // V-mix pair slots
  constexpr int PMAX = 48;                   // pairs per tile at most (attention_rows_rt)
  constexpr int PPT = (PMAX + S - 1) / S;    // pairs per V-mix thread at most
  static_assert(JC == 64 && NT % (HD / 2) == 0 && NT % NQ == 0, "tile shape");
  extern __shared__ __align__(16) float sm[];
  const int kvh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = NT / 32;
  const int KV = nkv * HD;
  const int2 tl = tiles[blockIdx.x];
  const int r0 = tl.x, nr = tl.y, P = nr * G;
  const int seq = rseq[r0], p0 = rpos[r0];
  const int lenmax = p0 + nr;
  const int scs = ((max_len + 3) & ~3) + 4;
  float *q = sm;                                     // [pair][HD]
  float *sc = q + (size_t)P * HD;                    // [pair][scs]
  float *red = sc + (size_t)P * scs;                 // [2][pair]
  size_t toff = (size_t)(red + 2 * P + 8 - sm);
  toff = (toff + 3) & ~(size_t)3;
  float *tiles_s = sm + toff;                        // [2][JC][TS]
  for (int x = tid; x < P * HD; x += NT) {
    const int pr = x / HD, d = x % HD, i = pr / G, g = pr % G;
    q[x] = qkv[(size_t)(r0 + i) * ld + ((size_t)kvh * G + g) * HD + d];
  }
  const float scale = rsqrt_cr(__int2float_rn(HD));
  const float *kbase = kc + (size_t)seq * max_pos * KV + (size_t)kvh * HD;
  const float *vbase = vc + (size_t)seq * max_pos * KV + (size_t)kvh * HD;
  const int nch = (lenmax + JC - 1) / JC;
  const uint32_t tbase = (uint32_t)__cvta_generic_to_shared(tiles_s);
  constexpr int RP = NT / NQ;
  const int sq = tid % NQ, sr = tid / NQ;
  auto stage = [&](const float *base, int c, int buf) {
    const int j0 = c * JC, jc = min(JC, lenmax - j0);
    const float *src = base + (size_t)(j0 + sr) * KV + 4 * sq;
    uint32_t dst = tbase + (uint32_t)(((buf * JC + sr) * TS + 4 * sq) * 4);
    for (int jj = sr; jj < jc; jj += RP) {
      cp_async16(dst, src);
      src += (size_t)RP * KV;
      dst += (uint32_t)(RP * TS * 4);
    }
    cp_async_commit();
  };

  // ---- scores
  stage(kbase, 0, 0);
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) stage(kbase, c + 1, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int j0 = c * JC;
    const float *tile = tiles_s + (size_t)(c & 1) * JC * TS;
    for (int u0 = tid; u0 < nr * JC; u0 += NT) {
      const int i = u0 / JC, jj = u0 % JC;     // row i of the tile, key j0 + jj: all G heads
      if (j0 + jj > p0 + i) continue;          // past this row's position (and past the chunk)
      const float4 *k4 = reinterpret_cast<const float4 *>(tile + jj * TS);
      const float4 *q4 = reinterpret_cast<const float4 *>(q + (size_t)i * G * HD);
      float d[G], t3[G], t4[G], t5[G];
#pragma unroll
      for (int g = 0; g < G; ++g) d[g] = t3[g] = t4[g] = t5[g] = 0.0f;
#pragma unroll
      for (int t = 0; t < NQ; ++t) {
        const float4 b = k4[t];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 a = q4[g * NQ + t];
          if (TREE) {
            tree_group(d[g], t3[g], t4[g], t5[g],
                       fadd(fadd(fmul(a.x, b.x), fmul(a.y, b.y)), fadd(fmul(a.z, b.z), fmul(a.w, b.w))), t & 7);
          } else {
            d[g] = fadd(d[g], fmul(a.x, b.x));
            d[g] = fadd(d[g], fmul(a.y, b.y));
            d[g] = fadd(d[g], fmul(a.z, b.z));
            d[g] = fadd(d[g], fmul(a.w, b.w));
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) sc[(size_t)(i * G + g) * scs + j0 + jj] = fmul(d[g], scale);
    }
    __syncthreads();
  }
  stage(vbase, 0, 0);  // V chunk 0 loads while the softmax runs
  // ---- max per (row, head), serial-scan semantics
  for (int pr = warp; pr < P; pr += NW) {
    const float *sg = sc + (size_t)pr * scs;
    const int len = p0 + pr / G + 1;
    float mx = bitsf(0x7fc00000u);
    for (int j = lane; j < len; j += 32) mx = max_comb(mx, sg[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max_comb(mx, __shfl_xor_sync(FULL, mx, o));
    if (lane == 0) red[pr] = is_nan(sg[0]) ? sg[0] : mx;
  }
  __syncthreads();
  for (int pr = 0; pr < P; ++pr) {
    float *sg = sc + (size_t)pr * scs;
    const int len = p0 + pr / G + 1;
    const float mg = red[pr];
    for (int j = tid; j < len; j += NT) sg[j] = exp_pinned(fsub(sg[j], mg));
  }
  __syncthreads();
  // ---- denominators: one lane per (row, head) chain, or in tree order one
  // warp per (row, head): 32-leaf blocks (zero-padded), block sums in order
  if (TREE) {
    for (int pr = warp; pr < P; pr += NW) {
      const float *sg = sc + (size_t)pr * scs;
      const int len = p0 + pr / G + 1;
      float acc = 0.0f;
      for (int j0 = 0; j0 < len; j0 += 32) acc = fadd(acc, warp_tree32(j0 + lane < len ? sg[j0 + lane] : 0.0f));
      if (lane == 0) red[P + pr] = acc;
    }
  } else {
    for (int pr = tid; pr < P; pr += NT) red[P + pr] = serial_sum4(sc + (size_t)pr * scs, p0 + pr / G + 1);
  }
  __syncthreads();
  for (int pr = 0; pr < P; ++pr) {
    float *sg = sc + (size_t)pr * scs;
    const int len = p0 + pr / G + 1;
    const float den = red[P + pr];
    for (int j = tid; j < len; j += NT) sg[j] = fdiv(sg[j], den);
  }
  // ---- V-mix: thread (d, d + 1) = 2 (tid % (HD/2)) of pairs tid / (HD/2) + k S
  const int d = 2 * (tid % (HD / 2)), slot = tid / (HD / 2);
  float2 acc[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) acc[k] = make_float2(0.0f, 0.0f);
  const int full_to = p0 + 1;  // keys [0, full_to) are read by every row of the tile
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) stage(vbase, c + 1, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int j0 = c * JC;
    const float *tile = tiles_s + (size_t)(c & 1) * JC * TS + d;
    if (j0 + JC <= full_to) {
      // every pair reads the whole chunk
#pragma unroll 1
      for (int jj = 0; jj < JC; jj += 4) {
        const float2 v0 = *reinterpret_cast<const float2 *>(tile + (jj + 0) * TS);
        const float2 v1 = *reinterpret_cast<const float2 *>(tile + (jj + 1) * TS);
        const float2 v2 = *reinterpret_cast<const float2 *>(tile + (jj + 2) * TS);
        const float2 v3 = *reinterpret_cast<const float2 *>(tile + (jj + 3) * TS);
#pragma unroll
        for (int k = 0; k < PPT; ++k) {
          const int pr = slot + k * S;
          if (pr < P) {
            const float4 w = *reinterpret_cast<const float4 *>(sc + (size_t)pr * scs + j0 + jj);
            float2 a = acc[k];
            a = fadd_pair(a, fmul(w.x, v0.x), fmul(w.x, v0.y));
            a = fadd_pair(a, fmul(w.y, v1.x), fmul(w.y, v1.y));
            a = fadd_pair(a, fmul(w.z, v2.x), fmul(w.z, v2.y));
            a = fadd_pair(a, fmul(w.w, v3.x), fmul(w.w, v3.y));
            acc[k] = a;
          }
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < PPT; ++k) {
        const int pr = slot + k * S;
        if (pr < P) {
          const int je = min(JC, p0 + pr / G + 1 - j0);  // keys of this chunk the row reads
          const float *pg = sc + (size_t)pr * scs + j0;
          float2 a = acc[k];
          for (int jj = 0; jj < je; ++jj) {
            const float p = pg[jj];
            const float2 v = *reinterpret_cast<const float2 *>(tile + jj * TS);
            a = fadd_pair(a, fmul(p, v.x), fmul(p, v.y));
          }
          acc[k] = a;
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int pr = slot + k * S;
    if (pr < P) {
      const int i = pr / G, g = pr % G;
      float *o = att + (size_t)(r0 + i) * ars + (((size_t)kvh * G + g) * HD + d) * acs;
      o[0] = acc[k].x;
      o[acs] = acc[k].y;
    }
  }
}

// Shared memory of k_attention_rows_s for tiles of up to rt rows.
size_t attention_rows_s_smem_floats(int rt, int G, int hd, int max_len) {
  const size_t P = (size_t)rt * G, scs = (((size_t)max_len + 3) & ~(size_t)3) + 4;
  size_t f = P * hd + P * scs + 2 * P + 8;
  f = (f + 3) & ~(size_t)3;
  return f + (size_t)2 * ATT_JC * (hd + 4);
}

template <int HD, int G, bool TREE>
static void run_attention_rows_s(const float *qkv, int ld, const int2 *tiles, int n_tiles, int rt, RowMap rm, int n_kv,
                                 const float *kc, const float *vc, int max_pos, float *att, int ars, int acs,
                                 int max_len, cudaStream_t s) {
  const size_t smem = attention_rows_s_smem_floats(rt, G, HD, max_len) * sizeof(float);
  static SmemLimit lim;
  lim.ensure(k_attention_rows_s<HD, G, TREE>, smem);
  k_attention_rows_s<HD, G, TREE><<<dim3(n_tiles, n_kv), ATTR_NT, smem, s>>>(qkv, ld, tiles, rm.seq, rm.pos, n_kv, kc, vc,
                                                                      max_pos, att, ars, acs, max_len);
}

void launch_attention_rows(const float *qkv, int ld, const int2 *tiles, int n_tiles, int rt, RowMap rm, int n_heads,
                           int n_kv, int hd, const float *kcache, const float *vcache, int max_pos, bool tree,
                           float *att, int ars, int acs, int max_len, cudaStream_t s) {
  if (n_tiles <= 0) return;
  const int G = n_heads / n_kv;
  if (rt * G <= 48 && attention_rows_s_smem_floats(rt, G, hd, max_len) * 4 <= 227 * 1024) {
#define CIS2B_ATTR(HD_, G_)                                                                                        \
    if (hd == HD_ && G == G_) {                                                                                    \
      if (tree)                                                                                                    \
        run_attention_rows_s<HD_, G_, true>(qkv, ld, tiles, n_tiles, rt, rm, n_kv, kcache, vcache, max_pos, att,  \
                                            ars, acs, max_len, s);                                                 \
      else                                                                                                         \
        run_attention_rows_s<HD_, G_, false>(qkv, ld, tiles, n_tiles, rt, rm, n_kv, kcache, vcache, max_pos, att, \
                                             ars, acs, max_len, s);                                                \
      return;                                                                                                      \
    }
    CIS2B_ATTR(64, 3)
    CIS2B_ATTR(64, 1)
    CIS2B_ATTR(128, 2)
#undef CIS2B_ATTR
  }
  const size_t smem = attention_rows_smem_floats(rt, G, hd, max_len) * sizeof(float);
  static SmemLimit lim;
  if (smem > 48 * 1024) lim.ensure(k_attention_rows, smem);
  k_attention_rows<<<dim3(n_tiles, n_kv), ATTR_NT, smem, s>>>(qkv, ld, tiles, rm.seq, rm.pos, rt, n_heads, n_kv, hd,
                                                             kcache, vcache, max_pos, tree ? 1 : 0, att, ars, acs,
                                                             max_len);
}

// ============================================================ token selection

struct ArgBest { float v; int i; };
// Lowest index among the maximal non-NaN values (the serial strict-'>' scan
// from index 0 of cis2_model.h:764-774, given element 0 is not NaN).
__device__ __forceinline__ ArgBest arg_comb(ArgBest a, ArgBest b) {
  if (a.i < 0) return b;
  if (b.i < 0) return a;
  if (b.v > a.v) return b;
  if (a.v > b.v) return a;
  return (b.i < a.i) ? b : a;
}

__global__ void k_argmax(const float *logits, int V, const int32_t *slot, size_t slot_stride,
                         uint32_t *next) {
  __shared__ ArgBest red[32];
  const int r = blockIdx.x, tid = threadIdx.x;
  const float *row = logits + (slot ? (size_t)(*slot) * slot_stride : 0) + (size_t)r * V;
  ArgBest b = {0.0f, -1};
  for (int i = tid; i < V; i += blockDim.x) {
    float v = row[i];
    if (is_nan(v)) continue;
    if (b.i < 0 || v > b.v) { b.v = v; b.i = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgBest c;
    c.v = __shfl_xor_sync(FULL, b.v, o);
    c.i = __shfl_xor_sync(FULL, b.i, o);
    b = arg_comb(b, c);
  }
  if ((tid & 31) == 0) red[tid >> 5] = b;
  __syncthreads();
  if (tid == 0) {
    ArgBest a = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) a = arg_comb(a, red[w]);
    uint32_t idx = (a.i < 0 || is_nan(row[0])) ? 0u : (uint32_t)a.i;
    next[r] = idx;
  }
}
void launch_argmax(const float *logits, int V, int rows, const int32_t *slot, size_t slot_stride,
                   uint32_t *next, cudaStream_t s) {
  if (rows <= 0) return;
  k_argmax<<<rows, 1024, 0, s>>>(logits, V, slot, slot_stride, next);
}

// ---- E23 pinned sampler (e23 patch, src/sampling.rs hunk :650-725) ----
//
// One CTA per row.  Element-wise steps run on all threads; the
// order-pinned folds (softmax denominator, nucleus cumulative sum, CDF walk)
// run in thread 0 over chunks that the other threads stage into shared
// memory.  The renormalisation total is not folded again: it is the sum of
// the nucleus in sorted order, the very sequence of additions the nucleus
// walk made, so it equals the nucleus walk's final sum bit for bit.  The
// (probability desc, index asc) order is a stable LSD radix sort of key =
// ~bits(p) (p >= +0, so bit order is value order) over ascending indices.
constexpr int SAMPLE_THREADS = 1024;
constexpr int FOLD_CHUNK = 1024;

__device__ __forceinline__ uint64_t sm64_round(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Pinned running sum: thread 0 forms acc_i = ((0 + v_0) + v_1) + ... + v_i
// for i = 0..n-1 in order, v_i = load(i), and stops at the first i with
// stop(acc_i).  The other threads compute load() for the next chunk and
// stage it in shared memory while thread 0 folds the current one.  Thread 0
// reads 8 values at a time with 16-byte loads, one batch ahead, and tests
// stop() once per 8 additions without a branch, so its chain waits only on
// the additions;
// stop must therefore be monotone along the walk, which holds for a running
// sum of non-negative values and a threshold test.  When a 64-value stretch
// has crossed, the stretch is walked again one value at a time from its
// saved start to find the exact index (the same additions, so the same
// values).  Result, after the final barrier: sh_i[1] = the stop index (n if
// none), sh_f[0] = acc at that index (the full sum if none).
// buf: 2 * FOLD_CHUNK floats, 16-byte aligned; sh_i[0] is the stop flag.
template <class Load, class Stop>
__device__ void fold_until(int n, Load load, Stop stop, float *buf, int *sh_i, float *sh_f) {
  const int tid = threadIdx.x;
  if (tid == 0) sh_i[0] = 0;
  for (int i = tid; i < FOLD_CHUNK && i < n; i += blockDim.x) buf[i] = load(i);
  __syncthreads();
  float acc = 0.0f;
  int at = n;
  const int nch = (n + FOLD_CHUNK - 1) / FOLD_CHUNK;
  for (int c = 0; c < nch; ++c) {
    float *cur = buf + (c & 1) * FOLD_CHUNK;
    float *nxt = buf + ((c + 1) & 1) * FOLD_CHUNK;
    const int base = c * FOLD_CHUNK, cnt = min(FOLD_CHUNK, n - base);
    if (tid == 0) {
      int i = 0;
      const float4 *q4 = reinterpret_cast<const float4 *>(cur);
      float4 na, nb;  // the next 8 values, loaded one batch ahead
      if (cnt >= 64) { na = q4[0]; nb = q4[1]; }
      for (; i + 64 <= cnt; i += 64) {
        const float a0 = acc;
        bool crossed = false;
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const float4 a = na, b = nb;
          const int nx = (i + 8 * h + 8) >> 2;  // float4 index of the next batch
          if (h < 7 || i + 128 <= cnt) { na = q4[nx]; nb = q4[nx + 1]; }
          acc = fadd(acc, a.x); acc = fadd(acc, a.y); acc = fadd(acc, a.z); acc = fadd(acc, a.w);
          acc = fadd(acc, b.x); acc = fadd(acc, b.y); acc = fadd(acc, b.z); acc = fadd(acc, b.w);
          crossed |= stop(acc);
        }
        if (crossed) {
          acc = a0;
          for (int u = 0; u < 64; ++u) {
            acc = fadd(acc, cur[i + u]);
            if (stop(acc)) { at = base + i + u; break; }
          }
          break;
        }
      }
      if (at == n)
        for (; i < cnt; ++i) {
          acc = fadd(acc, cur[i]);
          if (stop(acc)) { at = base + i; break; }
        }
      if (at != n) sh_i[0] = 1;
    } else if (c + 1 < nch) {
      const int nb = base + FOLD_CHUNK, ncnt = min(FOLD_CHUNK, n - nb);
      for (int i = tid - 1; i < ncnt; i += blockDim.x - 1) nxt[i] = load(nb + i);
    }
    __syncthreads();
    if (sh_i[0]) break;
  }
  if (tid == 0) { sh_i[1] = at; sh_f[0] = acc; }
  __syncthreads();
}

// Stable LSD radix sort of (key, value) pairs by key ascending, 4 passes of
// 8 bits, by the whole block; the result ends in (kA, vA).  Values that come
// in index order therefore keep index order among equal keys.
//
// Each warp owns one contiguous segment of the input.  Per pass it counts
// its segment's digits (32 at a time: lanes with equal digits find each
// other with match_any and the lowest of them adds the group's size), one
// block-wide scan turns the (digit, warp) counts into output offsets, and
// each warp then writes its segment in order, every element at
// offset(digit, warp) + (equal digits before it in the segment).  The
// output order is (digit, warp, position in segment) = (digit, index): the
// pass is stable, with block barriers only between the phases of a pass.
// A pass whose digit is the same for every key moves nothing and is
// skipped.  wcnt holds [blockDim.x / 32][256] counters.
__device__ void block_radix_sort(uint32_t *kA, uint32_t *vA, uint32_t *kB, uint32_t *vB, int V, int *hist,
                                 int *base, int (*wcnt)[256]) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int seg = (V + nw - 1) / nw;
  const int lo = min(V, warp * seg), hi = min(V, lo + seg);
  __shared__ int skip[4];  // per pass, so no flag is reset while another thread may still read it
  if (tid < 4) skip[tid] = 0;
  __syncthreads();
  uint32_t *ki = kA, *vi = vA, *ko = kB, *vo = vB;
  for (int pass = 0; pass < 4; ++pass) {
    const int sh = 8 * pass;
    for (int d = lane; d < 256; d += 32) wcnt[warp][d] = 0;
    __syncwarp();
    // ---- counts per (warp, digit)
#pragma unroll 4
    for (int g = lo; g < hi; g += 32) {
      const int i = g + lane;
      const bool valid = i < hi;
      const int dg = valid ? (int)((ki[i] >> sh) & 255u) : 256;
      const unsigned same = __match_any_sync(FULL, dg);
      if (valid && (same & lt_mask) == 0) wcnt[warp][dg] += __popc(same);
      __syncwarp();
    }
    __syncthreads();
    // ---- offsets: digit-major, then warp
    if (tid < 256) {
      int run = 0;
      for (int w = 0; w < nw; ++w) { const int c = wcnt[w][tid]; wcnt[w][tid] = run; run += c; }
      hist[tid] = run;
      if (run == V) skip[pass] = 1;  // every key has this digit: the pass is the identity
    }
    __syncthreads();
    if (skip[pass]) continue;  // uniform across the block (read after the barrier)
    if (tid < 32) {      // exclusive scan of the 256 digit totals by one warp
      int v[8], t = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) { v[j] = hist[tid * 8 + j]; t += v[j]; }
      int incl = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(FULL, incl, o);
        if (tid >= o) incl += n;
      }
      int run = incl - t;
#pragma unroll
      for (int j = 0; j < 8; ++j) { base[tid * 8 + j] = run; run += v[j]; }
    }
    __syncthreads();
    // ---- scatter, segment order kept within each digit
#pragma unroll 4
    for (int g = lo; g < hi; g += 32) {
      const int i = g + lane;
      const bool valid = i < hi;
      const uint32_t key = valid ? ki[i] : 0u, val = valid ? vi[i] : 0u;
      const int dg = valid ? (int)((key >> sh) & 255u) : 256;
      const unsigned same = __match_any_sync(FULL, dg);
      if (valid) {
        const int dst = base[dg] + wcnt[warp][dg] + __popc(same & lt_mask);
        ko[dst] = key;
        vo[dst] = val;
      }
      __syncwarp();
      if (valid && (same & lt_mask) == 0) wcnt[warp][dg] += __popc(same);
      __syncwarp();
    }
    __syncthreads();
    uint32_t *t;
    t = ki; ki = ko; ko = t;
    t = vi; vi = vo; vo = t;
  }
  if (ki != kA) {  // an odd number of passes moved data: bring the result back to (kA, vA)
    for (int i = tid; i < V; i += nt) { kA[i] = ki[i]; vA[i] = vi[i]; }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(SAMPLE_THREADS)
k_sample(const float *logits, int V, const int32_t *slot, size_t slot_stride, float temperature,
         float top_p, uint64_t seed, const int32_t *position, float *scratch, uint32_t *next) {
  __shared__ __align__(16) float buf[2 * FOLD_CHUNK];
  __shared__ int hist[256];
  __shared__ int base[256];
  __shared__ int wcnt[SAMPLE_THREADS / 32][256];
  __shared__ float redf[32];
  __shared__ float shared_f[4];
  __shared__ int shared_i[4];
  const int r = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const float *row = logits + (slot ? (size_t)(*slot) * slot_stride : 0) + (size_t)r * V;
  float *p = scratch + (size_t)r * 5 * V;                   // probabilities
  uint32_t *kA = reinterpret_cast<uint32_t *>(p + V), *vA = kA + V;
  uint32_t *kB = vA + V, *vB = kB + V;

  // Step 1-2: scale by temperature, max scan.
  float m = bitsf(0x7fc00000u);
  for (int i = tid; i < V; i += nt) {
    float s = fdiv(row[i], temperature);
    p[i] = s;
    m = max_comb(m, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max_comb(m, __shfl_xor_sync(FULL, m, o));
  if ((tid & 31) == 0) redf[tid >> 5] = m;
  __syncthreads();
  if (tid == 0) {
    float mm = redf[0];
    for (int w = 1; w < nt / 32; ++w) mm = max_comb(mm, redf[w]);
    if (is_nan(p[0])) mm = p[0];
    shared_f[0] = mm;
  }
  __syncthreads();
  const float mx = shared_f[0];
  for (int i = tid; i < V; i += nt) p[i] = exp_pinned(fsub(p[i], mx));
  __syncthreads();
  // Step 2b: denominator, strict left-to-right over index order.
  fold_until(V, [&](int i) { return p[i]; }, [](float) { return false; }, buf, shared_i, &shared_f[1]);
  const float den = shared_f[1];
  for (int i = tid; i < V; i += nt) {
    float pv = fdiv(p[i], den);
    p[i] = pv;
    kA[i] = ~__float_as_uint(pv);
    vA[i] = (uint32_t)i;
  }
  __syncthreads();
  // Step 3: stable LSD radix sort on ~bits(p): probability descending, index ascending.
  block_radix_sort(kA, vA, kB, vB, V, hist, base, wcnt);
  uint32_t *ki = kA, *vi = vA;
  // After 4 passes the sorted keys/indices are back in (kA, vA).
  // Step 4: nucleus = shortest prefix with cumulative sum >= top_p.  Step 5's
  // total (the nucleus summed again in the same order) is that prefix's sum.
  fold_until(V, [&](int i) { return __uint_as_float(~ki[i]); }, [&](float c) { return c >= top_p; }, buf,
             shared_i, &shared_f[2]);
  const int nuc = shared_i[1] < V ? shared_i[1] + 1 : V;
  const float total = shared_f[2];
  // Step 6: draw u = (word >> 11) * 2^-53, walk the CDF.
  const uint64_t pos64 = (uint64_t)(int64_t)position[r];
  const uint64_t word = sm64_round(seed ^ sm64_round(pos64));
  const double u = __dmul_rn((double)(word >> 11), 1.0 / 9007199254740992.0);
  fold_until(nuc, [&](int i) { return fdiv(__uint_as_float(~ki[i]), total); },
             [&](float c) { return (double)c > u; }, buf, shared_i, &shared_f[3]);
  const int pick = shared_i[1] < nuc ? shared_i[1] : nuc - 1;
  if (tid == 0) next[r] = vi[pick];
}

void launch_sample(const float *logits, int V, int rows, const int32_t *slot, size_t slot_stride,
                   float temperature, float top_p, uint64_t seed, const int32_t *position,
                   float *scratch, uint32_t *next, cudaStream_t s) {
  if (rows <= 0) return;
  k_sample<<<rows, SAMPLE_THREADS, 0, s>>>(logits, V, slot, slot_stride, temperature, top_p, seed,
                                           position, scratch, next);
}

// ------------------------------------------------------------ seeded Gumbel-max sampler
//
// The "CIS2-SAMPLE-1" clause (code/patches/cis2-spec__seeded-sampling.patch
// :81-145), one block per row:
//   s_i = l_i / T;  rank order = s descending, index ascending (stable radix
//   sort of an order-preserving key, -0 keyed as +0 since the clause compares
//   values);  top-k keeps ranks < k;  top-p walks the kept ranks with the
//   exp_pinned weights, their sequential denominator and running sum, keeping
//   rank r while r == 0 or c_{r-1} < top_p;  z_i = s_i + g_i for kept i,
//   g_i = -ln(-ln(u_i)) from MurmurHash3_x86_32(seed || step || i, 0x43495332);
//   next = the first index of the maximum z.
// MurmurHash3_x86_32 (Austin Appleby, public domain) is restated from the
// published algorithm for the clause's fixed 16-byte key.

__device__ __forceinline__ uint32_t mm3_rotl(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }
__device__ __forceinline__ uint32_t mm3_block(uint32_t h, uint32_t k) {
  k *= 0xcc9e2d51u;
  k = mm3_rotl(k, 15);
  k *= 0x1b873593u;
  h ^= k;
  h = mm3_rotl(h, 13);
  return h * 5u + 0xe6546b64u;
}
__device__ __forceinline__ float gumbel_noise(uint64_t seed, uint32_t step, uint32_t index) {
  uint32_t h = 0x43495332u;  // hash seed "CIS2"
  h = mm3_block(h, (uint32_t)seed);
  h = mm3_block(h, (uint32_t)(seed >> 32));
  h = mm3_block(h, step);
  h = mm3_block(h, index);
  h ^= 16u;  // key length
  h ^= h >> 16;
  h *= 0x85ebca6bu;
  h ^= h >> 13;
  h *= 0xc2b2ae35u;
  h ^= h >> 16;
  const float u = fmul(__uint2float_rn((h >> 9) * 2u + 1u), bitsf(0x33800000u));  // exact: m < 2^24, times 2^-24
  return fsub(0.0f, ln_pinned(fsub(0.0f, ln_pinned(u))));
}

__global__ void __launch_bounds__(SAMPLE_THREADS)
k_sample_gumbel(const float *logits, int V, const int32_t *slot, size_t slot_stride, float temperature,
                uint32_t top_k, float top_p, uint64_t seed, const int32_t *step, float *scratch, uint32_t *next) {
  __shared__ __align__(16) float buf[2 * FOLD_CHUNK];
  __shared__ int hist[256];
  __shared__ int base[256];
  __shared__ int wcnt[SAMPLE_THREADS / 32][256];
  __shared__ float bz[SAMPLE_THREADS / 32];
  __shared__ int bi[SAMPLE_THREADS / 32];
  __shared__ float shared_f[4];
  __shared__ int shared_i[4];
  const int r = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const float *row = logits + (slot ? (size_t)(*slot) * slot_stride : 0) + (size_t)r * V;
  float *sv = scratch + (size_t)r * 5 * V;  // s_i by index
  uint32_t *kA = reinterpret_cast<uint32_t *>(sv + V), *vA = kA + V;
  uint32_t *kB = vA + V, *vB = kB + V;
  for (int i = tid; i < V; i += nt) {
    const float x = fdiv(row[i], temperature);
    sv[i] = x;
    uint32_t u = __float_as_uint(x);
    if (u == 0x80000000u) u = 0u;                       // -0 ranks as +0
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // ascending with the value
    kA[i] = ~ord;                                        // descending
    vA[i] = (uint32_t)i;
  }
  __syncthreads();
  block_radix_sort(kA, vA, kB, vB, V, hist, base, wcnt);
  const uint32_t *order = vA;
  const int K = (top_k > 0 && top_k < (uint32_t)V) ? (int)top_k : V;
  int P = K;
  if (top_p < 1.0f) {
    const float m0 = sv[order[0]];
    float *e = reinterpret_cast<float *>(kB);  // e_r by rank
    for (int q = tid; q < K; q += nt) e[q] = exp_pinned(fsub(sv[order[q]], m0));
    __syncthreads();
    fold_until(K, [&](int q) { return e[q]; }, [](float) { return false; }, buf, shared_i, &shared_f[0]);
    const float den = shared_f[0];
    // Keep ranks up to and including the first whose cumulative sum is no
    // longer below top_p.
    fold_until(K, [&](int q) { return fdiv(e[q], den); }, [&](float c) { return !(c < top_p); }, buf,
               shared_i, &shared_f[1]);
    P = shared_i[1] < K ? shared_i[1] + 1 : K;
  }
  const uint32_t st = (uint32_t)*step;
  float best_z = 0.0f;
  int best_i = -1;
  for (int q = tid; q < P; q += nt) {
    const int i = (int)order[q];
    const float z = fadd(sv[i], gumbel_noise(seed, st, (uint32_t)i));
    if (best_i < 0 || z > best_z || (z == best_z && i < best_i)) { best_z = z; best_i = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float oz = __shfl_xor_sync(FULL, best_z, o);
    const int oi = __shfl_xor_sync(FULL, best_i, o);
    if (oi >= 0 && (best_i < 0 || oz > best_z || (oz == best_z && oi < best_i))) { best_z = oz; best_i = oi; }
  }
  if ((tid & 31) == 0) { bz[tid >> 5] = best_z; bi[tid >> 5] = best_i; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < nt / 32; ++w)
      if (bi[w] >= 0 && (best_i < 0 || bz[w] > best_z || (bz[w] == best_z && bi[w] < best_i))) {
        best_z = bz[w];
        best_i = bi[w];
      }
    next[r] = (uint32_t)best_i;
  }
}

void launch_sample_gumbel(const float *logits, int V, int rows, const int32_t *slot, size_t slot_stride,
                          float temperature, uint32_t top_k, float top_p, uint64_t seed, const int32_t *step,
                          float *scratch, uint32_t *next, cudaStream_t s) {
  if (rows <= 0) return;
  k_sample_gumbel<<<rows, SAMPLE_THREADS, 0, s>>>(logits, V, slot, slot_stride, temperature, top_k, top_p, seed,
                                                  step, scratch, next);
}

// ------------------------------------------------------------ sampler without allocation
//
// A second way to run the E23 sampler on one row, for callers that cannot
// allocate device memory themselves or through this library: code whose
// device memory belongs to its own allocator (a framework's caching pool or
// a pre-reserved arena) and must not be bypassed with cudaMalloc, and code
// on a latency-critical path where cudaMalloc/cudaFree would synchronise the
// device.  Its working memory is the file-scope array below, which every GPU
// that loads the library holds until the process exits.  Sized for rows of
// up to CIS2B_STATIC_SAMPLE_MAX logits: the sampler needs 5 floats per logit
// (probabilities, two key/index buffer pairs) plus one int for the position.
constexpr int kStaticSampleMax = CIS2B_STATIC_SAMPLE_MAX;
static_assert(kStaticSampleMax == 262144, "the error text below and the header state 262144");
static __device__ __align__(256) float g_sample_scratch[5 * kStaticSampleMax + 64];

// The host-side name g_sample_scratch is not a device address; the address
// is looked up once per device, with that device current, and kept for the
// life of the process (a device reset that destroys the primary context
// leaves it stale; the header says so).
static float *g_scratch_addr[64];
static std::mutex g_scratch_mu;

__global__ void k_store_position(int32_t *dst, int32_t v) { *dst = v; }

}  // namespace cis2b

extern "C" int cis2b_op_sample_static(int32_t device, const float *d_logits, int32_t n, float temperature,
                                      float top_p, uint64_t seed, uint64_t position, uint32_t *d_out_index,
                                      void *stream) {
  using namespace cis2b;
  if (!d_logits || !d_out_index) return set_last_error(1, "d_logits and d_out_index must be device pointers");
  if (n <= 0 || n > kStaticSampleMax)
    return set_last_error(1, "n must be in 1..262144: the static sampler scratch holds 5 floats per logit "
                             "for at most 262144 logits");
  if (!(temperature > 0.0f) || !(top_p > 0.0f && top_p <= 1.0f))
    return set_last_error(1, "temperature must be > 0 and top_p in (0, 1]");
  if (position > 0x7fffffffull) return set_last_error(1, "position must be < 2^31");
  if (device < 0 || device >= 64) return set_last_error(1, "device ordinal out of range");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return set_last_error(4, cudaGetErrorString(e));
  float *scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device]) {
      void *p = nullptr;
      e = cudaGetSymbolAddress(&p, g_sample_scratch);
      if (e != cudaSuccess) return set_last_error(4, cudaGetErrorString(e));
      g_scratch_addr[device] = static_cast<float *>(p);
    }
    scratch = g_scratch_addr[device];
  }
  // Every element of the scratch that the sampler reads it first writes, so
  // nothing is cleared between calls.  Only the position slot is set here.
  int32_t *pos_slot = reinterpret_cast<int32_t *>(scratch + 5 * (size_t)kStaticSampleMax);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  k_store_position<<<1, 1, 0, s>>>(pos_slot, (int32_t)position);
  k_sample<<<1, SAMPLE_THREADS, 0, s>>>(d_logits, n, nullptr, 0, temperature, top_p, seed, pos_slot, scratch,
                                        d_out_index);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(4, cudaGetErrorString(e));
  return 0;
}

namespace cis2b {

// After token selection: record the token, advance the row's position and
// the logits ring slot for the next step.
__global__ void k_step_advance(const uint32_t *next, int rows, const int32_t *step, int gen,
                               uint32_t *tokens_out, uint32_t *ids_hist, int32_t *pos,
                               int32_t *sample_pos, int32_t *slot, int ring, int32_t *step_ctr) {
  const int t = *step;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    tokens_out[(size_t)r * gen + t] = next[r];
    ids_hist[(size_t)t * rows + r] = next[r];
    pos[r] += 1;
    if (sample_pos) sample_pos[r] += 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (slot) *slot = (t + 1) % ring;
    if (step_ctr) *step_ctr = t + 1;
  }
}
void launch_step_advance(const uint32_t *next, int rows, const int32_t *step, int gen,
                         uint32_t *tokens_out, uint32_t *ids_hist, int32_t *pos, int32_t *sample_pos,
                         int32_t *slot, int ring, int32_t *step_ctr, cudaStream_t s) {
  // one block so that the counter update is ordered after every row's read
  k_step_advance<<<1, 1024, 0, s>>>(next, rows, step, gen, tokens_out, ids_hist, pos, sample_pos,
                                    slot, ring, step_ctr);
}

__global__ void k_gather_rows(const float *src, int ld, const int32_t *src_idx,
                              const int32_t *dst_idx, int H, float *dst) {
  int r = blockIdx.x;
  const float *s = src + (size_t)src_idx[r] * ld;
  float *d = dst + (size_t)dst_idx[r] * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) d[i] = s[i];
}
void launch_gather_rows(const float *src, int ld, const int32_t *src_idx, const int32_t *dst_idx,
                        int n, int H, float *dst, cudaStream_t s) {
  if (n <= 0) return;
  k_gather_rows<<<n, 256, 0, s>>>(src, ld, src_idx, dst_idx, H, dst);
}

// ============================================================ witness SHA-256

// Header / short input absorb: one thread per sequence, byte-serial.
__global__ void k_sha_absorb_bytes(ShaState *st, const uint8_t *bytes, const uint32_t *offsets,
                                   int n_seq) {
  int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n_seq) return;
  ShaState S = st[s];
  uint32_t bn = S.carry_n;
  const uint8_t *b = bytes + offsets[s];
  uint32_t n = offsets[s + 1] - offsets[s];
  for (uint32_t i = 0; i < n; ++i) sha_absorb_byte(S.h, S.carry, bn, b[i]);
  S.carry_n = bn;
  S.len += n;
  st[s] = S;
}
void launch_sha_absorb_bytes(ShaState *st, const uint8_t *bytes, const uint32_t *offsets, int n_seq,
                             cudaStream_t s) {
  if (n_seq <= 0) return;
  k_sha_absorb_bytes<<<(n_seq + 63) / 64, 64, 0, s>>>(st, bytes, offsets, n_seq);
}

// Step stream of one sequence = carry bytes || V logits (u32 LE) || next id.
__device__ __forceinline__ uint32_t step_dword(const uint32_t *data, int nd, uint32_t id, int i) {
  return i < nd ? data[i] : (i == nd ? id : 0u);
}
__device__ __forceinline__ uint8_t step_byte(const uint8_t *carry, int c, const uint32_t *data, int nd,
                                             uint32_t id, int p) {
  if (p < c) return carry[p];
  int q = p - c;
  return (uint8_t)(step_dword(data, nd, id, q >> 2) >> (8 * (q & 3)));
}
// Big-endian message word at stream byte offset p.
__device__ __forceinline__ uint32_t step_word(const uint8_t *carry, int c, const uint32_t *data,
                                              int nd, uint32_t id, int p) {
  if (p >= c) {
    int q = p - c;
    if ((q & 3) == 0) return __byte_perm(step_dword(data, nd, id, q >> 2), 0, 0x0123);
    if ((q & 3) == 2)
      return __byte_perm(step_dword(data, nd, id, q >> 2), step_dword(data, nd, id, (q >> 2) + 1),
                         0x2345);
  }
  uint32_t w = 0;
  for (int b = 0; b < 4; ++b) w = (w << 8) | step_byte(carry, c, data, nd, id, p + b);
  return w;
}

// W+K scratch: [block][warp][16 quads][32 lanes] uint4, so each step of the
// chain reads 512 contiguous bytes per warp and finds quad qd at a fixed
// offset from its block pointer.
size_t sha_wk_words(int V, int n_seq) {
  size_t nb_max = ((size_t)63 + 4 * (size_t)V + 4) / 64;
  return nb_max * 64 * (size_t)((n_seq + 31) / 32 * 32);
}

// Expand W+K for every full block of this step.  Layout [block][16 quads][seq]
// so the compression warp's 32 lanes read 512 contiguous bytes per quad.
__global__ void k_sha_prep(const ShaState *st, int n_seq, const float *logits, int V,
                           size_t row_stride, const uint32_t *next_ids, uint32_t *wk, int nb_max) {
  size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  int s = (int)(idx % n_seq), j = (int)(idx / n_seq);
  if (j >= nb_max) return;
  const int c = (int)st[s].carry_n;
  const int total = c + 4 * V + 4;
  if (j >= total / 64) return;
  const uint32_t *data = reinterpret_cast<const uint32_t *>(logits + (size_t)s * row_stride);
  const uint32_t id = next_ids[s];
  uint32_t m[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) m[i] = step_word(st[s].carry, c, data, V, id, 64 * j + 4 * i);
  uint32_t w[64];
  sha_expand_wk(m, w);
  const int nw = (n_seq + 31) / 32;
  uint4 *out = reinterpret_cast<uint4 *>(wk) + ((size_t)j * nw + s / 32) * 16 * 32 + (s & 31);
#pragma unroll
  for (int qd = 0; qd < 16; ++qd)
    out[qd * 32] = make_uint4(w[4 * qd], w[4 * qd + 1], w[4 * qd + 2], w[4 * qd + 3]);
}

// The same expansion for decode step t, without reading the chain state, so
// that it can run while the chain still compresses step t - 1 (which
// rewrites the state at its end).  The carry in front of step t's bytes is
// fully determined: its length is (c0 + t * (4V + 4)) mod 64, c0 being the
// carry length before step 0, and its bytes are the last ones of step t - 1's
// stream (logits || id), since a carry is shorter than a step.  At t = 0 the
// carry comes from the state, and c0 is recorded for the later steps.
__device__ __forceinline__ uint32_t prev_stream_byte(const uint32_t *prev, int V, uint32_t prev_id, int b) {
  const uint32_t d = (b >> 2) < V ? prev[b >> 2] : prev_id;
  return (d >> (8 * (b & 3))) & 0xffu;
}
__global__ void k_sha_prep_at(const ShaState *st, uint32_t *c0, int t, int n_seq, const float *prev_logits,
                              const uint32_t *prev_ids, const float *logits, int V, size_t row_stride,
                              const uint32_t *next_ids, uint32_t *wk, int nb_max) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int s = (int)(idx % n_seq), j = (int)(idx / n_seq);
  if (j >= nb_max) return;
  int c;
  if (t == 0) {
    c = (int)st[s].carry_n;
    if (j == 0) c0[s] = (uint32_t)c;
  } else {
    c = (int)(((uint64_t)c0[s] + (uint64_t)t * (4ull * (uint64_t)V + 4ull)) & 63ull);
  }
  const int total = c + 4 * V + 4;
  if (j >= total / 64) return;
  const uint32_t *data = reinterpret_cast<const uint32_t *>(logits + (size_t)s * row_stride);
  const uint32_t id = next_ids[s];
  uint32_t m[16];
  if (64 * j >= c) {
#pragma unroll
    for (int i = 0; i < 16; ++i) m[i] = step_word(nullptr, c, data, V, id, 64 * j + 4 * i);
  } else {  // block 0 starts with the carry
    uint8_t cb[64];
    if (t == 0) {
      for (int b = 0; b < c; ++b) cb[b] = st[s].carry[b];
    } else {
      const uint32_t *prev = reinterpret_cast<const uint32_t *>(prev_logits + (size_t)s * row_stride);
      const uint32_t pid = prev_ids[s];
      for (int b = 0; b < c; ++b) cb[b] = (uint8_t)prev_stream_byte(prev, V, pid, 4 * V + 4 - c + b);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) m[i] = step_word(cb, c, data, V, id, 64 * j + 4 * i);
  }
  uint32_t w[64];
  sha_expand_wk(m, w);
  const int nw = (n_seq + 31) / 32;
  uint4 *out = reinterpret_cast<uint4 *>(wk) + ((size_t)j * nw + s / 32) * 16 * 32 + (s & 31);
#pragma unroll
  for (int qd = 0; qd < 16; ++qd)
    out[qd * 32] = make_uint4(w[4 * qd], w[4 * qd + 1], w[4 * qd + 2], w[4 * qd + 3]);
}
void launch_sha_prep_at(const ShaState *st, uint32_t *c0, int t, int n_seq, const float *prev_logits,
                        const uint32_t *prev_ids, const float *logits, int V, size_t row_stride,
                        const uint32_t *next_ids, uint32_t *wk_scratch, cudaStream_t s) {
  if (n_seq <= 0) return;
  const int nb_max = (int)((63 + 4 * (size_t)V + 4) / 64);
  const size_t threads = (size_t)nb_max * n_seq;
  k_sha_prep_at<<<(unsigned)((threads + 127) / 128), 128, 0, s>>>(st, c0, t, n_seq, prev_logits, prev_ids, logits,
                                                                  V, row_stride, next_ids, wk_scratch, nb_max);
}

// The chain: one thread per sequence compresses the step's blocks in order,
// keeps the tail as the new carry and emits the per-step digest (a
// finalised copy of the running state).  The expanded W+K words stream
// into shared memory through an ST-deep cp.async pipeline, so the
// compression never waits on L2/HBM latency; each lane copies and reads
// only its own slots, so no warp-level synchronisation is involved.
//
// The chain is issue-bound (11 integer-pipe instructions and 5 multiply-adds
// per round, one warp), so a chain warp must not share its scheduler with
// forward-pass warps: a CTA asks for the whole shared memory of the SM,
// which keeps every other kernel's CTAs off that SM while the witness runs.
// With up to SHA_SOLO_WARPS chain warps, each gets an SM of its own and a
// SHA_SOLO_STAGES-deep ring: measured on B200, two chain warps on one SM
// slow down by a quarter while a vocabulary-wide decode GEMM loads L2 from
// the other SMs, and one warp per SM does not.  Beyond that, SHA_WARPS warps
// (one per SM sub-partition) share an SM with SHA_STAGES stages each.
constexpr int SHA_WARPS = 4;
constexpr int SHA_STAGES = 7;
constexpr int SHA_SOLO_WARPS = 4;
constexpr int SHA_SOLO_STAGES = 28;
constexpr size_t SHA_STAGE_BYTES = (size_t)16 * 32 * sizeof(uint4);          // one block, 32 chains
constexpr size_t SHA_SMEM = (size_t)227 * 1024;                              // SM's maximum per CTA
static_assert(SHA_WARPS * SHA_STAGES * SHA_STAGE_BYTES <= SHA_SMEM, "witness pipeline exceeds smem");
static_assert(SHA_SOLO_STAGES * SHA_STAGE_BYTES <= SHA_SMEM, "witness pipeline exceeds smem");


template <int ST>
__global__ void __launch_bounds__(32 * SHA_WARPS, 1)
k_sha_compress(ShaState *st, int n_seq, const float *logits, int V, size_t row_stride,
               const uint32_t *next_ids, const uint32_t *wk, uint8_t *digest_out, size_t digest_stride,
               uint32_t one) {
  extern __shared__ uint4 smem_all[];  // [warp][ST][16][32 lanes]
  const int lane = threadIdx.x & 31;
  uint4 *stg = smem_all + (size_t)(threadIdx.x >> 5) * ST * 16 * 32;
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n_seq) return;
  ShaState S = st[s];
  const int c = (int)S.carry_n;
  const int total = c + 4 * V + 4;
  const int nb = total / 64;
  // This lane's quad qd of block j is at src + j * bstride + qd * 32 (uint4).
  const int nw = (n_seq + 31) / 32;
  const uint4 *src = reinterpret_cast<const uint4 *>(wk) + (size_t)(s / 32) * 16 * 32 + lane;
  const size_t bstride = (size_t)nw * 16 * 32;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(stg) + (uint32_t)lane * 16;
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = S.h[i];
  // Stage slot k holds quads at sbase + (k*16 + qd) * 512 bytes (lane-interleaved).
  const uint4 *next_src = src;
  int next_j = 0, issue_slot = 0;
  auto issue = [&]() {
    if (next_j < nb) {
      const uint32_t d0 = sbase + (uint32_t)issue_slot * 16 * 512;
#pragma unroll
      for (int qd = 0; qd < 16; ++qd) cp_async16(d0 + (uint32_t)qd * 512, next_src + qd * 32);
    }
    cp_async_commit();  // empty groups keep the per-thread group count uniform
    next_src += bstride;
    ++next_j;
    issue_slot = issue_slot == ST - 1 ? 0 : issue_slot + 1;
  };
#pragma unroll
  for (int j = 0; j < ST - 1; ++j) issue();
  // The first two quads of block j+1 are read during block j, so a block's
  // first rounds never wait for a shared-memory load; the wait below
  // therefore keeps one block fewer in flight (blocks up to j+1 landed).
  int slot = 0;
  cp_async_wait<ST - 2>();
  uint4 qa = stg[lane], qb = stg[32 + lane];
  for (int j = 0; j < nb; ++j) {
    issue();
    cp_async_wait<ST - 2>();
    const uint4 *blk = stg + (size_t)slot * 16 * 32 + lane;
    const int nslot = slot == ST - 1 ? 0 : slot + 1;
    uint32_t w[64];
    w[0] = qa.x; w[1] = qa.y; w[2] = qa.z; w[3] = qa.w;
    w[4] = qb.x; w[5] = qb.y; w[6] = qb.z; w[7] = qb.w;
#pragma unroll
    for (int qd = 2; qd < 16; ++qd) {
      uint4 v = blk[qd * 32];
      w[4 * qd] = v.x; w[4 * qd + 1] = v.y; w[4 * qd + 2] = v.z; w[4 * qd + 3] = v.w;
    }
    const uint4 *nblk = stg + (size_t)nslot * 16 * 32 + lane;  // next block (stale past the last: unused)
    qa = nblk[0];
    qb = nblk[32];
    sha_compress_wk_m(h, w, one);
    slot = nslot;
  }
  cp_async_wait<0>();
  // New carry = stream bytes [64*nb, total).
  const uint32_t *data = reinterpret_cast<const uint32_t *>(logits + (size_t)s * row_stride);
  const uint32_t id = next_ids[s];
  uint8_t nc[64];
  const int cn = total - 64 * nb;
  for (int b = 0; b < cn; ++b) nc[b] = step_byte(S.carry, c, data, V, id, 64 * nb + b);
  for (int b = 0; b < cn; ++b) S.carry[b] = nc[b];
  S.carry_n = (uint32_t)cn;
  S.len += (uint64_t)4 * V + 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) S.h[i] = h[i];
  st[s] = S;
  if (digest_out) {
    uint8_t d[32];
    sha_final_copy(S.h, S.len, S.carry, S.carry_n, d);
    for (int i = 0; i < 32; ++i) digest_out[(size_t)s * digest_stride + i] = d[i];
  }
}

void launch_sha_prep(const ShaState *st, int n_seq, const float *logits, int V, size_t row_stride,
                     const uint32_t *next_ids, uint32_t *wk_scratch, cudaStream_t s) {
  if (n_seq <= 0) return;
  int nb_max = (int)((63 + 4 * (size_t)V + 4) / 64);
  size_t threads = (size_t)nb_max * n_seq;
  k_sha_prep<<<(unsigned)((threads + 127) / 128), 128, 0, s>>>(st, n_seq, logits, V, row_stride,
                                                              next_ids, wk_scratch, nb_max);
}
void launch_sha_compress(ShaState *st, int n_seq, const float *logits, int V, size_t row_stride,
                         const uint32_t *next_ids, const uint32_t *wk_scratch, uint8_t *step_digest_out,
                         size_t digest_stride, cudaStream_t s) {
  if (n_seq <= 0) return;
  static SmemLimit lim_shared, lim_solo;
  lim_shared.ensure(k_sha_compress<SHA_STAGES>, SHA_SMEM);
  lim_solo.ensure(k_sha_compress<SHA_SOLO_STAGES>, SHA_SMEM);
  const int warps = (n_seq + 31) / 32;
  if (warps <= SHA_SOLO_WARPS) {
    k_sha_compress<SHA_SOLO_STAGES><<<warps, 32, SHA_SMEM, s>>>(st, n_seq, logits, V, row_stride, next_ids,
                                                                 wk_scratch, step_digest_out, digest_stride, 1u);
    return;
  }
  const int ctas = (warps + SHA_WARPS - 1) / SHA_WARPS;
  k_sha_compress<SHA_STAGES><<<ctas, 32 * SHA_WARPS, SHA_SMEM, s>>>(st, n_seq, logits, V, row_stride, next_ids,
                                                                    wk_scratch, step_digest_out, digest_stride, 1u);
}
void launch_sha_step(ShaState *st, int n_seq, const float *logits, int V, size_t row_stride,
                     const uint32_t *next_ids, uint32_t *wk_scratch, uint8_t *step_digest_out,
                     size_t digest_stride, cudaStream_t s) {
  launch_sha_prep(st, n_seq, logits, V, row_stride, next_ids, wk_scratch, s);
  launch_sha_compress(st, n_seq, logits, V, row_stride, next_ids, wk_scratch, step_digest_out,
                      digest_stride, s);
}

__global__ void k_sha_finalize(const ShaState *st, int n_seq, uint8_t *out) {
  int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n_seq) return;
  uint8_t d[32];
  sha_final_copy(st[s].h, st[s].len, st[s].carry, st[s].carry_n, d);
  for (int i = 0; i < 32; ++i) out[(size_t)s * 32 + i] = d[i];
}
void launch_sha_finalize(const ShaState *st, int n_seq, uint8_t *out, cudaStream_t s) {
  if (n_seq <= 0) return;
  k_sha_finalize<<<(n_seq + 63) / 64, 64, 0, s>>>(st, n_seq, out);
}

__global__ void k_sha_ids(const uint32_t *prompt_flat, const uint32_t *prompt_off,
                          const uint32_t *prompt_len, const uint32_t *gen_tokens, int gen, int n_seq,
                          uint8_t *out) {
  int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n_seq) return;
  uint32_t h[8];
  sha_init(h);
  uint8_t buf[64];
  uint32_t bn = 0;
  uint64_t len = 0;
  auto put = [&](uint32_t v) {
    for (int b = 0; b < 4; ++b) sha_absorb_byte(h, buf, bn, (uint8_t)(v >> (8 * b)));
    len += 4;
  };
  for (uint32_t i = 0; i < prompt_len[s]; ++i) put(prompt_flat[prompt_off[s] + i]);
  for (int t = 0; t < gen; ++t) put(gen_tokens[(size_t)s * gen + t]);
  uint8_t d[32];
  sha_final_copy(h, len, buf, bn, d);
  for (int i = 0; i < 32; ++i) out[(size_t)s * 32 + i] = d[i];
}
void launch_sha_ids(const uint32_t *prompt_flat, const uint32_t *prompt_off, const uint32_t *prompt_len,
                    const uint32_t *gen_tokens, int gen, int n_seq, uint8_t *out, cudaStream_t s) {
  if (n_seq <= 0) return;
  k_sha_ids<<<(n_seq + 63) / 64, 64, 0, s>>>(prompt_flat, prompt_off, prompt_len, gen_tokens, gen,
                                             n_seq, out);
}

}  // namespace cis2b
