// cis2b_kernels.h -- host-side launchers for the sm_100a kernels of the
// CIS-2 decode path (implemented in cis2b_kernels.cu).  Internal interface
// between the runtime (cis2b_runtime.cu) and the kernels; not exported.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace cis2b {

struct ShaState;  // cis2b_sha256.cuh

// Where one activation row of a batch lives: sequence index and position.
struct RowMap {
  const int32_t *seq;  // [rows]
  const int32_t *pos;  // [rows]
};

// Pinned RoPE / inv_freq tables (built once per model).
void launch_inv_freq(float rope_theta_f32, int head_dim, float *inv_freq, cudaStream_t s);
void launch_rope_table(const float *inv_freq, int half, int max_pos, float *cos_t, float *sin_t,
                       cudaStream_t s);

void launch_embed(const uint16_t *E, int H, const uint32_t *tokens, int rows, float *h,
                  cudaStream_t s);
// out[r * ors + i * ocs]: (ors, ocs) = (n, 1) row-major or (1, ldm) k-major.
void launch_rmsnorm(const float *x, int ldx, const uint16_t *w, float eps, int n, int rows, bool tree,
                    float *out, int ors, int ocs, cudaStream_t s);

// Y[m][n] (+)= sum_k W[n][k] X[m][k] in the pinned order.  XT is X k-major
// [K][ldm] (ldm % 4 == 0, ldm >= M); Wp holds W bf16 in 8-row k-major
// panels and Wpf the same panels widened to fp32 (launch_panelize): the
// many-row form (M >= 64; tree order: K % 32 == 0) reads Wpf, the others Wp.  If
// resid != nullptr, Y = resid + dot.  If y_slot != nullptr, Y is offset by
// (*y_slot) * y_slot_stride floats.
void launch_gemm(const float *XT, int ldm, const uint16_t *Wp, const float *Wpf, int K, int N, int M, float *Y,
                 int ldy, const float *resid, int ldr, bool tree, const int32_t *y_slot, size_t y_slot_stride,
                 cudaStream_t s);
// The many-row form behind launch_gemm (M >= 64, sequential order or, when
// gemm_big_ok(K, true), tree order): Y[m * ysm + n * ysn], so the output may
// be written k-major for the next product.  glu: Wpf is a gate/up pair
// panelised with il_half = I (N = 2I); the output is silu(gate) * up, I columns.
void launch_gemm_big(const float *XT, int ldm, const float *Wpf, int K, int N, int M, float *Y, int ysm, int ysn,
                     const float *resid, int ldr, const int32_t *y_slot, size_t y_slot_stride, int glu,
                     cudaStream_t s, bool tree = false);
bool gemm_big_ok(int K, bool tree);
int gemm_big_choice(int M, int N, bool tree = false);
// Wp[n8][k][j] = W[8*n8 + j][k], zero rows past N; Wp holds panel_elems(N, K)
// elements, bf16 bits or (float overload) those widened to fp32.
// il_half = I > 0 (N = 2I): rows interleaved, panel row 2i = W row i (gate),
// 2i + 1 = W row I + i (up).
void launch_panelize(const uint16_t *W, int N, int K, uint16_t *Wp, cudaStream_t s, int il_half = 0);
void launch_panelize(const uint16_t *W, int N, int K, float *Wp, cudaStream_t s, int il_half = 0);
size_t panel_elems(int N, int K);

// Decode form of the same product for few rows, in sequential order or (tree)
// the v0.4 tree order.  X is row-major [M][ldx] (ldx % 4 == 0); Wt holds W
// bf16 in 32-column tiles (launch_tile32).  resid / y_slot as launch_gemm.
// Usable when gemm_dec_ok(K, tree).
// glu = I > 0: W is a gate/up pair tiled with launch_tile32(..., glu_half = I)
// and Y receives silu(gate) * up, [M][ldy] with I columns (N = 2I).
void launch_gemm_dec(const float *X, int ldx, const uint16_t *Wt, int K, int N, int M, float *Y, int ldy,
                     const float *resid, int ldr, const int32_t *y_slot, size_t y_slot_stride,
                     cudaStream_t s, int glu = 0, bool tree = false);
// Wt[n32][kq][j][q] = W[32*n32 + j][4*kq + q], zero columns past N; K % 4 == 0.
// glu_half = I (N = 2I, I % 16 == 0): tile n32 holds gate rows 16*n32 + j in
// columns j < 16 and up rows I + 16*n32 + j - 16 in columns j >= 16.
void launch_tile32(const uint16_t *W, int N, int K, uint16_t *Wt, cudaStream_t s, int glu_half = 0);
__host__ __device__ size_t tile32_elems(int N, int K);
bool gemm_dec_ok(int K, bool tree = false);
// Index into the decode tile list for (M, N, K): 0 (8x4) .. 3 (2x2).
int gemm_dec_choice(int M, int N, int K);

// q/k norm (optional), RoPE of q and k, and the KV-cache append.
// qkv rows: [q (n_heads*hd) | k (n_kv*hd) | v (n_kv*hd)].  Caches are laid
// out [seq][max_pos][kv_dim] for ONE layer (the caller offsets by layer).
void launch_qkv_post(float *qkv, int ld, int rows, RowMap rm, int n_heads, int n_kv, int hd,
                     const uint16_t *q_norm, const uint16_t *k_norm, float eps, bool tree,
                     const float *cos_t, const float *sin_t, float *kcache, float *vcache,
                     int max_pos, cudaStream_t s);
// fuse_post: also do launch_qkv_post's work for the row (decode only: every
// row must be a different sequence's newest position).  dbg (trace mode,
// rows == 1 only): receives the scaled scores [n_heads][pos+1] and then the
// softmax weights [n_heads][pos+1].
void launch_attention(float *qkv, int ld, int rows, RowMap rm, int n_heads, int n_kv, int hd,
                      float *kcache, float *vcache, int max_pos, bool tree, float *att,
                      int ars, int acs, int max_len, bool fuse_post, const uint16_t *q_norm,
                      const uint16_t *k_norm, float eps, const float *cos_t, const float *sin_t,
                      cudaStream_t s, float *dbg = nullptr);
// Trace mode: per-head q/k RMSNorm of one qkv row, in place.
void launch_qk_norm_row(float *row, int n_heads, int n_kv, int hd, const uint16_t *q_norm, const uint16_t *k_norm,
                        float eps, bool tree, cudaStream_t s);
// Shared memory (floats) the attention kernel needs; G = n_heads / n_kv.
size_t attention_smem_floats(int G, int hd, int max_len);
// Prompt-pass attention over tiles of consecutive rows of one sequence
// (consecutive positions): tiles[t] = (first row, rows <= rt).  Each K/V
// chunk is staged once per tile instead of once per row.  rt from
// attention_rows_rt (scores of rt rows fit the shared-memory budget);
// max_len >= the largest position + 1 of the pass; hd <= 256.
int attention_rows_rt(int G, int hd, int max_len);
size_t attention_rows_smem_floats(int rt, int G, int hd, int max_len);
void launch_attention_rows(const float *qkv, int ld, const int2 *tiles, int n_tiles, int rt, RowMap rm, int n_heads,
                           int n_kv, int hd, const float *kcache, const float *vcache, int max_pos, bool tree,
                           float *att, int ars, int acs, int max_len, cudaStream_t s);
// Index of the GEMM tile the dispatcher picks for (M, N, K).
int gemm_tile_choice(int M, int N, int K, bool tree);
// gu rows [rows][2I] with gate i at 2i and up i at 2i + 1 (interleaved panels).
void launch_silu_mul(const float *gu, int I, int rows, float *hid, int hrs, int hcs, cudaStream_t s);
void launch_add_bias(float *x, int ld, int rows, const uint16_t *b, int n, cudaStream_t s);

// Token selection.  logits rows at logits + slot*slot_stride (slot from device).
void launch_argmax(const float *logits, int V, int rows, const int32_t *slot, size_t slot_stride,
                   uint32_t *next, cudaStream_t s);
void launch_sample(const float *logits, int V, int rows, const int32_t *slot, size_t slot_stride,
                   float temperature, float top_p, uint64_t seed, const int32_t *position,
                   float *scratch, uint32_t *next, cudaStream_t s);
// Seeded Gumbel-max sampler ("CIS2-SAMPLE-1"); step = 0-based generation step (device).
void launch_sample_gumbel(const float *logits, int V, int rows, const int32_t *slot, size_t slot_stride,
                          float temperature, uint32_t top_k, float top_p, uint64_t seed, const int32_t *step,
                          float *scratch, uint32_t *next, cudaStream_t s);
// Record the chosen ids (tokens_out[r][step], ids_hist[step][r]), advance positions, ring slot, step.
void launch_step_advance(const uint32_t *next, int rows, const int32_t *step, int gen,
                         uint32_t *tokens_out, uint32_t *ids_hist, int32_t *pos, int32_t *sample_pos,
                         int32_t *slot, int ring, int32_t *step_ctr, cudaStream_t s);
// dst[dst_idx[r]][:H] = src[src_idx[r]][:H], r < n
void launch_gather_rows(const float *src, int ld, const int32_t *src_idx, const int32_t *dst_idx,
                        int n, int H, float *dst, cudaStream_t s);

// Witness.
void launch_sha_absorb_bytes(ShaState *st, const uint8_t *bytes, const uint32_t *offsets, int n_seq,
                             cudaStream_t s);
size_t sha_wk_words(int V, int n_seq);
void launch_sha_step(ShaState *st, int n_seq, const float *logits, int V, size_t row_stride,
                     const uint32_t *next_ids, uint32_t *wk_scratch, uint8_t *step_digest_out,
                     size_t digest_stride, cudaStream_t s);
// The two halves of launch_sha_step: W+K expansion (many threads), then the
// per-sequence compression chain.
void launch_sha_prep(const ShaState *st, int n_seq, const float *logits, int V, size_t row_stride,
                     const uint32_t *next_ids, uint32_t *wk_scratch, cudaStream_t s);
// launch_sha_prep for decode step t that does not read the chain state, so
// it may overlap the chain's step t - 1: prev_logits / prev_ids are step
// t - 1's (unused at t = 0); c0[n_seq] is written at t = 0 and read after.
void launch_sha_prep_at(const ShaState *st, uint32_t *c0, int t, int n_seq, const float *prev_logits,
                        const uint32_t *prev_ids, const float *logits, int V, size_t row_stride,
                        const uint32_t *next_ids, uint32_t *wk_scratch, cudaStream_t s);
void launch_sha_compress(ShaState *st, int n_seq, const float *logits, int V, size_t row_stride,
                         const uint32_t *next_ids, const uint32_t *wk_scratch, uint8_t *step_digest_out,
                         size_t digest_stride, cudaStream_t s);
void launch_sha_finalize(const ShaState *st, int n_seq, uint8_t *out, cudaStream_t s);
// Argmax digest: SHA-256 over prompt ids then generated ids (u32 LE).
void launch_sha_ids(const uint32_t *prompt_flat, const uint32_t *prompt_off, const uint32_t *prompt_len,
                    const uint32_t *gen_tokens, int gen, int n_seq, uint8_t *out, cudaStream_t s);

// Records `msg` as this thread's cis2b_last_error() and returns `code`.
int set_last_error(int code, const char *msg);

// Element-wise pinned function map (test entry point).
void launch_pinned_map(int fn, const float *x, float *y, size_t n, cudaStream_t s);

}  // namespace cis2b
