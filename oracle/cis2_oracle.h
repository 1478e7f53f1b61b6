/* oracle/cis2_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C11 CPU restatement of the CIS-2 deterministic decode path, used
 * as the parity checker for the CUDA build and as the "port" CPU baseline.
 * Nothing in the product links against this.  Every function cites the
 * reference location it restates (paths inside Aefinity-AI/cis2-lab-archive).
 *
 * Parity pins: the restatement is checked against (1) the reference's own
 * C++ port compiled from its sources (oracle/_ref, built by oracle/Makefile)
 * on every synthetic configuration, (2) the weight-independent golden
 * vectors of the spec (table digest, inv_freq digest, dot_seq order case,
 * bf16 widen bits, SHA-256 KATs) -- see tests/test_oracle.py.
 */
#ifndef CIS2_ORACLE_H
#define CIS2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-layer tensor slots, in this order, for cis2o_model_new(). */
enum {
  CIS2O_IN_NORM = 0, CIS2O_POST_NORM, CIS2O_Q, CIS2O_K, CIS2O_V, CIS2O_O,
  CIS2O_GATE, CIS2O_UP, CIS2O_DOWN, CIS2O_Q_NORM, CIS2O_K_NORM,
  CIS2O_Q_BIAS, CIS2O_K_BIAS, CIS2O_V_BIAS, CIS2O_LAYER_SLOTS
};

typedef struct {
  int32_t hidden, inter, n_layers, n_heads, n_kv_heads, head_dim, vocab;
  float eps;          /* already narrowed once from the f64 config value */
  double rope_theta;  /* f64 as parsed; narrowed to f32 inside ln_pinned's arg */
  int32_t tied;       /* 1: lm_head is embed_tokens */
  int32_t tree;       /* 0 sequential (v0.3b default), 1 v0.4 tree candidate */
} cis2o_config;

typedef struct {
  int32_t enabled;    /* 0: greedy argmax; 1: E23 pinned sampler; 2: seeded Gumbel-max "CIS2-SAMPLE-1" */
  uint64_t seed;
  float temperature;
  float top_p;
  uint32_t top_k;     /* scheme 2 only; 0 = disabled */
} cis2o_sample;

/* tensors: embed, final_norm, lm_head (NULL if tied), then n_layers *
 * CIS2O_LAYER_SLOTS bf16 pointers (NULL for absent optional tensors).
 * The pointers are borrowed and must outlive the model. */
void *cis2o_model_new(const cis2o_config *cfg, const uint16_t *embed,
                      const uint16_t *final_norm, const uint16_t *lm_head,
                      const uint16_t *const *layer_tensors);
void cis2o_model_free(void *model);

/* Digests folded into the witness header (spec §12.1 items 4 and 5). */
void cis2o_table_digest(uint8_t out[32]);
void cis2o_inv_freq(const void *model, float *out_half, uint8_t out_digest[32]);

/* Greedy or sampled decode of n_seq independent sequences.
 * prompt_ids: concatenated prompts; prompt_lens[n_seq].
 * hdr: weights_sha256 || tokenizer_sha256 || config_sha256 (96 raw bytes).
 * out_tokens [n_seq][gen], out_step_digests [n_seq][gen][32] (may be NULL),
 * out_witness [n_seq][32], out_argmax [n_seq][32].
 * trace_path: if non-NULL, per-(pos, layer, op) SHA-256 lines in the
 * reference's --trace format (sequence 0 only).  Returns 0 on success. */
int cis2o_generate(const void *model, const uint32_t *prompt_ids, const uint32_t *prompt_lens,
                   uint32_t n_seq, uint32_t gen, const cis2o_sample *sample,
                   const uint8_t hdr[96], uint32_t *out_tokens, uint8_t *out_step_digests,
                   uint8_t *out_witness, uint8_t *out_argmax, const char *trace_path);

/* Teacher-forced logits: runs prompt+claimed tokens of ONE sequence and
 * writes the fp32 logits of positions [n_prompt-1, n_prompt-1+n_claim) into
 * out_logits [n_claim+... rows][vocab] (row i = logits after position
 * n_prompt-1+i).  Used by op-level parity tests. */
int cis2o_logits(const void *model, const uint32_t *ids, uint32_t n_prompt, uint32_t n_rows,
                 float *out_logits);

/* Pinned scalar math (spec §6) and reductions (spec §5, v0.4 tree). */
float cis2o_exp(float x);
float cis2o_sin(float x);
float cis2o_cos(float x);
float cis2o_ln(float x);
float cis2o_silu(float x);
float cis2o_rsqrt(float x);
float cis2o_dot(const float *a, const float *b, int32_t n, int32_t tree);
float cis2o_sum(const float *a, int32_t n, int32_t tree);
/* y[r][o] = dot(W[o,:], X[r,:]) with W bf16 [n_out][k], X fp32 [rows][k]. */
void cis2o_matmul_bf16(const uint16_t *W, const float *X, int32_t rows, int32_t n_out, int32_t k,
                       int32_t tree, float *Y);
void cis2o_softmax(float *v, int32_t n, int32_t tree);
uint32_t cis2o_argmax(const float *v, int32_t n);
uint32_t cis2o_sample_pinned(const float *logits, int32_t n, float temperature, float top_p,
                             uint64_t seed, uint64_t position);
uint64_t cis2o_rng_word(uint64_t seed, uint64_t position);
/* Seeded Gumbel-max sampling ("CIS2-SAMPLE-1"): MurmurHash3_x86_32 over a
 * byte key, the noise of one (seed, step, index), and one draw. */
uint32_t cis2o_murmur3_32(const uint8_t *key, size_t len, uint32_t seed);
void cis2o_gumbel_noise(uint64_t seed, uint32_t step, uint32_t index, uint32_t *hash, float *u, float *g);
uint32_t cis2o_sample_gumbel(const float *logits, int32_t n, float temperature, uint32_t top_k, float top_p,
                             uint64_t seed, uint32_t step, float *z_out);
void cis2o_sha256(const uint8_t *data, size_t n, uint8_t out[32]);
/* The 242,428 points of the pinned-function sweep (math_sweep.h); out may be NULL. */
size_t cis2o_math_sweep(float *out);
/* Evaluate one pinned function over an array (f: 0 exp,1 sin,2 cos,3 ln,4 silu,5 rsqrt). */
void cis2o_map(int32_t f, const float *x, float *y, size_t n);

#ifdef __cplusplus
}
#endif
#endif
