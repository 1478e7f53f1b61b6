/* include/cis2b.h -- C ABI of the B200 (sm_100a) CIS-2 deterministic decoder.
 *
 * Drop-in boundary for the reference's model-load / generate / witness
 * surface.  Plain C types only.  Every function returns CIS2B_OK (0) or an
 * error code and never exits the process; the message of the last failure
 * on the calling thread is available from cis2b_last_error().
 *
 * Reference interfaces each entry point replaces (paths inside
 * Aefinity-AI/cis2-lab-archive):
 *   cis2b_load      cis2_model_load()            code/cis2-fp/verify3/model.h:56
 *                   + the load half of main()    code/cis2-fp/gpu/cis2_host.cpp:87-163
 *                                                (config, artifact sha256, table digest,
 *                                                 inv_freq table, bf16 weights)
 *   cis2b_generate  cis2_run_decode()            code/cis2-fp/verify3/model.h:71-76
 *                   + the decode half of main()  code/cis2-fp/gpu/cis2_host.cpp:165-218
 *                   + run_one_prompt (sampled)   code/patches/cis2-fp__cm_e23-pinned-sampling.patch:581-780
 *                   batched over sequences as in code/patches/cis2-fp__cm_gpu3-batched-full.patch:687-763
 *   cis2b_free      cis2_model_free()            code/cis2-fp/verify3/model.h:57
 *   cis2b_info_get  the printed header lines     code/cis2-fp/gpu/cis2_host.cpp:222-227
 *   cis2b_logits    teacher-forced logits        code/cis2-fp/verify3/model.h:138-158
 *                   (cis2_verify_receipt_prefill's all_logits)
 *
 * Threading: a model handle belongs to one device and must not be used by
 * two threads at once (the reference's verify3 state is global and not
 * thread-safe at all, model.c:49).  Different handles are independent.
 */
#ifndef CIS2B_H
#define CIS2B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CIS2B_OK 0
#define CIS2B_ERR_ARG 1      /* invalid argument or size */
#define CIS2B_ERR_IO 2       /* artifact missing / unreadable / malformed */
#define CIS2B_ERR_CONFIG 3   /* architecture this decoder refuses */
#define CIS2B_ERR_CUDA 4     /* CUDA runtime or kernel failure */
#define CIS2B_ERR_NOMEM 5    /* host or device allocation failed */

#define CIS2B_REDUCTION_SEQUENTIAL 0 /* CIS-2 v0.3b default: strict left-to-right folds */
#define CIS2B_REDUCTION_TREE 1       /* v0.4 candidate: 32-leaf pairwise blocks */

typedef struct cis2b_model cis2b_model;

/* Architecture gate run on config.json before the weights are read.
 * CIS2B_GATE_REFERENCE (0, the default): the Rust reference's gate
 *   (code/cis2-fp/src/main.rs:545-644) key for key and reason for reason:
 *   model_type llama or qwen2, head_dim equal to hidden/heads, ...
 * CIS2B_GATE_QWEN3_PORT (1): the same, but model_type qwen3 is admitted with
 *   its explicit head_dim, as the lab's Qwen3 port of the C++ path decodes it
 *   (labs/w1x-qwen3/scripts/qwen3-port.diff). */
#define CIS2B_GATE_REFERENCE 0
#define CIS2B_GATE_QWEN3_PORT 1

typedef struct {
  int32_t device;        /* CUDA device ordinal */
  int32_t reduction;     /* CIS2B_REDUCTION_* */
  int32_t max_positions; /* prompt + generated positions per sequence; 0 = 4096 */
  int32_t arch_gate;     /* CIS2B_GATE_* */
  int32_t reserved[4];   /* must be zero */
} cis2b_opts;

/* Sampled-mode parameters.  Pass NULL for greedy.
 * scheme CIS2B_SAMPLE_E23 (0): the E23 pinned sampler (SplitMix64 word,
 *   nucleus over the sorted softmax, CDF walk), witness prefix
 *   "CIS2_SAMPLE_V1" before the header; top_k must be 0.
 * scheme CIS2B_SAMPLE_GUMBEL (1): the seeded Gumbel-max clause
 *   "CIS2-SAMPLE-1" (MurmurHash3 noise, top-k then top-p on rank order),
 *   its header absorbed after the prompt ids. */
#define CIS2B_SAMPLE_E23 0
#define CIS2B_SAMPLE_GUMBEL 1
typedef struct {
  uint64_t seed;
  float temperature; /* > 0, finite */
  float top_p;       /* (0, 1]; 1 = disabled */
  uint32_t scheme;   /* CIS2B_SAMPLE_* */
  uint32_t top_k;    /* CIS2B_SAMPLE_GUMBEL only; 0 (or >= vocab) = disabled */
} cis2b_sample;

typedef struct {
  int32_t hidden, intermediate, n_layers, n_heads, n_kv_heads, head_dim, vocab, tied;
  float rms_norm_eps;  /* narrowed once from the f64 config value */
  double rope_theta;
  int32_t reduction;
  int32_t max_positions;
  uint8_t weights_sha256[32];
  uint8_t tokenizer_sha256[32];
  uint8_t config_sha256[32];
  uint8_t table_digest[32];
  uint8_t inv_freq_table_digest[32];
} cis2b_info;

/* Device-side timing of the last cis2b_generate (CUDA events). */
typedef struct {
  double total_ms;    /* first kernel to last witness kernel */
  double prefill_ms;  /* prompt positions through the model */
  double decode_ms;   /* token steps (forward + selection), main stream */
  double witness_tail_ms; /* witness work left after the last decode step */
  int64_t kernel_launches; /* kernels this library launched for the call */
  int64_t h2d_bytes;       /* host -> device bytes copied by the call */
  int64_t d2h_bytes;       /* device -> host bytes copied by the call */
} cis2b_timing;

/* Per-kernel-class CUDA-event timing (for roofline measurement).  Classes: */
#define CIS2B_PROF_LM_HEAD 1u     /* lm_head GEMM (final norm output x vocab) */
#define CIS2B_PROF_LAYER_GEMM 2u  /* q/k/v, o, gate/up and down GEMMs */
#define CIS2B_PROF_ATTENTION 4u   /* scores + softmax + V-mix kernel */
#define CIS2B_PROF_WITNESS 8u     /* witness SHA-256 compression chain */
typedef struct {
  int64_t launches;
  double total_ms;  /* sum of per-launch event durations on the launching stream */
} cis2b_kernel_time;

/* Loads weights_dir/{model.safetensors,config.json,tokenizer.json}: hashes
 * the three artifacts, parses the config (numbers as f64, eps narrowed once),
 * uploads the bf16 weights to the device and builds the pinned inv_freq and
 * RoPE tables there. */
int cis2b_load(const char *weights_dir, const cis2b_opts *opts, cis2b_model **out);

int cis2b_info_get(const cis2b_model *m, cis2b_info *out);

/* Decodes n_seq independent sequences in one batch.
 *   prompt_ids   concatenated prompts (u32 token ids), prompt_lens[n_seq] >= 1
 *   gen_toks     tokens to generate per sequence (>= 0)
 *   sample       NULL = greedy argmax (first maximum wins); else the E23
 *                sampler with position = prompt_len + step
 * Outputs (caller-owned host buffers, any may be NULL except out_witness):
 *   out_tokens        [n_seq][gen_toks]
 *   out_step_digests  [n_seq][gen_toks][32]  witness state finalised after each step
 *   out_witness       [n_seq][32]  final witness digest (CIS2_REF / CIS2_SAMPLE digest)
 *   out_argmax        [n_seq][32]  SHA-256 over prompt ids then generated ids
 * Each sequence's outputs equal its own batch-1 run. */
int cis2b_generate(cis2b_model *m, const uint32_t *prompt_ids, const uint32_t *prompt_lens,
                   uint32_t n_seq, uint32_t gen_toks, const cis2b_sample *sample,
                   uint32_t *out_tokens, uint8_t *out_step_digests, uint8_t *out_witness,
                   uint8_t *out_argmax);

int cis2b_last_timing(const cis2b_model *m, cis2b_timing *out);

/* Times every launch of the classes in `class_mask` (CIS2B_PROF_*) with a
 * CUDA event pair in later cis2b_generate calls; 0 turns it off. */
int cis2b_profile(cis2b_model *m, uint32_t class_mask);
/* Totals of the last cis2b_generate for ONE class bit. */
int cis2b_profile_read(const cis2b_model *m, uint32_t class_bit, cis2b_kernel_time *out);

/* Receipt verification, teacher-forced (replaces cis2_verify_receipt_prefill,
 * code/cis2-fp/verify3/model.h:151-157, and the claim check of
 * verify3/main.c:230-265, batched over sequences).  For each sequence ONE
 * forward pass over prompt + claimed[0 .. gen-2] gives the logits of every
 * claimed step; the token of each step is RECOMPUTED from them (argmax, or
 * the sampler in `sample`) and the witness is rebuilt exactly as
 * cis2b_generate builds it.  An honest claim therefore reproduces the
 * generation's tokens and digests.
 *   claimed           [n_seq][gen]  the receipt's generated ids
 *   out_tokens        [n_seq][gen]  recomputed ids (may be NULL)
 *   out_first_mismatch [n_seq]      first step whose recomputed id differs
 *                                   from the claim, -1 if none (may be NULL)
 *   out_step_digests, out_witness, out_argmax as cis2b_generate. */
int cis2b_verify(cis2b_model *m, const uint32_t *prompt_ids, const uint32_t *prompt_lens, uint32_t n_seq,
                 const uint32_t *claimed, uint32_t gen_toks, const cis2b_sample *sample, uint32_t *out_tokens,
                 int32_t *out_first_mismatch, uint8_t *out_step_digests, uint8_t *out_witness,
                 uint8_t *out_argmax);

/* Teacher-forced logits of ONE sequence: runs ids[0 .. n_prompt+n_rows-2]
 * and writes the fp32 logits after positions n_prompt-1 .. n_prompt+n_rows-2
 * into out_logits[n_rows][vocab]. */
int cis2b_logits(cis2b_model *m, const uint32_t *ids, uint32_t n_prompt, uint32_t n_rows,
                 float *out_logits);

/* Per-op trace, for localising a parity failure (debug only; the
 * reference CLI's --trace F, code/cis2-fp/gpu/cis2_host.cpp:76, 173-193, and
 * its emit points, gpu/cis2_model.h:482-496, 685-760).  Runs ids[0 .. n_ids)
 * as ONE sequence, position by position, and writes one line per op output
 *   pos=P layer=L op=NAME sha256=HEX
 * (SHA-256 over the output's fp32 bits, u32 LE) in the reference's op order:
 * embedding; per layer norm1 q k v [q_norm k_norm] rope_q rope_k scores
 * softmax attn_out o_proj resid1 norm2 gate up silu_mul down resid2; then
 * final_norm and logits.  To trace a generation of G tokens as the
 * reference does, pass the prompt followed by the G generated ids. */
int cis2b_trace(cis2b_model *m, const uint32_t *ids, uint32_t n_ids, const char *trace_path);

void cis2b_free(cis2b_model *m);

/* Message of the last failed call on this thread ("" if none). */
const char *cis2b_last_error(void);

/* ---- kernel-level entry points (host buffers in and out) ---------------
 * Used by the parity tests to check single kernels against the CPU oracle. */

/* y[i] = f(x[i]); f: 0 exp, 1 sin, 2 cos, 3 ln, 4 silu, 5 rsqrt (spec §6). */
int cis2b_op_pinned_map(int32_t device, int32_t fn, const float *x, float *y, size_t n);
/* Y[r][o] = dot(W[o,:], X[r,:]) in the pinned order; W bf16 [n_out][k], k % 8 == 0.
 * reduction: CIS2B_REDUCTION_SEQUENTIAL or _TREE through the panel kernel the
 * prompt pass uses, or CIS2B_OP_MATMUL_DECODE / _DECODE_TREE: sequential or
 * tree order through the few-row kernel decode steps use (rows <= 1024; tree
 * order: k % 32 == 0). */
#define CIS2B_OP_MATMUL_DECODE 2
#define CIS2B_OP_MATMUL_DECODE_TREE 3
int cis2b_op_matmul(int32_t device, const uint16_t *W, const float *X, int32_t rows, int32_t n_out,
                    int32_t k, int32_t reduction, float *Y);
/* Index (0-based) of the register tile the many-row product picks for
 * rows x n_out (sequential order, rows >= 64), or -1; lets the parity tests
 * confirm that their shapes reach every tile of that kernel. */
int cis2b_op_gemm_tile(int32_t rows, int32_t n_out);
/* Witness stream check: absorbs `prefix` (byte path), then n_chunks chunks of
 * chunk_words u32 words through the device step path (last word of each
 * chunk plays the token id); writes the digest after each chunk. */
int cis2b_op_sha256_stream(int32_t device, const uint8_t *prefix, size_t prefix_len,
                           const uint32_t *words, uint32_t chunk_words, uint32_t n_chunks,
                           uint8_t *out_digests);
/* Greedy token selection on `rows` logits rows of n values each, through
 * the kernel the decode steps use: the first index of the strict maximum
 * (code/cis2-fp/src/main.rs:1161-1169; gpu/cis2_model.h:764-774), so an
 * exact tie -- +0 against -0 included -- keeps the lower index, a NaN at
 * index 0 selects 0 and a NaN elsewhere is never selected. */
int cis2b_op_argmax(int32_t device, const float *logits, int32_t rows, int32_t n, uint32_t *out_index);
/* E23 sampler on one logits row; position < 2^31. */
int cis2b_op_sample(int32_t device, const float *logits, int32_t n, float temperature, float top_p,
                    uint64_t seed, uint64_t position, uint32_t *out_index);
/* Seeded Gumbel-max ("CIS2-SAMPLE-1") draw on one logits row; step is the
 * 0-based generation step. */
int cis2b_op_sample_gumbel(int32_t device, const float *logits, int32_t n, float temperature, uint32_t top_k,
                           float top_p, uint64_t seed, uint32_t step, uint32_t *out_index);

/* No counterpart in the reference.  The E23 sampler on one logits row that
 * ALLOCATES NOTHING: for callers that cannot call cudaMalloc -- code whose
 * device memory is owned by its own allocator (a framework's caching pool,
 * a pre-reserved arena) that must not be bypassed, or code on a
 * latency-critical path where cudaMalloc/cudaFree would synchronise the
 * device.  The caller passes device pointers for the input row and the
 * output index; the sampler's working memory is a fixed array inside the
 * library (5 floats per logit for CIS2B_STATIC_SAMPLE_MAX logits, about
 * 5 MiB) that every GPU which loads the library keeps until the process
 * exits.
 *   d_logits     device pointer to n fp32 logits, 1 <= n <= CIS2B_STATIC_SAMPLE_MAX
 *   d_out_index  device pointer to one uint32, written with the drawn index
 *   stream       cudaStream_t to run on (NULL: the legacy default stream)
 *   position     < 2^31
 * Makes `device` current on the calling thread.  The first call on a device
 * looks up the array's device address and keeps it; make that first call
 * before any stream capture.  A device reset that destroys the primary
 * context (cudaDeviceReset) makes the kept address stale: do not call this
 * entry point again in that process afterwards.  The call is asynchronous:
 * the index is valid once `stream` has reached it.  All calls on one device
 * in one process share the one array, whichever model handle or thread
 * makes them, and it keeps the last call's contents (every element the
 * sampler reads it writes first), so calls whose work overlaps on the GPU --
 * two streams, or two threads -- race and must be ordered by the caller.
 * Only this entry point uses the array: it never races with cis2b_generate,
 * cis2b_verify or the other entry points, and separate processes each have
 * their own copy.  Sizes above the maximum are rejected with CIS2B_ERR_ARG.
 * Same result as cis2b_op_sample. */
#define CIS2B_STATIC_SAMPLE_MAX 262144
int cis2b_op_sample_static(int32_t device, const float *d_logits, int32_t n, float temperature, float top_p,
                           uint64_t seed, uint64_t position, uint32_t *d_out_index, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* CIS2B_H */
