// cis2b_runtime.cu -- host runtime behind the C ABI (include/cis2b.h).
//
// Load: artifact hashes, config (code/cis2-fp/gpu/cis2_host.cpp:87-117 and
// qwen3-port.diff:109-110), bf16 weights uploaded as-is into one device
// arena (the exact widen happens inside the kernels), pinned inv_freq and
// RoPE tables built on the device.
//
// Generate: all sequences of a call run as one batch.  Prompt positions go
// through the model position-batched (each row's arithmetic is identical to
// a per-token run, code/cis2-fp/verify3/model.h:128-139); then one decode
// step per token: select (argmax or E23 sampler) -> witness absorb on a
// second, high-priority stream -> forward of the chosen tokens.  The
// witness of step t only needs step t's logits, so it lags the forward and
// overlaps it; logits live in a ring sized to the step count where memory
// allows, otherwise the forward waits for the witness to free a slot.
#include "../../include/cis2b.h"
#include "cis2b_host.h"
#include "cis2b_kernels.h"
#include "cis2b_pinned.cuh"
#include "cis2b_sha256.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <string>
#include <vector>

using namespace cis2b;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string &msg) {
  g_err = msg;
  return code;
}

}  // namespace

// Lets entry points defined next to their kernels report through
// cis2b_last_error() like every other call.
int cis2b::set_last_error(int code, const char *msg) { return fail(code, msg); }

namespace {

#define CU(x)                                                                               \
  do {                                                                                      \
    cudaError_t e_ = (x);                                                                   \
    if (e_ != cudaSuccess)                                                                  \
      return fail(CIS2B_ERR_CUDA, std::string(#x) + " -> " + cudaGetErrorString(e_));        \
  } while (0)

// Kernel launches report errors asynchronously; check after each batch.
#define CU_LAUNCHED()                                                                       \
  do {                                                                                      \
    cudaError_t e_ = cudaGetLastError();                                                    \
    if (e_ != cudaSuccess)                                                                  \
      return fail(CIS2B_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e_)); \
  } while (0)

struct DevBuf {
  void *p = nullptr;
  size_t bytes = 0;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  cudaError_t ensure(size_t want) {
    if (want <= bytes && p) return cudaSuccess;
    release();
    cudaError_t e = cudaMalloc(&p, want ? want : 16);
    if (e == cudaSuccess) bytes = want;
    return e;
  }
  template <class T> T *as() const { return reinterpret_cast<T *>(p); }
};

struct LayerW {
  const uint16_t *in_norm, *post_norm, *wqkv, *wo, *wgu, *wdown;  // row-major [N][K] as on disk
  const uint16_t *q_norm, *k_norm, *q_bias, *k_bias, *v_bias;
  const uint16_t *pqkv, *po, *pgu, *pdown;  // the same weights in GEMM panel layout
  const float *fqkv = nullptr, *fo = nullptr, *fgu = nullptr, *fdown = nullptr;  // ... widened to fp32
  const uint16_t *tqkv, *to, *tgu, *tdown;  // and in 32-column decode tiles (sequential mode)
};

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

constexpr int PREFILL_CHUNK = 8192;            // rows per prefill pass
// lm_head rows up to which the decode GEMM is used; from 64 rows on the
// prompt-pass GEMM's 64 x 64 tile is faster (B200: 156 vs 178 us at 64 x
// 49,152 x 576, 557 vs 985 us at 300 x 32,000 x 768; 737 vs 629 us for the
// decode GEMM at 32 x 151,936 x 1,024).
constexpr int DEC_HEAD_ROWS = 48;
// Decode-step rows from which the layer products leave the few-row kernel
// for the register-tiled one (k-major activations).
constexpr int DEC_BIG_ROWS = 128;
constexpr size_t RING_BUDGET = 8ull << 30;     // bytes of logits kept for the witness

}  // namespace

struct cis2b_model {
  int dev = 0;
  cis2b_info info{};
  bool tree = false;
  int H = 0, I = 0, L = 0, NH = 0, NKV = 0, HD = 0, V = 0, QD = 0, KVD = 0, max_pos = 0;
  float eps = 0.f;
  std::vector<LayerW> layers;
  const uint16_t *embed = nullptr, *final_norm = nullptr, *lm_head = nullptr;
  DevBuf arena;   // all weights as on disk (embedding rows, norms, biases are read from here)
  DevBuf panels;  // GEMM weights re-laid in 8-row k-major panels
  const uint16_t *lm_head_p = nullptr;
  // The same panels widened to fp32 for the many-row product: it then
  // spends no issue slots on widening, and HBM has room.
  DevBuf panels_f;
  const float *lm_head_f = nullptr;
  DevBuf tiles;   // the same weights in 32-column tiles for the decode GEMM
  const uint16_t *lm_head_t = nullptr;
  bool dec_tiles = false;  // decode steps use launch_gemm_dec (K % 4 == 0; tree mode K % 32 == 0)
  int dec_big_rows = DEC_BIG_ROWS;  // ... below this many rows (above: the register-tiled product)
  DevBuf inv_freq, cos_t, sin_t;
  cudaStream_t s_main = nullptr, s_sha = nullptr, s_prep = nullptr;
  // workspace
  DevBuf h, ln, qkv, att, gu, hid, hlast, lnlast, kc, vc, ring, scratch;
  int act_ldm = 0;  // column count of the k-major activation buffers
  DevBuf rows_seq, rows_pos, rows_tok, gsrc, gdst, att_tiles;
  DevBuf d_next, d_pos, d_spos, d_seq, d_ctl, d_tokens, d_ids_hist;
  DevBuf sha_state, sha_wk, sha_c0, step_dig, d_witness, d_argmax;
  DevBuf hdr_bytes, hdr_off, p_flat, p_off, p_len;
  std::vector<cudaEvent_t> ev_sha;
  cudaEvent_t ev_sel = nullptr, ev0 = nullptr, ev_pref = nullptr, ev_dec = nullptr, ev_end = nullptr;
  cudaEvent_t ev_prep[2] = {nullptr, nullptr}, ev_comp[2] = {nullptr, nullptr};  // witness expansion halves
  cis2b_timing timing{};
  int64_t launches = 0, h2d = 0, d2h = 0;
  // per-launch event timing of selected kernel classes (cis2b_profile)
  struct ProfEvent { uint32_t cls; cudaEvent_t a, b; };
  uint32_t prof_mask = 0;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<ProfEvent> prof_events;
  cis2b_kernel_time prof[4]{};
};

namespace {

cudaEvent_t pool_event(cis2b_model *m) {
  if (m->ev_used == m->ev_pool.size()) {
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    m->ev_pool.push_back(e);
  }
  return m->ev_pool[m->ev_used++];
}

// Brackets the launches made in its scope with an event pair on stream `s`
// when the class is selected for profiling.
struct ProfScope {
  cis2b_model *m;
  uint32_t cls;
  cudaStream_t s;
  cudaEvent_t a = nullptr;
  ProfScope(cis2b_model *m_, uint32_t cls_, cudaStream_t s_) : m(m_), cls(cls_), s(s_) {
    if (m->prof_mask & cls) {
      a = pool_event(m);
      cudaEventRecord(a, s);
    }
  }
  ~ProfScope() {
    if (!a) return;
    cudaEvent_t b = pool_event(m);
    cudaEventRecord(b, s);
    m->prof_events.push_back({cls, a, b});
  }
};

int class_index(uint32_t bit) {
  switch (bit) {
    case CIS2B_PROF_LM_HEAD: return 0;
    case CIS2B_PROF_LAYER_GEMM: return 1;
    case CIS2B_PROF_ATTENTION: return 2;
    case CIS2B_PROF_WITNESS: return 3;
    default: return -1;
  }
}

const char *kSlotNames[] = {"input_layernorm.weight", "post_attention_layernorm.weight"};

struct TensorRef {
  size_t begin = 0, end = 0;
  std::vector<size_t> shape;
  std::string dtype;
};

// ------------------------------------------------------------------ loading

// Shortest decimal that reads back as the same f64, in positional notation
// (how Rust's Display prints an f64 in the gate's reasons).
std::string f64_display(double x) {
  char buf[512];
  for (int p = 1; p <= 17; ++p) {
    snprintf(buf, sizeof buf, "%.*g", p, x);
    if (strtod(buf, nullptr) == x) break;
  }
  if (!strchr(buf, 'e')) return buf;
  for (int d = 0; d <= 340; ++d) {  // no exponent form: widen the fixed form until it round-trips
    snprintf(buf, sizeof buf, "%.*f", d, x);
    if (strtod(buf, nullptr) == x) break;
  }
  return buf;
}

// The architecture gate: the checkpoints whose arithmetic this decoder
// reproduces, and a refusal by name for the rest, with the reference's keys,
// order and reason texts (code/cis2-fp/src/main.rs:545-644, which refuses
// with CIS2_REF_UNSUPPORTED and exit status 2).  With CIS2B_GATE_QWEN3_PORT
// model_type "qwen3" is admitted as well, because the lab's Qwen3 port of the
// C++ path decodes it (labs/w1x-qwen3/scripts/qwen3-port.diff); for it the
// explicit head_dim is the one used (Qwen3-0.6B declares 128 against a
// derived 64).
bool gate_architecture(JsonRef cfg, int gate, std::string &why) {
  auto present = [&](const char *k) { return cfg[k] && !cfg[k].is(JsonRef::Null); };
  const bool qwen3_port = gate == CIS2B_GATE_QWEN3_PORT;
  std::string mt;
  if (cfg["model_type"].is(JsonRef::String)) {
    mt = cfg["model_type"].text();
    if (mt != "llama" && mt != "qwen2" && !(qwen3_port && mt == "qwen3")) {
      why = "model_type=\"" + mt + "\" is not in the CIS-2 specified subset " +
            (qwen3_port ? "[\"llama\", \"qwen2\", \"qwen3\"]" : "[\"llama\", \"qwen2\"]");
      return false;
    }
  }
  if (cfg["torch_dtype"].is(JsonRef::String) && cfg["torch_dtype"].text() != "bfloat16") {
    why = "torch_dtype=\"" + cfg["torch_dtype"].text() + "\"; CIS-2 pins bf16-on-disk weights (\u00a73.5)";
    return false;
  }
  const JsonRef h = cfg["hidden_size"], nh = cfg["num_attention_heads"];
  if (h.is(JsonRef::Number) && nh.is(JsonRef::Number)) {
    if (nh.number() == 0) { why = "num_attention_heads=0"; return false; }
    const long derived = (long)h.number() / (long)nh.number();
    long used = derived;
    if (const JsonRef j = cfg["head_dim"]; j.is(JsonRef::Number)) {
      if ((long)j.number() != derived && !(qwen3_port && mt == "qwen3")) {
        why = "config declares head_dim=" + std::to_string((long)j.number()) +
              " but this implementation derives hidden_size/num_attention_heads=" + std::to_string(derived) +
              "; the decode path uses the derived value, so the explicit one would be silently ignored";
        return false;
      }
      used = (long)j.number();
    }
    if (used % 2 != 0) {
      why = "derived head_dim=" + std::to_string(used) + " is odd; RoPE pairs require even";
      return false;
    }
  }
  if (const JsonRef j = cfg["partial_rotary_factor"]; j.is(JsonRef::Number) && j.number() != 1.0) {
    why = "partial_rotary_factor=" + f64_display(j.number()) + "; only full rotary is specified";
    return false;
  }
  if (present("rope_scaling")) { why = "rope_scaling is set; only unscaled RoPE is specified"; return false; }
  if (cfg["use_sliding_window"].boolean()) {
    why = "use_sliding_window=true; only full causal attention is specified";
    return false;
  }
  if (present("quantization_config")) {
    why = "quantization_config is present; CIS-2 reads unquantized bf16 weights";
    return false;
  }
  for (const char *k : {"attention_multiplier", "embedding_multiplier", "residual_multiplier", "logits_scaling",
                        "attn_logit_softcapping", "final_logit_softcapping", "query_pre_attn_scalar"})
    if (present(k)) {
      why = std::string(k) + " is set; this implementation hardcodes rsqrt(head_dim) attention scaling and no "
            "logit scaling, so the result would be silently wrong";
      return false;
    }
  for (const char *k : {"num_local_experts", "num_experts", "n_routed_experts", "moe_intermediate_size"})
    if (present(k)) { why = std::string(k) + " is set; MoE routing is not specified"; return false; }
  return true;
}

int load_impl(const char *dir_c, const cis2b_opts *opts, cis2b_model *m) {
  if (!dir_c) return fail(CIS2B_ERR_ARG, "weights_dir is NULL");
  cis2b_opts o{};
  if (opts) o = *opts;
  for (int i = 0; i < 4; ++i)
    if (o.reserved[i] != 0) return fail(CIS2B_ERR_ARG, "cis2b_opts.reserved must be zero");
  if (o.arch_gate != CIS2B_GATE_REFERENCE && o.arch_gate != CIS2B_GATE_QWEN3_PORT)
    return fail(CIS2B_ERR_ARG, "unknown architecture gate");
  if (o.reduction != CIS2B_REDUCTION_SEQUENTIAL && o.reduction != CIS2B_REDUCTION_TREE)
    return fail(CIS2B_ERR_ARG, "unknown reduction mode");
  if (o.max_positions < 0) return fail(CIS2B_ERR_ARG, "max_positions < 0");
  m->dev = o.device;
  m->tree = o.reduction == CIS2B_REDUCTION_TREE;
  if (const char *e = getenv("CIS2B_DEC_BIG_ROWS")) m->dec_big_rows = atoi(e);  // tuning override
  m->max_pos = o.max_positions ? o.max_positions : 4096;

  // Everything up to the upload is host work, so artifact and config errors
  // are reported the same way with or without a device.  The config is read
  // and gated first, so an unsupported checkpoint is refused by name even
  // without its weights (code/cis2-fp/src/main.rs:812-823).
  const std::string dir(dir_c);
  std::string wbytes, tok, cfgtxt;
  if (!read_file(dir + "/config.json", cfgtxt)) return fail(CIS2B_ERR_IO, "cannot read " + dir + "/config.json");
  JsonDoc cfg_doc;
  std::string jerr;
  if (!cfg_doc.parse(cfgtxt.data(), cfgtxt.data() + cfgtxt.size(), jerr) || !cfg_doc.root().is(JsonRef::Object))
    return fail(CIS2B_ERR_IO, "config.json: " + (jerr.empty() ? std::string("not an object") : jerr));
  const JsonRef cfg = cfg_doc.root();
  {
    std::string why;
    if (!gate_architecture(cfg, o.arch_gate, why)) return fail(CIS2B_ERR_CONFIG, why);
  }
  if (!read_file(dir + "/model.safetensors", wbytes))
    return fail(CIS2B_ERR_IO, "cannot read " + dir + "/model.safetensors");
  if (!read_file(dir + "/tokenizer.json", tok)) return fail(CIS2B_ERR_IO, "cannot read " + dir + "/tokenizer.json");
  {
    Sha256 a, b, c;
    a.update(wbytes.data(), wbytes.size());
    a.final(m->info.weights_sha256);
    b.update(tok.data(), tok.size());
    b.final(m->info.tokenizer_sha256);
    c.update(cfgtxt.data(), cfgtxt.size());
    c.final(m->info.config_sha256);
  }

  // ---- config (cis2_host.cpp:97-117, qwen3-port.diff:109-110)
  auto need = [&](const char *k, double &v) -> bool {
    if (!cfg[k].is(JsonRef::Number)) return false;
    v = cfg[k].number();
    return true;
  };
  double hid, inter, nl, nh, nkv, voc, eps, theta;
  if (!need("hidden_size", hid) || !need("intermediate_size", inter) || !need("num_hidden_layers", nl) ||
      !need("num_attention_heads", nh) || !need("num_key_value_heads", nkv) || !need("vocab_size", voc) ||
      !need("rms_norm_eps", eps) || !need("rope_theta", theta))
    return fail(CIS2B_ERR_CONFIG, "config.json lacks a required numeric key");
  m->H = (int)hid; m->I = (int)inter; m->L = (int)nl; m->NH = (int)nh; m->NKV = (int)nkv; m->V = (int)voc;
  m->eps = (float)eps;
  if (m->NH <= 0 || m->NKV <= 0 || m->H <= 0 || m->I <= 0 || m->L <= 0 || m->V <= 0)
    return fail(CIS2B_ERR_CONFIG, "non-positive model dimension");
  m->HD = m->H / m->NH;
  if (cfg["head_dim"].is(JsonRef::Number)) m->HD = (int)cfg["head_dim"].number();
  bool tied = true;
  if (cfg["tie_word_embeddings"].is(JsonRef::Bool)) tied = cfg["tie_word_embeddings"].boolean();
  m->QD = m->NH * m->HD;
  m->KVD = m->NKV * m->HD;
  if (m->NH % m->NKV) return fail(CIS2B_ERR_CONFIG, "num_attention_heads % num_key_value_heads != 0");
  if (m->HD <= 0 || m->HD % 4) return fail(CIS2B_ERR_CONFIG, "head_dim must be a positive multiple of 4");
  if (m->H % 8 || m->QD % 8 || m->I % 8)
    return fail(CIS2B_ERR_CONFIG, "hidden, q_dim and intermediate sizes must be multiples of 8");
  m->info.hidden = m->H; m->info.intermediate = m->I; m->info.n_layers = m->L;
  m->info.n_heads = m->NH; m->info.n_kv_heads = m->NKV; m->info.head_dim = m->HD;
  m->info.vocab = m->V; m->info.tied = tied ? 1 : 0; m->info.rms_norm_eps = m->eps;
  m->info.rope_theta = theta; m->info.reduction = o.reduction; m->info.max_positions = m->max_pos;

  // ---- safetensors index (cis2_model.h:296-326)
  if (wbytes.size() < 8) return fail(CIS2B_ERR_IO, "safetensors too short");
  uint64_t hlen = 0;
  for (int i = 0; i < 8; ++i) hlen |= (uint64_t)(uint8_t)wbytes[i] << (8 * i);
  if (8 + hlen > wbytes.size()) return fail(CIS2B_ERR_IO, "safetensors header length out of range");
  JsonDoc hdr_doc;
  if (!hdr_doc.parse(wbytes.data() + 8, wbytes.data() + 8 + hlen, jerr) || !hdr_doc.root().is(JsonRef::Object))
    return fail(CIS2B_ERR_IO, "safetensors header: " + (jerr.empty() ? std::string("not an object") : jerr));
  const JsonRef hdr = hdr_doc.root();
  const size_t data0 = 8 + hlen, data_len = wbytes.size() - data0;
  auto find = [&](const std::string &name, TensorRef &t) -> bool {
    const JsonRef j = hdr[name.c_str()];
    const JsonRef dt = j["dtype"], sh = j["shape"], of = j["data_offsets"];
    if (!dt.is(JsonRef::String) || !sh.is(JsonRef::Array) || !of.is(JsonRef::Array) || of.size() != 2)
      return false;
    t.dtype = dt.text();
    t.shape.clear();
    for (size_t i = 0; i < sh.size(); ++i) t.shape.push_back((size_t)sh.item(i).number());
    t.begin = (size_t)of.item(0).number();
    t.end = (size_t)of.item(1).number();
    return true;
  };
  struct Piece { size_t dst_off; const uint8_t *src; size_t bytes; };
  std::vector<Piece> pieces;
  size_t arena_bytes = 0;
  auto reserve = [&](size_t bytes) {
    size_t off = arena_bytes;
    arena_bytes += (bytes + 255) & ~(size_t)255;
    return off;
  };
  std::string err;
  // Adds tensor `name` of `shape` at byte offset `dst` within a reserved region.
  auto take = [&](const std::string &name, std::vector<size_t> shape, size_t dst, bool optional,
                  bool &present) -> bool {
    TensorRef t;
    present = find(name, t);
    if (!present) {
      if (!optional) err = "tensor " + name + " missing";
      return optional;
    }
    if (t.dtype != "BF16") { err = "tensor " + name + " dtype " + t.dtype + ", expected BF16"; return false; }
    if (t.shape != shape) { err = "tensor " + name + " shape mismatch"; return false; }
    size_t n = 1;
    for (size_t d : shape) n *= d;
    if (t.end < t.begin || t.end > data_len || t.end - t.begin != 2 * n) {
      err = "tensor " + name + " byte range invalid";
      return false;
    }
    pieces.push_back({dst, (const uint8_t *)wbytes.data() + data0 + t.begin, 2 * n});
    return true;
  };
  const size_t H = m->H, I = m->I, QD = m->QD, KVD = m->KVD, V = m->V, HD = m->HD;
  bool pr;
  size_t off_embed = reserve(2 * V * H);
  if (!take("model.embed_tokens.weight", {V, H}, off_embed, false, pr)) return fail(CIS2B_ERR_IO, err);
  size_t off_norm = reserve(2 * H);
  if (!take("model.norm.weight", {H}, off_norm, false, pr)) return fail(CIS2B_ERR_IO, err);
  size_t off_lm = 0;
  if (!tied) {
    off_lm = reserve(2 * V * H);
    if (!take("lm_head.weight", {V, H}, off_lm, false, pr)) return fail(CIS2B_ERR_IO, err);
  }
  struct LOff { size_t in, post, qkv, o, gu, down, qn, kn, qb, kb, vb; bool hqn, hkn, hqb, hkb, hvb; };
  std::vector<LOff> lo((size_t)m->L);
  for (int l = 0; l < m->L; ++l) {
    char pfx[64];
    snprintf(pfx, sizeof pfx, "model.layers.%d.", l);
    std::string p(pfx);
    LOff &x = lo[(size_t)l];
    x.in = reserve(2 * H);
    x.post = reserve(2 * H);
    x.qkv = reserve(2 * (QD + 2 * KVD) * H);
    x.o = reserve(2 * H * QD);
    x.gu = reserve(2 * 2 * I * H);
    x.down = reserve(2 * H * I);
    x.qn = reserve(2 * HD);
    x.kn = reserve(2 * HD);
    x.qb = reserve(2 * QD);
    x.kb = reserve(2 * KVD);
    x.vb = reserve(2 * KVD);
    if (!take(p + kSlotNames[0], {H}, x.in, false, pr) || !take(p + kSlotNames[1], {H}, x.post, false, pr) ||
        !take(p + "self_attn.q_proj.weight", {QD, H}, x.qkv, false, pr) ||
        !take(p + "self_attn.k_proj.weight", {KVD, H}, x.qkv + 2 * QD * H, false, pr) ||
        !take(p + "self_attn.v_proj.weight", {KVD, H}, x.qkv + 2 * (QD + KVD) * H, false, pr) ||
        !take(p + "self_attn.o_proj.weight", {H, QD}, x.o, false, pr) ||
        !take(p + "mlp.gate_proj.weight", {I, H}, x.gu, false, pr) ||
        !take(p + "mlp.up_proj.weight", {I, H}, x.gu + 2 * I * H, false, pr) ||
        !take(p + "mlp.down_proj.weight", {H, I}, x.down, false, pr) ||
        !take(p + "self_attn.q_norm.weight", {HD}, x.qn, true, x.hqn) ||
        !take(p + "self_attn.k_norm.weight", {HD}, x.kn, true, x.hkn) ||
        !take(p + "self_attn.q_proj.bias", {QD}, x.qb, true, x.hqb) ||
        !take(p + "self_attn.k_proj.bias", {KVD}, x.kb, true, x.hkb) ||
        !take(p + "self_attn.v_proj.bias", {KVD}, x.vb, true, x.hvb))
      return fail(CIS2B_ERR_IO, err);
  }
  CU(cudaSetDevice(m->dev));
  CU(cudaStreamCreateWithFlags(&m->s_main, cudaStreamNonBlocking));
  int lo_pri = 0, hi_pri = 0;
  CU(cudaDeviceGetStreamPriorityRange(&lo_pri, &hi_pri));
  CU(cudaStreamCreateWithPriority(&m->s_sha, cudaStreamNonBlocking, hi_pri));
  CU(cudaStreamCreateWithPriority(&m->s_prep, cudaStreamNonBlocking, hi_pri));
  if (m->arena.ensure(arena_bytes) != cudaSuccess)
    return fail(CIS2B_ERR_NOMEM, "device allocation of the weight arena failed");
  uint8_t *base = m->arena.as<uint8_t>();
  for (const Piece &pc : pieces) CU(cudaMemcpy(base + pc.dst_off, pc.src, pc.bytes, cudaMemcpyHostToDevice));
  auto at = [&](size_t off) { return reinterpret_cast<const uint16_t *>(base + off); };
  m->embed = at(off_embed);
  m->final_norm = at(off_norm);
  m->lm_head = tied ? m->embed : at(off_lm);
  m->layers.resize((size_t)m->L);
  for (int l = 0; l < m->L; ++l) {
    const LOff &x = lo[(size_t)l];
    LayerW &w = m->layers[(size_t)l];
    w.in_norm = at(x.in); w.post_norm = at(x.post); w.wqkv = at(x.qkv); w.wo = at(x.o);
    w.wgu = at(x.gu); w.wdown = at(x.down);
    w.q_norm = x.hqn ? at(x.qn) : nullptr; w.k_norm = x.hkn ? at(x.kn) : nullptr;
    w.q_bias = x.hqb ? at(x.qb) : nullptr; w.k_bias = x.hkb ? at(x.kb) : nullptr;
    w.v_bias = x.hvb ? at(x.vb) : nullptr;
  }
  wbytes.clear();
  wbytes.shrink_to_fit();

  // ---- GEMM weights in panel layout (same bf16 bits, k-major 8-row panels)
  {
    const int NQKV = m->QD + 2 * m->KVD;
    size_t total = 0;
    auto preserve = [&](int N, int K) {
      size_t off = total;
      total += (panel_elems(N, K) * 2 + 255) & ~(size_t)255;
      return off;
    };
    std::vector<size_t> offs;
    for (int l = 0; l < m->L; ++l) {
      offs.push_back(preserve(NQKV, m->H));
      offs.push_back(preserve(m->H, m->QD));
      offs.push_back(preserve(2 * m->I, m->H));
      offs.push_back(preserve(m->H, m->I));
    }
    size_t off_lmp = preserve(m->V, m->H);
    if (m->panels.ensure(total) != cudaSuccess)
      return fail(CIS2B_ERR_NOMEM, "device allocation of the weight panels failed");
    uint8_t *pb = m->panels.as<uint8_t>();
    auto pat = [&](size_t off) { return reinterpret_cast<uint16_t *>(pb + off); };
    for (int l = 0; l < m->L; ++l) {
      LayerW &w = m->layers[(size_t)l];
      w.pqkv = pat(offs[4 * l]);
      w.po = pat(offs[4 * l + 1]);
      w.pgu = pat(offs[4 * l + 2]);
      w.pdown = pat(offs[4 * l + 3]);
      launch_panelize(w.wqkv, NQKV, m->H, const_cast<uint16_t *>(w.pqkv), m->s_main);
      launch_panelize(w.wo, m->H, m->QD, const_cast<uint16_t *>(w.po), m->s_main);
      launch_panelize(w.wgu, 2 * m->I, m->H, const_cast<uint16_t *>(w.pgu), m->s_main, m->I);  // gate/up interleaved
      launch_panelize(w.wdown, m->H, m->I, const_cast<uint16_t *>(w.pdown), m->s_main);
    }
    m->lm_head_p = pat(off_lmp);
    launch_panelize(m->lm_head, m->V, m->H, const_cast<uint16_t *>(m->lm_head_p), m->s_main);
    {  // fp32 panels at twice the offsets (4 bytes per element instead of 2)
      if (m->panels_f.ensure(2 * total) != cudaSuccess)
        return fail(CIS2B_ERR_NOMEM, "device allocation of the fp32 weight panels failed");
      uint8_t *fb = m->panels_f.as<uint8_t>();
      auto fat = [&](size_t off) { return reinterpret_cast<float *>(fb + 2 * off); };
      for (int l = 0; l < m->L; ++l) {
        LayerW &w = m->layers[(size_t)l];
        w.fqkv = fat(offs[4 * l]);
        w.fo = fat(offs[4 * l + 1]);
        w.fgu = fat(offs[4 * l + 2]);
        w.fdown = fat(offs[4 * l + 3]);
        launch_panelize(w.wqkv, NQKV, m->H, const_cast<float *>(w.fqkv), m->s_main);
        launch_panelize(w.wo, m->H, m->QD, const_cast<float *>(w.fo), m->s_main);
        launch_panelize(w.wgu, 2 * m->I, m->H, const_cast<float *>(w.fgu), m->s_main, m->I);
        launch_panelize(w.wdown, m->H, m->I, const_cast<float *>(w.fdown), m->s_main);
      }
      m->lm_head_f = fat(off_lmp);
      launch_panelize(m->lm_head, m->V, m->H, const_cast<float *>(m->lm_head_f), m->s_main);
    }
    CU_LAUNCHED();
    CU(cudaStreamSynchronize(m->s_main));
  }

  // ---- decode tiles (same bf16 bits, 32 columns x 4 k per lane-row)
  m->dec_tiles = gemm_dec_ok(m->H, m->tree) && gemm_dec_ok(m->QD, m->tree) && gemm_dec_ok(m->I, m->tree) &&
                 m->I % 16 == 0;
  if (m->dec_tiles) {
    const int NQKV = m->QD + 2 * m->KVD;
    size_t total = 0;
    auto reserve = [&](int N, int K) {
      size_t off = total;
      total += (tile32_elems(N, K) * 2 + 255) & ~(size_t)255;
      return off;
    };
    std::vector<size_t> offs;
    for (int l = 0; l < m->L; ++l) {
      offs.push_back(reserve(NQKV, m->H));
      offs.push_back(reserve(m->H, m->QD));
      offs.push_back(reserve(2 * m->I, m->H));
      offs.push_back(reserve(m->H, m->I));
    }
    size_t off_lm = reserve(m->V, m->H);
    if (m->tiles.ensure(total) != cudaSuccess)
      return fail(CIS2B_ERR_NOMEM, "device allocation of the decode weight tiles failed");
    uint16_t *tb = m->tiles.as<uint16_t>();
    auto tat = [&](size_t off) { return tb + off / 2; };
    for (int l = 0; l < m->L; ++l) {
      LayerW &w = m->layers[(size_t)l];
      w.tqkv = tat(offs[4 * l]);
      w.to = tat(offs[4 * l + 1]);
      w.tgu = tat(offs[4 * l + 2]);
      w.tdown = tat(offs[4 * l + 3]);
      launch_tile32(w.wqkv, NQKV, m->H, const_cast<uint16_t *>(w.tqkv), m->s_main);
      launch_tile32(w.wo, m->H, m->QD, const_cast<uint16_t *>(w.to), m->s_main);
      launch_tile32(w.wgu, 2 * m->I, m->H, const_cast<uint16_t *>(w.tgu), m->s_main, m->I);
      launch_tile32(w.wdown, m->H, m->I, const_cast<uint16_t *>(w.tdown), m->s_main);
    }
    m->lm_head_t = tat(off_lm);
    launch_tile32(m->lm_head, m->V, m->H, const_cast<uint16_t *>(m->lm_head_t), m->s_main);
    CU_LAUNCHED();
    CU(cudaStreamSynchronize(m->s_main));
  }

  // ---- pinned tables on the device (cis2_model.h:456-476, 547-568)
  const int half = m->HD / 2;
  if (m->inv_freq.ensure(sizeof(float) * half) != cudaSuccess ||
      m->cos_t.ensure(sizeof(float) * half * (size_t)m->max_pos) != cudaSuccess ||
      m->sin_t.ensure(sizeof(float) * half * (size_t)m->max_pos) != cudaSuccess)
    return fail(CIS2B_ERR_NOMEM, "device allocation of the RoPE tables failed");
  launch_inv_freq((float)theta, m->HD, m->inv_freq.as<float>(), m->s_main);
  launch_rope_table(m->inv_freq.as<float>(), half, m->max_pos, m->cos_t.as<float>(), m->sin_t.as<float>(),
                    m->s_main);
  CU_LAUNCHED();
  std::vector<float> invf((size_t)half);
  CU(cudaMemcpyAsync(invf.data(), m->inv_freq.p, sizeof(float) * half, cudaMemcpyDeviceToHost, m->s_main));
  CU(cudaStreamSynchronize(m->s_main));
  {
    Sha256 s;
    for (float f : invf) { uint32_t u; memcpy(&u, &f, 4); s.u32le(u); }
    s.final(m->info.inv_freq_table_digest);
  }
  {
    // §6.6 table digest: the coefficient bit patterns in declared order
    // (cis2_model.h:414-450), the same constants the kernels use.
    Sha256 s;
    const uint32_t a[] = {EXP_LOG2E, EXP_C1, EXP_C2, EXP_P0, EXP_P1, EXP_P2, EXP_P3, EXP_P4, EXP_P5};
    for (uint32_t u : a) s.u32le(u);
    uint8_t le[8];
    for (int i = 0; i < 8; ++i) le[i] = (uint8_t)(PI_2_F64 >> (8 * i));
    s.update(le, 8);
    const uint32_t b[] = {SIN_C0, SIN_C1, SIN_C2, COS_C0, COS_C1, COS_C2, LOG_SQRTHF, LOG_Q1, LOG_Q2,
                          LOG_P0, LOG_P1, LOG_P2, LOG_P3, LOG_P4, LOG_P5, LOG_P6, LOG_P7, LOG_P8};
    for (uint32_t u : b) s.u32le(u);
    s.final(m->info.table_digest);
  }
  CU(cudaEventCreate(&m->ev_sel, cudaEventDisableTiming));
  CU(cudaEventCreate(&m->ev0));
  CU(cudaEventCreate(&m->ev_pref));
  CU(cudaEventCreate(&m->ev_dec));
  CU(cudaEventCreate(&m->ev_end));
  for (int i = 0; i < 2; ++i) {
    CU(cudaEventCreateWithFlags(&m->ev_prep[i], cudaEventDisableTiming));
    CU(cudaEventCreateWithFlags(&m->ev_comp[i], cudaEventDisableTiming));
  }
  return CIS2B_OK;
}

// ------------------------------------------------------------------ forward
// Runs `rows` activation rows (token ids, sequence index and position per
// row, all on the device) through every layer.  Leaves the final hidden
// state in m->h.  kv caches are [layer][seq][maxP][kvd].  `decode`: every
// row is a different sequence's newest position, so the q/k post-processing
// and the cache append run inside the attention kernel.
// Row tiles for the prompt-pass attention (launch_attention_rows).
struct AttTiles {
  const int2 *tiles = nullptr;
  int n = 0, rt = 0, max_len = 0;
};

int forward_rows(cis2b_model *m, int rows, const uint32_t *tok, const int32_t *seq,
                 const int32_t *pos, int n_seq_cache, int maxP, bool decode, const AttTiles *at = nullptr) {
  cudaStream_t s = m->s_main;
  const int H = m->H, I = m->I, QD = m->QD, KVD = m->KVD, NQKV = QD + 2 * KVD;
  float *h = m->h.as<float>(), *ln = m->ln.as<float>(), *qkv = m->qkv.as<float>();
  float *att = m->att.as<float>(), *gu = m->gu.as<float>(), *hid = m->hid.as<float>();
  const size_t layer_kv = (size_t)n_seq_cache * maxP * KVD;
  const int ldm = m->act_ldm;  // ln, att, hid are k-major [K][ldm] GEMM operands
  RowMap rm{seq, pos};
  launch_embed(m->embed, H, tok, rows, h, s);
  m->launches += 1;
  // Decode steps in sequential mode with fewer than dec_big_rows rows run the
  // GEMMs in the few-row form: its activations are row-major, so every
  // producer writes (row stride K, 1).  Everything else -- the prompt pass,
  // tree mode, and decode steps with many rows -- uses k-major operands and
  // the register-tiled product.
  const bool dec = decode && m->dec_tiles && rows < m->dec_big_rows;
  const int lnr = dec ? H : 1, lnc = dec ? 1 : ldm;      // ln / att / hid (row, column) strides
  const int atr = dec ? QD : 1, hir = dec ? I : 1;
  auto gemm = [&](const float *X, const uint16_t *Wp, const float *Wpf, const uint16_t *Wt, int K, int N, float *Y,
                  int ldy, const float *R, int ldr) {
    ProfScope p(m, CIS2B_PROF_LAYER_GEMM, s);
    if (dec) launch_gemm_dec(X, K, Wt, K, N, rows, Y, ldy, R, ldr, nullptr, 0, s, 0, m->tree);
    else launch_gemm(X, ldm, Wp, Wpf, K, N, rows, Y, ldy, R, ldr, m->tree, nullptr, 0, s);
  };
  for (int l = 0; l < m->L; ++l) {
    const LayerW &w = m->layers[(size_t)l];
    float *kc = m->kc.as<float>() + (size_t)l * layer_kv;
    float *vc = m->vc.as<float>() + (size_t)l * layer_kv;
    launch_rmsnorm(h, H, w.in_norm, m->eps, H, rows, m->tree, ln, lnr, lnc, s);
    gemm(ln, w.pqkv, w.fqkv, w.tqkv, H, NQKV, qkv, NQKV, nullptr, 0);
    m->launches += 2;
    if (w.q_bias) { launch_add_bias(qkv, NQKV, rows, w.q_bias, QD, s); m->launches++; }
    if (w.k_bias) { launch_add_bias(qkv + QD, NQKV, rows, w.k_bias, KVD, s); m->launches++; }
    if (w.v_bias) { launch_add_bias(qkv + QD + KVD, NQKV, rows, w.v_bias, KVD, s); m->launches++; }
    if (!decode) {
      launch_qkv_post(qkv, NQKV, rows, rm, m->NH, m->NKV, m->HD, w.q_norm, w.k_norm, m->eps, m->tree,
                      m->cos_t.as<float>(), m->sin_t.as<float>(), kc, vc, maxP, s);
      m->launches++;
    }
    { ProfScope p(m, CIS2B_PROF_ATTENTION, s);
      if (!decode && at && at->n > 0)
        launch_attention_rows(qkv, NQKV, at->tiles, at->n, at->rt, rm, m->NH, m->NKV, m->HD, kc, vc, maxP, m->tree,
                              att, atr, ldm, at->max_len, s);
      else
        launch_attention(qkv, NQKV, rows, rm, m->NH, m->NKV, m->HD, kc, vc, maxP, m->tree, att, atr,
                         dec ? 1 : ldm, maxP, decode, w.q_norm, w.k_norm, m->eps, m->cos_t.as<float>(),
                         m->sin_t.as<float>(), s); }
    gemm(att, w.po, w.fo, w.to, QD, H, h, H, h, H);
    launch_rmsnorm(h, H, w.post_norm, m->eps, H, rows, m->tree, ln, lnr, lnc, s);
    if (dec) {  // SwiGLU in the gate/up GEMM's epilogue
      ProfScope p(m, CIS2B_PROF_LAYER_GEMM, s);
      launch_gemm_dec(ln, H, w.tgu, H, 2 * I, rows, hid, I, nullptr, 0, nullptr, 0, s, I, m->tree);
    } else if (rows >= 64 && gemm_big_ok(H, m->tree)) {  // SwiGLU in the epilogue, hid written k-major
      ProfScope p(m, CIS2B_PROF_LAYER_GEMM, s);
      launch_gemm_big(ln, ldm, w.fgu, H, 2 * I, rows, hid, 1, ldm, nullptr, 0, nullptr, 0, 1, s, m->tree);
    } else {
      gemm(ln, w.pgu, w.fgu, w.tgu, H, 2 * I, gu, 2 * I, nullptr, 0);
      launch_silu_mul(gu, I, rows, hid, hir, ldm, s);
      m->launches++;
    }
    gemm(hid, w.pdown, w.fdown, w.tdown, I, H, h, H, h, H);
    m->launches += 5;
  }
  CU_LAUNCHED();
  return CIS2B_OK;
}

// Final norm + lm_head of `rows` hidden rows -> Y (rows x V).
int head_rows(cis2b_model *m, const float *hin, int rows, float *Y, const int32_t *y_slot,
              size_t slot_stride) {
  cudaStream_t s = m->s_main;
  const int ldb = round_up(rows, 64);  // lnlast is k-major [H][ldb] for the panel GEMM
  // Row-major [rows][H] for the decode GEMM.  In tree mode the panel kernel
  // is the slower one from 64 rows on too, so decode steps keep the decode GEMM.
  const bool dec = m->dec_tiles && (rows <= DEC_HEAD_ROWS || (m->tree && rows < m->dec_big_rows));
  launch_rmsnorm(hin, m->H, m->final_norm, m->eps, m->H, rows, m->tree, m->lnlast.as<float>(),
                 dec ? m->H : 1, dec ? 1 : ldb, s);
  {
    ProfScope p(m, CIS2B_PROF_LM_HEAD, s);
    if (dec)
      launch_gemm_dec(m->lnlast.as<float>(), m->H, m->lm_head_t, m->H, m->V, rows, Y, m->V, nullptr, 0, y_slot,
                      slot_stride, s, 0, m->tree);
    else
      launch_gemm(m->lnlast.as<float>(), ldb, m->lm_head_p, m->lm_head_f, m->H, m->V, rows, Y, m->V, nullptr, 0,
                  m->tree, y_slot, slot_stride, s);
  }
  m->launches += 2;
  CU_LAUNCHED();
  return CIS2B_OK;
}

// Activation buffers for up to `rows` rows.  The GEMM operands (ln, att,
// hid) are k-major with act_ldm = rows rounded up to 64 columns.
int ensure_act(cis2b_model *m, int rows) {
  const size_t r = (size_t)std::max(rows, 1);
  const size_t ldm = (size_t)round_up((int)r, 64);
  const size_t H = m->H, I = m->I, QD = m->QD, KVD = m->KVD;
  if (m->h.ensure(4 * r * H) || m->ln.ensure(4 * ldm * H) || m->qkv.ensure(4 * r * (QD + 2 * KVD)) ||
      m->att.ensure(4 * ldm * QD) || m->gu.ensure(4 * r * 2 * I) || m->hid.ensure(4 * ldm * I))
    return fail(CIS2B_ERR_NOMEM, "device allocation of activations failed");
  m->act_ldm = (int)ldm;
  return CIS2B_OK;
}

// Position-batched pass over prompt rows.  rows_* are host arrays (row order
// must list each sequence's positions ascending).  For out_rows[i] >= 0,
// the final hidden state of row out_src[i] lands in hlast row out_dst[i].
int prefill(cis2b_model *m, const std::vector<uint32_t> &tok, const std::vector<int32_t> &seq,
            const std::vector<int32_t> &pos, const std::vector<int32_t> &out_src,
            const std::vector<int32_t> &out_dst, int n_seq_cache, int maxP) {
  const int total = (int)tok.size();
  const int chunk = std::min(total, PREFILL_CHUNK);
  int rc = ensure_act(m, std::max(chunk, n_seq_cache));
  if (rc) return rc;
  if (m->rows_tok.ensure(4 * (size_t)total) || m->rows_seq.ensure(4 * (size_t)total) ||
      m->rows_pos.ensure(4 * (size_t)total) || m->gsrc.ensure(4 * out_src.size() + 4) ||
      m->gdst.ensure(4 * out_dst.size() + 4))
    return fail(CIS2B_ERR_NOMEM, "device allocation of row maps failed");
  cudaStream_t s = m->s_main;
  CU(cudaMemcpyAsync(m->rows_tok.p, tok.data(), 4 * (size_t)total, cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->rows_seq.p, seq.data(), 4 * (size_t)total, cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->rows_pos.p, pos.data(), 4 * (size_t)total, cudaMemcpyHostToDevice, s));
  // Per chunk gather lists, uploaded once (host memory must stay valid until
  // the copies run, so stage everything before the first launch).
  std::vector<int32_t> gs, gd;
  std::vector<std::pair<int, int>> ranges;  // [first, count) into gs/gd per chunk
  for (int c0 = 0; c0 < total; c0 += chunk) {
    int first = (int)gs.size();
    for (size_t i = 0; i < out_src.size(); ++i)
      if (out_src[i] >= c0 && out_src[i] < c0 + chunk) {
        gs.push_back(out_src[i] - c0);
        gd.push_back(out_dst[i]);
      }
    ranges.push_back({first, (int)gs.size() - first});
  }
  if (!gs.empty()) {
    CU(cudaMemcpyAsync(m->gsrc.p, gs.data(), 4 * gs.size(), cudaMemcpyHostToDevice, s));
    CU(cudaMemcpyAsync(m->gdst.p, gd.data(), 4 * gd.size(), cudaMemcpyHostToDevice, s));
  }
  // Attention row tiles per chunk: runs of rows of one sequence at
  // consecutive positions, at most rt long (rt from the chunk's longest row).
  std::vector<int2> tl;
  std::vector<AttTiles> ats;
  const bool tiled = m->HD <= 256;
  for (int c0 = 0; c0 < total && tiled; c0 += chunk) {
    const int n = std::min(chunk, total - c0);
    int maxpos = 0;
    for (int i = c0; i < c0 + n; ++i) maxpos = std::max(maxpos, (int)pos[(size_t)i]);
    AttTiles a;
    a.max_len = maxpos + 1;
    a.rt = attention_rows_rt(m->NH / m->NKV, m->HD, a.max_len);
    a.n = (int)tl.size();  // index of the chunk's first tile until the pointers are known
    for (int i = c0; i < c0 + n;) {
      int k = 1;
      while (k < a.rt && i + k < c0 + n && seq[(size_t)(i + k)] == seq[(size_t)i] &&
             pos[(size_t)(i + k)] == pos[(size_t)i] + k)
        ++k;
      tl.push_back(make_int2(i - c0, k));
      i += k;
    }
    ats.push_back(a);
  }
  if (!tl.empty()) {
    if (m->att_tiles.ensure(sizeof(int2) * tl.size()))
      return fail(CIS2B_ERR_NOMEM, "device allocation of attention tiles failed");
    CU(cudaMemcpyAsync(m->att_tiles.p, tl.data(), sizeof(int2) * tl.size(), cudaMemcpyHostToDevice, s));
    for (size_t c = 0; c < ats.size(); ++c) {
      const int first = ats[c].n, last = c + 1 < ats.size() ? ats[c + 1].n : (int)tl.size();
      ats[c].tiles = m->att_tiles.as<int2>() + first;
      ats[c].n = last - first;
    }
  }
  int ci = 0;
  for (int c0 = 0; c0 < total; c0 += chunk, ++ci) {
    const int n = std::min(chunk, total - c0);
    rc = forward_rows(m, n, m->rows_tok.as<uint32_t>() + c0, m->rows_seq.as<int32_t>() + c0,
                      m->rows_pos.as<int32_t>() + c0, n_seq_cache, maxP, false,
                      tiled ? &ats[(size_t)ci] : nullptr);
    if (rc) return rc;
    const auto &rg = ranges[(size_t)ci];
    if (rg.second) {
      launch_gather_rows(m->h.as<float>(), m->H, m->gsrc.as<int32_t>() + rg.first,
                         m->gdst.as<int32_t>() + rg.first, rg.second, m->H, m->hlast.as<float>(), s);
      m->launches++;
    }
  }
  // The host vectors above are read by the async copies; make sure they ran.
  CU(cudaStreamSynchronize(s));
  CU_LAUNCHED();
  return CIS2B_OK;
}

int alloc_cache(cis2b_model *m, int n_seq, int maxP) {
  size_t kv = (size_t)m->L * n_seq * maxP * m->KVD * sizeof(float);
  if (m->kc.ensure(kv) || m->vc.ensure(kv))
    return fail(CIS2B_ERR_NOMEM, "device allocation of the KV cache failed (" + std::to_string(kv >> 20) + " MiB each)");
  return CIS2B_OK;
}

// Generation, or -- with `claimed` ([n_seq][gen] ids) -- teacher-forced
// receipt verification (verify3/model.c:923-1004): ONE prompt pass over
// prompt + claimed[0 .. gen-2] per sequence yields the hidden state of every
// claimed position; each step then runs the same head, the same selection
// (argmax or sampler: the token is RECOMPUTED, never taken from the claim)
// and the same witness absorb as generation, so an honest claim reproduces
// the generation digests exactly.
int generate_impl(cis2b_model *m, const uint32_t *prompt_ids, const uint32_t *prompt_lens,
                  uint32_t n_seq, uint32_t gen, const cis2b_sample *sample, uint32_t *out_tokens,
                  uint8_t *out_steps, uint8_t *out_witness, uint8_t *out_argmax,
                  const uint32_t *claimed = nullptr) {
  if (!m) return fail(CIS2B_ERR_ARG, "model is NULL");
  if (n_seq == 0) return CIS2B_OK;
  if (!prompt_ids || !prompt_lens || !out_witness) return fail(CIS2B_ERR_ARG, "NULL input/output buffer");
  if (sample && !(sample->temperature > 0.0f && sample->temperature <= 3.402823466e38f))
    return fail(CIS2B_ERR_ARG, "temperature must be finite and > 0");
  if (sample && sample->scheme != CIS2B_SAMPLE_E23 && sample->scheme != CIS2B_SAMPLE_GUMBEL)
    return fail(CIS2B_ERR_ARG, "unknown sampling scheme");
  if (sample && sample->scheme == CIS2B_SAMPLE_E23 && sample->top_k != 0)
    return fail(CIS2B_ERR_ARG, "top_k applies to the Gumbel-max scheme only");
  if (sample && !(sample->top_p > 0.0f && sample->top_p <= 1.0f)) return fail(CIS2B_ERR_ARG, "top_p must be in (0, 1]");
  CU(cudaSetDevice(m->dev));
  const int B = (int)n_seq, G = (int)gen;
  uint32_t maxP0 = 0;
  size_t total_prompt = 0;
  for (int b = 0; b < B; ++b) {
    if (prompt_lens[b] == 0) return fail(CIS2B_ERR_ARG, "empty prompt (the reference needs >= 1 id)");
    maxP0 = std::max(maxP0, prompt_lens[b]);
    total_prompt += prompt_lens[b];
  }
  for (size_t i = 0; i < total_prompt; ++i)
    if (prompt_ids[i] >= (uint32_t)m->V) return fail(CIS2B_ERR_ARG, "prompt id out of vocabulary range");
  const bool tf = claimed != nullptr;  // teacher-forced verification
  if (tf)
    for (size_t i = 0; i < (size_t)B * G; ++i)
      if (claimed[i] >= (uint32_t)m->V) return fail(CIS2B_ERR_ARG, "claimed id out of vocabulary range");
  const int maxP = (int)maxP0 + G;
  if (maxP > m->max_pos)
    return fail(CIS2B_ERR_ARG, "prompt + gen_toks exceeds max_positions (" + std::to_string(m->max_pos) + ")");
  const size_t V = m->V;
  int ring = std::max(1, G);
  size_t per_slot = (size_t)B * V * sizeof(float);
  if ((size_t)ring * per_slot > RING_BUDGET) ring = (int)std::max<size_t>(2, RING_BUDGET / per_slot);
  ring = std::min(ring, std::max(1, G));
  int rc = alloc_cache(m, B, maxP);
  if (rc) return rc;
  const size_t hrows = tf ? (size_t)B * std::max(G, 1) : (size_t)B;  // hidden rows kept from the prompt pass
  if (m->ring.ensure((size_t)ring * per_slot) || m->hlast.ensure(4 * hrows * m->H) ||
      m->lnlast.ensure(4 * (size_t)round_up(B, 64) * m->H) || m->d_next.ensure(4 * (size_t)B) ||
      m->d_pos.ensure(4 * (size_t)B) || m->d_spos.ensure(4 * (size_t)B) || m->d_seq.ensure(4 * (size_t)B) ||
      m->d_ctl.ensure(64) || m->d_tokens.ensure(4 * (size_t)B * std::max(G, 1)) ||
      m->d_ids_hist.ensure(4 * (size_t)B * std::max(G, 1)) ||
      m->sha_state.ensure(sizeof(ShaState) * (size_t)B) ||
      m->sha_wk.ensure(2 * 4 * sha_wk_words(m->V, B)) || m->sha_c0.ensure(4 * (size_t)B) || m->step_dig.ensure(32 * (size_t)B * std::max(G, 1)) ||
      m->d_witness.ensure(32 * (size_t)B) || m->d_argmax.ensure(32 * (size_t)B) ||
      (sample && m->scratch.ensure(4 * (size_t)B * 5 * V)))
    return fail(CIS2B_ERR_NOMEM, "device allocation of decode buffers failed");
  if ((int)m->ev_sha.size() < ring) {
    for (int i = (int)m->ev_sha.size(); i < ring; ++i) {
      cudaEvent_t e;
      CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      m->ev_sha.push_back(e);
    }
  }
  cudaStream_t s = m->s_main, ss = m->s_sha, sp = m->s_prep;
  const size_t wk_words = sha_wk_words(m->V, B);
  m->launches = 0;
  m->ev_used = 0;
  m->prof_events.clear();

  // ---- host-side staging (all before the first launch)
  const size_t tf_rows = tf && G > 1 ? (size_t)B * (G - 1) : 0;  // claimed tokens fed back as inputs
  std::vector<uint32_t> rtok(total_prompt + tf_rows);
  std::vector<int32_t> rseq(total_prompt + tf_rows), rpos(total_prompt + tf_rows), osrc, odst;
  std::vector<int32_t> iota(B), pos0(B), spos0(B);
  std::vector<uint32_t> poff(B), plen(B);
  {
    size_t r = 0, pr = 0;
    for (int b = 0; b < B; ++b) {
      poff[b] = (uint32_t)pr;
      plen[b] = prompt_lens[b];
      const size_t r0 = r;
      for (uint32_t p = 0; p < prompt_lens[b]; ++p, ++r, ++pr) {
        rtok[r] = prompt_ids[pr];
        rseq[r] = b;
        rpos[r] = (int32_t)p;
      }
      if (tf) {
        for (int t = 0; t + 1 < G; ++t, ++r) {
          rtok[r] = claimed[(size_t)b * G + t];
          rseq[r] = b;
          rpos[r] = (int32_t)(prompt_lens[b] + t);
        }
        // step t's logits come from position prompt_len - 1 + t (model.c:936-941)
        for (int t = 0; t < G; ++t) {
          osrc.push_back((int32_t)(r0 + prompt_lens[b] - 1 + t));
          odst.push_back(t * B + b);
        }
      } else {
        osrc.push_back((int32_t)(r - 1));
        odst.push_back(b);
      }
      iota[b] = b;
      pos0[b] = (int32_t)prompt_lens[b] - 1;
      spos0[b] = (int32_t)prompt_lens[b];
    }
  }
  // witness header bytes (cis2_host.cpp:180-186; e23 patch :617-624)
  std::vector<uint8_t> hb;
  std::vector<uint32_t> hoff(B + 1);
  for (int b = 0; b < B; ++b) {
    hoff[b] = (uint32_t)hb.size();
    if (sample && sample->scheme == CIS2B_SAMPLE_E23) {
      const char tag[] = "CIS2_SAMPLE_V1";
      hb.insert(hb.end(), tag, tag + 14);
      for (int i = 0; i < 8; ++i) hb.push_back((uint8_t)(sample->seed >> (8 * i)));
      uint32_t tb, pb;
      memcpy(&tb, &sample->temperature, 4);
      memcpy(&pb, &sample->top_p, 4);
      for (int i = 0; i < 4; ++i) hb.push_back((uint8_t)(tb >> (8 * i)));
      for (int i = 0; i < 4; ++i) hb.push_back((uint8_t)(pb >> (8 * i)));
    }
    hb.insert(hb.end(), m->info.weights_sha256, m->info.weights_sha256 + 32);
    hb.insert(hb.end(), m->info.tokenizer_sha256, m->info.tokenizer_sha256 + 32);
    hb.insert(hb.end(), m->info.config_sha256, m->info.config_sha256 + 32);
    hb.insert(hb.end(), m->info.table_digest, m->info.table_digest + 32);
    hb.insert(hb.end(), m->info.inv_freq_table_digest, m->info.inv_freq_table_digest + 32);
    for (uint32_t p = 0; p < prompt_lens[b]; ++p) {
      uint32_t v = prompt_ids[poff[b] + p];
      for (int i = 0; i < 4; ++i) hb.push_back((uint8_t)(v >> (8 * i)));
    }
    if (sample && sample->scheme == CIS2B_SAMPLE_GUMBEL) {
      // seeded-sampling patch :128-134: tag, seed, T bits, top_k, top_p bits, after the prompt ids
      const char tag[] = "CIS2-SAMPLE-1";
      hb.insert(hb.end(), tag, tag + 13);
      for (int i = 0; i < 8; ++i) hb.push_back((uint8_t)(sample->seed >> (8 * i)));
      uint32_t tb, pb;
      memcpy(&tb, &sample->temperature, 4);
      memcpy(&pb, &sample->top_p, 4);
      for (int i = 0; i < 4; ++i) hb.push_back((uint8_t)(tb >> (8 * i)));
      for (int i = 0; i < 4; ++i) hb.push_back((uint8_t)(sample->top_k >> (8 * i)));
      for (int i = 0; i < 4; ++i) hb.push_back((uint8_t)(pb >> (8 * i)));
    }
  }
  hoff[B] = (uint32_t)hb.size();
  std::vector<ShaState> st0((size_t)B);
  for (auto &x : st0) {
    memset(&x, 0, sizeof x);
    const uint32_t iv[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                            0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    memcpy(x.h, iv, sizeof iv);
  }
  if (m->hdr_bytes.ensure(hb.size()) || m->hdr_off.ensure(4 * (size_t)(B + 1)) ||
      m->p_flat.ensure(4 * total_prompt) || m->p_off.ensure(4 * (size_t)B) || m->p_len.ensure(4 * (size_t)B))
    return fail(CIS2B_ERR_NOMEM, "device allocation of header buffers failed");

  CU(cudaEventRecord(m->ev0, s));
  CU(cudaMemcpyAsync(m->hdr_bytes.p, hb.data(), hb.size(), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->hdr_off.p, hoff.data(), 4 * hoff.size(), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->sha_state.p, st0.data(), sizeof(ShaState) * st0.size(), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->p_flat.p, prompt_ids, 4 * total_prompt, cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->p_off.p, poff.data(), 4 * (size_t)B, cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->p_len.p, plen.data(), 4 * (size_t)B, cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->d_seq.p, iota.data(), 4 * (size_t)B, cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->d_pos.p, pos0.data(), 4 * (size_t)B, cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->d_spos.p, spos0.data(), 4 * (size_t)B, cudaMemcpyHostToDevice, s));
  CU(cudaMemsetAsync(m->d_ctl.p, 0, 64, s));  // [0] step counter, [1] ring slot
  // Header absorb on the witness stream, ordered after the copies.
  CU(cudaEventRecord(m->ev_sel, s));
  CU(cudaStreamWaitEvent(ss, m->ev_sel, 0));
  launch_sha_absorb_bytes(m->sha_state.as<ShaState>(), m->hdr_bytes.as<uint8_t>(), m->hdr_off.as<uint32_t>(),
                          B, ss);
  m->launches++;
  CU(cudaEventRecord(m->ev_comp[0], ss));  // step 0's expansion reads the carry the header left

  // ---- prefill: every prompt position of every sequence
  rc = prefill(m, rtok, rseq, rpos, osrc, odst, B, maxP);
  if (rc) return rc;
  float *ring_base = m->ring.as<float>();
  rc = head_rows(m, m->hlast.as<float>(), B, ring_base, nullptr, 0);  // step-0 logits -> slot 0
  if (rc) return rc;
  CU(cudaEventRecord(m->ev_pref, s));

  int32_t *d_step = m->d_ctl.as<int32_t>(), *d_slot = m->d_ctl.as<int32_t>() + 1;
  uint32_t *d_next = m->d_next.as<uint32_t>();
  // Token selection for the step whose logits sit in ring slot *d_slot,
  // then the bookkeeping that points the next forward at its position.
  auto select = [&]() {
    if (sample && sample->scheme == CIS2B_SAMPLE_GUMBEL)
      launch_sample_gumbel(ring_base, m->V, B, d_slot, (size_t)B * V, sample->temperature, sample->top_k,
                           sample->top_p, sample->seed, d_step, m->scratch.as<float>(), d_next, s);
    else if (sample)
      launch_sample(ring_base, m->V, B, d_slot, (size_t)B * V, sample->temperature, sample->top_p,
                    sample->seed, m->d_spos.as<int32_t>(), m->scratch.as<float>(), d_next, s);
    else
      launch_argmax(ring_base, m->V, B, d_slot, (size_t)B * V, d_next, s);
    launch_step_advance(d_next, B, d_step, G, m->d_tokens.as<uint32_t>(), m->d_ids_hist.as<uint32_t>(),
                        m->d_pos.as<int32_t>(), m->d_spos.as<int32_t>(), d_slot, ring, d_step, s);
    m->launches += 2;
  };
  // One decode step on the main stream: forward of the chosen ids, lm_head
  // into the next ring slot, selection.  Every argument is a fixed device
  // pointer (positions, ids, slot and step live in device memory), so the
  // step is captured once as a CUDA graph and replayed.
  auto step_body = [&]() -> int {
    int r = forward_rows(m, B, d_next, m->d_seq.as<int32_t>(), m->d_pos.as<int32_t>(), B, maxP, true);
    if (r) return r;
    r = head_rows(m, m->h.as<float>(), B, ring_base, d_slot, (size_t)B * V);
    if (r) return r;
    select();
    return CIS2B_OK;
  };
  const uint32_t in_graph = CIS2B_PROF_LM_HEAD | CIS2B_PROF_LAYER_GEMM | CIS2B_PROF_ATTENTION;
  const bool use_graph = !tf && G >= 3 && !(m->prof_mask & in_graph);
  cudaGraphExec_t gexec = nullptr;
  int64_t step_launches = 0;
  if (use_graph) {
    cudaGraph_t g = nullptr;
    const int64_t l0 = m->launches;
    CU(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    rc = step_body();
    cudaError_t ce = cudaStreamEndCapture(s, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (ce != cudaSuccess) return fail(CIS2B_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
    ce = cudaGraphInstantiate(&gexec, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(CIS2B_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ce));
    step_launches = m->launches - l0;
    m->launches = l0;
  }
  struct GraphGuard {
    cudaGraphExec_t e;
    ~GraphGuard() { if (e) cudaGraphExecDestroy(e); }
  } guard{gexec};
  for (int t = 0; t < G; ++t) {
    if (t == 0) {
      select();
    } else if (tf) {
      if (t >= ring) CU(cudaStreamWaitEvent(s, m->ev_sha[(size_t)(t % ring)], 0));
      rc = head_rows(m, m->hlast.as<float>() + (size_t)t * B * m->H, B, ring_base, d_slot, (size_t)B * V);
      if (rc) return rc;
      select();
    } else {
      if (t >= ring) CU(cudaStreamWaitEvent(s, m->ev_sha[(size_t)(t % ring)], 0));
      if (use_graph) {
        CU(cudaGraphLaunch(gexec, s));
        m->launches += step_launches;
      } else {
        rc = step_body();
        if (rc) return rc;
      }
    }
    // Witness of step t.  The W+K expansion runs on s_prep into one half of
    // the double buffer and may overlap the chain's step t - 1; it needs this
    // step's logits and the chain to be done with the half (step t - 2).
    // Ring slot t - 1 is released once the chain has finished it and this
    // expansion has read its tail (the carry in front of step t).
    uint32_t *wk_t = m->sha_wk.as<uint32_t>() + (size_t)(t & 1) * wk_words;
    const float *logits_t = ring_base + (size_t)(t % ring) * B * V;
    CU(cudaEventRecord(m->ev_sel, s));
    CU(cudaStreamWaitEvent(sp, m->ev_sel, 0));
    CU(cudaStreamWaitEvent(sp, m->ev_comp[t & 1], 0));
    launch_sha_prep_at(m->sha_state.as<ShaState>(), m->sha_c0.as<uint32_t>(), t, B,
                       t ? ring_base + (size_t)((t - 1) % ring) * B * V : nullptr,
                       t ? m->d_ids_hist.as<uint32_t>() + (size_t)(t - 1) * B : nullptr, logits_t, m->V, V,
                       m->d_ids_hist.as<uint32_t>() + (size_t)t * B, wk_t, sp);
    CU(cudaEventRecord(m->ev_prep[t & 1], sp));
    CU(cudaStreamWaitEvent(ss, m->ev_prep[t & 1], 0));
    if (t > 0) CU(cudaEventRecord(m->ev_sha[(size_t)((t - 1) % ring)], ss));
    {
      ProfScope p(m, CIS2B_PROF_WITNESS, ss);
      launch_sha_compress(m->sha_state.as<ShaState>(), B, logits_t, m->V, V,
                          m->d_ids_hist.as<uint32_t>() + (size_t)t * B, wk_t,
                          m->step_dig.as<uint8_t>() + (size_t)t * 32, (size_t)G * 32, ss);
    }
    m->launches += 2;
    CU(cudaEventRecord(m->ev_comp[t & 1], ss));
  }
  if (G > 0) CU(cudaEventRecord(m->ev_sha[(size_t)((G - 1) % ring)], ss));
  CU_LAUNCHED();
  CU(cudaEventRecord(m->ev_dec, s));
  // Join the witness stream; the final digest and the argmax digest run on
  // the main stream after its last step.
  CU(cudaEventRecord(m->ev_sel, ss));
  CU(cudaStreamWaitEvent(s, m->ev_sel, 0));
  launch_sha_finalize(m->sha_state.as<ShaState>(), B, m->d_witness.as<uint8_t>(), s);
  launch_sha_ids(m->p_flat.as<uint32_t>(), m->p_off.as<uint32_t>(), m->p_len.as<uint32_t>(),
                 m->d_tokens.as<uint32_t>(), G, B, m->d_argmax.as<uint8_t>(), s);
  m->launches += 2;
  CU(cudaEventRecord(m->ev_end, s));
  CU_LAUNCHED();
  if (out_tokens && G) CU(cudaMemcpyAsync(out_tokens, m->d_tokens.p, 4 * (size_t)B * G, cudaMemcpyDeviceToHost, s));
  if (out_steps && G) CU(cudaMemcpyAsync(out_steps, m->step_dig.p, 32 * (size_t)B * G, cudaMemcpyDeviceToHost, s));
  CU(cudaMemcpyAsync(out_witness, m->d_witness.p, 32 * (size_t)B, cudaMemcpyDeviceToHost, s));
  if (out_argmax) CU(cudaMemcpyAsync(out_argmax, m->d_argmax.p, 32 * (size_t)B, cudaMemcpyDeviceToHost, s));
  CU(cudaStreamSynchronize(s));
  CU(cudaStreamSynchronize(ss));
  float t_tot = 0, t_pre = 0, t_dec = 0, t_tail = 0;
  CU(cudaEventElapsedTime(&t_tot, m->ev0, m->ev_end));
  CU(cudaEventElapsedTime(&t_pre, m->ev0, m->ev_pref));
  CU(cudaEventElapsedTime(&t_dec, m->ev_pref, m->ev_dec));
  CU(cudaEventElapsedTime(&t_tail, m->ev_dec, m->ev_end));
  m->timing.total_ms = t_tot;
  m->timing.prefill_ms = t_pre;
  m->timing.decode_ms = t_dec;
  m->timing.witness_tail_ms = t_tail;
  m->timing.kernel_launches = m->launches;
  // bytes the call moved across PCIe: header bytes, offsets, states, prompt
  // ids and row maps in; tokens, digests out.
  m->timing.h2d_bytes = (int64_t)(hb.size() + 4 * hoff.size() + sizeof(ShaState) * st0.size() +
                                  4 * total_prompt + 4 * rtok.size() * 3 + 8 * osrc.size() +
                                  4 * (size_t)B * 6 + 8 * (size_t)B);
  m->timing.d2h_bytes = (int64_t)((out_tokens ? 4 * (size_t)B * G : 0) + (out_steps ? 32 * (size_t)B * G : 0) +
                                  32 * (size_t)B + (out_argmax ? 32 * (size_t)B : 0));
  for (auto &k : m->prof) k = cis2b_kernel_time{0, 0.0};
  for (const auto &pe : m->prof_events) {
    float ms = 0;
    CU(cudaEventElapsedTime(&ms, pe.a, pe.b));
    int ci = class_index(pe.cls);
    m->prof[ci].launches += 1;
    m->prof[ci].total_ms += ms;
  }
  return CIS2B_OK;
}

int logits_impl(cis2b_model *m, const uint32_t *ids, uint32_t n_prompt, uint32_t n_rows, float *out) {
  if (!m || !ids || !out) return fail(CIS2B_ERR_ARG, "NULL argument");
  if (n_prompt == 0 || n_rows == 0) return fail(CIS2B_ERR_ARG, "n_prompt and n_rows must be >= 1");
  CU(cudaSetDevice(m->dev));
  const int total = (int)(n_prompt + n_rows - 1);
  if (total > m->max_pos) return fail(CIS2B_ERR_ARG, "sequence exceeds max_positions");
  for (int i = 0; i < total; ++i)
    if (ids[i] >= (uint32_t)m->V) return fail(CIS2B_ERR_ARG, "id out of vocabulary range");
  int rc = alloc_cache(m, 1, total);
  if (rc) return rc;
  std::vector<uint32_t> tok(ids, ids + total);
  std::vector<int32_t> seq((size_t)total, 0), pos((size_t)total), osrc(n_rows), odst(n_rows);
  for (int i = 0; i < total; ++i) pos[(size_t)i] = i;
  for (uint32_t r = 0; r < n_rows; ++r) { osrc[r] = (int32_t)(n_prompt - 1 + r); odst[r] = (int32_t)r; }
  if (m->hlast.ensure(4 * (size_t)n_rows * m->H) || m->lnlast.ensure(4 * (size_t)round_up((int)n_rows, 64) * m->H) ||
      m->ring.ensure(4 * (size_t)n_rows * m->V) || ensure_act(m, 1))
    return fail(CIS2B_ERR_NOMEM, "device allocation failed");
  rc = prefill(m, tok, seq, pos, osrc, odst, 1, total);
  if (rc) return rc;
  rc = head_rows(m, m->hlast.as<float>(), (int)n_rows, m->ring.as<float>(), nullptr, 0);
  if (rc) return rc;
  CU(cudaMemcpyAsync(out, m->ring.p, 4 * (size_t)n_rows * m->V, cudaMemcpyDeviceToHost, m->s_main));
  CU(cudaStreamSynchronize(m->s_main));
  return CIS2B_OK;
}

template <class T>
struct Scoped {
  T *p = nullptr;
  ~Scoped() { if (p) cudaFree(p); }
};

// ------------------------------------------------------------------ trace
// Per-op trace (debug mode, off the timed path; cis2_model.h:482-496 and the
// emit points of cis2_forward_token, :685-760; q_norm / k_norm lines from
// labs/w1x-qwen3/scripts/qwen3-port.diff:66-80).  Every position of `ids`
// runs alone through the position-batched (prompt-pass) kernels, one row,
// so each op's output exists in device memory; its fp32 bits are copied out
// and hashed (SHA-256 over u32 LE) into one line per op:
//   pos=P layer=L op=NAME sha256=HEX      (layer -1 for embedding, final_norm, logits)
// The decode-step kernels fuse several of these ops and are checked against
// the same arithmetic by the parity tests.  Three outputs that no production
// kernel writes on its own are made here from production kernels: o_proj and
// down are the residual GEMMs run once without their residual; scores and
// softmax come from the attention kernel's trace output.
int trace_impl(cis2b_model *m, const uint32_t *ids, uint32_t n_ids, const char *path) {
  if (!m || !ids || !path) return fail(CIS2B_ERR_ARG, "NULL argument");
  if (n_ids == 0) return fail(CIS2B_ERR_ARG, "n_ids must be >= 1");
  if ((int)n_ids > m->max_pos) return fail(CIS2B_ERR_ARG, "ids exceed max_positions");
  for (uint32_t i = 0; i < n_ids; ++i)
    if (ids[i] >= (uint32_t)m->V) return fail(CIS2B_ERR_ARG, "id out of vocabulary range");
  CU(cudaSetDevice(m->dev));
  const int maxP = (int)n_ids, H = m->H, I = m->I, QD = m->QD, KVD = m->KVD, NQKV = QD + 2 * KVD;
  int rc = alloc_cache(m, 1, maxP);
  if (rc) return rc;
  rc = ensure_act(m, 1);
  if (rc) return rc;
  DevBuf d_tok, d_seq, d_pos, d_o, d_dbg, d_logits;
  if (d_tok.ensure(4) || d_seq.ensure(4) || d_pos.ensure(4) || d_o.ensure(4 * (size_t)H) ||
      d_dbg.ensure(4 * 2 * (size_t)m->NH * maxP) || d_logits.ensure(4 * (size_t)m->V) ||
      m->lnlast.ensure(4 * (size_t)64 * H))
    return fail(CIS2B_ERR_NOMEM, "device allocation of trace buffers failed");
  FILE *fp = fopen(path, "wb");
  if (!fp) return fail(CIS2B_ERR_IO, std::string("cannot write ") + path);
  struct Closer { FILE *f; ~Closer() { fclose(f); } } closer{fp};
  cudaStream_t s = m->s_main;
  const int ldm = m->act_ldm;
  std::vector<float> host;
  // Copies n floats (element stride `stride`) and writes the op's line.
  auto emit = [&](int pos, int layer, const char *op, const float *dev, size_t n, size_t stride) -> int {
    host.resize(n);
    if (stride == 1) CU(cudaMemcpyAsync(host.data(), dev, 4 * n, cudaMemcpyDeviceToHost, s));
    else CU(cudaMemcpy2DAsync(host.data(), 4, dev, 4 * stride, 4, n, cudaMemcpyDeviceToHost, s));
    CU(cudaStreamSynchronize(s));
    Sha256 h;
    for (float f : host) { uint32_t u; memcpy(&u, &f, 4); h.u32le(u); }
    uint8_t d[32];
    h.final(d);
    fprintf(fp, "pos=%d layer=%d op=%s sha256=%s\n", pos, layer, op, hex(d, 32).c_str());
    return CIS2B_OK;
  };
#define EMIT(...) do { int e_ = emit(__VA_ARGS__); if (e_) return e_; } while (0)
  float *h = m->h.as<float>(), *ln = m->ln.as<float>(), *qkv = m->qkv.as<float>();
  float *att = m->att.as<float>(), *gu = m->gu.as<float>(), *hid = m->hid.as<float>();
  float *o = d_o.as<float>(), *dbg = d_dbg.as<float>();
  const size_t layer_kv = (size_t)maxP * KVD;
  RowMap rm{d_seq.as<int32_t>(), d_pos.as<int32_t>()};
  const int32_t zero = 0;
  CU(cudaMemcpyAsync(d_seq.p, &zero, 4, cudaMemcpyHostToDevice, s));
  for (int pos = 0; pos < maxP; ++pos) {
    const int32_t p32 = pos;
    CU(cudaMemcpyAsync(d_tok.p, &ids[pos], 4, cudaMemcpyHostToDevice, s));
    CU(cudaMemcpyAsync(d_pos.p, &p32, 4, cudaMemcpyHostToDevice, s));
    launch_embed(m->embed, H, d_tok.as<uint32_t>(), 1, h, s);
    EMIT(pos, -1, "embedding", h, (size_t)H, 1);
    for (int l = 0; l < m->L; ++l) {
      const LayerW &w = m->layers[(size_t)l];
      float *kc = m->kc.as<float>() + (size_t)l * layer_kv, *vc = m->vc.as<float>() + (size_t)l * layer_kv;
      launch_rmsnorm(h, H, w.in_norm, m->eps, H, 1, m->tree, ln, 1, ldm, s);
      EMIT(pos, l, "norm1", ln, (size_t)H, (size_t)ldm);
      launch_gemm(ln, ldm, w.pqkv, w.fqkv, H, NQKV, 1, qkv, NQKV, nullptr, 0, m->tree, nullptr, 0, s);
      if (w.q_bias) launch_add_bias(qkv, NQKV, 1, w.q_bias, QD, s);
      if (w.k_bias) launch_add_bias(qkv + QD, NQKV, 1, w.k_bias, KVD, s);
      if (w.v_bias) launch_add_bias(qkv + QD + KVD, NQKV, 1, w.v_bias, KVD, s);
      EMIT(pos, l, "q", qkv, (size_t)QD, 1);
      EMIT(pos, l, "k", qkv + QD, (size_t)KVD, 1);
      EMIT(pos, l, "v", qkv + QD + KVD, (size_t)KVD, 1);
      if (w.q_norm || w.k_norm) {
        launch_qk_norm_row(qkv, m->NH, m->NKV, m->HD, w.q_norm, w.k_norm, m->eps, m->tree, s);
        if (w.q_norm) EMIT(pos, l, "q_norm", qkv, (size_t)QD, 1);
        if (w.k_norm) EMIT(pos, l, "k_norm", qkv + QD, (size_t)KVD, 1);
      }
      launch_qkv_post(qkv, NQKV, 1, rm, m->NH, m->NKV, m->HD, nullptr, nullptr, m->eps, m->tree,
                      m->cos_t.as<float>(), m->sin_t.as<float>(), kc, vc, maxP, s);
      EMIT(pos, l, "rope_q", qkv, (size_t)QD, 1);
      EMIT(pos, l, "rope_k", qkv + QD, (size_t)KVD, 1);
      launch_attention(qkv, NQKV, 1, rm, m->NH, m->NKV, m->HD, kc, vc, maxP, m->tree, att, 1, ldm, maxP, false,
                       nullptr, nullptr, m->eps, m->cos_t.as<float>(), m->sin_t.as<float>(), s, dbg);
      EMIT(pos, l, "scores", dbg, (size_t)m->NH * (pos + 1), 1);
      EMIT(pos, l, "softmax", dbg + (size_t)m->NH * (pos + 1), (size_t)m->NH * (pos + 1), 1);
      EMIT(pos, l, "attn_out", att, (size_t)QD, (size_t)ldm);
      launch_gemm(att, ldm, w.po, w.fo, QD, H, 1, o, H, nullptr, 0, m->tree, nullptr, 0, s);
      EMIT(pos, l, "o_proj", o, (size_t)H, 1);
      launch_gemm(att, ldm, w.po, w.fo, QD, H, 1, h, H, h, H, m->tree, nullptr, 0, s);
      EMIT(pos, l, "resid1", h, (size_t)H, 1);
      launch_rmsnorm(h, H, w.post_norm, m->eps, H, 1, m->tree, ln, 1, ldm, s);
      EMIT(pos, l, "norm2", ln, (size_t)H, (size_t)ldm);
      launch_gemm(ln, ldm, w.pgu, w.fgu, H, 2 * I, 1, gu, 2 * I, nullptr, 0, m->tree, nullptr, 0, s);
      EMIT(pos, l, "gate", gu, (size_t)I, 2);  // gate and up interleaved (launch_panelize)
      EMIT(pos, l, "up", gu + 1, (size_t)I, 2);
      launch_silu_mul(gu, I, 1, hid, 1, ldm, s);
      EMIT(pos, l, "silu_mul", hid, (size_t)I, (size_t)ldm);
      launch_gemm(hid, ldm, w.pdown, w.fdown, I, H, 1, o, H, nullptr, 0, m->tree, nullptr, 0, s);
      EMIT(pos, l, "down", o, (size_t)H, 1);
      launch_gemm(hid, ldm, w.pdown, w.fdown, I, H, 1, h, H, h, H, m->tree, nullptr, 0, s);
      EMIT(pos, l, "resid2", h, (size_t)H, 1);
    }
    launch_rmsnorm(h, H, m->final_norm, m->eps, H, 1, m->tree, m->lnlast.as<float>(), 1, 64, s);
    EMIT(pos, -1, "final_norm", m->lnlast.as<float>(), (size_t)H, 64);
    launch_gemm(m->lnlast.as<float>(), 64, m->lm_head_p, m->lm_head_f, H, m->V, 1, d_logits.as<float>(), m->V,
                nullptr, 0, m->tree, nullptr, 0, s);
    EMIT(pos, -1, "logits", d_logits.as<float>(), (size_t)m->V, 1);
    CU_LAUNCHED();
  }
#undef EMIT
  return CIS2B_OK;
}

}  // namespace

// ================================================================== C ABI
extern "C" {

const char *cis2b_last_error(void) { return g_err.c_str(); }

int cis2b_load(const char *weights_dir, const cis2b_opts *opts, cis2b_model **out) {
  if (!out) return fail(CIS2B_ERR_ARG, "out is NULL");
  *out = nullptr;
  cis2b_model *m = new (std::nothrow) cis2b_model();
  if (!m) return fail(CIS2B_ERR_NOMEM, "host allocation failed");
  int rc = load_impl(weights_dir, opts, m);
  if (rc) {
    cis2b_free(m);
    return rc;
  }
  *out = m;
  g_err.clear();
  return CIS2B_OK;
}

int cis2b_info_get(const cis2b_model *m, cis2b_info *out) {
  if (!m || !out) return fail(CIS2B_ERR_ARG, "NULL argument");
  *out = m->info;
  return CIS2B_OK;
}

int cis2b_generate(cis2b_model *m, const uint32_t *prompt_ids, const uint32_t *prompt_lens, uint32_t n_seq,
                   uint32_t gen_toks, const cis2b_sample *sample, uint32_t *out_tokens,
                   uint8_t *out_step_digests, uint8_t *out_witness, uint8_t *out_argmax) {
  int rc = generate_impl(m, prompt_ids, prompt_lens, n_seq, gen_toks, sample, out_tokens, out_step_digests,
                         out_witness, out_argmax);
  if (rc == CIS2B_OK) g_err.clear();
  return rc;
}

int cis2b_verify(cis2b_model *m, const uint32_t *prompt_ids, const uint32_t *prompt_lens, uint32_t n_seq,
                 const uint32_t *claimed, uint32_t gen_toks, const cis2b_sample *sample, uint32_t *out_tokens,
                 int32_t *out_first_mismatch, uint8_t *out_step_digests, uint8_t *out_witness,
                 uint8_t *out_argmax) {
  if (!claimed && n_seq && gen_toks) return fail(CIS2B_ERR_ARG, "claimed ids are NULL");
  std::vector<uint32_t> toks((size_t)n_seq * gen_toks + 1);
  static const uint32_t no_claim = 0;
  int rc = generate_impl(m, prompt_ids, prompt_lens, n_seq, gen_toks, sample, toks.data(), out_step_digests,
                         out_witness, out_argmax, claimed ? claimed : &no_claim);
  if (rc) return rc;
  for (uint32_t b = 0; b < n_seq; ++b) {
    int32_t first = -1;
    for (uint32_t t = 0; t < gen_toks; ++t)
      if (toks[(size_t)b * gen_toks + t] != claimed[(size_t)b * gen_toks + t]) { first = (int32_t)t; break; }
    if (out_first_mismatch) out_first_mismatch[b] = first;
  }
  if (out_tokens && n_seq && gen_toks) memcpy(out_tokens, toks.data(), 4 * (size_t)n_seq * gen_toks);
  g_err.clear();
  return CIS2B_OK;
}

int cis2b_last_timing(const cis2b_model *m, cis2b_timing *out) {
  if (!m || !out) return fail(CIS2B_ERR_ARG, "NULL argument");
  *out = m->timing;
  return CIS2B_OK;
}

int cis2b_profile(cis2b_model *m, uint32_t class_mask) {
  if (!m) return fail(CIS2B_ERR_ARG, "model is NULL");
  if (class_mask & ~15u) return fail(CIS2B_ERR_ARG, "unknown profile class bit");
  m->prof_mask = class_mask;
  return CIS2B_OK;
}

int cis2b_profile_read(const cis2b_model *m, uint32_t class_bit, cis2b_kernel_time *out) {
  if (!m || !out) return fail(CIS2B_ERR_ARG, "NULL argument");
  int ci = class_index(class_bit);
  if (ci < 0) return fail(CIS2B_ERR_ARG, "class_bit must be exactly one CIS2B_PROF_* bit");
  *out = m->prof[ci];
  return CIS2B_OK;
}

int cis2b_logits(cis2b_model *m, const uint32_t *ids, uint32_t n_prompt, uint32_t n_rows, float *out_logits) {
  int rc = logits_impl(m, ids, n_prompt, n_rows, out_logits);
  if (rc == CIS2B_OK) g_err.clear();
  return rc;
}

int cis2b_trace(cis2b_model *m, const uint32_t *ids, uint32_t n_ids, const char *trace_path) {
  int rc = trace_impl(m, ids, n_ids, trace_path);
  if (rc == CIS2B_OK) g_err.clear();
  return rc;
}

void cis2b_free(cis2b_model *m) {
  if (!m) return;
  cudaSetDevice(m->dev);
  if (m->s_main) cudaStreamSynchronize(m->s_main);
  if (m->s_sha) cudaStreamSynchronize(m->s_sha);
  if (m->s_prep) cudaStreamSynchronize(m->s_prep);
  for (cudaEvent_t e : m->ev_sha) cudaEventDestroy(e);
  for (int i = 0; i < 2; ++i) {
    if (m->ev_prep[i]) cudaEventDestroy(m->ev_prep[i]);
    if (m->ev_comp[i]) cudaEventDestroy(m->ev_comp[i]);
  }
  for (cudaEvent_t e : m->ev_pool) cudaEventDestroy(e);
  cudaEvent_t evs[] = {m->ev_sel, m->ev0, m->ev_pref, m->ev_dec, m->ev_end};
  for (cudaEvent_t e : evs)
    if (e) cudaEventDestroy(e);
  if (m->s_main) cudaStreamDestroy(m->s_main);
  if (m->s_sha) cudaStreamDestroy(m->s_sha);
  if (m->s_prep) cudaStreamDestroy(m->s_prep);
  delete m;
}

// ---------------------------------------------------------------- op entry points

int cis2b_op_pinned_map(int32_t device, int32_t fn, const float *x, float *y, size_t n) {
  if (!x || !y) return fail(CIS2B_ERR_ARG, "NULL buffer");
  if (fn < 0 || fn > 5) return fail(CIS2B_ERR_ARG, "unknown function id");
  CU(cudaSetDevice(device));
  Scoped<float> dx, dy;
  CU(cudaMalloc(&dx.p, 4 * n + 4));
  CU(cudaMalloc(&dy.p, 4 * n + 4));
  CU(cudaMemcpy(dx.p, x, 4 * n, cudaMemcpyHostToDevice));
  launch_pinned_map(fn, dx.p, dy.p, n, 0);
  CU_LAUNCHED();
  CU(cudaMemcpy(y, dy.p, 4 * n, cudaMemcpyDeviceToHost));
  return CIS2B_OK;
}

int cis2b_op_matmul(int32_t device, const uint16_t *W, const float *X, int32_t rows, int32_t n_out, int32_t k,
                    int32_t reduction, float *Y) {
  if (!W || !X || !Y) return fail(CIS2B_ERR_ARG, "NULL buffer");
  if (rows <= 0 || n_out <= 0 || k <= 0 || k % 8) return fail(CIS2B_ERR_ARG, "bad shape (k must be a multiple of 8)");
  if (reduction < 0 || reduction > CIS2B_OP_MATMUL_DECODE_TREE) return fail(CIS2B_ERR_ARG, "bad reduction");
  const bool dec_form = reduction >= CIS2B_OP_MATMUL_DECODE, dec_tree = reduction == CIS2B_OP_MATMUL_DECODE_TREE;
  if (dec_form && (rows > 1024 || !gemm_dec_ok(k, dec_tree)))
    return fail(CIS2B_ERR_ARG, "decode form: rows <= 1024 and k a multiple of 4 (tree order: of 32)");
  CU(cudaSetDevice(device));
  if (dec_form) {
    Scoped<uint16_t> dw, dt;
    Scoped<float> dx, dy;
    CU(cudaMalloc(&dw.p, 2 * (size_t)n_out * k));
    CU(cudaMalloc(&dt.p, 2 * tile32_elems(n_out, k)));
    CU(cudaMalloc(&dx.p, 4 * (size_t)rows * k));
    CU(cudaMalloc(&dy.p, 4 * (size_t)rows * n_out));
    CU(cudaMemcpy(dw.p, W, 2 * (size_t)n_out * k, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(dx.p, X, 4 * (size_t)rows * k, cudaMemcpyHostToDevice));
    launch_tile32(dw.p, n_out, k, dt.p, 0);
    launch_gemm_dec(dx.p, k, dt.p, k, n_out, rows, dy.p, n_out, nullptr, 0, nullptr, 0, 0, 0, dec_tree);
    CU_LAUNCHED();
    CU(cudaMemcpy(Y, dy.p, 4 * (size_t)rows * n_out, cudaMemcpyDeviceToHost));
    return CIS2B_OK;
  }
  // Same operand layouts as the decoder: W in 8-row panels, X k-major.
  const int ldm = round_up(rows, 4);
  std::vector<float> xt((size_t)k * ldm, 0.0f);
  for (int r = 0; r < rows; ++r)
    for (int i = 0; i < k; ++i) xt[(size_t)i * ldm + r] = X[(size_t)r * k + i];
  Scoped<uint16_t> dw, dp;
  Scoped<float> dx, dy, dpf;
  CU(cudaMalloc(&dw.p, 2 * (size_t)n_out * k));
  CU(cudaMalloc(&dp.p, 2 * panel_elems(n_out, k)));
  CU(cudaMalloc(&dpf.p, 4 * panel_elems(n_out, k)));
  CU(cudaMalloc(&dx.p, 4 * xt.size()));
  CU(cudaMalloc(&dy.p, 4 * (size_t)rows * n_out));
  CU(cudaMemcpy(dw.p, W, 2 * (size_t)n_out * k, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(dx.p, xt.data(), 4 * xt.size(), cudaMemcpyHostToDevice));
  launch_panelize(dw.p, n_out, k, dp.p, 0);
  launch_panelize(dw.p, n_out, k, dpf.p, 0);
  launch_gemm(dx.p, ldm, dp.p, dpf.p, k, n_out, rows, dy.p, n_out, nullptr, 0, reduction == CIS2B_REDUCTION_TREE,
              nullptr, 0, 0);
  CU_LAUNCHED();
  CU(cudaMemcpy(Y, dy.p, 4 * (size_t)rows * n_out, cudaMemcpyDeviceToHost));
  return CIS2B_OK;
}

int cis2b_op_gemm_tile(int32_t rows, int32_t n_out) {
  if (rows < 64 || n_out <= 0) return fail(CIS2B_ERR_ARG, "rows >= 64 and n_out >= 1"), -1;
  return gemm_big_choice(rows, n_out);
}

int cis2b_op_sha256_stream(int32_t device, const uint8_t *prefix, size_t prefix_len, const uint32_t *words,
                           uint32_t chunk_words, uint32_t n_chunks, uint8_t *out_digests) {
  if ((!prefix && prefix_len) || (!words && n_chunks) || !out_digests) return fail(CIS2B_ERR_ARG, "NULL buffer");
  if (chunk_words < 2 && n_chunks) return fail(CIS2B_ERR_ARG, "chunk_words must be >= 2");
  CU(cudaSetDevice(device));
  Scoped<ShaState> st;
  Scoped<uint8_t> pre, dig;
  Scoped<uint32_t> off, w, wk;
  ShaState s0;
  memset(&s0, 0, sizeof s0);
  const uint32_t iv[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                          0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
  memcpy(s0.h, iv, sizeof iv);
  CU(cudaMalloc(&st.p, sizeof(ShaState)));
  CU(cudaMemcpy(st.p, &s0, sizeof s0, cudaMemcpyHostToDevice));
  CU(cudaMalloc(&pre.p, prefix_len + 1));
  CU(cudaMalloc(&off.p, 8));
  uint32_t offs[2] = {0, (uint32_t)prefix_len};
  if (prefix_len) CU(cudaMemcpy(pre.p, prefix, prefix_len, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(off.p, offs, 8, cudaMemcpyHostToDevice));
  launch_sha_absorb_bytes(st.p, pre.p, off.p, 1, 0);
  const int V = (int)chunk_words - 1;
  CU(cudaMalloc(&w.p, 4 * (size_t)chunk_words * n_chunks + 4));
  CU(cudaMalloc(&wk.p, 4 * sha_wk_words(V, 1)));
  CU(cudaMalloc(&dig.p, 32 * (size_t)n_chunks + 32));
  if (n_chunks) CU(cudaMemcpy(w.p, words, 4 * (size_t)chunk_words * n_chunks, cudaMemcpyHostToDevice));
  for (uint32_t c = 0; c < n_chunks; ++c) {
    const uint32_t *base = w.p + (size_t)c * chunk_words;
    launch_sha_step(st.p, 1, reinterpret_cast<const float *>(base), V, (size_t)V, base + V, wk.p,
                    dig.p + 32 * (size_t)c, 32, 0);
  }
  CU_LAUNCHED();
  if (n_chunks) CU(cudaMemcpy(out_digests, dig.p, 32 * (size_t)n_chunks, cudaMemcpyDeviceToHost));
  else {
    launch_sha_finalize(st.p, 1, dig.p, 0);
    CU(cudaMemcpy(out_digests, dig.p, 32, cudaMemcpyDeviceToHost));
  }
  return CIS2B_OK;
}

int cis2b_op_sample(int32_t device, const float *logits, int32_t n, float temperature, float top_p, uint64_t seed,
                    uint64_t position, uint32_t *out_index) {
  if (!logits || !out_index || n <= 0) return fail(CIS2B_ERR_ARG, "bad argument");
  if (!(temperature > 0.0f) || !(top_p > 0.0f && top_p <= 1.0f)) return fail(CIS2B_ERR_ARG, "bad sampler parameters");
  if (position > 0x7fffffffull) return fail(CIS2B_ERR_ARG, "position must be below 2^31");
  CU(cudaSetDevice(device));
  Scoped<float> dl, scr;
  Scoped<uint32_t> nx;
  Scoped<int32_t> dp;
  CU(cudaMalloc(&dl.p, 4 * (size_t)n));
  CU(cudaMalloc(&scr.p, 4 * 5 * (size_t)n));
  CU(cudaMalloc(&nx.p, 4));
  CU(cudaMalloc(&dp.p, 4));
  int32_t pos32 = (int32_t)position;
  CU(cudaMemcpy(dl.p, logits, 4 * (size_t)n, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(dp.p, &pos32, 4, cudaMemcpyHostToDevice));
  launch_sample(dl.p, n, 1, nullptr, 0, temperature, top_p, seed, dp.p, scr.p, nx.p, 0);
  CU_LAUNCHED();
  CU(cudaMemcpy(out_index, nx.p, 4, cudaMemcpyDeviceToHost));
  return CIS2B_OK;
}

int cis2b_op_argmax(int32_t device, const float *logits, int32_t rows, int32_t n, uint32_t *out_index) {
  if (!logits || !out_index || rows <= 0 || n <= 0) return fail(CIS2B_ERR_ARG, "bad argument");
  CU(cudaSetDevice(device));
  Scoped<float> dl;
  Scoped<uint32_t> nx;
  CU(cudaMalloc(&dl.p, 4 * (size_t)rows * n));
  CU(cudaMalloc(&nx.p, 4 * (size_t)rows));
  CU(cudaMemcpy(dl.p, logits, 4 * (size_t)rows * n, cudaMemcpyHostToDevice));
  launch_argmax(dl.p, n, rows, nullptr, 0, nx.p, 0);
  CU_LAUNCHED();
  CU(cudaMemcpy(out_index, nx.p, 4 * (size_t)rows, cudaMemcpyDeviceToHost));
  return CIS2B_OK;
}

int cis2b_op_sample_gumbel(int32_t device, const float *logits, int32_t n, float temperature, uint32_t top_k,
                           float top_p, uint64_t seed, uint32_t step, uint32_t *out_index) {
  if (!logits || !out_index || n <= 0) return fail(CIS2B_ERR_ARG, "bad argument");
  if (!(temperature > 0.0f && temperature <= 3.402823466e38f) || !(top_p > 0.0f && top_p <= 1.0f))
    return fail(CIS2B_ERR_ARG, "bad sampler parameters");
  CU(cudaSetDevice(device));
  Scoped<float> dl, scr;
  Scoped<uint32_t> nx;
  Scoped<int32_t> dst;
  CU(cudaMalloc(&dl.p, 4 * (size_t)n));
  CU(cudaMalloc(&scr.p, 4 * 5 * (size_t)n));
  CU(cudaMalloc(&nx.p, 4));
  CU(cudaMalloc(&dst.p, 4));
  CU(cudaMemcpy(dl.p, logits, 4 * (size_t)n, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(dst.p, &step, 4, cudaMemcpyHostToDevice));
  launch_sample_gumbel(dl.p, n, 1, nullptr, 0, temperature, top_k, top_p, seed, dst.p, scr.p, nx.p, 0);
  CU_LAUNCHED();
  CU(cudaMemcpy(out_index, nx.p, 4, cudaMemcpyDeviceToHost));
  return CIS2B_OK;
}

}  // extern "C"
