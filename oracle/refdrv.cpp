// oracle/refdrv.cpp -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// A thin driver around the reference's own single-source C++ port
// (code/cis2-fp/gpu/cis2_model.h, cis2_math.h, cis2_sha256.h, cis2_fpenv.h),
// compiled from the reference's header files where they lie, with the
// reference's own host flags (code/cis2-fp/gpu/Makefile:46-58).  Every
// arithmetic operation on the decode path is the reference's:
//   cis2_forward_token   (cis2_model.h:685-760)
//   cis2_argmax          (cis2_model.h:764-774)
//   Cis2Sha256           (cis2_sha256.h:12-111)
//   cis2_table_digest / cis2_build_inv_freq (cis2_model.h:414-476)
//
// What this driver adds over the reference's cis2_host.cpp main():
//   * many sequences per process (one ids line each), workspace reused;
//   * a per-step witness digest: SHA-256 finalised on a COPY of the running
//     witness state after each step's update, so the last one equals the
//     final CIS2_REF digest (cis2_host.cpp:196-214);
//   * the E23 pinned sampler (no C/C++ source exists in the reference; this is
//     a restatement of code/patches/cis2-fp__cm_e23-pinned-sampling.patch,
//     src/sampling.rs hunk, lines 619-725) with its witness prefix
//     "CIS2_SAMPLE_V1" || seed || T || top_p before the header (patch :610-624);
//   * per-phase wall-clock timings for the CPU baseline and, with
//     --step-times, the time at which every decode step ended.
// It prints one JSON object per sequence.
//
// Build variants (oracle/Makefile): sequential, -DCIS2_REDUCTION_TREE, and a
// Qwen3 variant built against a patched copy of the headers
// (labs/w1x-qwen3/scripts/qwen3-port.diff) with -DREFDRV_QWEN3.

#include "cis2_fpenv.h"
#include "cis2_math.h"
#include "cis2_model.h"
#include "cis2_sha256.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <string>
#include <vector>

static double now_s() {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static std::vector<std::vector<uint32_t>> read_id_lines(const std::string &path) {
  std::string text = cis2_read_file(path);
  std::vector<std::vector<uint32_t>> out;
  std::vector<uint32_t> cur;
  size_t i = 0;
  while (i <= text.size()) {
    char c = i < text.size() ? text[i] : '\n';
    if (c == '\n') {
      if (!cur.empty()) out.push_back(cur);
      cur.clear();
      ++i;
      continue;
    }
    if (c >= '0' && c <= '9') {
      size_t j = i;
      while (j < text.size() && text[j] >= '0' && text[j] <= '9') ++j;
      cur.push_back((uint32_t)strtoul(text.substr(i, j - i).c_str(), nullptr, 10));
      i = j;
      continue;
    }
    ++i;  // separators: space, tab, comma, CR
  }
  return out;
}

// ---- E23 pinned sampler (restated from the sampling.rs text) -------------
static uint64_t sm64_round(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static uint64_t rng_word(uint64_t seed, uint64_t position) {
  return sm64_round(seed ^ sm64_round(position));
}
static double uniform01(uint64_t word) {
  return (double)(word >> 11) * (1.0 / 9007199254740992.0);  // 2^-53
}

static uint32_t sample_pinned(const float *logits, int n, float temperature, float top_p,
                              uint64_t seed, uint64_t position) {
  std::vector<float> probs((size_t)n);
  for (int i = 0; i < n; ++i) probs[(size_t)i] = logits[i] / temperature;
  float max_v = probs[0];
  for (int i = 1; i < n; ++i)
    if (probs[(size_t)i] > max_v) max_v = probs[(size_t)i];
  for (int i = 0; i < n; ++i) probs[(size_t)i] = cis2_exp_pinned(probs[(size_t)i] - max_v);
  float denom = cis2_sum_seq(probs.data(), n);
  for (int i = 0; i < n; ++i) probs[(size_t)i] = probs[(size_t)i] / denom;
  std::vector<uint32_t> order((size_t)n);
  for (int i = 0; i < n; ++i) order[(size_t)i] = (uint32_t)i;
  std::sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
    float pa = probs[a], pb = probs[b];
    if (pa != pb) return pa > pb;
    return a < b;
  });
  float cum = 0.0f;
  size_t nucleus = order.size();
  for (size_t i = 0; i < order.size(); ++i) {
    cum = cum + probs[order[i]];
    if (cum >= top_p) { nucleus = i + 1; break; }
  }
  float total = 0.0f;
  for (size_t i = 0; i < nucleus; ++i) total = total + probs[order[i]];
  double u = uniform01(rng_word(seed, position));
  float cdf = 0.0f;
  for (size_t i = 0; i < nucleus; ++i) {
    float p = probs[order[i]] / total;
    cdf = cdf + p;
    if ((double)cdf > u) return order[i];
  }
  return order[nucleus - 1];
}

int main(int argc, char **argv) {
  cis2_fpenv_init();

  std::string weights_dir = "weights", ids_path, out_path;
  int gen_toks = 16, first = 0, count = -1;
  bool step_digests = false, sampled = false, step_times = false;
  uint64_t seed = 0;
  float temperature = 0.8f, top_p = 0.95f;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    if (a == "--weights-dir" && i + 1 < argc) weights_dir = argv[++i];
    else if (a == "--ids" && i + 1 < argc) ids_path = argv[++i];
    else if (a == "--gen-toks" && i + 1 < argc) gen_toks = atoi(argv[++i]);
    else if (a == "--first" && i + 1 < argc) first = atoi(argv[++i]);
    else if (a == "--count" && i + 1 < argc) count = atoi(argv[++i]);
    else if (a == "--out" && i + 1 < argc) out_path = argv[++i];
    else if (a == "--step-digests") step_digests = true;
    else if (a == "--step-times") step_times = true;
    else if (a == "--sample" && i + 3 < argc) {
      sampled = true;
      seed = strtoull(argv[++i], nullptr, 10);
      temperature = strtof(argv[++i], nullptr);
      top_p = strtof(argv[++i], nullptr);
    } else { fprintf(stderr, "FATAL: unknown argument %s\n", a.c_str()); return 2; }
  }
  if (ids_path.empty()) { fprintf(stderr, "FATAL: --ids FILE required\n"); return 2; }

  double t_load0 = now_s();
  const std::string weights_path = weights_dir + "/model.safetensors";
  const std::string tokenizer_path = weights_dir + "/tokenizer.json";
  const std::string config_path = weights_dir + "/config.json";
  unsigned char weights_sha[32], tokenizer_sha[32], config_sha[32];
  cis2_sha256_file(weights_path, weights_sha);
  cis2_sha256_file(tokenizer_path, tokenizer_sha);
  cis2_sha256_file(config_path, config_sha);

  // Config exactly as cis2_host.cpp:97-117 (+ qwen3-port.diff:109-110).
  Cis2Json cfg = cis2_json_parse(cis2_read_file(config_path));
  auto need = [&](const char *k) -> const Cis2Json & {
    const Cis2Json *v = cfg.get(k);
    if (!v) { fprintf(stderr, "FATAL: config.json missing %s\n", k); exit(2); }
    return *v;
  };
  Cis2Model model;
  model.hidden = (int)need("hidden_size").num;
  model.inter = (int)need("intermediate_size").num;
  model.n_layers = (int)need("num_hidden_layers").num;
  model.n_heads = (int)need("num_attention_heads").num;
  model.n_kv_heads = (int)need("num_key_value_heads").num;
  model.vocab = (int)need("vocab_size").num;
  model.eps = (float)need("rms_norm_eps").num;
  const double rope_theta = need("rope_theta").num;
  model.head_dim = model.hidden / model.n_heads;
#ifdef REFDRV_QWEN3
  if (const Cis2Json *hd = cfg.get("head_dim")) model.head_dim = (int)hd->num;
  model.q_dim = model.n_heads * model.head_dim;
  const size_t QD = (size_t)model.q_dim;
#else
  if (cfg.get("head_dim") && (int)cfg.get("head_dim")->num != model.head_dim) {
    fprintf(stderr, "FATAL: explicit head_dim needs the Qwen3 build (refdrv_qwen3)\n");
    return 2;
  }
  const size_t QD = (size_t)model.hidden;
#endif
  bool tie = true;
  if (const Cis2Json *t = cfg.get("tie_word_embeddings"))
    tie = (t->kind == Cis2Json::BOOL) ? t->b : true;

  unsigned char table_dig[32];
  cis2_table_digest(table_dig);
  cis2_build_inv_freq(model, rope_theta);

  Cis2SafeTensors st;
  st.open(weights_path);
  const size_t H = (size_t)model.hidden, I = (size_t)model.inter;
  const size_t KV = (size_t)model.n_kv_heads * (size_t)model.head_dim;
  const size_t V = (size_t)model.vocab;
  model.embed_tokens = st.load_bf16("model.embed_tokens.weight", {V, H});
  model.layers.resize((size_t)model.n_layers);
  for (int i = 0; i < model.n_layers; ++i) {
    char nb[160];
    auto nm = [&](const char *suffix) {
      snprintf(nb, sizeof(nb), "model.layers.%d.%s", i, suffix);
      return std::string(nb);
    };
    Cis2Layer &L = model.layers[(size_t)i];
    L.input_layernorm = st.load_bf16(nm("input_layernorm.weight"), {H});
    L.post_attention_layernorm = st.load_bf16(nm("post_attention_layernorm.weight"), {H});
    L.q_proj = st.load_bf16(nm("self_attn.q_proj.weight"), {QD, H});
    L.k_proj = st.load_bf16(nm("self_attn.k_proj.weight"), {KV, H});
    L.v_proj = st.load_bf16(nm("self_attn.v_proj.weight"), {KV, H});
    L.o_proj = st.load_bf16(nm("self_attn.o_proj.weight"), {H, QD});
    L.gate_proj = st.load_bf16(nm("mlp.gate_proj.weight"), {I, H});
    L.up_proj = st.load_bf16(nm("mlp.up_proj.weight"), {I, H});
    L.down_proj = st.load_bf16(nm("mlp.down_proj.weight"), {H, I});
    L.q_bias = st.has(nm("self_attn.q_proj.bias")) ? st.load_bf16(nm("self_attn.q_proj.bias"), {QD}) : nullptr;
    L.k_bias = st.has(nm("self_attn.k_proj.bias")) ? st.load_bf16(nm("self_attn.k_proj.bias"), {KV}) : nullptr;
    L.v_bias = st.has(nm("self_attn.v_proj.bias")) ? st.load_bf16(nm("self_attn.v_proj.bias"), {KV}) : nullptr;
#ifdef REFDRV_QWEN3
    const size_t HD = (size_t)model.head_dim;
    L.q_norm = st.has(nm("self_attn.q_norm.weight")) ? st.load_bf16(nm("self_attn.q_norm.weight"), {HD}) : nullptr;
    L.k_norm = st.has(nm("self_attn.k_norm.weight")) ? st.load_bf16(nm("self_attn.k_norm.weight"), {HD}) : nullptr;
#else
    if (st.has(nm("self_attn.q_norm.weight"))) {
      fprintf(stderr, "FATAL: q_norm tensors need the Qwen3 build (refdrv_qwen3)\n");
      return 2;
    }
#endif
  }
  model.final_norm = st.load_bf16("model.norm.weight", {H});
  model.lm_head = tie ? nullptr : st.load_bf16("lm_head.weight", {V, H});
  st.blob.clear();
  st.blob.shrink_to_fit();
  double t_load = now_s() - t_load0;

  std::vector<std::vector<uint32_t>> seqs = read_id_lines(ids_path);
  int last = count < 0 ? (int)seqs.size() : std::min((int)seqs.size(), first + count);
  size_t max_prompt = 0;
  for (int s = first; s < last; ++s) max_prompt = std::max(max_prompt, seqs[(size_t)s].size());

  FILE *out = stdout;
  if (!out_path.empty()) {
    out = fopen(out_path.c_str(), "w");
    if (!out) { fprintf(stderr, "FATAL: cannot write %s\n", out_path.c_str()); return 2; }
  }
  fprintf(out, "{\"kind\":\"header\",\"weights_sha256\":\"%s\",\"tokenizer_sha256\":\"%s\","
               "\"config_sha256\":\"%s\",\"table_digest\":\"%s\",\"inv_freq_table_digest\":\"%s\","
               "\"load_s\":%.6f,\"reduction_mode\":\"%s\"}\n",
          cis2_hex(weights_sha, 32).c_str(), cis2_hex(tokenizer_sha, 32).c_str(),
          cis2_hex(config_sha, 32).c_str(), cis2_hex(table_dig, 32).c_str(),
          cis2_hex(model.inv_freq_table_digest, 32).c_str(), t_load,
#ifdef CIS2_REDUCTION_TREE
          "tree"
#else
          "sequential"
#endif
  );
  fflush(out);

  Cis2Workspace ws;
  ws.alloc(model, (int)max_prompt + gen_toks);
  std::vector<float> logits((size_t)model.vocab);

  for (int s = first; s < last; ++s) {
    const std::vector<uint32_t> &prompt = seqs[(size_t)s];
    double t0 = now_s();
    Cis2Sha256 witness;
    if (sampled) {
      const char tag[] = "CIS2_SAMPLE_V1";
      witness.update(tag, 14);
      unsigned char le[8];
      for (int i = 0; i < 8; ++i) le[i] = (unsigned char)((seed >> (8 * i)) & 0xFF);
      witness.update(le, 8);
      witness.update_u32le(cis2_f32_bits(temperature));
      witness.update_u32le(cis2_f32_bits(top_p));
    }
    witness.update(weights_sha, 32);
    witness.update(tokenizer_sha, 32);
    witness.update(config_sha, 32);
    witness.update(table_dig, 32);
    witness.update(model.inv_freq_table_digest, 32);
    for (size_t i = 0; i < prompt.size(); ++i) witness.update_u32le(prompt[i]);

    std::vector<uint32_t> all = prompt;
    for (size_t pos = 0; pos < prompt.size(); ++pos)
      cis2_forward_token(model, ws, (int)pos, prompt[pos], nullptr);
    cis2_download(logits.data(), ws.logits, (size_t)model.vocab);
    double t1 = now_s();

    std::vector<std::string> step_hex;
    std::vector<double> step_end;  // seconds since the decode started, after each step's forward
    Cis2Sha256 steps_hash;
    for (int step = 0; step < gen_toks; ++step) {
      uint32_t next_id;
      if (sampled)
        next_id = sample_pinned(logits.data(), model.vocab, temperature, top_p, seed,
                                (uint64_t)(prompt.size() + (size_t)step));
      else
        next_id = cis2_argmax(logits.data(), model.vocab);
      for (int i = 0; i < model.vocab; ++i) witness.update_u32le(cis2_f32_bits(logits[(size_t)i]));
      witness.update_u32le(next_id);
      {
        Cis2Sha256 copy = witness;
        unsigned char d[32];
        copy.finalize(d);
        steps_hash.update(d, 32);
        if (step_digests) step_hex.push_back(cis2_hex(d, 32));
      }
      all.push_back(next_id);
      int pos = (int)prompt.size() + step;
      // The reference computes one more forward after the last draw
      // (cis2_host.cpp:208); its logits never enter the witness, so it is
      // skipped for the final step here.
      if (step + 1 < gen_toks) {
        cis2_forward_token(model, ws, pos, next_id, nullptr);
        cis2_download(logits.data(), ws.logits, (size_t)model.vocab);
      }
      if (step_times) step_end.push_back(now_s() - t1);
    }
    double t2 = now_s();
    unsigned char wdig[32], adig[32], sdig[32];
    witness.finalize(wdig);
    Cis2Sha256 ah;
    for (size_t i = 0; i < all.size(); ++i) ah.update_u32le(all[i]);
    ah.finalize(adig);
    steps_hash.finalize(sdig);

    fprintf(out, "{\"kind\":\"seq\",\"seq\":%d,\"prompt_toks\":%zu,\"gen_toks\":%d,\"tokens\":[", s,
            prompt.size(), gen_toks);
    for (size_t i = prompt.size(); i < all.size(); ++i)
      fprintf(out, "%s%u", i == prompt.size() ? "" : ",", all[i]);
    fprintf(out, "],\"witness\":\"%s\",\"argmax\":\"%s\",\"steps_sha\":\"%s\"",
            cis2_hex(wdig, 32).c_str(), cis2_hex(adig, 32).c_str(), cis2_hex(sdig, 32).c_str());
    if (step_digests) {
      fprintf(out, ",\"step_digests\":[");
      for (size_t i = 0; i < step_hex.size(); ++i)
        fprintf(out, "%s\"%s\"", i ? "," : "", step_hex[i].c_str());
      fprintf(out, "]");
    }
    if (step_times) {
      fprintf(out, ",\"step_end_s\":[");
      for (size_t i = 0; i < step_end.size(); ++i) fprintf(out, "%s%.6f", i ? "," : "", step_end[i]);
      fprintf(out, "]");
    }
    fprintf(out, ",\"prefill_s\":%.6f,\"decode_s\":%.6f}\n", t1 - t0, t2 - t1);
    fflush(out);
  }
  if (out != stdout) fclose(out);
  ws.free_all();
  return 0;
}
