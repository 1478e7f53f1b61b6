// cis2b_ref -- command-line front end of libcis2b.so that prints the
// reference's stdout contract, so harnesses that parse the reference's
// lines by regex keep working unchanged:
//   weights_sha256= / tokenizer_sha256= / config_sha256= / table_digest= /
//   inv_freq_table_digest= / prompt_idx=N prompt_tokens=[..] / run1_tokens= /
//   run1_witness_digest= / run1_argmax_digest= / reduction_mode= /
//   CIS2_REF digest=<hex> prompt_idx=N prompt_toks=N gen_toks=N dtype=fp32 reduction_mode=M
// (code/cis2-fp/gpu/cis2_host.cpp:222-245; src/main.rs:1231-1262) and, in
// sampled mode, the E23 line
//   CIS2_SAMPLE digest=<hex> mode=sampled seed=S temperature=T top_p=P prompt_idx=N ...
// (code/patches/cis2-fp__cm_e23-pinned-sampling.patch:770-779).  With
// --sample SEED,T,K,P (the seeded Gumbel-max clause "CIS2-SAMPLE-1", flag as
// in labs/w1x-sample/reports/w1x-sample/RESULTS-hq-builder.md:11-12) the
// lines are the greedy ones, the digest being that of the sampled run.
//
//   cis2b_ref --weights-dir D --ids F [--gen-toks N] [--reduction sequential|tree]
//             [--mode greedy|sampled --seed S --temperature T --top-p P]
//             [--sample SEED,T,K,P] [--receipt F] [--arch-gate reference|qwen3-port]
//             [--device I] [--prompt-idx I] [--step-digests] [--trace F] [--verify2]
// With --trace F the first prompt's run is also written to F as the
// reference's per-op trace (code/cis2-fp/gpu/cis2_host.cpp:76, 173-208):
// one "pos=P layer=L op=NAME sha256=HEX" line per op of every position, the
// prompt's and the generated tokens', so `make gate`-style diffs against the
// reference's trace work with this binary (see cis2b_trace in cis2b.h).
// The architecture gate runs on config.json first, as in the reference
// (code/cis2-fp/src/main.rs:812-823): a refused checkpoint prints the two
// CIS2_REF_UNSUPPORTED lines and exits 2 whatever else is missing; a failure
// after the gate admitted the checkpoint (say, absent weights) exits 101, the
// status the reference's panic gives, so refusal suites
// (code/cis2-fp/tests/fixtures/run_refusal_suite.sh) tell the two apart.
// With --receipt F (one line of claimed generated ids per prompt, all the
// same length) the prompts are VERIFIED instead of decoded: one
// teacher-forced pass (cis2b_verify), and per prompt the lines
//   CIS2_VERIFY3 digest=<hex> prompt_idx=N prompt_toks=N gen_toks=N dtype=fp32
//   CIS2_VERIFY3 argmax_digest= / table_digest= / inv_freq_table_digest=
//   CIS2_VERIFY3 generated_token_ids=a,b,... / first_mismatch_pos=K
// of code/cis2-fp/verify3/main.c:272-318; exit status 1 if any claim differs.
// Each non-empty line of F is one prompt (decimal ids); all prompts are
// decoded as one batch and reported in file order.
// With --verify2 the run is the spec's pinned reference vector unless --ids
// and --gen-toks say otherwise: prompt "Once upon a time" as its token ids
// 6403 1980 253 655 (the ids code/cis2-fp/verify2/src/main.rs:446-451
// asserts after tokenising), 16 greedy tokens; the output is then the five
// lines of that verifier (verify2/src/main.rs:489-500)
//   CIS2_VERIFY2 digest=<hex> prompt_toks=4 gen_toks=16 dtype=fp32 / argmax_digest= /
//   table_digest= / inv_freq table_digest= / generated_token_ids=[a, b, ...]
// which the receipt server parses (code/cis2-llm/server/app/runner.py:25-88);
// its witness is the same byte stream as CIS2_REF's.
#include "cis2b.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

static std::string hexs(const uint8_t *b, size_t n) {
  static const char *d = "0123456789abcdef";
  std::string s;
  for (size_t i = 0; i < n; ++i) { s.push_back(d[b[i] >> 4]); s.push_back(d[b[i] & 15]); }
  return s;
}

static std::string ids_list(const uint32_t *v, size_t n) {
  std::string s = "[";
  for (size_t i = 0; i < n; ++i) {
    if (i) s += ", ";
    s += std::to_string(v[i]);
  }
  return s + "]";
}

// Shortest decimal that reads back as the same f32 (how Rust prints f32).
static std::string f32_str(float x) {
  char buf[64];
  for (int p = 1; p <= 9; ++p) {
    snprintf(buf, sizeof buf, "%.*g", p, (double)x);
    if (strtof(buf, nullptr) == x) break;
  }
  return buf;
}

// Lines of decimal ids separated by blanks or commas; empty lines skipped.
static bool read_id_lines(const std::string &path, std::vector<std::vector<uint32_t>> &lines) {
  FILE *f = fopen(path.c_str(), "rb");
  if (!f) { fprintf(stderr, "FATAL: cannot open %s\n", path.c_str()); return false; }
  std::vector<uint32_t> cur;
  std::string num;
  int c;
  auto flush_num = [&]() {
    if (!num.empty()) { cur.push_back((uint32_t)strtoul(num.c_str(), nullptr, 10)); num.clear(); }
  };
  bool ok = true;
  while ((c = fgetc(f)) != EOF) {
    if (c >= '0' && c <= '9') num.push_back((char)c);
    else if (c == '\n') { flush_num(); if (!cur.empty()) lines.push_back(cur); cur.clear(); }
    else if (c == ' ' || c == '\t' || c == ',' || c == '\r') flush_num();
    else { fprintf(stderr, "FATAL: %s: unexpected character\n", path.c_str()); ok = false; break; }
  }
  flush_num();
  if (!cur.empty()) lines.push_back(cur);
  fclose(f);
  return ok;
}

int main(int argc, char **argv) {
  std::string weights_dir = "weights", ids_path, receipt_path, trace_path;
  int gen = 16, device = 0, prompt_idx = 0;
  bool tree = false, sampled = false, gumbel = false, step_digests = false, verify2 = false;
  int arch_gate = CIS2B_GATE_REFERENCE;
  cis2b_sample smp{0, 0.8f, 0.95f, CIS2B_SAMPLE_E23, 0};
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() -> const char * {
      if (i + 1 >= argc) { fprintf(stderr, "FATAL: %s needs a value\n", a.c_str()); exit(2); }
      return argv[++i];
    };
    if (a == "--weights-dir") weights_dir = next();
    else if (a == "--ids") ids_path = next();
    else if (a == "--gen-toks") gen = atoi(next());
    else if (a == "--verify2") verify2 = true;
    else if (a == "--device") device = atoi(next());
    else if (a == "--prompt-idx") prompt_idx = atoi(next());
    else if (a == "--step-digests") step_digests = true;
    else if (a == "--reduction") {
      std::string v = next();
      if (v == "tree") tree = true;
      else if (v != "sequential") { fprintf(stderr, "FATAL: --reduction sequential|tree\n"); return 2; }
    } else if (a == "--mode") {
      std::string v = next();
      if (v == "sampled") sampled = true;
      else if (v != "greedy") { fprintf(stderr, "FATAL: --mode greedy|sampled\n"); return 2; }
    } else if (a == "--sample") {
      // SEED,T,K,P: decimal seed, temperature and top_p as strtof reads them, top_k
      std::string v = next();
      unsigned long long sd = 0;
      unsigned k = 0;
      char tbuf[64], pbuf[64];
      if (sscanf(v.c_str(), "%llu,%63[^,],%u,%63s", &sd, tbuf, &k, pbuf) != 4) {
        fprintf(stderr, "FATAL: --sample SEED,T,K,P\n");
        return 2;
      }
      smp.seed = sd;
      smp.temperature = strtof(tbuf, nullptr);
      smp.top_k = k;
      smp.top_p = strtof(pbuf, nullptr);
      smp.scheme = CIS2B_SAMPLE_GUMBEL;
      gumbel = true;
    } else if (a == "--arch-gate") {
      std::string v = next();
      if (v == "qwen3-port") arch_gate = CIS2B_GATE_QWEN3_PORT;
      else if (v != "reference") { fprintf(stderr, "FATAL: --arch-gate reference|qwen3-port\n"); return 2; }
    } else if (a == "--receipt") receipt_path = next();
    else if (a == "--trace") trace_path = next();
    else if (a == "--seed") smp.seed = strtoull(next(), nullptr, 10);
    else if (a == "--temperature") smp.temperature = strtof(next(), nullptr);
    else if (a == "--top-p") smp.top_p = strtof(next(), nullptr);
    else { fprintf(stderr, "FATAL: unknown CLI argument: %s\n", a.c_str()); return 2; }
  }
  if (gen < 0) { fprintf(stderr, "FATAL: --gen-toks must be >= 0\n"); return 2; }

  std::vector<std::vector<uint32_t>> prompts, claims;
  if (!ids_path.empty()) {
    if (!read_id_lines(ids_path, prompts)) return 2;
    if (prompts.empty()) { fprintf(stderr, "FATAL: %s: no token ids\n", ids_path.c_str()); return 2; }
  } else if (verify2) {
    prompts.push_back({6403u, 1980u, 253u, 655u});  // "Once upon a time"
  }
  if (verify2 && (sampled || gumbel || tree)) {
    fprintf(stderr, "FATAL: --verify2 is the greedy sequential vector\n");
    return 2;
  }
  const bool verify = !receipt_path.empty();
  if (verify) {
    if (!read_id_lines(receipt_path, claims)) return 2;
    if (claims.size() != prompts.size()) {
      fprintf(stderr, "FATAL: %s: %zu claim lines for %zu prompts\n", receipt_path.c_str(), claims.size(),
              prompts.size());
      return 2;
    }
    gen = claims.empty() ? 0 : (int)claims[0].size();
    for (auto &c : claims)
      if ((int)c.size() != gen) { fprintf(stderr, "FATAL: %s: claim lines differ in length\n", receipt_path.c_str()); return 2; }
  }

  cis2b_opts o{};
  o.device = device;
  o.arch_gate = arch_gate;
  o.reduction = tree ? CIS2B_REDUCTION_TREE : CIS2B_REDUCTION_SEQUENTIAL;
  size_t maxp = 0;
  for (auto &p : prompts) maxp = p.size() > maxp ? p.size() : maxp;
  o.max_positions = (int32_t)(maxp + (size_t)gen > 4096 ? maxp + (size_t)gen : 4096);
  cis2b_model *m = nullptr;
  const int lrc = cis2b_load(weights_dir.c_str(), &o, &m);
  if (lrc == CIS2B_ERR_CONFIG) {  // the reference's refusal lines (code/cis2-fp/src/main.rs:818-822)
    fprintf(stderr, "CIS2_REF_UNSUPPORTED reason=%s\n", cis2b_last_error());
    fprintf(stderr, "This checkpoint is outside the CIS-2 specified subset; no digest emitted.\n");
    return 2;
  }
  if (lrc != CIS2B_OK) {
    fprintf(stderr, "FATAL: %s\n", cis2b_last_error());
    return 101;
  }
  if (prompts.empty()) {
    fprintf(stderr, "FATAL: --ids FILE is required\n");
    cis2b_free(m);
    return 2;
  }
  cis2b_info info;
  cis2b_info_get(m, &info);

  const uint32_t n = (uint32_t)prompts.size();
  std::vector<uint32_t> flat, lens;
  for (auto &p : prompts) { flat.insert(flat.end(), p.begin(), p.end()); lens.push_back((uint32_t)p.size()); }
  std::vector<uint32_t> toks((size_t)n * gen);
  std::vector<uint8_t> steps((size_t)n * gen * 32), wit((size_t)n * 32), arg((size_t)n * 32);
  if (sampled && gumbel) {
    fprintf(stderr, "FATAL: --mode sampled (E23) and --sample (CIS2-SAMPLE-1) exclude each other\n");
    return 2;
  }
  const cis2b_sample *sp = (sampled || gumbel) ? &smp : nullptr;
  if (verify) {
    std::vector<uint32_t> cl;
    for (auto &c : claims) cl.insert(cl.end(), c.begin(), c.end());
    std::vector<int32_t> first(n);
    if (cis2b_verify(m, flat.data(), lens.data(), n, cl.data(), (uint32_t)gen, sp, toks.data(), first.data(),
                     nullptr, wit.data(), arg.data()) != CIS2B_OK) {
      fprintf(stderr, "FATAL: %s\n", cis2b_last_error());
      cis2b_free(m);
      return 2;
    }
    int bad = 0;
    for (uint32_t s = 0; s < n; ++s) {
      const int pi = prompt_idx + (int)s;
      printf("CIS2_VERIFY3 digest=%s prompt_idx=%d prompt_toks=%u gen_toks=%d dtype=fp32\n",
             hexs(&wit[(size_t)s * 32], 32).c_str(), pi, lens[s], gen);
      printf("CIS2_VERIFY3 argmax_digest=%s\n", hexs(&arg[(size_t)s * 32], 32).c_str());
      printf("CIS2_VERIFY3 table_digest=%s\n", hexs(info.table_digest, 32).c_str());
      printf("CIS2_VERIFY3 inv_freq_table_digest=%s\n", hexs(info.inv_freq_table_digest, 32).c_str());
      printf("CIS2_VERIFY3 generated_token_ids=");
      for (int t = 0; t < gen; ++t) printf("%s%u", t ? "," : "", toks[(size_t)s * gen + t]);
      printf("\nCIS2_VERIFY3 first_mismatch_pos=%d\n", first[s]);
      bad += first[s] >= 0;
    }
    cis2b_free(m);
    return bad ? 1 : 0;
  }
  if (cis2b_generate(m, flat.data(), lens.data(), n, (uint32_t)gen, sp, toks.data(), steps.data(), wit.data(),
                     arg.data()) != CIS2B_OK) {
    fprintf(stderr, "FATAL: %s\n", cis2b_last_error());
    cis2b_free(m);
    return 2;
  }
  if (!trace_path.empty()) {
    std::vector<uint32_t> run(prompts[0]);
    run.insert(run.end(), toks.begin(), toks.begin() + gen);
    if (cis2b_trace(m, run.data(), (uint32_t)run.size(), trace_path.c_str()) != CIS2B_OK) {
      fprintf(stderr, "FATAL: %s\n", cis2b_last_error());
      cis2b_free(m);
      return 2;
    }
  }
  if (verify2) {
    for (uint32_t s = 0; s < n; ++s) {
      printf("CIS2_VERIFY2 digest=%s prompt_toks=%u gen_toks=%d dtype=fp32\n", hexs(&wit[(size_t)s * 32], 32).c_str(),
             lens[s], gen);
      printf("argmax_digest=%s\n", hexs(&arg[(size_t)s * 32], 32).c_str());
      printf("table_digest=%s\n", hexs(info.table_digest, 32).c_str());
      printf("inv_freq table_digest=%s\n", hexs(info.inv_freq_table_digest, 32).c_str());
      printf("generated_token_ids=%s\n", ids_list(toks.data() + (size_t)s * gen, (size_t)gen).c_str());
    }
    cis2b_free(m);
    return 0;
  }
  printf("weights_sha256=%s\n", hexs(info.weights_sha256, 32).c_str());
  printf("tokenizer_sha256=%s\n", hexs(info.tokenizer_sha256, 32).c_str());
  printf("config_sha256=%s\n", hexs(info.config_sha256, 32).c_str());
  printf("table_digest=%s\n", hexs(info.table_digest, 32).c_str());
  printf("inv_freq_table_digest=%s\n", hexs(info.inv_freq_table_digest, 32).c_str());
  const char *mode = tree ? "tree" : "sequential";
  size_t off = 0;
  for (uint32_t s = 0; s < n; ++s) {
    const int pi = prompt_idx + (int)s;
    const uint32_t *p = flat.data() + off;
    off += lens[s];
    std::vector<uint32_t> all(p, p + lens[s]);
    all.insert(all.end(), toks.begin() + (size_t)s * gen, toks.begin() + (size_t)(s + 1) * gen);
    printf("prompt_idx=%d prompt_tokens=%s\n", pi, ids_list(p, lens[s]).c_str());
    printf("prompt_idx=%d run1_tokens=%s\n", pi, ids_list(all.data(), all.size()).c_str());
    printf("prompt_idx=%d run1_witness_digest=%s\n", pi, hexs(&wit[(size_t)s * 32], 32).c_str());
    printf("prompt_idx=%d run1_argmax_digest=%s\n", pi, hexs(&arg[(size_t)s * 32], 32).c_str());
    if (step_digests)
      for (int t = 0; t < gen; ++t)
        printf("prompt_idx=%d step=%d witness=%s\n", pi, t,
               hexs(&steps[((size_t)s * gen + t) * 32], 32).c_str());
    printf("prompt_idx=%d reduction_mode=%s\n", pi, mode);
    if (sampled)
      printf("CIS2_SAMPLE digest=%s mode=sampled seed=%llu temperature=%s top_p=%s prompt_idx=%d "
             "prompt_toks=%u gen_toks=%d dtype=fp32\n",
             hexs(&wit[(size_t)s * 32], 32).c_str(), (unsigned long long)smp.seed,
             f32_str(smp.temperature).c_str(), f32_str(smp.top_p).c_str(), pi, lens[s], gen);
    else
      printf("CIS2_REF digest=%s prompt_idx=%d prompt_toks=%u gen_toks=%d dtype=fp32 reduction_mode=%s\n",
             hexs(&wit[(size_t)s * 32], 32).c_str(), pi, lens[s], gen, mode);
  }
  cis2b_free(m);
  return 0;
}
