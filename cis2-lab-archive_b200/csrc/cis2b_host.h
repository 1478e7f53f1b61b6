// cis2b_host.h -- host-side plumbing for the CIS-2 runtime: a minimal JSON
// reader (config.json and the safetensors header), the safetensors index,
// and SHA-256 for the artifact hashes (spec §12.1 items 1-3).
#pragma once
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <utility>
#include <vector>

namespace cis2b {

// ------------------------------------------------------------------ JSON
struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0.0;  // strtod: correctly rounded decimal -> f64
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json *get(const char *k) const {
    if (kind != OBJ) return nullptr;
    for (auto &kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class JsonParser {
 public:
  JsonParser(const char *p, const char *e) : p_(p), e_(e) {}
  bool parse(Json &out, std::string &err) {
    ok_ = true;
    value(out, 0);
    ws();
    if (ok_ && p_ != e_) fail("trailing characters");
    err = err_;
    return ok_;
  }

 private:
  const char *p_, *e_;
  bool ok_ = true;
  std::string err_;
  void fail(const char *m) {
    if (ok_) err_ = m;
    ok_ = false;
    p_ = e_;
  }
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  void str(std::string &s) {
    if (p_ >= e_ || *p_ != '"') return fail("expected string");
    ++p_;
    while (p_ < e_ && *p_ != '"') {
      char c = *p_++;
      if (c != '\\') { s.push_back(c); continue; }
      if (p_ >= e_) return fail("bad escape");
      char x = *p_++;
      switch (x) {
        case 'n': s.push_back('\n'); break;
        case 't': s.push_back('\t'); break;
        case 'r': s.push_back('\r'); break;
        case 'b': s.push_back('\b'); break;
        case 'f': s.push_back('\f'); break;
        case 'u': {
          if (e_ - p_ < 4) return fail("bad \\u");
          unsigned v = (unsigned)strtoul(std::string(p_, 4).c_str(), nullptr, 16);
          p_ += 4;
          s.push_back(v < 0x80 ? (char)v : '?');
          break;
        }
        default: s.push_back(x);
      }
    }
    if (p_ >= e_) return fail("unterminated string");
    ++p_;
  }
  void value(Json &v, int depth) {
    if (depth > 64) return fail("nesting too deep");
    ws();
    if (p_ >= e_) return fail("unexpected end");
    char c = *p_;
    if (c == '{') {
      v.kind = Json::OBJ;
      ++p_;
      ws();
      if (p_ < e_ && *p_ == '}') { ++p_; return; }
      while (ok_) {
        ws();
        std::string k;
        str(k);
        ws();
        if (p_ >= e_ || *p_ != ':') return fail("expected ':'");
        ++p_;
        Json child;
        value(child, depth + 1);
        v.obj.emplace_back(std::move(k), std::move(child));
        ws();
        if (p_ < e_ && *p_ == ',') { ++p_; continue; }
        if (p_ < e_ && *p_ == '}') { ++p_; return; }
        return fail("expected ',' or '}'");
      }
      return;
    }
    if (c == '[') {
      v.kind = Json::ARR;
      ++p_;
      ws();
      if (p_ < e_ && *p_ == ']') { ++p_; return; }
      while (ok_) {
        Json child;
        value(child, depth + 1);
        v.arr.push_back(std::move(child));
        ws();
        if (p_ < e_ && *p_ == ',') { ++p_; continue; }
        if (p_ < e_ && *p_ == ']') { ++p_; return; }
        return fail("expected ',' or ']'");
      }
      return;
    }
    if (c == '"') { v.kind = Json::STR; return str(v.str); }
    if (e_ - p_ >= 4 && !memcmp(p_, "true", 4)) { v.kind = Json::BOOL; v.b = true; p_ += 4; return; }
    if (e_ - p_ >= 5 && !memcmp(p_, "false", 5)) { v.kind = Json::BOOL; p_ += 5; return; }
    if (e_ - p_ >= 4 && !memcmp(p_, "null", 4)) { p_ += 4; return; }
    // number: copy the lexeme so strtod never reads past the buffer
    const char *q = p_;
    while (q < e_ && (strchr("+-0123456789.eE", *q) != nullptr)) ++q;
    if (q == p_) return fail("expected value");
    std::string lex(p_, q);
    char *stop = nullptr;
    v.num = strtod(lex.c_str(), &stop);
    if (stop != lex.c_str() + lex.size()) return fail("bad number");
    v.kind = Json::NUM;
    p_ = q;
  }
};

// ------------------------------------------------------------------ SHA-256 (host)
class Sha256 {
 public:
  Sha256() { reset(); }
  void reset() {
    static const uint32_t iv[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    memcpy(h_, iv, sizeof iv);
    len_ = 0;
    n_ = 0;
  }
  void update(const void *data, size_t n) {
    const uint8_t *p = (const uint8_t *)data;
    len_ += n;
    if (n_) {
      size_t t = 64 - n_;
      if (t > n) t = n;
      memcpy(buf_ + n_, p, t);
      n_ += t; p += t; n -= t;
      if (n_ == 64) { block(buf_); n_ = 0; }
    }
    while (n >= 64) { block(p); p += 64; n -= 64; }
    if (n) { memcpy(buf_, p, n); n_ = n; }
  }
  void u32le(uint32_t v) {
    uint8_t b[4] = {(uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24)};
    update(b, 4);
  }
  void final(uint8_t out[32]) const {
    Sha256 c = *this;
    uint64_t bits = c.len_ * 8;
    uint8_t pad[72] = {0x80};
    size_t padn = (c.n_ < 56) ? 56 - c.n_ : 120 - c.n_;
    for (int i = 0; i < 8; ++i) pad[padn + i] = (uint8_t)(bits >> (56 - 8 * i));
    c.update(pad, padn + 8);
    for (int i = 0; i < 8; ++i) {
      out[4 * i] = (uint8_t)(c.h_[i] >> 24); out[4 * i + 1] = (uint8_t)(c.h_[i] >> 16);
      out[4 * i + 2] = (uint8_t)(c.h_[i] >> 8); out[4 * i + 3] = (uint8_t)c.h_[i];
    }
  }

 private:
  uint32_t h_[8];
  uint64_t len_;
  uint8_t buf_[64];
  size_t n_;
  static uint32_t ror(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void block(const uint8_t *p) {
    static const uint32_t K[64] = {
        0x428a2f98u,0x71374491u,0xb5c0fbcfu,0xe9b5dba5u,0x3956c25bu,0x59f111f1u,0x923f82a4u,0xab1c5ed5u,
        0xd807aa98u,0x12835b01u,0x243185beu,0x550c7dc3u,0x72be5d74u,0x80deb1feu,0x9bdc06a7u,0xc19bf174u,
        0xe49b69c1u,0xefbe4786u,0x0fc19dc6u,0x240ca1ccu,0x2de92c6fu,0x4a7484aau,0x5cb0a9dcu,0x76f988dau,
        0x983e5152u,0xa831c66du,0xb00327c8u,0xbf597fc7u,0xc6e00bf3u,0xd5a79147u,0x06ca6351u,0x14292967u,
        0x27b70a85u,0x2e1b2138u,0x4d2c6dfcu,0x53380d13u,0x650a7354u,0x766a0abbu,0x81c2c92eu,0x92722c85u,
        0xa2bfe8a1u,0xa81a664bu,0xc24b8b70u,0xc76c51a3u,0xd192e819u,0xd6990624u,0xf40e3585u,0x106aa070u,
        0x19a4c116u,0x1e376c08u,0x2748774cu,0x34b0bcb5u,0x391c0cb3u,0x4ed8aa4au,0x5b9cca4fu,0x682e6ff3u,
        0x748f82eeu,0x78a5636fu,0x84c87814u,0x8cc70208u,0x90befffau,0xa4506cebu,0xbef9a3f7u,0xc67178f2u};
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = ((uint32_t)p[4 * i] << 24) | ((uint32_t)p[4 * i + 1] << 16) |
             ((uint32_t)p[4 * i + 2] << 8) | (uint32_t)p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      uint32_t s0 = ror(w[i - 15], 7) ^ ror(w[i - 15], 18) ^ (w[i - 15] >> 3);
      uint32_t s1 = ror(w[i - 2], 17) ^ ror(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], hh = h_[7];
    for (int i = 0; i < 64; ++i) {
      uint32_t t1 = hh + (ror(e, 6) ^ ror(e, 11) ^ ror(e, 25)) + ((e & f) ^ (~e & g)) + K[i] + w[i];
      uint32_t t2 = (ror(a, 2) ^ ror(a, 13) ^ ror(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d; h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += hh;
  }
};

inline bool read_file(const std::string &path, std::string &out) {
  FILE *f = fopen(path.c_str(), "rb");
  if (!f) return false;
  if (fseek(f, 0, SEEK_END) != 0) { fclose(f); return false; }
  long n = ftell(f);
  if (n < 0) { fclose(f); return false; }
  fseek(f, 0, SEEK_SET);
  out.resize((size_t)n);
  bool ok = n == 0 || fread(&out[0], 1, (size_t)n, f) == (size_t)n;
  fclose(f);
  return ok;
}

inline std::string hex(const uint8_t *b, size_t n) {
  static const char *d = "0123456789abcdef";
  std::string s;
  for (size_t i = 0; i < n; ++i) { s.push_back(d[b[i] >> 4]); s.push_back(d[b[i] & 15]); }
  return s;
}

}  // namespace cis2b
