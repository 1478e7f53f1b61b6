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
// A parsed JSON text held as one flat array of nodes.  Containers list
// their children by node index; an object's children alternate key, value.
// Strings are decoded to UTF-8 (\uXXXX escapes included, surrogate pairs
// joined), numbers are checked against the JSON grammar and converted once
// with strtod (correctly rounded decimal -> f64; the loader narrows eps to
// f32 from that f64 afterwards).  Access goes through JsonRef, a (document,
// node) pair that is empty when a lookup misses, so chained lookups need no
// null checks.
class JsonDoc;

class JsonRef {
 public:
  enum Type { None, Null, Bool, Number, String, Array, Object };
  JsonRef() = default;
  JsonRef(const JsonDoc *d, int n) : doc_(d), node_(n) {}
  explicit operator bool() const { return doc_ && node_ >= 0; }
  inline Type type() const;
  bool is(Type t) const { return type() == t; }
  inline bool boolean() const;        // Bool's value (false otherwise)
  inline double number() const;       // Number's value (0 otherwise)
  inline const std::string &text() const;  // String's value ("" otherwise)
  inline size_t size() const;         // Array items / Object members
  inline JsonRef item(size_t i) const;           // i-th Array item
  inline JsonRef operator[](const char *key) const;  // Object member (first match)

 private:
  const JsonDoc *doc_ = nullptr;
  int node_ = -1;
};

class JsonDoc {
 public:
  // Parses [b, e); on failure returns false with a message in `err`.
  bool parse(const char *b, const char *e, std::string &err) {
    nodes_.clear();
    cur_ = b;
    end_ = e;
    err_.clear();
    int root = parse_value(0);
    skip_space();
    if (root >= 0 && cur_ != end_) root = error("trailing characters after the top-level value");
    err = err_;
    return root >= 0;
  }
  JsonRef root() const { return nodes_.empty() ? JsonRef() : JsonRef(this, 0); }

 private:
  friend class JsonRef;
  struct Node {
    JsonRef::Type type = JsonRef::Null;
    bool flag = false;
    double value = 0.0;
    std::string text;
    std::vector<int> kids;
  };
  std::vector<Node> nodes_;
  const char *cur_ = nullptr, *end_ = nullptr;
  std::string err_;
  static const std::string &empty() {
    static const std::string e;
    return e;
  }

  int error(const char *what) {
    if (err_.empty()) err_ = what;
    cur_ = end_;
    return -1;
  }
  void skip_space() {
    while (cur_ < end_ && (*cur_ == ' ' || *cur_ == '\n' || *cur_ == '\r' || *cur_ == '\t')) ++cur_;
  }
  int add(JsonRef::Type t) {
    nodes_.emplace_back();
    nodes_.back().type = t;
    return (int)nodes_.size() - 1;
  }
  bool literal(const char *word) {
    size_t n = strlen(word);
    if ((size_t)(end_ - cur_) < n || memcmp(cur_, word, n) != 0) return false;
    cur_ += n;
    return true;
  }
  static void put_utf8(std::string &out, uint32_t cp) {
    if (cp < 0x80) {
      out.push_back((char)cp);
    } else if (cp < 0x800) {
      out.push_back((char)(0xC0 | (cp >> 6)));
      out.push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      out.push_back((char)(0xE0 | (cp >> 12)));
      out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back((char)(0x80 | (cp & 0x3F)));
    } else {
      out.push_back((char)(0xF0 | (cp >> 18)));
      out.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
      out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back((char)(0x80 | (cp & 0x3F)));
    }
  }
  bool hex4(uint32_t &cp) {
    if (end_ - cur_ < 4) return false;
    cp = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *cur_++;
      int d = (c >= '0' && c <= '9') ? c - '0' : (c >= 'a' && c <= 'f') ? c - 'a' + 10
                                                : (c >= 'A' && c <= 'F') ? c - 'A' + 10 : -1;
      if (d < 0) return false;
      cp = cp * 16 + (uint32_t)d;
    }
    return true;
  }
  // Reads a string token (cur_ at the opening quote) into `out`.
  bool read_string(std::string &out) {
    ++cur_;
    while (cur_ < end_) {
      unsigned char c = (unsigned char)*cur_++;
      if (c == '"') return true;
      if (c < 0x20) return false;  // raw control characters are not allowed
      if (c != '\\') { out.push_back((char)c); continue; }
      if (cur_ >= end_) return false;
      char esc = *cur_++;
      switch (esc) {
        case '"': case '\\': case '/': out.push_back(esc); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          uint32_t cp;
          if (!hex4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: a low one must follow
            uint32_t lo;
            if (end_ - cur_ < 2 || cur_[0] != '\\' || cur_[1] != 'u') return false;
            cur_ += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            return false;
          }
          put_utf8(out, cp);
          break;
        }
        default: return false;
      }
    }
    return false;
  }
  // Number per the JSON grammar: -? (0 | [1-9][0-9]*) (.[0-9]+)? ([eE][+-]?[0-9]+)?
  int parse_number() {
    const char *s = cur_;
    auto digits = [&]() {
      const char *d = cur_;
      while (cur_ < end_ && *cur_ >= '0' && *cur_ <= '9') ++cur_;
      return cur_ > d;
    };
    if (cur_ < end_ && *cur_ == '-') ++cur_;
    if (cur_ < end_ && *cur_ == '0') ++cur_;
    else if (!digits()) return error("malformed number");
    if (cur_ < end_ && *cur_ == '.') { ++cur_; if (!digits()) return error("malformed number"); }
    if (cur_ < end_ && (*cur_ == 'e' || *cur_ == 'E')) {
      ++cur_;
      if (cur_ < end_ && (*cur_ == '+' || *cur_ == '-')) ++cur_;
      if (!digits()) return error("malformed number");
    }
    const std::string lexeme(s, cur_);  // strtod must not read past the token
    int n = add(JsonRef::Number);
    nodes_[(size_t)n].value = strtod(lexeme.c_str(), nullptr);
    return n;
  }
  int parse_value(int depth) {
    if (depth > 64) return error("nesting deeper than 64 levels");
    skip_space();
    if (cur_ >= end_) return error("unexpected end of input");
    const char c = *cur_;
    if (c == '"') {
      std::string t;
      if (!read_string(t)) return error("malformed string");
      int n = add(JsonRef::String);
      nodes_[(size_t)n].text = std::move(t);
      return n;
    }
    if (c == '{' || c == '[') {
      const bool obj = c == '{';
      const char close = obj ? '}' : ']';
      int n = add(obj ? JsonRef::Object : JsonRef::Array);
      ++cur_;
      skip_space();
      if (cur_ < end_ && *cur_ == close) { ++cur_; return n; }
      for (;;) {
        if (obj) {
          skip_space();
          if (cur_ >= end_ || *cur_ != '"') return error("object key must be a string");
          std::string key;
          if (!read_string(key)) return error("malformed object key");
          int k = add(JsonRef::String);
          nodes_[(size_t)k].text = std::move(key);
          nodes_[(size_t)n].kids.push_back(k);
          skip_space();
          if (cur_ >= end_ || *cur_ != ':') return error("expected ':' after an object key");
          ++cur_;
        }
        int v = parse_value(depth + 1);
        if (v < 0) return -1;
        nodes_[(size_t)n].kids.push_back(v);
        skip_space();
        if (cur_ < end_ && *cur_ == ',') { ++cur_; continue; }
        if (cur_ < end_ && *cur_ == close) { ++cur_; return n; }
        return error(obj ? "expected ',' or '}'" : "expected ',' or ']'");
      }
    }
    if (literal("true")) { int n = add(JsonRef::Bool); nodes_[(size_t)n].flag = true; return n; }
    if (literal("false")) return add(JsonRef::Bool);
    if (literal("null")) return add(JsonRef::Null);
    if (c == '-' || (c >= '0' && c <= '9')) return parse_number();
    return error("unexpected character");
  }
};

JsonRef::Type JsonRef::type() const { return *this ? doc_->nodes_[(size_t)node_].type : None; }
bool JsonRef::boolean() const { return is(Bool) && doc_->nodes_[(size_t)node_].flag; }
double JsonRef::number() const { return is(Number) ? doc_->nodes_[(size_t)node_].value : 0.0; }
const std::string &JsonRef::text() const { return is(String) ? doc_->nodes_[(size_t)node_].text : JsonDoc::empty(); }
size_t JsonRef::size() const {
  if (is(Array)) return doc_->nodes_[(size_t)node_].kids.size();
  if (is(Object)) return doc_->nodes_[(size_t)node_].kids.size() / 2;
  return 0;
}
JsonRef JsonRef::item(size_t i) const {
  if (!is(Array) || i >= size()) return JsonRef();
  return JsonRef(doc_, doc_->nodes_[(size_t)node_].kids[i]);
}
JsonRef JsonRef::operator[](const char *key) const {
  if (!is(Object)) return JsonRef();
  const std::vector<int> &k = doc_->nodes_[(size_t)node_].kids;
  for (size_t i = 0; i + 1 < k.size(); i += 2)
    if (doc_->nodes_[(size_t)k[i]].text == key) return JsonRef(doc_, k[i + 1]);
  return JsonRef();
}

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
