// artifact.hpp — θ_v artifact reader (INTEGER_LLM/runtime/src/loader.rs:322-560),
// host side: weights_manifest.json and luts.json, every file checked against
// its shape and SHA-256 before anything is accepted, then 2-D tensors
// registered on the device with myl_weight_register / myl_weight16_register.
//
// Included by myl_w8a16.cu (uses its fail() / TRY machinery).
#pragma once

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

namespace myl_artifact_detail {

// ---- SHA-256 (FIPS 180-4) -----------------------------------------------------
// The constants are derived exactly instead of transcribed: K[i] is the first
// 32 fractional bits of the cube root of the i-th prime and H0[i] those of the
// square root, i.e. floor(root(p * 2^(32 n))) mod 2^32 with an integer root.
using u128 = unsigned __int128;

static uint32_t frac_root_bits(uint64_t p, int n) {
  const u128 target = u128(p) << (32 * n);
  u128 lo = 0, hi = u128(1) << 36;  // root < 2^36 for p < 2^12, n <= 3
  while (lo < hi) {                 // largest r with r^n <= target
    const u128 mid = (lo + hi + 1) >> 1;
    u128 pw = 1;
    for (int i = 0; i < n; ++i) pw *= mid;
    if (pw <= target) lo = mid;
    else hi = mid - 1;
  }
  return uint32_t(uint64_t(lo) & 0xFFFFFFFFull);
}

struct Sha256Tables {
  uint32_t k[64], h0[8];
  Sha256Tables() {
    uint64_t primes[64];
    int n = 0;
    for (uint64_t c = 2; n < 64; ++c) {
      bool prime = true;
      for (uint64_t d = 2; d * d <= c; ++d)
        if (c % d == 0) { prime = false; break; }
      if (prime) primes[n++] = c;
    }
    for (int i = 0; i < 64; ++i) k[i] = frac_root_bits(primes[i], 3);
    for (int i = 0; i < 8; ++i) h0[i] = frac_root_bits(primes[i], 2);
  }
};

static const Sha256Tables& sha_tables() {
  static const Sha256Tables t;
  return t;
}

static inline uint32_t rotr(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }

// Incremental form: update() any number of times, then finish().
struct Sha256Stream {
  uint32_t h[8];
  uint8_t buf[64];
  size_t fill = 0;
  uint64_t total = 0;

  Sha256Stream() {
    const Sha256Tables& T = sha_tables();
    for (int i = 0; i < 8; ++i) h[i] = T.h0[i];
  }

  void block(const uint8_t* blk) {
    const Sha256Tables& T = sha_tables();
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t(blk[4 * i]) << 24) | (uint32_t(blk[4 * i + 1]) << 16) |
             (uint32_t(blk[4 * i + 2]) << 8) | uint32_t(blk[4 * i + 3]);
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      const uint32_t ch = (e & f) ^ (~e & g);
      const uint32_t t1 = hh + S1 + ch + T.k[i] + w[i];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
      const uint32_t t2 = S0 + mj;
      hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }

  void update(const uint8_t* data, size_t len) {
    total += len;
    if (fill) {
      const size_t take = std::min(len, size_t(64) - fill);
      std::memcpy(buf + fill, data, take);
      fill += take;
      data += take;
      len -= take;
      if (fill < 64) return;
      block(buf);
      fill = 0;
    }
    for (; len >= 64; data += 64, len -= 64) block(data);
    if (len) {
      std::memcpy(buf, data, len);
      fill = len;
    }
  }

  void finish(uint8_t out[32]) {
    const uint64_t bits = total * 8;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (fill != 56) update(&zero, 1);
    uint8_t len_be[8];
    for (int i = 0; i < 8; ++i) len_be[i] = uint8_t(bits >> (56 - 8 * i));
    update(len_be, 8);
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < 4; ++j) out[4 * i + j] = uint8_t(h[i] >> (24 - 8 * j));
  }
};

static void sha256(const uint8_t* data, size_t len, uint8_t out[32]) {
  Sha256Stream st;
  st.update(data, len);
  st.finish(out);
}

static std::string sha256_hex(const std::vector<uint8_t>& v) {
  uint8_t d[32];
  sha256(v.data(), v.size(), d);
  static const char* hex = "0123456789abcdef";
  std::string s(64, '0');
  for (int i = 0; i < 32; ++i) {
    s[size_t(2 * i)] = hex[d[i] >> 4];
    s[size_t(2 * i + 1)] = hex[d[i] & 15];
  }
  return s;
}

// ---- a small JSON reader (objects, arrays, strings, numbers, literals) ---------
struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonParser {
  const std::string& s;
  size_t i = 0;
  std::string err;
  explicit JsonParser(const std::string& src) : s(src) {}
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool fail_at(const char* what) {
    if (err.empty()) err = std::string(what) + " at byte " + std::to_string(i);
    return false;
  }
  bool parse_string(std::string& out) {
    if (i >= s.size() || s[i] != '"') return fail_at("expected a string");
    ++i;
    while (i < s.size() && s[i] != '"') {
      char c = s[i++];
      if (c == '\\') {
        if (i >= s.size()) return fail_at("bad escape");
        const char e = s[i++];
        switch (e) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (i + 4 > s.size()) return fail_at("bad \\u escape");
            const unsigned cp = unsigned(std::stoul(s.substr(i, 4), nullptr, 16));
            i += 4;
            if (cp < 0x80) out += char(cp);  // names and files are ASCII; others kept as UTF-8
            else if (cp < 0x800) { out += char(0xC0 | (cp >> 6)); out += char(0x80 | (cp & 0x3F)); }
            else { out += char(0xE0 | (cp >> 12)); out += char(0x80 | ((cp >> 6) & 0x3F)); out += char(0x80 | (cp & 0x3F)); }
            break;
          }
          default: return fail_at("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (i >= s.size()) return fail_at("unterminated string");
    ++i;
    return true;
  }
  bool parse(Json& v, int depth = 0) {
    if (depth > 64) return fail_at("nesting too deep");
    ws();
    if (i >= s.size()) return fail_at("unexpected end");
    const char c = s[i];
    if (c == '{') {
      v.kind = Json::OBJ;
      ++i;
      ws();
      if (i < s.size() && s[i] == '}') { ++i; return true; }
      for (;;) {
        ws();
        std::string k;
        if (!parse_string(k)) return false;
        ws();
        if (i >= s.size() || s[i] != ':') return fail_at("expected ':'");
        ++i;
        Json val;
        if (!parse(val, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(val));
        ws();
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        if (i < s.size() && s[i] == '}') { ++i; return true; }
        return fail_at("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::ARR;
      ++i;
      ws();
      if (i < s.size() && s[i] == ']') { ++i; return true; }
      for (;;) {
        Json val;
        if (!parse(val, depth + 1)) return false;
        v.arr.push_back(std::move(val));
        ws();
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        if (i < s.size() && s[i] == ']') { ++i; return true; }
        return fail_at("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Json::STR;
      return parse_string(v.str);
    }
    if (s.compare(i, 4, "true") == 0) { v.kind = Json::BOOL; v.b = true; i += 4; return true; }
    if (s.compare(i, 5, "false") == 0) { v.kind = Json::BOOL; v.b = false; i += 5; return true; }
    if (s.compare(i, 4, "null") == 0) { v.kind = Json::NUL; i += 4; return true; }
    const size_t start = i;
    while (i < s.size() && (std::isdigit(static_cast<unsigned char>(s[i])) || s[i] == '-' ||
                            s[i] == '+' || s[i] == '.' || s[i] == 'e' || s[i] == 'E'))
      ++i;
    if (i == start) return fail_at("unexpected character");
    v.kind = Json::NUM;
    v.num = std::strtod(s.substr(start, i - start).c_str(), nullptr);
    return true;
  }
};

static bool read_file(const std::string& path, std::vector<uint8_t>& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  out.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  return true;
}

static bool as_int(const Json* j, int64_t& v) {
  if (!j || j->kind != Json::NUM) return false;
  v = int64_t(j->num);
  return double(v) == j->num;
}

}  // namespace myl_artifact_detail

// One tensor of weights_manifest.json.
struct ArtifactTensor {
  std::string key, original_name, file;
  int dtype = 0;  // 1 = int8, 2 = int16
  std::vector<int64_t> shape;
  std::vector<uint8_t> bytes;   // as read (little-endian int16 for dtype 2)
  std::vector<uint8_t> shifts;  // one per row (shape[0])
};

struct myl_artifact {
  std::vector<ArtifactTensor> tensors;
  std::map<std::string, std::vector<int16_t>> luts;
};
