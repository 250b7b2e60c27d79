// SHA-256 from FIPS 180-4 section 6.2, and a strict recursive-descent JSON reader.
#include "vb/contract.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <set>
#include <sstream>

namespace vb {
namespace {

// FIPS 180-4 section 4.2.2: first 32 bits of the fractional parts of the cube
// roots of the first 64 primes.
const uint32_t K[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void compress(uint32_t h[8], const unsigned char* block) {
  uint32_t w[64];
  for (int t = 0; t < 16; ++t)
    w[t] = (uint32_t)block[4 * t] << 24 | (uint32_t)block[4 * t + 1] << 16 | (uint32_t)block[4 * t + 2] << 8 |
           (uint32_t)block[4 * t + 3];
  for (int t = 16; t < 64; ++t) {
    uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
    uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
    w[t] = w[t - 16] + s0 + w[t - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
  for (int t = 0; t < 64; ++t) {
    uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    uint32_t ch = (e & f) ^ (~e & g);
    uint32_t t1 = hh + S1 + ch + K[t] + w[t];
    uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    uint32_t t2 = S0 + maj;
    hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

}  // namespace

std::string sha256_hex(const std::string& data) {
  // FIPS 180-4 section 5.3.3 initial hash value.
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  std::string msg = data;
  uint64_t bits = (uint64_t)data.size() * 8;
  msg.push_back((char)0x80);
  while (msg.size() % 64 != 56) msg.push_back('\0');
  for (int i = 7; i >= 0; --i) msg.push_back((char)((bits >> (8 * i)) & 0xff));
  for (size_t off = 0; off < msg.size(); off += 64) compress(h, reinterpret_cast<const unsigned char*>(msg.data()) + off);
  char out[65];
  for (int i = 0; i < 8; ++i) snprintf(out + 8 * i, 9, "%08x", h[i]);
  return std::string(out, 64);
}

namespace {

class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}
  Json document() {
    Json v = value(0);
    ws();
    if (p_ != s_.size()) fail("trailing data");
    return v;
  }

 private:
  [[noreturn]] void fail(const std::string& m) { throw JsonError("json: " + m + " at " + std::to_string(p_)); }
  void ws() { while (p_ < s_.size() && (s_[p_] == ' ' || s_[p_] == '\n' || s_[p_] == '\t' || s_[p_] == '\r')) ++p_; }
  bool lit(const char* w) {
    size_t n = strlen(w);
    if (s_.compare(p_, n, w) == 0) { p_ += n; return true; }
    return false;
  }
  Json value(int depth) {
    if (depth > 64) fail("nesting deeper than 64");
    ws();
    if (p_ >= s_.size()) fail("unexpected end");
    Json v;
    char c = s_[p_];
    if (c == '{') {
      v.kind = Json::Object;
      ++p_;
      std::set<std::string> seen;
      ws();
      if (p_ < s_.size() && s_[p_] == '}') { ++p_; return v; }
      while (true) {
        ws();
        if (p_ >= s_.size() || s_[p_] != '"') fail("expected a key");
        std::string key = string();
        if (!seen.insert(key).second) fail("duplicate key '" + key + "'");
        ws();
        if (p_ >= s_.size() || s_[p_] != ':') fail("expected ':'");
        ++p_;
        v.obj.emplace_back(key, value(depth + 1));
        ws();
        if (p_ < s_.size() && s_[p_] == ',') { ++p_; continue; }
        if (p_ < s_.size() && s_[p_] == '}') { ++p_; return v; }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::Array;
      ++p_;
      ws();
      if (p_ < s_.size() && s_[p_] == ']') { ++p_; return v; }
      while (true) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (p_ < s_.size() && s_[p_] == ',') { ++p_; continue; }
        if (p_ < s_.size() && s_[p_] == ']') { ++p_; return v; }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') { v.kind = Json::String; v.str = string(); return v; }
    if (lit("true")) { v.kind = Json::Bool; v.b = true; return v; }
    if (lit("false")) { v.kind = Json::Bool; v.b = false; return v; }
    if (lit("null")) return v;
    if (c == '-' || (c >= '0' && c <= '9')) {
      size_t b = p_;
      if (s_[p_] == '-') ++p_;
      while (p_ < s_.size() && (isdigit((unsigned char)s_[p_]) || s_[p_] == '.' || s_[p_] == 'e' || s_[p_] == 'E' ||
                                s_[p_] == '+' || s_[p_] == '-'))
        ++p_;
      std::string t = s_.substr(b, p_ - b);
      char* end = nullptr;
      double d = strtod(t.c_str(), &end);
      if (*end != '\0' || !std::isfinite(d)) fail("invalid number " + t);
      v.kind = Json::Number;
      v.num = d;
      return v;
    }
    fail(std::string("unexpected character '") + c + "'");
  }
  std::string string() {
    ++p_;
    std::string out;
    while (p_ < s_.size() && s_[p_] != '"') {
      char c = s_[p_++];
      if (c == '\\') {
        if (p_ >= s_.size()) fail("bad escape");
        char e = s_[p_++];
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
            if (p_ + 4 > s_.size()) fail("bad \\u escape");
            unsigned cp = (unsigned)strtoul(s_.substr(p_, 4).c_str(), nullptr, 16);
            p_ += 4;
            if (cp < 0x80) out += (char)cp;
            else if (cp < 0x800) { out += (char)(0xc0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3f)); }
            else { out += (char)(0xe0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3f)); out += (char)(0x80 | (cp & 0x3f)); }
            break;
          }
          default: fail("bad escape");
        }
      } else {
        if ((unsigned char)c < 0x20) fail("control character in string");
        out += c;
      }
    }
    if (p_ >= s_.size()) fail("unterminated string");
    ++p_;
    return out;
  }
  const std::string& s_;
  size_t p_ = 0;
};

void dump_to(const Json& j, std::ostringstream& o) {
  switch (j.kind) {
    case Json::Null: o << "null"; break;
    case Json::Bool: o << (j.b ? "true" : "false"); break;
    case Json::Number: {
      if (j.num == (double)(long long)j.num && std::fabs(j.num) < 9e15) o << (long long)j.num;
      else { char buf[32]; snprintf(buf, sizeof buf, "%.17g", j.num); o << buf; }
      break;
    }
    case Json::String: {
      o << '"';
      for (char c : j.str) {
        if (c == '"' || c == '\\') o << '\\' << c;
        else if ((unsigned char)c < 0x20) { char buf[8]; snprintf(buf, sizeof buf, "\\u%04x", c); o << buf; }
        else o << c;
      }
      o << '"';
      break;
    }
    case Json::Array: {
      o << '[';
      for (size_t i = 0; i < j.arr.size(); ++i) { if (i) o << ','; dump_to(j.arr[i], o); }
      o << ']';
      break;
    }
    case Json::Object: {
      o << '{';
      for (size_t i = 0; i < j.obj.size(); ++i) {
        if (i) o << ',';
        Json k; k.kind = Json::String; k.str = j.obj[i].first;
        dump_to(k, o);
        o << ':';
        dump_to(j.obj[i].second, o);
      }
      o << '}';
      break;
    }
  }
}

}  // namespace

Json parse_json(const std::string& text) { return Parser(text).document(); }

const Json* Json::get(const std::string& key) const {
  for (auto& kv : obj) if (kv.first == key) return &kv.second;
  return nullptr;
}

const Json& Json::at(const std::string& key) const {
  const Json* v = get(key);
  if (!v) throw JsonError("json: missing key '" + key + "'");
  return *v;
}

long long Json::as_int() const {
  if (kind != Number || num != (double)(long long)num) throw JsonError("json: expected an integer");
  return (long long)num;
}

double Json::as_double() const {
  if (kind != Number) throw JsonError("json: expected a number");
  return num;
}

const std::string& Json::as_string() const {
  if (kind != String) throw JsonError("json: expected a string");
  return str;
}

std::string Json::dump() const {
  std::ostringstream o;
  dump_to(*this, o);
  return o.str();
}

void require_exact_keys(const Json& obj, const std::vector<std::string>& keys, const std::string& where) {
  if (obj.kind != Json::Object) throw JsonError(where + " must be an object");
  std::set<std::string> allowed(keys.begin(), keys.end());
  for (auto& kv : obj.obj)
    if (!allowed.count(kv.first)) throw JsonError(where + " has unknown key '" + kv.first + "'");
  for (auto& k : keys)
    if (!obj.get(k)) throw JsonError(where + " lacks key '" + k + "'");
}

}  // namespace vb
