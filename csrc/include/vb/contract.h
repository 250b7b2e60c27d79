// Contract utilities shared by the native runtime: SHA-256, a strict JSON
// reader, deadlines and overflow-checked arithmetic.
#pragma once
#include <chrono>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace vb {

// SHA-256 (FIPS 180-4) of a byte string, lowercase hex.
std::string sha256_hex(const std::string& data);

// Strict JSON: rejects duplicate keys, non-finite numbers, trailing data and
// nesting deeper than 64 levels.
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json* get(const std::string& key) const;
  const Json& at(const std::string& key) const;
  long long as_int() const;
  double as_double() const;
  const std::string& as_string() const;
  std::string dump() const;
};

struct JsonError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

Json parse_json(const std::string& text);
// Only the listed keys may appear.
void require_exact_keys(const Json& obj, const std::vector<std::string>& keys, const std::string& where);

using Clock = std::chrono::steady_clock;

struct Deadline {
  Clock::time_point at;
  static Deadline after(double seconds) {
    return Deadline{Clock::now() + std::chrono::duration_cast<Clock::duration>(std::chrono::duration<double>(seconds))};
  }
  double remaining() const { return std::chrono::duration<double>(at - Clock::now()).count(); }
  bool expired() const { return Clock::now() >= at; }
  // A child deadline never extends its parent.
  Deadline child(double seconds) const {
    Deadline d = after(seconds);
    return d.at < at ? d : *this;
  }
};

inline size_t checked_mul(size_t a, size_t b) {
  if (a && b > SIZE_MAX / a) throw std::overflow_error("size overflow");
  return a * b;
}

}  // namespace vb
