// Minimal ordered JSON values for the request front end, with the behaviour
// of serde_json (preserve_order) that the reference's request handling
// depends on (laya-rust Cargo.toml:25; systemone.rs:48-118):
//   - objects keep insertion order; inserting an existing key replaces its
//     value in place;
//   - integer literals that fit i64 (negative) or u64 (non-negative) stay
//     integers, every other number is an f64;
//   - serialisation is compact, strings escape '"', '\\', \b \f \n \r \t and
//     other control characters as \u00xx, and f64 values print with ryu's
//     shortest digits in its layout (see fmt_f64).
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace laya {
namespace json {

struct Value {
  enum Kind { Null, Bool, Int, UInt, Float, String, Array, Object };
  Kind kind = Null;
  bool b = false;
  int64_t i = 0;
  uint64_t u = 0;
  double f = 0.0;
  std::string s;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;

  bool is_null() const { return kind == Null; }
  bool is_string() const { return kind == String; }
  bool is_array() const { return kind == Array; }
  bool is_object() const { return kind == Object; }
  bool is_number() const { return kind == Int || kind == UInt || kind == Float; }
  // object member, or nullptr (also for non-objects)
  const Value* get(const std::string& key) const;
  // insert or replace in place
  void set(const std::string& key, Value v);
  double as_f64() const;

  static Value str(std::string v) {
    Value x;
    x.kind = String;
    x.s = std::move(v);
    return x;
  }
  static Value num(double v) {
    Value x;
    x.kind = Float;
    x.f = v;
    return x;
  }
  static Value integer(int64_t v) {
    Value x;
    if (v >= 0) {
      x.kind = UInt;
      x.u = static_cast<uint64_t>(v);
    } else {
      x.kind = Int;
      x.i = v;
    }
    return x;
  }
  static Value object() {
    Value x;
    x.kind = Object;
    return x;
  }
};

struct ParseError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// Parses one JSON document (UTF-8); throws ParseError.
Value parse(const char* text, size_t len);
// Compact serialisation (serde_json::to_string).
std::string dump(const Value& v);
void dump_to(const Value& v, std::string& out);
void dump_string(const std::string& s, std::string& out);
// An f64 as serde_json prints it: ryu's shortest round-trip digits, laid
// out as digits ".0" for decimal exponents 0..16, with a decimal point inside
// the digits, as "0.000ddd" down to 1e-5, else "d.ddde<exp>".
std::string fmt_f64(double x);
// Number::to_string (integers in decimal, floats by fmt_f64).
std::string number_string(const Value& v);

}  // namespace json
}  // namespace laya
