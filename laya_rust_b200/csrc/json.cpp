// Ordered JSON parse / serialise with serde_json's observable behaviour; see
// json.h.
#include "json.h"

#include <charconv>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <unordered_map>

namespace laya {
namespace json {

const Value* Value::get(const std::string& key) const {
  if (kind != Object) return nullptr;
  for (const auto& kv : obj)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

void Value::set(const std::string& key, Value v) {
  for (auto& kv : obj)
    if (kv.first == key) {
      kv.second = std::move(v);
      return;
    }
  obj.emplace_back(key, std::move(v));
}

double Value::as_f64() const {
  switch (kind) {
    case Int: return static_cast<double>(i);
    case UInt: return static_cast<double>(u);
    case Float: return f;
    default: return std::numeric_limits<double>::quiet_NaN();
  }
}

namespace {

constexpr int kMaxDepth = 128;  // serde_json's recursion limit

struct Parser {
  const char* p;
  const char* end;
  int depth = 0;

  [[noreturn]] void fail(const char* what) { throw ParseError(what); }

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }

  static void put_utf8(uint32_t cp, std::string& out) {
    if (cp < 0x80) {
      out.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
      out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
      out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
  }

  uint32_t hex4() {
    if (end - p < 4) fail("EOF while parsing a string");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("invalid escape");
    }
    return v;
  }

  // one UTF-8 code point starting at p (validated), appended raw
  void utf8_char(std::string& out) {
    const unsigned char c = static_cast<unsigned char>(*p);
    int n = 0;
    uint32_t cp = 0;
    if (c < 0x80) {
      n = 1;
      cp = c;
    } else if ((c & 0xE0) == 0xC0) {
      n = 2;
      cp = c & 0x1F;
    } else if ((c & 0xF0) == 0xE0) {
      n = 3;
      cp = c & 0x0F;
    } else if ((c & 0xF8) == 0xF0) {
      n = 4;
      cp = c & 0x07;
    } else {
      fail("invalid unicode code point");
    }
    if (end - p < n) fail("invalid unicode code point");
    for (int k = 1; k < n; ++k) {
      const unsigned char d = static_cast<unsigned char>(p[k]);
      if ((d & 0xC0) != 0x80) fail("invalid unicode code point");
      cp = (cp << 6) | (d & 0x3F);
    }
    static const uint32_t kMin[5] = {0, 0, 0x80, 0x800, 0x10000};
    if (cp < kMin[n] || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) fail("invalid unicode code point");
    out.append(p, n);
    p += n;
  }

  std::string string() {
    ++p;  // opening quote
    std::string out;
    for (;;) {
      if (p >= end) fail("EOF while parsing a string");
      const char c = *p;
      if (c == '"') {
        ++p;
        return out;
      }
      if (static_cast<unsigned char>(c) < 0x20) fail("control character (\\u0000-\\u001F) found while parsing a string");
      if (c != '\\') {
        utf8_char(out);
        continue;
      }
      ++p;
      if (p >= end) fail("EOF while parsing a string");
      const char e = *p++;
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            if (end - p < 2 || p[0] != '\\' || p[1] != 'u') fail("unexpected end of hex escape");
            p += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo > 0xDFFF) fail("lone leading surrogate in hex escape");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
            fail("lone leading surrogate in hex escape");
          }
          put_utf8(cp, out);
          break;
        }
        default: fail("invalid escape");
      }
    }
  }

  Value number() {
    const char* s = p;
    if (*p == '-') ++p;
    if (p >= end) fail("invalid number");
    if (*p == '0') {
      ++p;
    } else if (*p >= '1' && *p <= '9') {
      while (p < end && *p >= '0' && *p <= '9') ++p;
    } else {
      fail("invalid number");
    }
    bool is_float = false;
    if (p < end && *p == '.') {
      is_float = true;
      ++p;
      if (p >= end || !(*p >= '0' && *p <= '9')) fail("invalid number");
      while (p < end && *p >= '0' && *p <= '9') ++p;
    }
    if (p < end && (*p == 'e' || *p == 'E')) {
      is_float = true;
      ++p;
      if (p < end && (*p == '+' || *p == '-')) ++p;
      if (p >= end || !(*p >= '0' && *p <= '9')) fail("invalid number");
      while (p < end && *p >= '0' && *p <= '9') ++p;
    }
    const std::string text(s, p);
    Value v;
    if (!is_float) {
      if (text[0] == '-') {
        int64_t x = 0;
        const auto r = std::from_chars(text.data(), text.data() + text.size(), x);
        if (r.ec == std::errc()) {
          if (x >= 0) {  // "-0" is the float -0.0
            v.kind = Value::Float;
            v.f = -0.0;
          } else {
            v.kind = Value::Int;
            v.i = x;
          }
          return v;
        }
      } else {
        uint64_t x = 0;
        const auto r = std::from_chars(text.data(), text.data() + text.size(), x);
        if (r.ec == std::errc()) {
          v.kind = Value::UInt;
          v.u = x;
          return v;
        }
      }
    }
    v.kind = Value::Float;
    v.f = std::strtod(text.c_str(), nullptr);
    if (!std::isfinite(v.f)) fail("number out of range");
    return v;
  }

  Value value() {
    ws();
    if (p >= end) fail("EOF while parsing a value");
    const char c = *p;
    if (c == '{' || c == '[') {
      if (++depth > kMaxDepth) fail("recursion limit exceeded");
      Value v;
      ++p;
      ws();
      if (c == '{') {
        v.kind = Value::Object;
        if (p < end && *p == '}') {
          ++p;
          --depth;
          return v;
        }
        // large objects (a tokenizer's vocabulary) get a key index so that
        // duplicate detection stays linear
        std::unordered_map<std::string, size_t> index;
        for (;;) {
          ws();
          if (p >= end || *p != '"') fail("key must be a string");
          std::string key = string();
          ws();
          if (p >= end || *p != ':') fail("expected `:`");
          ++p;
          Value item = value();
          if (v.obj.size() < 32) {
            v.set(key, std::move(item));
            if (v.obj.size() == 32)
              for (size_t q = 0; q < v.obj.size(); ++q) index.emplace(v.obj[q].first, q);
          } else {
            const auto it = index.find(key);
            if (it != index.end()) {
              v.obj[it->second].second = std::move(item);
            } else {
              index.emplace(key, v.obj.size());
              v.obj.emplace_back(std::move(key), std::move(item));
            }
          }
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == '}') {
            ++p;
            break;
          }
          fail("expected `,` or `}`");
        }
      } else {
        v.kind = Value::Array;
        if (p < end && *p == ']') {
          ++p;
          --depth;
          return v;
        }
        for (;;) {
          v.arr.push_back(value());
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == ']') {
            ++p;
            break;
          }
          fail("expected `,` or `]`");
        }
      }
      --depth;
      return v;
    }
    if (c == '"') return Value::str(string());
    if (c == '-' || (c >= '0' && c <= '9')) return number();
    auto lit = [&](const char* w, size_t n) {
      if (static_cast<size_t>(end - p) < n || std::memcmp(p, w, n) != 0) fail("expected value");
      p += n;
    };
    Value v;
    if (c == 't') {
      lit("true", 4);
      v.kind = Value::Bool;
      v.b = true;
    } else if (c == 'f') {
      lit("false", 5);
      v.kind = Value::Bool;
    } else if (c == 'n') {
      lit("null", 4);
    } else {
      fail("expected value");
    }
    return v;
  }
};

}  // namespace

Value parse(const char* text, size_t len) {
  Parser ps{text, text + len};
  Value v = ps.value();
  ps.ws();
  if (ps.p != ps.end) throw ParseError("trailing characters");
  return v;
}

std::string fmt_f64(double x) {
  if (!std::isfinite(x)) return "null";
  if (x == 0.0) return std::signbit(x) ? "-0.0" : "0.0";
  char buf[64];
  const auto r = std::to_chars(buf, buf + sizeof buf, std::fabs(x), std::chars_format::scientific);
  const std::string sci(buf, r.ptr);
  const size_t epos = sci.find('e');
  std::string digits;
  for (size_t q = 0; q < epos; ++q)
    if (sci[q] != '.') digits.push_back(sci[q]);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  const int e = std::atoi(sci.c_str() + epos + 1);
  const int length = static_cast<int>(digits.size());
  const int kk = e + 1;  // 10^(kk-1) <= |x| < 10^kk
  const int k = kk - length;
  std::string out = x < 0 ? "-" : "";
  if (0 <= k && kk <= 16) {
    out += digits;
    out.append(static_cast<size_t>(k), '0');
    out += ".0";
  } else if (0 < kk && kk <= 16) {
    out += digits.substr(0, kk);
    out += '.';
    out += digits.substr(kk);
  } else if (-5 < kk && kk <= 0) {
    out += "0.";
    out.append(static_cast<size_t>(-kk), '0');
    out += digits;
  } else if (length == 1) {
    out += digits;
    out += 'e';
    out += std::to_string(kk - 1);
  } else {
    out += digits[0];
    out += '.';
    out += digits.substr(1);
    out += 'e';
    out += std::to_string(kk - 1);
  }
  return out;
}

std::string number_string(const Value& v) {
  switch (v.kind) {
    case Value::Int: return std::to_string(v.i);
    case Value::UInt: return std::to_string(v.u);
    case Value::Float: return fmt_f64(v.f);
    default: return "";
  }
}

void dump_string(const std::string& s, std::string& out) {
  static const char* hex = "0123456789abcdef";
  out.push_back('"');
  for (const char ch : s) {
    const unsigned char c = static_cast<unsigned char>(ch);
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      default:
        if (c < 0x20) {
          out += "\\u00";
          out.push_back(hex[c >> 4]);
          out.push_back(hex[c & 15]);
        } else {
          out.push_back(ch);
        }
    }
  }
  out.push_back('"');
}

void dump_to(const Value& v, std::string& out) {
  switch (v.kind) {
    case Value::Null: out += "null"; break;
    case Value::Bool: out += v.b ? "true" : "false"; break;
    case Value::Int:
    case Value::UInt:
    case Value::Float: out += number_string(v); break;
    case Value::String: dump_string(v.s, out); break;
    case Value::Array:
      out.push_back('[');
      for (size_t k = 0; k < v.arr.size(); ++k) {
        if (k) out.push_back(',');
        dump_to(v.arr[k], out);
      }
      out.push_back(']');
      break;
    case Value::Object:
      out.push_back('{');
      for (size_t k = 0; k < v.obj.size(); ++k) {
        if (k) out.push_back(',');
        dump_string(v.obj[k].first, out);
        out.push_back(':');
        dump_to(v.obj[k].second, out);
      }
      out.push_back('}');
      break;
  }
}

std::string dump(const Value& v) {
  std::string out;
  dump_to(v, out);
  return out;
}

}  // namespace json
}  // namespace laya
