#include "gguf_reader.h"

#include <cstdarg>
#include <cstring>
#include <stdexcept>

namespace laya {

namespace {

constexpr uint32_t kMagic = 0x46554747u;
constexpr uint64_t kAlign = 32;

std::string fmt(const char* f, ...) __attribute__((format(printf, 1, 2)));
std::string fmt(const char* f, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof buf, f, ap);
  va_end(ap);
  return buf;
}

struct Rd {
  FILE* f;
  uint64_t pos, len;
  void take(void* dst, uint64_t n, const std::string& ctx) {
    if (pos + n > len || pos + n < pos)
      throw std::runtime_error(fmt("gguf: %s: read of %llu bytes at %llu passes end of file (%llu)",
                                   ctx.c_str(), (unsigned long long)n, (unsigned long long)pos,
                                   (unsigned long long)len));
    if (n && fread(dst, 1, n, f) != n) throw std::runtime_error("gguf: " + ctx + ": short read");
    pos += n;
  }
  template <class T>
  T get(const std::string& ctx) {
    T v;
    take(&v, sizeof v, ctx);
    return v;
  }
  std::string str(const std::string& ctx) {
    uint64_t n = get<uint64_t>(ctx);
    if (n > len - pos) throw std::runtime_error(fmt("gguf: %s: string passes end of file", ctx.c_str()));
    std::string s(n, '\0');
    take(s.data(), n, ctx);
    return s;
  }
};

void read_value(Rd& r, uint32_t ty, const std::string& ctx, GgufValue* out, int depth) {
  GgufValue tmp;
  GgufValue& v = out ? *out : tmp;
  v.ty = ty;
  switch (ty) {
    case 0: v.u = r.get<uint8_t>(ctx); v.has_u = true; break;
    case 1: v.u = (uint64_t)(int64_t)r.get<int8_t>(ctx); v.has_u = true; break;
    case 2: v.u = r.get<uint16_t>(ctx); v.has_u = true; break;
    case 3: v.u = (uint64_t)(int64_t)r.get<int16_t>(ctx); v.has_u = true; break;
    case 4: v.u = r.get<uint32_t>(ctx); v.has_u = true; break;
    case 5: v.u = (uint64_t)(int64_t)r.get<int32_t>(ctx); v.has_u = true; break;
    case 6: v.f = r.get<float>(ctx); v.has_f = true; break;
    case 7: r.get<uint8_t>(ctx); break;
    case 8: v.s = r.str(ctx); v.has_s = true; break;
    case 9: {
      uint32_t et = r.get<uint32_t>(ctx);
      uint64_t n = r.get<uint64_t>(ctx);
      if (n > (r.len - 1) / 8)
        throw std::runtime_error(fmt("gguf: %s: array of %llu elements is not plausible in %llu bytes",
                                     ctx.c_str(), (unsigned long long)n, (unsigned long long)r.len));
      if (depth > 16) throw std::runtime_error("gguf: " + ctx + ": arrays nested too deep");
      for (uint64_t i = 0; i < n; ++i) read_value(r, et, ctx, nullptr, depth + 1);
      break;
    }
    case 10: v.u = r.get<uint64_t>(ctx); v.has_u = true; break;
    case 11: v.u = (uint64_t)r.get<int64_t>(ctx); v.has_u = true; break;
    case 12: v.f = r.get<double>(ctx); v.has_f = true; break;
    default:
      throw std::runtime_error(fmt("gguf: %s: unknown metadata value type %u", ctx.c_str(), ty));
  }
}

}  // namespace

uint64_t gguf_elem_size(uint32_t ty) {
  if (ty == 0) return 4;
  if (ty == 1 || ty == 30) return 2;
  throw std::runtime_error(fmt("gguf: unsupported tensor type %u", ty));
}

uint64_t GgufTensor::elems() const {
  uint64_t e = 1;
  for (uint64_t d : dims) e *= d;
  return e;
}

uint64_t GgufTensor::nbytes() const { return elems() * gguf_elem_size(ty); }

std::vector<int64_t> GgufTensor::stored_dims() const {
  std::vector<int64_t> d;
  for (auto it = dims.rbegin(); it != dims.rend(); ++it) d.push_back((int64_t)*it);
  return d;
}

GgufFile::GgufFile(const std::string& path) : path_(path) {
  f_ = fopen(path.c_str(), "rb");
  if (!f_) throw std::runtime_error(path + ": cannot open");
  fseek(f_, 0, SEEK_END);
  len_ = (uint64_t)ftell(f_);
  fseek(f_, 0, SEEK_SET);
  Rd r{f_, 0, len_};
  uint32_t magic = r.get<uint32_t>(path);
  if (magic != kMagic)
    throw std::runtime_error(fmt("%s: not a GGUF file (magic %#010x, want %#010x)", path.c_str(), magic, kMagic));
  uint32_t version = r.get<uint32_t>(path);
  if (version != 3) throw std::runtime_error(fmt("%s: GGUF version %u, want 3", path.c_str(), version));
  uint64_t tc = r.get<uint64_t>(path), kc = r.get<uint64_t>(path);
  if (tc > len_ / 64 || kc > len_ / 16 || tc * 64 + kc * 16 > len_)
    throw std::runtime_error(fmt("%s: header claims %llu tensors and %llu metadata entries in %llu bytes",
                                 path.c_str(), (unsigned long long)tc, (unsigned long long)kc,
                                 (unsigned long long)len_));
  for (uint64_t i = 0; i < kc; ++i) {
    std::string key = r.str(path);
    uint32_t ty = r.get<uint32_t>(path);
    GgufValue v;
    read_value(r, ty, key, &v, 0);
    kv.emplace_back(std::move(key), std::move(v));
  }
  for (uint64_t i = 0; i < tc; ++i) {
    GgufTensor t;
    t.name = r.str(path);
    uint32_t nd = r.get<uint32_t>(path);
    if (nd == 0 || nd > 4) throw std::runtime_error(fmt("gguf: tensor %s has %u dimensions", t.name.c_str(), nd));
    for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(r.get<uint64_t>(t.name));
    t.ty = r.get<uint32_t>(t.name);
    t.offset = r.get<uint64_t>(t.name);
    tensors.push_back(std::move(t));
  }
  data_off = (r.pos + kAlign - 1) / kAlign * kAlign;
  if (data_off > len_) throw std::runtime_error(path + ": tensor data starts past end of file");
  for (const auto& t : tensors) {
    if (t.offset % kAlign)
      throw std::runtime_error(fmt("gguf: tensor %s offset %llu is not a multiple of %llu", t.name.c_str(),
                                   (unsigned long long)t.offset, (unsigned long long)kAlign));
    if (data_off + t.offset + t.nbytes() > len_)
      throw std::runtime_error("gguf: tensor " + t.name + " data is outside the file");
  }
}

GgufFile::~GgufFile() {
  if (f_) fclose(f_);
}

const GgufValue* GgufFile::get(const std::string& key) const {
  for (const auto& p : kv)
    if (p.first == key) return &p.second;
  return nullptr;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
  for (const auto& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}

void GgufFile::read_bytes(const GgufTensor& t, void* dst) const {
  if (fseek(f_, (long)(data_off + t.offset), SEEK_SET) != 0 || fread(dst, 1, t.nbytes(), f_) != t.nbytes())
    throw std::runtime_error(path_ + ": short read of " + t.name);
}

}  // namespace laya
