// GGUF v3 reader for the engine's own loader.  Restates the validation of
// laya-rust src/gguf.rs:289-357 (magic, version 3, plausible counts, 1..4
// dimensions, 32-byte aligned offsets, data inside the file) and the metadata
// accessors of :140-163.  Errors throw std::runtime_error with the
// reference's wording.
#pragma once
#include <stdint.h>

#include <cstdio>
#include <string>
#include <vector>

namespace laya {

struct GgufValue {
  uint32_t ty = 0;
  bool has_u = false, has_f = false, has_s = false;
  uint64_t u = 0;
  double f = 0;
  std::string s;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;  // GGUF order (reverse of the framework shape)
  uint32_t ty = 0;
  uint64_t offset = 0;
  uint64_t elems() const;
  uint64_t nbytes() const;
  std::vector<int64_t> stored_dims() const;  // weights.rs:261-268
};

class GgufFile {
 public:
  explicit GgufFile(const std::string& path);
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;

  const GgufValue* get(const std::string& key) const;
  const GgufTensor* tensor(const std::string& name) const;
  void read_bytes(const GgufTensor& t, void* dst) const;
  const std::string& path() const { return path_; }

  std::vector<std::pair<std::string, GgufValue>> kv;
  std::vector<GgufTensor> tensors;
  uint64_t data_off = 0;

 private:
  std::string path_;
  FILE* f_ = nullptr;
  uint64_t len_ = 0;
};

uint64_t gguf_elem_size(uint32_t ty);

}  // namespace laya
