// Minimal GGUF v3 reader (mmap, zero-copy) for the model loader.
//
// Parses the same file structure the reference's mi_gguf_open does (reference
// src/gguf.cpp:259-436): magic "GGUF", version 3, KV metadata, tensor infos,
// data section aligned to general.alignment (default 32). Only what the
// loader needs is kept: u32/f32 scalars by key and tensor (type, shape, bytes).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace mi {

constexpr uint32_t kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ8_0 = 8;

struct GgufTensor {
  std::string name;
  uint32_t type = 0;
  int n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
};

class GgufFile {
 public:
  ~GgufFile();
  bool open(const std::string& path, std::string* err);
  bool get_u32(const std::string& key, uint32_t* out) const;
  bool get_f32(const std::string& key, float* out) const;
  const GgufTensor* find(const std::string& name) const;

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, uint64_t> u32_;
  std::map<std::string, float> f32_;
  std::map<std::string, GgufTensor> tensors_;
};

}  // namespace mi
