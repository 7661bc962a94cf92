#include "gguf_reader.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

namespace mi {

namespace {

struct Cursor {
  const uint8_t* p;
  size_t size, off = 0;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (off + sizeof(T) > size) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p + off, sizeof(T));
    off += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t n = get<uint64_t>();
    if (!ok || off + n > size) {
      ok = false;
      return {};
    }
    std::string s((const char*)p + off, (size_t)n);
    off += (size_t)n;
    return s;
  }
  void skip(size_t n) {
    if (off + n > size) ok = false;
    else off += n;
  }
};

// Byte size of one scalar of GGUF value type t (0 for string/array).
size_t scalar_size(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;   // u8, i8, bool
    case 2: case 3: return 2;           // u16, i16
    case 4: case 5: case 6: return 4;   // u32, i32, f32
    case 10: case 11: case 12: return 8;  // u64, i64, f64
    default: return 0;
  }
}

}  // namespace

GgufFile::~GgufFile() {
  if (map_) munmap(map_, size_);
}

bool GgufFile::open(const std::string& path, std::string* err) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    *err = "failed to open '" + path + "': " + std::strerror(errno);
    return false;
  }
  struct stat st {};
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    *err = "'" + path + "' is too small to be a GGUF file";
    return false;
  }
  size_ = (size_t)st.st_size;
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    *err = std::string("mmap failed: ") + std::strerror(errno);
    return false;
  }
  Cursor c{(const uint8_t*)map_, size_};
  if (std::memcmp(map_, "GGUF", 4) != 0) {
    *err = "not a GGUF file (bad magic)";
    return false;
  }
  c.skip(4);
  const uint32_t version = c.get<uint32_t>();
  if (version != 3) {
    *err = "unsupported GGUF version (only v3)";
    return false;
  }
  const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
  size_t alignment = 32;
  for (uint64_t i = 0; i < n_kv && c.ok; i++) {
    const std::string key = c.str();
    const uint32_t t = c.get<uint32_t>();
    if (t == 8) {
      c.str();
    } else if (t == 9) {
      const uint32_t et = c.get<uint32_t>();
      const uint64_t n = c.get<uint64_t>();
      if (et == 8) {
        for (uint64_t k = 0; k < n && c.ok; k++) c.str();
      } else if (scalar_size(et) != 0) {
        c.skip((size_t)(n * scalar_size(et)));
      } else {
        c.ok = false;
      }
    } else if (t == 4 || t == 5) {
      const uint32_t v = c.get<uint32_t>();
      u32_[key] = v;
      if (key == "general.alignment") alignment = v;
    } else if (t == 6) {
      f32_[key] = c.get<float>();
    } else if (scalar_size(t) != 0) {
      c.skip(scalar_size(t));
    } else {
      c.ok = false;
    }
  }
  if (!c.ok) {
    *err = "truncated or corrupt GGUF metadata";
    return false;
  }
  if (alignment == 0 || (alignment & (alignment - 1)) != 0) {
    *err = "invalid general.alignment";
    return false;
  }
  std::vector<std::pair<GgufTensor, uint64_t>> infos;
  for (uint64_t i = 0; i < n_tensors && c.ok; i++) {
    GgufTensor t;
    t.name = c.str();
    t.n_dims = (int)c.get<uint32_t>();
    if (t.n_dims < 1 || t.n_dims > 4) {
      c.ok = false;
      break;
    }
    for (int d = 0; d < t.n_dims; d++) t.ne[d] = (int64_t)c.get<uint64_t>();
    t.type = c.get<uint32_t>();
    const uint64_t off = c.get<uint64_t>();
    infos.emplace_back(t, off);
  }
  if (!c.ok) {
    *err = "truncated or corrupt GGUF tensor table";
    return false;
  }
  const size_t data_start = (c.off + alignment - 1) / alignment * alignment;
  for (auto& it : infos) {
    GgufTensor t = it.first;
    const int64_t n = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
    if (t.type == kGgmlF32) t.nbytes = (size_t)n * 4;
    else if (t.type == kGgmlF16) t.nbytes = (size_t)n * 2;
    else if (t.type == kGgmlQ8_0 && t.ne[0] % 32 == 0) t.nbytes = (size_t)(n / 32 * 34);
    else {
      *err = "tensor '" + t.name + "' has an unsupported type (F32, F16, Q8_0 only)";
      return false;
    }
    const size_t start = data_start + (size_t)it.second;
    if (start + t.nbytes > size_) {
      *err = "tensor '" + t.name + "' runs past the end of the file";
      return false;
    }
    t.data = (const uint8_t*)map_ + start;
    tensors_[t.name] = t;
  }
  return true;
}

bool GgufFile::get_u32(const std::string& key, uint32_t* out) const {
  auto it = u32_.find(key);
  if (it == u32_.end()) return false;
  *out = (uint32_t)it->second;
  return true;
}

bool GgufFile::get_f32(const std::string& key, float* out) const {
  auto it = f32_.find(key);
  if (it == f32_.end()) return false;
  *out = it->second;
  return true;
}

const GgufTensor* GgufFile::find(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

}  // namespace mi
