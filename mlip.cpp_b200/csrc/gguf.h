// Minimal GGUF (v2/v3) reader: metadata key/values and tensors, loaded into
// host memory.  Replaces mlip.cpp's ggml-backed GGUFLoader
// (src/core/gguf_loader.{h,cpp}) for the "pet" layout.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace pet {

struct GGUFTensor {
  std::string name;
  std::vector<int64_t> ne;  // ggml order: ne[0] is the fastest dimension
  uint32_t type = 0;        // ggml type id (0 = F32, 1 = F16, 26 = I32)
  std::vector<uint8_t> data;
  int64_t numel() const {
    int64_t n = 1;
    for (auto v : ne) n *= v;
    return n;
  }
};

struct GGUFValue {
  uint32_t type = 0;
  double num = 0.0;  // numeric scalars (ints, floats, bools)
  std::string str;   // strings
};

class GGUFFile {
 public:
  explicit GGUFFile(const std::string &path);
  bool has(const std::string &key) const { return kv_.count(key) != 0; }
  std::string get_string(const std::string &key, const std::string &dflt = "") const;
  float get_f32(const std::string &key, float dflt) const;
  int32_t get_i32(const std::string &key, int32_t dflt) const;
  const GGUFTensor *tensor(const std::string &name) const;
  const std::map<std::string, GGUFTensor> &tensors() const { return tensors_; }

 private:
  std::map<std::string, GGUFValue> kv_;
  std::map<std::string, GGUFTensor> tensors_;
};

// Element size in bytes of the ggml types this reader accepts.
size_t ggml_type_size(uint32_t type);

}  // namespace pet
