// GGUF reader (format: magic "GGUF", version, tensor count, KV count, KV
// pairs, tensor infos, aligned tensor data).  Only unquantised tensor types
// are accepted; "pet" GGUFs are all F32/I32 (scripts/convert_pet_mad.py:270).
#include "gguf.h"

#include <cstdio>
#include <cstring>
#include <fstream>

#include "common.cuh"

namespace pet {

size_t ggml_type_size(uint32_t type) {
  switch (type) {
    case 0: return 4;   // F32
    case 1: return 2;   // F16
    case 24: return 1;  // I8
    case 25: return 2;  // I16
    case 26: return 4;  // I32
    case 27: return 8;  // I64
    case 28: return 8;  // F64
    case 30: return 2;  // BF16
    default: return 0;
  }
}

namespace {

struct Reader {
  std::vector<uint8_t> buf;
  size_t pos = 0;
  std::string path;
  void need(size_t n) {
    if (pos + n > buf.size()) throw Error(kErrIO, "truncated GGUF file: " + path);
  }
  template <class T> T rd() {
    need(sizeof(T));
    T v;
    std::memcpy(&v, buf.data() + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t n = rd<uint64_t>();
    need(n);
    std::string s(reinterpret_cast<const char *>(buf.data() + pos), n);
    pos += n;
    return s;
  }
};

// GGUF value types
enum : uint32_t {
  T_U8 = 0, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY,
  T_U64, T_I64, T_F64
};

double read_scalar(Reader &r, uint32_t t) {
  switch (t) {
    case T_U8: return r.rd<uint8_t>();
    case T_I8: return r.rd<int8_t>();
    case T_U16: return r.rd<uint16_t>();
    case T_I16: return r.rd<int16_t>();
    case T_U32: return r.rd<uint32_t>();
    case T_I32: return r.rd<int32_t>();
    case T_F32: return r.rd<float>();
    case T_BOOL: return r.rd<uint8_t>() ? 1.0 : 0.0;
    case T_U64: return static_cast<double>(r.rd<uint64_t>());
    case T_I64: return static_cast<double>(r.rd<int64_t>());
    case T_F64: return r.rd<double>();
    default: throw Error(kErrIO, "bad GGUF value type " + std::to_string(t));
  }
}

void skip_value(Reader &r, uint32_t t) {
  if (t == T_STRING) {
    r.str();
  } else if (t == T_ARRAY) {
    uint32_t et = r.rd<uint32_t>();
    uint64_t n = r.rd<uint64_t>();
    for (uint64_t i = 0; i < n; ++i) skip_value(r, et);
  } else {
    read_scalar(r, t);
  }
}

}  // namespace

GGUFFile::GGUFFile(const std::string &path) {
  Reader r;
  r.path = path;
  {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw Error(kErrIO, "Failed to load GGUF file: " + path);
    std::streamsize sz = f.tellg();
    f.seekg(0);
    r.buf.resize(static_cast<size_t>(sz));
    if (sz > 0 && !f.read(reinterpret_cast<char *>(r.buf.data()), sz))
      throw Error(kErrIO, "Failed to read GGUF file: " + path);
  }
  uint32_t magic = r.rd<uint32_t>();
  if (magic != 0x46554747u) throw Error(kErrIO, "not a GGUF file: " + path);
  uint32_t version = r.rd<uint32_t>();
  if (version < 2 || version > 3) throw Error(kErrIO, "unsupported GGUF version " + std::to_string(version));
  uint64_t n_tensors = r.rd<uint64_t>();
  uint64_t n_kv = r.rd<uint64_t>();
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = r.str();
    uint32_t t = r.rd<uint32_t>();
    GGUFValue v;
    v.type = t;
    if (t == T_STRING) {
      v.str = r.str();
    } else if (t == T_ARRAY) {
      skip_value(r, t);
    } else {
      v.num = read_scalar(r, t);
    }
    kv_[key] = v;
  }
  struct Info { std::string name; std::vector<int64_t> ne; uint32_t type; uint64_t off; };
  std::vector<Info> infos(n_tensors);
  for (auto &in : infos) {
    in.name = r.str();
    uint32_t nd = r.rd<uint32_t>();
    if (nd > 4) throw Error(kErrIO, "bad tensor rank in " + in.name);
    in.ne.resize(nd);
    for (auto &x : in.ne) x = static_cast<int64_t>(r.rd<uint64_t>());
    in.type = r.rd<uint32_t>();
    in.off = r.rd<uint64_t>();
  }
  uint64_t align = 32;
  auto it = kv_.find("general.alignment");
  if (it != kv_.end() && it->second.num > 0) align = static_cast<uint64_t>(it->second.num);
  size_t data_start = (r.pos + align - 1) / align * align;
  for (auto &in : infos) {
    size_t es = ggml_type_size(in.type);
    if (es == 0) throw Error(kErrUnsupported, "unsupported tensor type for " + in.name);
    GGUFTensor t;
    t.name = in.name;
    t.ne = in.ne;
    t.type = in.type;
    size_t bytes = static_cast<size_t>(t.numel()) * es;
    size_t beg = data_start + in.off;
    if (beg + bytes > r.buf.size()) throw Error(kErrIO, "tensor data out of range: " + in.name);
    t.data.assign(r.buf.begin() + beg, r.buf.begin() + beg + bytes);
    tensors_[in.name] = std::move(t);
  }
}

std::string GGUFFile::get_string(const std::string &key, const std::string &dflt) const {
  auto it = kv_.find(key);
  return (it == kv_.end() || it->second.type != T_STRING) ? dflt : it->second.str;
}

float GGUFFile::get_f32(const std::string &key, float dflt) const {
  auto it = kv_.find(key);
  return (it == kv_.end() || it->second.type == T_STRING || it->second.type == T_ARRAY)
             ? dflt : static_cast<float>(it->second.num);
}

int32_t GGUFFile::get_i32(const std::string &key, int32_t dflt) const {
  auto it = kv_.find(key);
  return (it == kv_.end() || it->second.type == T_STRING || it->second.type == T_ARRAY)
             ? dflt : static_cast<int32_t>(it->second.num);
}

const GGUFTensor *GGUFFile::tensor(const std::string &name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

}  // namespace pet
