// gguf_host.cc -- GGUF v1-v3 reader (see gguf_host.h).
#include "gguf_host.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>
#include <unordered_set>

namespace rpgc {

bool ggml_block(uint32_t type, int64_t* elems, int64_t* bytes) {
  switch (type) {
    case 0: *elems = 1; *bytes = 4; return true;       // F32
    case 1: *elems = 1; *bytes = 2; return true;       // F16
    case 30: *elems = 1; *bytes = 2; return true;      // BF16
    case 2: *elems = 32; *bytes = 18; return true;     // Q4_0
    case 3: *elems = 32; *bytes = 20; return true;     // Q4_1
    case 6: *elems = 32; *bytes = 22; return true;     // Q5_0
    case 7: *elems = 32; *bytes = 24; return true;     // Q5_1
    case 8: *elems = 32; *bytes = 34; return true;     // Q8_0
    case 9: *elems = 32; *bytes = 36; return true;     // Q8_1
    case 10: *elems = 256; *bytes = 84; return true;   // Q2_K
    case 11: *elems = 256; *bytes = 110; return true;  // Q3_K
    case 12: *elems = 256; *bytes = 144; return true;  // Q4_K
    case 13: *elems = 256; *bytes = 176; return true;  // Q5_K
    case 14: *elems = 256; *bytes = 210; return true;  // Q6_K
    case 15: *elems = 256; *bytes = 292; return true;  // Q8_K
    default: return false;
  }
}

namespace {

struct Cursor {
  const uint8_t* p;
  size_t n, pos = 0;
  void need(size_t k) {
    if (pos + k > n) throw std::runtime_error("GGUF: truncated file");
  }
  template <typename T>
  T get() {
    need(sizeof(T));
    T v;
    std::memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t len = get<uint64_t>();
    if (len > (1ull << 31)) throw std::runtime_error("GGUF: string length out of range");
    need(len);
    std::string s(reinterpret_cast<const char*>(p + pos), len);
    pos += len;
    return s;
  }
};

void skip_or_read(Cursor& c, uint32_t type, GgufValue* out, int depth) {
  GgufValue v;
  switch (type) {
    case 0: v.kind = GgufValue::kInt; v.i = c.get<uint8_t>(); break;
    case 1: v.kind = GgufValue::kInt; v.i = c.get<int8_t>(); break;
    case 2: v.kind = GgufValue::kInt; v.i = c.get<uint16_t>(); break;
    case 3: v.kind = GgufValue::kInt; v.i = c.get<int16_t>(); break;
    case 4: v.kind = GgufValue::kInt; v.i = c.get<uint32_t>(); break;
    case 5: v.kind = GgufValue::kInt; v.i = c.get<int32_t>(); break;
    case 6: v.kind = GgufValue::kFloat; v.f = c.get<float>(); break;
    case 7: v.kind = GgufValue::kBool; v.b = c.get<uint8_t>() != 0; break;
    case 8: v.kind = GgufValue::kString; v.s = c.str(); break;
    case 10: v.kind = GgufValue::kInt; v.i = (int64_t)c.get<uint64_t>(); break;
    case 11: v.kind = GgufValue::kInt; v.i = c.get<int64_t>(); break;
    case 12: v.kind = GgufValue::kFloat; v.f = c.get<double>(); break;
    case 9: {
      if (depth > 2) throw std::runtime_error("GGUF: nested arrays too deep");
      const uint32_t et = c.get<uint32_t>();
      const uint64_t n = c.get<uint64_t>();
      if (n >= (1ull << 32)) throw std::runtime_error("GGUF: array length out of range");
      v.kind = GgufValue::kArray;
      v.array_len = n;
      if (et == 8 && depth == 0 && out) {  // strings: kept (the vocabulary)
        v.strs.reserve(n);
        for (uint64_t k = 0; k < n; ++k) v.strs.push_back(c.str());
        break;
      }
      for (uint64_t k = 0; k < n; ++k) skip_or_read(c, et, nullptr, depth + 1);
      break;
    }
    default:
      throw std::runtime_error("GGUF: unknown metadata type " + std::to_string(type));
  }
  if (out) *out = std::move(v);
}

}  // namespace

GgufReader::~GgufReader() {
  if (map_) munmap(map_, size_);
}

void GgufReader::Open(const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("cannot open " + path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    throw std::runtime_error("not a GGUF file (too small): " + path);
  }
  size_ = (size_t)st.st_size;
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    throw std::runtime_error("mmap failed: " + path);
  }
  Cursor c{static_cast<const uint8_t*>(map_), size_};
  if (c.get<uint32_t>() != 0x46554747u) throw std::runtime_error("bad GGUF magic: " + path);
  const uint32_t version = c.get<uint32_t>();
  if (version < 1 || version > 3) throw std::runtime_error("unsupported GGUF version");
  // Version 1 differs only in the two counts (32-bit); strings, array
  // lengths and dimensions are 64-bit in every version, as the reference
  // reads them (src/gguf.cc:84-93, 124).
  const bool v1 = version == 1;
  const uint64_t n_t = v1 ? c.get<uint32_t>() : c.get<uint64_t>();
  const uint64_t n_kv = v1 ? c.get<uint32_t>() : c.get<uint64_t>();
  for (uint64_t i = 0; i < n_kv; ++i) {
    const std::string key = c.str();
    GgufValue v;
    skip_or_read(c, c.get<uint32_t>(), &v, 0);
    meta_[key] = std::move(v);
  }
  if (Str("general.architecture", "").empty())
    throw std::runtime_error("GGUF: general.architecture missing");  // src/gguf.cc:105-106
  std::unordered_set<std::string> names;
  for (uint64_t i = 0; i < n_t; ++i) {
    GgufTensorInfo t;
    t.name = c.str();
    if (!names.insert(t.name).second)  // src/gguf.cc:139-141
      throw std::runtime_error("GGUF: duplicate tensor name " + t.name);
    const uint32_t nd = c.get<uint32_t>();
    if (nd < 1 || nd > 4) throw std::runtime_error("GGUF: bad n_dims for " + t.name);
    t.n_elements = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      const uint64_t dim = c.get<uint64_t>();
      if (dim == 0 || dim >= (1ull << 40)) throw std::runtime_error("GGUF: bad dim for " + t.name);
      t.dims.push_back((int64_t)dim);
      t.n_elements *= (int64_t)dim;
    }
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    int64_t be, bb;
    if (!ggml_block(t.type, &be, &bb) || t.n_elements % be)
      throw std::runtime_error("GGUF: unsupported type/shape for " + t.name);
    t.n_bytes = t.n_elements / be * bb;
    tensors_.push_back(std::move(t));
  }
  const int64_t align = Int("general.alignment", 32);
  if (align <= 0 || (align & 7)) throw std::runtime_error("GGUF: bad alignment");
  data_start_ = (c.pos + align - 1) / align * align;
  for (const auto& t : tensors_)
    if (data_start_ + t.offset + t.n_bytes > size_)
      throw std::runtime_error("GGUF: tensor " + t.name + " runs past the end of the file");
}

const GgufValue* GgufReader::Find(const std::string& key) const {
  auto it = meta_.find(key);
  return it == meta_.end() ? nullptr : &it->second;
}
int64_t GgufReader::Int(const std::string& key, int64_t def) const {
  const GgufValue* v = Find(key);
  if (!v) return def;
  if (v->kind == GgufValue::kInt) return v->i;
  if (v->kind == GgufValue::kFloat) return (int64_t)v->f;
  if (v->kind == GgufValue::kBool) return v->b ? 1 : 0;
  return def;
}
double GgufReader::Float(const std::string& key, double def) const {
  const GgufValue* v = Find(key);
  if (!v) return def;
  if (v->kind == GgufValue::kFloat) return v->f;
  if (v->kind == GgufValue::kInt) return (double)v->i;
  return def;
}
std::string GgufReader::Str(const std::string& key, const std::string& def) const {
  const GgufValue* v = Find(key);
  return (v && v->kind == GgufValue::kString) ? v->s : def;
}
size_t GgufReader::ArrayLen(const std::string& key) const {
  const GgufValue* v = Find(key);
  return (v && v->kind == GgufValue::kArray) ? v->array_len : 0;
}
const uint8_t* GgufReader::TensorData(const GgufTensorInfo& t) const {
  return static_cast<const uint8_t*>(map_) + data_start_ + t.offset;
}

}  // namespace rpgc
