// gguf_host.h -- GGUF v1-v3 reader for the host upload path.
//
// Reads the same file structure as the reference (src/gguf.cc:69-160):
// header, typed metadata, tensor table, tensor data aligned to
// general.alignment.  The whole file is memory-mapped read-only and tensor
// bytes are handed to the device upload unchanged.
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace rpgc {

struct GgufValue {
  enum Kind { kNone, kInt, kFloat, kBool, kString, kArray } kind = kNone;
  int64_t i = 0;
  double f = 0;
  bool b = false;
  std::string s;
  size_t array_len = 0;
  std::vector<std::string> strs;  // elements of a top-level array of strings
};

struct GgufTensorInfo {
  std::string name;
  std::vector<int64_t> dims;  // dims[0] fastest
  uint32_t type = 0;
  uint64_t offset = 0;        // relative to the data section
  int64_t n_elements = 0;
  int64_t n_bytes = 0;
};

class GgufReader {
 public:
  GgufReader() = default;
  ~GgufReader();
  GgufReader(const GgufReader&) = delete;
  GgufReader& operator=(const GgufReader&) = delete;

  // Throws std::runtime_error on malformed input.
  void Open(const std::string& path);

  const GgufValue* Find(const std::string& key) const;
  int64_t Int(const std::string& key, int64_t def) const;
  double Float(const std::string& key, double def) const;
  std::string Str(const std::string& key, const std::string& def) const;
  size_t ArrayLen(const std::string& key) const;

  const std::vector<GgufTensorInfo>& tensors() const { return tensors_; }
  const uint8_t* TensorData(const GgufTensorInfo& t) const;

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  uint64_t data_start_ = 0;
  std::map<std::string, GgufValue> meta_;
  std::vector<GgufTensorInfo> tensors_;
};

// Block geometry of the ggml types (reference src/quant.cc:29-45).
bool ggml_block(uint32_t type, int64_t* elems, int64_t* bytes);

}  // namespace rpgc
