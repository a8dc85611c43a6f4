// Minimal GGUF (v2/v3) reader for the GWP-0.5 artifact: metadata key/values
// and tensor descriptors, with payload reads by file offset. Replaces the
// engine's use of the reference's GgufReader (src/models/common/gguf_reader.cpp:26-97,
// 179-189), which depends on ggml.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace wamb {

enum GgmlType : uint32_t {
  GGML_F32 = 0,
  GGML_F16 = 1,
  GGML_Q8_0 = 8,
  GGML_BF16 = 30,
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> ne;  // ggml order: ne[0] is the contiguous dimension
  uint32_t type = 0;
  uint64_t offset = 0;  // absolute file offset of the payload
  uint64_t bytes = 0;
  uint64_t elements() const {
    uint64_t n = 1;
    for (uint64_t d : ne) n *= d;
    return n;
  }
};

struct GgufValue {
  uint32_t type = 0;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  std::vector<double> arr;  // numeric arrays only
};

class GgufFile {
 public:
  // Parses header, metadata and tensor descriptors. Returns false and fills
  // error on malformed or truncated files.
  bool open(const std::string& path, std::string* error);
  bool has(const std::string& key) const { return kv_.count(key) != 0; }
  bool get_u32(const std::string& key, uint32_t* out) const;
  bool get_f32(const std::string& key, float* out) const;
  bool get_str(const std::string& key, std::string* out) const;
  // Numeric array (<= 4096 elements) as floats.
  bool get_f32_array(const std::string& key, std::vector<float>* out) const;
  const GgufTensor* tensor(const std::string& name) const;
  const std::vector<GgufTensor>& tensors() const { return tensors_; }
  const std::string& path() const { return path_; }
  uint64_t file_size() const { return file_size_; }
  // Reads `bytes` payload bytes of a tensor starting at `start` into dst.
  bool read(const GgufTensor& t, uint64_t start, void* dst, uint64_t bytes) const;

 private:
  std::string path_;
  uint64_t file_size_ = 0;
  std::map<std::string, GgufValue> kv_;
  std::vector<GgufTensor> tensors_;
  std::map<std::string, size_t> index_;
};

// Bytes of `elements` values of a ggml type (0 if unsupported).
uint64_t ggml_type_bytes(uint32_t type, uint64_t elements);

}  // namespace wamb
