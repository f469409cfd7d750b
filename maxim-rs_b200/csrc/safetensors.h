// A read-only safetensors file: an 8-byte little-endian header length, a JSON
// header mapping tensor names to {dtype, shape, data_offsets}, then the raw
// tensor bytes. This is the format `tools/convert.py:88-126` writes and the
// reference reads through `lightgpu::safetensors::File` (src/weights.rs:15-41).
//
// The file is memory-mapped; tensors are returned as fp32 (F16 and F64 blobs,
// which the converter may also emit, are widened or narrowed on read).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace mx {

struct TensorInfo {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte range within the data section
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

class SafeTensors {
 public:
  explicit SafeTensors(const std::string& path);
  ~SafeTensors();
  SafeTensors(const SafeTensors&) = delete;
  SafeTensors& operator=(const SafeTensors&) = delete;

  bool contains(const std::string& name) const { return tensors_.count(name) != 0; }
  const TensorInfo& info(const std::string& name) const;
  // The tensor's values as fp32, in the file's own (row-major) order.
  std::vector<float> f32(const std::string& name) const;
  const std::map<std::string, TensorInfo>& tensors() const { return tensors_; }
  const std::map<std::string, std::string>& metadata() const { return metadata_; }
  const std::string& path() const { return path_; }

 private:
  std::string path_;
  void* map_ = nullptr;
  size_t map_len_ = 0;
  const uint8_t* data_ = nullptr;  // start of the data section
  size_t data_len_ = 0;
  std::map<std::string, TensorInfo> tensors_;
  std::map<std::string, std::string> metadata_;
};

}  // namespace mx
