// Minimal local safetensors reader (header JSON + mmap'd data).
// Replaces the HTTP-Range / Cache-API reader of src/io/safetensors.ts:24-341
// for a local file; keeps its dtype and shape asserts (177-190).
#pragma once
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace g4m {

struct TensorInfo {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
  }
};

class SafeTensors {
 public:
  ~SafeTensors();
  // Returns false with `err` set on a missing or malformed file.
  bool open(const std::string& path, std::string& err);
  const TensorInfo* find(const std::string& name) const;
  const void* data(const TensorInfo& t) const { return base_ + data_off_ + t.begin; }
  size_t bytes(const TensorInfo& t) const { return (size_t)(t.end - t.begin); }
  const std::map<std::string, TensorInfo>& tensors() const { return t_; }

 private:
  std::map<std::string, TensorInfo> t_;
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  uint64_t data_off_ = 0;
};

std::string shape_str(const TensorInfo& t);

}  // namespace g4m
