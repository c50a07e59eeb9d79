// blob.h -- reader of the reference engine's model.mmfree weight blob (host side).
//
// Format (matmulfreellmCPU cpp/src/io/weights.cpp:1-8, tools/provision.py:126-163):
// "MMFREE1\n", u64 LE header length, JSON header {config, tensors{name: {dtype, shape, offset,
// nbytes}}}, zero padding to 64 bytes, then the data section with 64-byte aligned tensors
// (offsets relative to the data-section start). Errors throw std::runtime_error with the
// same wording as the reference loader (weights.cpp:193-242, weights.hpp:49).
//
// model.mmfree2 ("MMFREE2\n", this engine's load cache) is the same container with every
// ternary weight stored as dtype "t2": the tiled 2-bit format of common.cuh for the logical
// shape [out, in] (packed_bytes(out, in) bytes), so loading uploads it without a repack.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace mmfree_cuda {

struct BlobConfig {
  size_t vocab_size = 32000;
  size_t hidden_size = 1024;
  size_t num_hidden_layers = 24;
  size_t num_heads = 1;
  size_t expand_ratio = 1;
  size_t intermediate_size = 2816;
  bool use_lower_bound = true;
  bool use_short_conv = false;
  float rms_norm_eps = 1e-6f;
};

struct BlobTensor {
  bool is_int8 = false;
  bool is_packed = false;  // dtype "t2" (model.mmfree2): tiled 2-bit ternary
  std::vector<size_t> shape;
  size_t offset = 0;  // absolute file offset
  size_t nbytes = 0;
  size_t numel() const {
    size_t n = 1;
    for (size_t s : shape) n *= s;
    return shape.empty() ? 0 : n;
  }
};

class Blob {
 public:
  explicit Blob(const std::string& path);  // mmaps the file read-only
  ~Blob();
  Blob(const Blob&) = delete;
  Blob& operator=(const Blob&) = delete;

  const BlobConfig& config() const { return cfg_; }
  bool has(const std::string& name) const { return tensors_.count(name) != 0; }
  const BlobTensor& get(const std::string& name) const;  // throws "weights: missing tensor X"
  const void* data(const BlobTensor& t) const { return static_cast<const char*>(base_) + t.offset; }

 private:
  BlobConfig cfg_;
  std::map<std::string, BlobTensor> tensors_;
  void* base_ = nullptr;
  size_t size_ = 0;
  int fd_ = -1;
};

}  // namespace mmfree_cuda
