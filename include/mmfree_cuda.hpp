// mmfree_cuda.hpp -- header-only C++ front of libmmfree_cuda.so with the reference engine's
// signatures (matmulfreellmCPU cpp/include/mmfree/{model,kernels,config}.hpp), so its C++
// callers switch by changing a namespace: mmfree::Model -> mmfree::cuda::Model.
// Errors surface as std::runtime_error carrying mmfree_cuda_last_error(), as the reference's
// do. Needs only this header, mmfree_cuda.h and the shared library (no CUDA headers).
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "mmfree_cuda.h"

namespace mmfree {
namespace cuda {

inline void check(int rc) {
  if (rc != MMFREE_OK) throw std::runtime_error(mmfree_cuda_last_error());
}

enum class ActQuant { Float, FixedQ510 };  // kernels.hpp:26

struct Sampling {  // model.hpp:27-31
  float temperature = 0.0f;
  int top_k = 0;
  std::uint64_t seed = 0;
};

struct Config {  // config.hpp:8-21
  std::size_t vocab_size = 0, hidden_size = 0, num_hidden_layers = 0, num_heads = 1,
              expand_ratio = 1, intermediate_size = 0;
  bool use_lower_bound = true, use_short_conv = false;
  float rms_norm_eps = 1e-6f;
};

inline int act(ActQuant aq) {
  return aq == ActQuant::FixedQ510 ? MMFREE_ACT_FIXED_Q510 : MMFREE_ACT_FLOAT;
}

// mmfree::Model (model.hpp:33-80) on one GPU. Opening the blob replaces
// Weights w(path); Model m(w, aq, frac_bits).
class Model {
 public:
  explicit Model(const std::string& blob_path, ActQuant aq = ActQuant::Float, int frac_bits = 10,
                 int device = 0) {
    check(mmfree_cuda_model_open(blob_path.c_str(), device, act(aq), frac_bits, &h_));
    mmfree_cuda_config c;
    check(mmfree_cuda_model_config(h_, &c));
    cfg_.vocab_size = c.vocab_size;
    cfg_.hidden_size = c.hidden_size;
    cfg_.num_hidden_layers = c.num_hidden_layers;
    cfg_.num_heads = c.num_heads;
    cfg_.expand_ratio = c.expand_ratio;
    cfg_.intermediate_size = c.intermediate_size;
    cfg_.use_lower_bound = c.use_lower_bound != 0;
    cfg_.use_short_conv = c.use_short_conv != 0;
    cfg_.rms_norm_eps = c.rms_norm_eps;
  }
  ~Model() { mmfree_cuda_model_close(h_); }
  Model(const Model&) = delete;
  Model& operator=(const Model&) = delete;

  const Config& config() const { return cfg_; }

  // Model::forward: logits [T, vocab_size] from a zero state.
  void forward(const std::int64_t* ids, std::size_t T, std::vector<float>& logits) {
    logits.resize(T * cfg_.vocab_size);
    check(mmfree_cuda_forward(h_, ids, T, logits.data()));
  }

  // Model::generate: prompt + up to new_tokens ids. on_token fires once per generated id, in
  // order, as soon as the host has it (every step when eos_id >= 0).
  std::vector<std::int64_t> generate(const std::vector<std::int64_t>& ids, std::size_t new_tokens,
                                     std::int64_t eos_id = -1, const Sampling& samp = {},
                                     const std::function<void(std::int64_t)>& on_token = {}) {
    std::vector<std::int64_t> out(ids.size() + new_tokens);
    std::size_t n = 0;
    auto relay = [](std::int64_t id, void* ctx) {
      (*static_cast<const std::function<void(std::int64_t)>*>(ctx))(id);
    };
    check(mmfree_cuda_generate_stream(
        h_, ids.data(), ids.size(), new_tokens, eos_id, samp.temperature, samp.top_k, samp.seed,
        on_token ? +relay : nullptr, const_cast<std::function<void(std::int64_t)>*>(&on_token),
        out.data(), out.size(), &n));
    out.resize(n);
    return out;
  }

  // Model::generate_serve: B lockstep streams.
  std::vector<std::vector<std::int64_t>> generate_serve(
      const std::vector<std::vector<std::int64_t>>& prompts, std::size_t new_tokens,
      std::int64_t eos_id = -1, const Sampling& samp = {}) {
    const std::size_t B = prompts.size();
    std::vector<const std::int64_t*> ptrs(B);
    std::vector<std::size_t> lens(B), out_lens(B);
    std::size_t stride = 0;
    for (std::size_t b = 0; b < B; ++b) {
      ptrs[b] = prompts[b].data();
      lens[b] = prompts[b].size();
      stride = std::max(stride, lens[b] + (new_tokens > 0 ? new_tokens : 1));
    }
    std::vector<std::int64_t> out(B * stride);
    check(mmfree_cuda_generate_serve(h_, B, ptrs.data(), lens.data(), new_tokens, eos_id,
                                     samp.temperature, samp.top_k, samp.seed, out.data(), stride,
                                     out_lens.data()));
    std::vector<std::vector<std::int64_t>> streams(B);
    for (std::size_t b = 0; b < B; ++b)
      streams[b].assign(out.begin() + b * stride, out.begin() + b * stride + out_lens[b]);
    return streams;
  }

  mmfree_cuda_model* handle() { return h_; }

 private:
  mmfree_cuda_model* h_ = nullptr;
  Config cfg_;
};

// mmfree::bitlinear (kernels.hpp:41-44) on device buffers; wq is the packed form produced by
// mmfree_cuda_repack_ternary. stream is a cudaStream_t (nullptr = default stream).
inline void bitlinear(float* out, const float* x, const float* norm_weight, const void* wq_packed,
                      float scale_w, std::size_t rows, std::size_t in_dim, std::size_t out_dim,
                      float eps, float* norm_out = nullptr, ActQuant aq = ActQuant::Float,
                      int frac_bits = 10, std::int32_t* acc_out = nullptr, void* stream = nullptr) {
  check(mmfree_cuda_bitlinear(out, x, norm_weight, wq_packed, scale_w, rows, in_dim, out_dim, eps,
                              norm_out, act(aq), frac_bits, acc_out, stream));
}

inline void rmsnorm(float* y, const float* x, const float* weight, std::size_t rows,
                    std::size_t cols, float eps, void* stream = nullptr) {
  check(mmfree_cuda_rmsnorm(y, x, weight, rows, cols, eps, stream));
}

inline void swiglu(float* out, const float* a, const float* b, std::size_t n,
                   void* stream = nullptr) {
  check(mmfree_cuda_swiglu(out, a, b, n, stream));
}

inline void hgrn_scan(float* out, const float* i, const float* f, std::size_t T, std::size_t D,
                      float* state_io = nullptr, void* stream = nullptr) {
  check(mmfree_cuda_hgrn_scan(out, i, f, T, D, state_io, stream));
}

inline void rmsnorm_swishgate(float* out, const float* g, const float* o, const float* weight,
                              std::size_t rows, std::size_t cols, float eps,
                              void* stream = nullptr) {
  check(mmfree_cuda_rmsnorm_swishgate(out, g, o, weight, rows, cols, eps, stream));
}

}  // namespace cuda
}  // namespace mmfree
