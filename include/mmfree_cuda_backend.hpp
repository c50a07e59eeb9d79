// mmfree_cuda_backend.hpp -- a mmfree::TernaryBackend that runs the integer accumulate of the
// reference engine's FixedQ510 BitLinear on the GPU (libmmfree_cuda.so, mmfree_cuda_seam_*).
//
// This is the file a maintainer adds to the reference tree to keep its own Model, kernels
// and numerics and offload only the ternary accumulate -- the seam the reference opens for
// accelerators (matmulfreellmCPU cpp/include/mmfree/ternary_backend.hpp:26-103). Include it
// after the reference's headers are on the include path:
//
//   mmfree::Weights w(path);
//   mmfree::Model m(w, mmfree::ActQuant::FixedQ510, 10);
//   mmfree::cuda::CudaTernaryBackend be(/*device=*/0);
//   m.set_backend(&be, {});   // model.hpp:74-79; proj_id is not needed (weights are keyed
//                             // by their host pointer), so an empty registry is enough
//
// Results are bit-identical to the reference's CpuBackend: the accumulate is exact integer
// arithmetic either way. Every call pays a host<->device round trip of its activations and
// accumulators; the whole-model API (mmfree_cuda.hpp) keeps everything on the GPU instead.
// Needs no CUDA headers: only mmfree_cuda.h and the shared library.
#pragma once

#include <cstddef>
#include <cstdint>

#include "mmfree/ternary_backend.hpp"
#include "mmfree_cuda.hpp"

namespace mmfree {
namespace cuda {

struct CudaTernaryBackend final : mmfree::TernaryBackend {
  // batch: the rows per matmul_batch call the reference's bitlinear chunks into
  // (TernaryBackend::batch_size, ternary_backend.hpp:33-37); larger is fewer round trips.
  explicit CudaTernaryBackend(int device = 0, std::size_t batch = 256) : batch_(batch) {
    check(mmfree_cuda_seam_open(device, &seam_));
  }
  ~CudaTernaryBackend() override { mmfree_cuda_seam_close(seam_); }
  CudaTernaryBackend(const CudaTernaryBackend&) = delete;
  CudaTernaryBackend& operator=(const CudaTernaryBackend&) = delete;

  void matmul(int /*proj_id*/, const std::int32_t* x, std::int32_t* acc, const std::int8_t* wq,
              std::size_t N, std::size_t M) override {
    check(mmfree_cuda_seam_matmul(seam_, wq, N, M, x, acc, 1));
  }
  std::size_t batch_size() const override { return batch_; }
  void matmul_batch(int /*proj_id*/, const std::int32_t* x, std::int32_t* acc,
                    const std::int8_t* wq, std::size_t N, std::size_t M,
                    std::size_t b) override {
    check(mmfree_cuda_seam_matmul(seam_, wq, N, M, x, acc, b));
  }

 private:
  mmfree_cuda_seam* seam_ = nullptr;
  std::size_t batch_;
};

}  // namespace cuda
}  // namespace mmfree
