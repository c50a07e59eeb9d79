// tp.h -- tensor-parallel prefill support: the NCCL communicator (loaded at run time) and the
// kernels that glue column / row shards of the BitLinear projections together.
//
// The layer split (matmulfreellmCPU cpp/src/model/hgrn_model.cpp:80-195, one rank per GPU):
//   FixedQ510  every projection is column-parallel (a rank owns N/P output features, the
//              SwiGLU pair of gate_proj included); a full row is gathered (NCCL all-gather
//              of the column slices) before each exact norm -- g and the recurrence before
//              g_norm, the residual before mlp_norm, z before down_proj, h before the next
//              layer -- because the reference's sum of squares is one serial AVX2-order
//              chain over the whole row. Results are bit-identical to one GPU.
//   Float      i/f/g and gate_proj column-parallel, o_proj and down_proj row-parallel (a rank
//              owns K/P input features): the norms before g_norm, o_proj and down_proj take
//              the row's sum of squares as an all-reduce of per-rank partial sums ([T]
//              floats), and the row-parallel outputs are summed by an all-reduce of [T, H].
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace mmfree_cuda {

constexpr int kNcclIdBytes = 128;

// One NCCL communicator over `world` ranks (libnccl.so.2 is loaded on first use; the library
// has no link-time dependency on it). Collectives are enqueued on the given stream.
class TpComm {
 public:
  static void unique_id(unsigned char out[kNcclIdBytes]);
  TpComm(const unsigned char id[kNcclIdBytes], int rank, int world);
  ~TpComm();
  TpComm(const TpComm&) = delete;
  TpComm& operator=(const TpComm&) = delete;
  int rank() const { return rank_; }
  int world() const { return world_; }
  // recv [world][bytes] = every rank's send [bytes]
  void all_gather(const void* send, void* recv, size_t bytes, cudaStream_t s);
  // in-place sums over ranks
  void all_reduce_f32(float* buf, size_t count, cudaStream_t s);

 private:
  void* comm_ = nullptr;
  int rank_ = 0, world_ = 1;
};

// full[t][p * n + c] = panels[p][t][c] for p < P (the layout an all-gather of column slices
// [T, n] produces, back to row-major [T, P n]).
cudaError_t launch_interleave(float* full, const float* panels, int P, int T, int n,
                              cudaStream_t s);
// Float-mode row-parallel helpers (fp32; the sums are re-associated, which Float allows).
// ss[t] = sum_c x[t, c]^2 over this rank's n columns (row stride ld).
cudaError_t launch_row_sumsq(float* ss, const float* x, int T, int n, int ld, cudaStream_t s);
// t = g * rstd(ss_g, K) * w * silu(o) on this rank's columns, and ss_t = its partial sum of
// squares (rmsnorm_swishgate.cpp:13-30 on a column slice; K = the full row length).
cudaError_t launch_gate_slice(float* t, float* ss_t, const float* g, const float* o,
                              const float* ss_g, const float* w, int T, int n, int K, float eps,
                              cudaStream_t s);
// yf[t][c] = x[t, c] * rstd(ss, K) * w[c] for c < n, 0 up to kp (the BitLinear norm of a
// column slice, bitlinear.cpp:95-105, into the float matmul's activation layout).
cudaError_t launch_norm_slice(float* yf, const float* x, const float* ss, const float* w, int T,
                              int n, int kp, int K, float eps, cudaStream_t s);
// The same as bf16 hi / lo planes [2][T][kp] (the tensor-core Float BitLinear's input).
cudaError_t launch_norm_slice_planes(int8_t* planes, const float* x, const float* ss, const float* w, int T,
                                     int n, int kp, int K, float eps, cudaStream_t s);
// out[i] = a[i] + b[i]
cudaError_t launch_add(float* out, const float* a, const float* b, int64_t n, cudaStream_t s);

}  // namespace mmfree_cuda
