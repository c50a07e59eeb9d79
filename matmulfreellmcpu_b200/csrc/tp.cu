// tp.cu -- tensor-parallel prefill: NCCL communicator and shard glue kernels (see tp.h).
#include "tp.h"

#include <dlfcn.h>
#include <cstring>
#include <nccl.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "exact.cuh"

namespace mmfree_cuda {

// ------------------------------------------------------------------------------ NCCL
// The entry points used here, resolved from libnccl.so.2 at run time. A process that already
// loaded NCCL (e.g. through torch.distributed) gets that copy back from dlopen.
namespace {
struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  static std::string failure;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      failure = std::string("tensor parallelism needs NCCL: ") + dlerror();
      return;
    }
    auto sym = [&](const char* name) {
      void* p = dlsym(h, name);
      if (!p) failure = std::string("NCCL symbol missing: ") + name;
      return p;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
  });
  if (!failure.empty()) throw std::runtime_error(failure);
  return api;
}

void nck(ncclResult_t r, const char* what) {
  if (r != ncclSuccess)
    throw std::runtime_error(std::string("cuda: ") + what + ": " + nccl().error_string(r));
}
}  // namespace

void TpComm::unique_id(unsigned char out[kNcclIdBytes]) {
  static_assert(sizeof(ncclUniqueId) == kNcclIdBytes, "NCCL unique id size");
  ncclUniqueId id;
  nck(nccl().get_unique_id(&id), "ncclGetUniqueId");
  std::memcpy(out, &id, kNcclIdBytes);
}

TpComm::TpComm(const unsigned char id[kNcclIdBytes], int rank, int world) : rank_(rank), world_(world) {
  if (world < 1 || rank < 0 || rank >= world) throw std::invalid_argument("bad rank / world size");
  ncclUniqueId uid;
  std::memcpy(&uid, id, kNcclIdBytes);
  ncclComm_t c = nullptr;
  nck(nccl().comm_init_rank(&c, world, uid, rank), "ncclCommInitRank");
  comm_ = c;
}

TpComm::~TpComm() {
  if (comm_) nccl().comm_destroy(static_cast<ncclComm_t>(comm_));
}

void TpComm::all_gather(const void* send, void* recv, size_t bytes, cudaStream_t s) {
  nck(nccl().all_gather(send, recv, bytes, ncclUint8, static_cast<ncclComm_t>(comm_), s),
      "ncclAllGather");
}

void TpComm::all_reduce_f32(float* buf, size_t count, cudaStream_t s) {
  nck(nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm_), s),
      "ncclAllReduce");
}

// ------------------------------------------------------------------------------ kernels
// One thread per 4 consecutive columns of one row: 16-byte loads and stores when n % 4 == 0.
__global__ void interleave_kernel(float* __restrict__ full, const float* __restrict__ panels, int P,
                                  int T, int n) {
  const int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;  // quad index
  const int nq = n / 4;
  const int64_t total = static_cast<int64_t>(P) * T * nq;
  if (q >= total) return;
  const int c4 = static_cast<int>(q % nq);
  const int64_t pt = q / nq;
  const int t = static_cast<int>(pt % T), p = static_cast<int>(pt / T);
  const float4 v = *reinterpret_cast<const float4*>(panels + (static_cast<int64_t>(p) * T + t) * n + 4 * c4);
  *reinterpret_cast<float4*>(full + static_cast<int64_t>(t) * P * n + static_cast<int64_t>(p) * n + 4 * c4) = v;
}

__global__ void interleave1_kernel(float* __restrict__ full, const float* __restrict__ panels, int P,
                                   int T, int n) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<int64_t>(P) * T * n) return;
  const int c = static_cast<int>(i % n);
  const int64_t pt = i / n;
  const int t = static_cast<int>(pt % T), p = static_cast<int>(pt / T);
  full[static_cast<int64_t>(t) * P * n + static_cast<int64_t>(p) * n + c] = panels[i];
}

cudaError_t launch_interleave(float* full, const float* panels, int P, int T, int n, cudaStream_t s) {
  if (P <= 0 || T <= 0 || n <= 0) return cudaSuccess;
  const bool vec = n % 4 == 0 && (reinterpret_cast<uintptr_t>(full) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(panels) & 15) == 0;
  const int64_t items = static_cast<int64_t>(P) * T * (vec ? n / 4 : n);
  const unsigned grid = static_cast<unsigned>(ceil_div(items, 256));
  if (vec) interleave_kernel<<<grid, 256, 0, s>>>(full, panels, P, T, n);
  else interleave1_kernel<<<grid, 256, 0, s>>>(full, panels, P, T, n);
  return cudaGetLastError();
}

// one warp per row: strided partial sums, then a shuffle tree
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void row_sumsq_kernel(float* __restrict__ ss, const float* __restrict__ x, int T, int n,
                                 int ld) {
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (t >= T) return;
  const float* r = x + static_cast<int64_t>(t) * ld;
  float a = 0.0f;
  for (int c = lane; c < n; c += 32) a = __fmaf_rn(r[c], r[c], a);
  a = warp_sum(a);
  if (lane == 0) ss[t] = a;
}

cudaError_t launch_row_sumsq(float* ss, const float* x, int T, int n, int ld, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  row_sumsq_kernel<<<static_cast<unsigned>(ceil_div(T, 8)), 256, 0, s>>>(ss, x, T, n, ld);
  return cudaGetLastError();
}

__global__ void gate_slice_kernel(float* __restrict__ t_out, float* __restrict__ ss_t,
                                  const float* __restrict__ g, const float* __restrict__ o,
                                  const float* __restrict__ ss_g, const float* __restrict__ w, int T,
                                  int n, int K, float eps) {
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (t >= T) return;
  const float r = rstd_of(ss_g[t], static_cast<float>(K), eps);
  const int64_t base = static_cast<int64_t>(t) * n;
  float a = 0.0f;
  for (int c = lane; c < n; c += 32) {
    const float v = __fmul_rn(norm_x(g[base + c], r, w[c]), silu_x(o[base + c], true));
    t_out[base + c] = v;
    a = __fmaf_rn(v, v, a);
  }
  a = warp_sum(a);
  if (lane == 0) ss_t[t] = a;
}

cudaError_t launch_gate_slice(float* t, float* ss_t, const float* g, const float* o,
                              const float* ss_g, const float* w, int T, int n, int K, float eps,
                              cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  gate_slice_kernel<<<static_cast<unsigned>(ceil_div(T, 8)), 256, 0, s>>>(t, ss_t, g, o, ss_g, w, T,
                                                                         n, K, eps);
  return cudaGetLastError();
}

__global__ void norm_slice_kernel(float* __restrict__ yf, const float* __restrict__ x,
                                  const float* __restrict__ ss, const float* __restrict__ w, int T,
                                  int n, int kp, int K, float eps) {
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T || c >= kp) return;
  const float r = rstd_of(ss[t], static_cast<float>(K), eps);
  yf[static_cast<int64_t>(t) * kp + c] = c < n ? norm_x(x[static_cast<int64_t>(t) * n + c], r, w[c]) : 0.0f;
}

cudaError_t launch_norm_slice(float* yf, const float* x, const float* ss, const float* w, int T,
                              int n, int kp, int K, float eps, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (T > 65535) return cudaErrorInvalidValue;
  norm_slice_kernel<<<dim3(static_cast<unsigned>(ceil_div(kp, 256)), T), 256, 0, s>>>(yf, x, ss, w, T,
                                                                                      n, kp, K, eps);
  return cudaGetLastError();
}

// The same rows as bf16 hi / lo planes [2][T][kp] for the tensor-core Float BitLinear (hi =
// bf16(y), lo = bf16(y - hi)), four elements per thread.
__global__ void norm_slice_planes_kernel(int8_t* __restrict__ planes, const float* __restrict__ x,
                                         const float* __restrict__ ss, const float* __restrict__ w, int T,
                                         int n, int kp, int K, float eps) {
  const int t = blockIdx.y;
  const int c0 = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (t >= T || c0 >= kp) return;
  const float r = rstd_of(ss[t], static_cast<float>(K), eps);
  float y[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int c = c0 + u;
    y[u] = c < n ? norm_x(x[static_cast<int64_t>(t) * n + c], r, w[c]) : 0.0f;
  }
  uint2 hi, lo;
  bf16_split4(y, hi, lo);
  *reinterpret_cast<uint2*>(planes + 2 * (static_cast<int64_t>(t) * kp + c0)) = hi;
  *reinterpret_cast<uint2*>(planes + 2 * ((static_cast<int64_t>(T) + t) * kp + c0)) = lo;
}

cudaError_t launch_norm_slice_planes(int8_t* planes, const float* x, const float* ss, const float* w, int T,
                                     int n, int kp, int K, float eps, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (T > 65535 || kp % 4 != 0 || (reinterpret_cast<uintptr_t>(planes) & 7) != 0) return cudaErrorInvalidValue;
  norm_slice_planes_kernel<<<dim3(static_cast<unsigned>(ceil_div(kp / 4, 256)), T), 256, 0, s>>>(
      planes, x, ss, w, T, n, kp, K, eps);
  return cudaGetLastError();
}

__global__ void add_kernel(float* __restrict__ out, const float* __restrict__ a,
                           const float* __restrict__ b, int64_t n) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) out[i] = __fadd_rn(a[i], b[i]);
}

cudaError_t launch_add(float* out, const float* a, const float* b, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  add_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, s>>>(out, a, b, n);
  return cudaGetLastError();
}

}  // namespace mmfree_cuda
