// capi.cu -- the extern "C" boundary of libmmfree_cuda.so (declared in include/mmfree_cuda.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/mmfree_cuda.h"
#include "common.cuh"
#include "kernels.h"
#include "blob.h"
#include "model.h"
#include "tp.h"

using namespace mmfree_cuda;

struct mmfree_cuda_model {
  Model* impl;
};

namespace {

thread_local std::string g_last_error;

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct TimeoutError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

// Map exceptions to status codes; the message is kept for mmfree_cuda_last_error().
template <class F>
int guard(F&& f) {
  try {
    f();
    return MMFREE_OK;
  } catch (const std::invalid_argument& e) {
    g_last_error = e.what();
    return MMFREE_E_INVALID;
  } catch (const std::out_of_range& e) {
    g_last_error = e.what();
    return MMFREE_E_RANGE;
  } catch (const std::logic_error& e) {
    g_last_error = e.what();
    return MMFREE_E_STATE;
  } catch (const CudaError& e) {
    g_last_error = e.what();
    return MMFREE_E_CUDA;
  } catch (const TimeoutError& e) {
    g_last_error = e.what();
    return MMFREE_E_TIMEOUT;
  } catch (const std::bad_alloc&) {
    g_last_error = "host out of memory";
    return MMFREE_E_INTERNAL;
  } catch (const std::runtime_error& e) {
    g_last_error = e.what();
    const bool cuda = std::strncmp(e.what(), "cuda:", 5) == 0;
    return cuda ? MMFREE_E_CUDA : MMFREE_E_IO;
  } catch (...) {
    g_last_error = "unknown error";
    return MMFREE_E_INTERNAL;
  }
}

void need(bool ok, const char* what) {
  if (!ok) throw std::invalid_argument(what);
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Library-owned scratch of the kernel entry points: one grow-only arena per device. Its first
// 256 bytes hold two words of device error flags: word 0 for the synchronous entry points
// (repack, ternary_matmul: checked and cleared before they return), word 1 for the
// asynchronous ones (bitlinear, bitlinear_cluster: read and cleared by
// mmfree_cuda_kernel_status).
struct Scratch {
  void* base = nullptr;
  size_t bytes = 0;
};
std::mutex g_scratch_mu;
Scratch g_scratch[64];
constexpr size_t kAsyncFlagWord = 1;  // index of the asynchronous entry points' word

char* scratch(size_t bytes) {
  int dev = 0;
  ck(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  Scratch& s = g_scratch[dev & 63];
  bytes += 256;
  if (bytes > s.bytes) {
    uint32_t words[2] = {0, 0};  // flags not yet reported survive the move to a larger arena
    if (s.base) {
      ck(cudaMemcpy(words, s.base, sizeof(words), cudaMemcpyDeviceToHost), "cudaMemcpy(flags)");
      ck(cudaFree(s.base), "cudaFree");  // synchronizes with work still using it
    }
    s.base = nullptr;
    s.bytes = 0;
    const size_t grow = bytes < (size_t(1) << 20) ? (size_t(1) << 20) : bytes;
    ck(cudaMalloc(&s.base, grow), "cudaMalloc(scratch)");
    ck(cudaMemset(s.base, 0, 256), "cudaMemset(scratch)");
    ck(cudaMemcpy(s.base, words, sizeof(words), cudaMemcpyHostToDevice), "cudaMemcpy(flags)");
    ck(cudaDeviceSynchronize(), "cudaDeviceSynchronize");  // order before any caller stream
    s.bytes = grow;
  }
  return static_cast<char*>(s.base);
}

// Reads and clears one device flag word on `st` (synchronizing it); returns the flags.
uint32_t take_flags(uint32_t* word, cudaStream_t st) {
  uint32_t f = 0;
  ck(cudaMemcpyAsync(&f, word, 4, cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync(flags)");
  ck(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  if (f) {
    ck(cudaMemsetAsync(word, 0, 4, st), "cudaMemsetAsync(flags)");
    ck(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  }
  return f;
}

size_t a256(size_t n) { return (n + 255) / 256 * 256; }

void check_flags(uint32_t* flags, cudaStream_t st) {
  const uint32_t f = take_flags(flags, st);
  if (f) {
    if (f & kErrRange) throw std::out_of_range("activation code outside int16");
    if (f & kErrNotTernary) throw std::out_of_range("weight outside {-1,0,+1}");
    if (f & kErrTimeout) throw TimeoutError("a bounded wait inside a kernel gave up");
    throw std::runtime_error("device error flag set");
  }
}

void check_dims(size_t rows, size_t in_dim, size_t out_dim) {
  need(in_dim > 0 && out_dim > 0, "in_dim and out_dim must be positive");
  need(in_dim <= MMFREE_CUDA_MAX_IN_DIM, "in_dim above MMFREE_CUDA_MAX_IN_DIM");
  need(out_dim <= (size_t(1) << 30) && rows <= (size_t(1) << 30), "dimension too large");
}

int sm_count_of_device() {
  int dev = 0, n = 0;
  ck(cudaGetDevice(&dev), "cudaGetDevice");
  ck(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
  return n > 0 ? n : 148;
}

// One or more BitLinear projections sharing x (bitlinear / bitlinear_cluster).
void run_bitlinear(int k, float* const* outs, const float* x, const float* const* nws,
                   const void* const* ws, const float* scales, size_t rows, size_t in_dim,
                   size_t out_dim, float eps, float* norm_out, bool fixed, int frac_bits,
                   int32_t* acc_out, cudaStream_t st) {
  check_dims(rows, in_dim, out_dim);
  need(frac_bits >= 0 && frac_bits <= 30, "frac_bits must be in [0, 30]");
  need(x != nullptr, "null x");
  for (int j = 0; j < k; ++j) need(outs[j] && nws[j] && ws[j], "null output, norm weight or weights");
  if (rows == 0) return;
  if (k == 1 && rows <= static_cast<size_t>(kDecMaxRows) && !norm_out && !acc_out) {
    // a few rows: one fused launch (each CTA normalises and quantises the rows itself, its
    // first weight unit staged in shared memory), the batch-1 decode kernel of the model
    DecArgs d;
    d.x = x;
    d.normw[0] = nws[0];
    d.w[0] = ws[0];
    d.M = static_cast<int>(rows);
    d.K = static_cast<int>(in_dim);
    d.N = static_cast<int>(out_dim);
    d.eps = eps;
    d.qs = static_cast<float>(1u << frac_bits);
    d.scale[0] = fixed ? 1.0f / (d.qs * scales[0]) : 1.0f / scales[0];
    d.out[0] = outs[0];
    d.fl = fixed ? 0 : 1;
    const int grid = std::max(1, std::min(dec_units(d, kDecEpiResid), 2 * sm_count_of_device()));
    // as a programmatic dependent: back-to-back calls stream the next call's first weight
    // units while this one finishes (before its dependency wait the kernel reads only weights
    // and writes nothing; a previous kernel that does not trigger early, like the repack,
    // still completes before it starts)
    if (launch_dec(d, kDecProPlain, kDecEpiResid, grid, st, true) == cudaSuccess) return;
    (void)cudaGetLastError();  // shape the fused kernel cannot stage: the general path below
  }
  const size_t kp = static_cast<size_t>(padded_k(static_cast<int64_t>(in_dim)));
  const size_t per = fixed ? a256(2 * rows * kp) + a256(rows * 4) : a256(rows * kp * 4);
  char* base = scratch(static_cast<size_t>(k) * per);
  PrepArgs p;
  p.x = x;
  p.nproj = k;
  p.norm_out = norm_out;
  p.M = static_cast<int>(rows);
  p.K = static_cast<int>(in_dim);
  p.eps = eps;
  p.qs = static_cast<float>(1u << frac_bits);
  p.fixed = fixed;
  // the tensor-core matmul (taken for >= kTcMinRows fixed rows) reads the low plane as lo - 128
  p.lo_signed = fixed && static_cast<int>(rows) >= kTcMinRows;
  // Float rows on the tensor cores too: the activations as bf16 hi / lo planes (the same 4
  // bytes per element as fp32 activations)
  p.bf16 = !fixed && static_cast<int>(rows) >= kTcMinRows;
  uint32_t* err = reinterpret_cast<uint32_t*>(base) + kAsyncFlagWord;
  p.err = err;
  for (int j = 0; j < k; ++j) {
    char* b = base + 256 + j * per;
    p.normw[j] = nws[j];
    if (fixed) {
      p.planes[j] = reinterpret_cast<int8_t*>(b);
      p.rowsum[j] = reinterpret_cast<int32_t*>(b + a256(2 * rows * kp));
    } else if (p.bf16) {
      p.planes[j] = reinterpret_cast<int8_t*>(b);
    } else {
      p.yf[j] = reinterpret_cast<float*>(b);
    }
  }
  ck(launch_prep(p, st), "prep kernel");
  for (int j = 0; j < k; ++j) {
    MatmulArgs a;
    a.w = ws[j];
    a.planes = p.planes[j];
    a.rowsum = p.rowsum[j];
    a.yf = p.yf[j];
    a.M = static_cast<int>(rows);
    a.N = static_cast<int>(out_dim);
    a.K = static_cast<int>(in_dim);
    a.scale = fixed ? 1.0f / (p.qs * scales[j]) : 1.0f / scales[j];
    a.out = outs[j];
    a.ldo = static_cast<int>(out_dim);
    a.acc_out = (acc_out && fixed) ? acc_out + static_cast<size_t>(j) * rows * out_dim : nullptr;
    a.fixed = fixed;
    a.allow_tc = true;
    a.lo_signed = p.lo_signed;
    a.bf16 = p.bf16;
    a.err = err;
    ck(launch_matmul(a, st), "matmul kernel");
  }
}

}  // namespace

// ---- allocation-free BitLinear scratch ------------------------------------------------------
// Compiled into the library: each device that loads this module holds one copy until the
// process exits. Bytes [0, 256) hold the calls' device error word; the activation planes
// follow. Host code must not use the symbol as an address (it names a host-side stand-in);
// the device address comes from cudaGetSymbolAddress, looked up per device with that device
// current and kept only once the lookup succeeded.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MMFREE_CUDA_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr size_t kNoallocHeader = 256;
std::mutex g_noalloc_mu;
char* g_noalloc_addr[64];

char* noalloc_base(int dev) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    char* p = nullptr;
    ck(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_scratch),
       "cudaGetSymbolAddress(noalloc scratch)");
    ck(cudaMemset(p, 0, kNoallocHeader), "cudaMemset(noalloc error word)");
    ck(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    g_noalloc_addr[dev] = p;
  }
  return g_noalloc_addr[dev];
}

char* noalloc_base_if_ready(int dev) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  return g_noalloc_addr[dev];
}

}  // namespace

extern "C" {

const char* mmfree_cuda_last_error(void) { return g_last_error.c_str(); }
int mmfree_cuda_abi_version(void) { return MMFREE_CUDA_ABI_VERSION; }

size_t mmfree_cuda_packed_bytes(size_t out_dim, size_t in_dim) {
  return static_cast<size_t>(packed_bytes(static_cast<int64_t>(out_dim), static_cast<int64_t>(in_dim)));
}

int mmfree_cuda_repack_ternary(void* dst, const int8_t* wq, size_t out_dim, size_t in_dim,
                               void* stream) {
  return guard([&] {
    need(dst && wq && out_dim > 0 && in_dim > 0, "repack: null pointer or zero dimension");
    uint32_t* flags = reinterpret_cast<uint32_t*>(scratch(0));
    ck(launch_repack(dst, wq, static_cast<int64_t>(out_dim), static_cast<int64_t>(in_dim), flags,
                     as_stream(stream)),
       "repack kernel");
    check_flags(flags, as_stream(stream));
  });
}

int mmfree_cuda_pack_ternary_host(void* dst, const int8_t* wq, size_t out_dim, size_t in_dim) {
  return guard([&] {
    need(dst && wq && out_dim > 0 && in_dim > 0, "pack: null pointer or zero dimension");
    const int64_t kc = packed_chunks(static_cast<int64_t>(in_dim));
    const int64_t ng = packed_groups(static_cast<int64_t>(out_dim));
    auto* out = static_cast<uint32_t*>(dst);
    for (int64_t g = 0; g < ng; ++g)
      for (int64_t c = 0; c < kc; ++c)
        for (int r = 0; r < kRowsPerGroup; ++r)
          for (int w = 0; w < 4; ++w) {
            const int64_t row = g * kRowsPerGroup + r;
            uint32_t word = 0;
            for (int i = 0; i < 16; ++i) {
              const int64_t k = c * kChunkK + w * 16 + i;
              uint32_t u = 1;
              if (row < static_cast<int64_t>(out_dim) && k < static_cast<int64_t>(in_dim)) {
                const int v = wq[row * static_cast<int64_t>(in_dim) + k];
                if (v < -1 || v > 1) throw std::out_of_range("weight outside {-1,0,+1}");
                u = static_cast<uint32_t>(v + 1);
              }
              word |= u << (8 * (i & 3) + 2 * (i >> 2));
            }
            out[((g * kc + c) * kRowsPerGroup + r) * 4 + w] = word;
          }
  });
}

int mmfree_cuda_bitlinear(float* out, const float* x, const float* norm_weight,
                          const void* wpacked, float scale_w, size_t rows, size_t in_dim,
                          size_t out_dim, float eps, float* norm_out, int act_quant,
                          int frac_bits, int32_t* acc_out, void* stream) {
  return guard([&] {
    need(act_quant == MMFREE_ACT_FLOAT || act_quant == MMFREE_ACT_FIXED_Q510, "bad act_quant");
    float* outs[1] = {out};
    const float* nws[1] = {norm_weight};
    const void* ws[1] = {wpacked};
    run_bitlinear(1, outs, x, nws, ws, &scale_w, rows, in_dim, out_dim, eps, norm_out,
                  act_quant == MMFREE_ACT_FIXED_Q510, frac_bits, acc_out, as_stream(stream));
  });
}

// ---- allocation-free BitLinear -------------------------------------------------------------
int mmfree_cuda_bitlinear_noalloc(float* out, const float* x, const float* norm_weight,
                                  const void* wpacked, float scale_w, size_t rows,
                                  size_t in_dim, size_t out_dim, float eps, float* norm_out,
                                  int act_quant, int frac_bits, int32_t* acc_out, void* stream) {
  return guard([&] {
    need(act_quant == MMFREE_ACT_FLOAT || act_quant == MMFREE_ACT_FIXED_Q510, "bad act_quant");
    check_dims(rows, in_dim, out_dim);
    need(frac_bits >= 0 && frac_bits <= 30, "frac_bits must be in [0, 30]");
    need(out && x && norm_weight && wpacked, "null output, input, norm weight or weights");
    if (rows == 0) return;
    const bool fixed = act_quant == MMFREE_ACT_FIXED_Q510;
    const size_t kp = static_cast<size_t>(padded_k(static_cast<int64_t>(in_dim)));
    const size_t planes_bytes = fixed ? a256(2 * rows * kp) : a256(rows * kp * 4);
    const size_t need_bytes = kNoallocHeader + planes_bytes + (fixed ? a256(rows * 4) : 0);
    need(need_bytes <= MMFREE_CUDA_NOALLOC_SCRATCH_BYTES,
         "bitlinear_noalloc: rows x in_dim needs more scratch than "
         "MMFREE_CUDA_NOALLOC_SCRATCH_BYTES (use mmfree_cuda_bitlinear or fewer rows per call)");
    int dev = 0;
    ck(cudaGetDevice(&dev), "cudaGetDevice");
    need(dev >= 0 && dev < 64, "device index above 63");
    char* const head = noalloc_base(dev);
    auto* err = reinterpret_cast<uint32_t*>(head);
    char* const base = head + kNoallocHeader;
    cudaStream_t st = as_stream(stream);
    PrepArgs p;
    p.x = x;
    p.nproj = 1;
    p.normw[0] = norm_weight;
    p.norm_out = norm_out;
    p.M = static_cast<int>(rows);
    p.K = static_cast<int>(in_dim);
    p.eps = eps;
    p.qs = static_cast<float>(1u << frac_bits);
    p.fixed = fixed;
    // the same kernels as mmfree_cuda_bitlinear: tensor cores from kTcMinRows fixed rows
    p.lo_signed = fixed && static_cast<int>(rows) >= kTcMinRows;
    p.err = err;
    if (fixed) {
      p.planes[0] = reinterpret_cast<int8_t*>(base);
      p.rowsum[0] = reinterpret_cast<int32_t*>(base + planes_bytes);
    } else {
      p.yf[0] = reinterpret_cast<float*>(base);
    }
    ck(launch_prep(p, st), "prep kernel");
    MatmulArgs a;
    a.w = wpacked;
    a.planes = p.planes[0];
    a.rowsum = p.rowsum[0];
    a.yf = p.yf[0];
    a.M = static_cast<int>(rows);
    a.N = static_cast<int>(out_dim);
    a.K = static_cast<int>(in_dim);
    a.scale = fixed ? 1.0f / (p.qs * scale_w) : 1.0f / scale_w;
    a.out = out;
    a.ldo = static_cast<int>(out_dim);
    a.acc_out = fixed ? acc_out : nullptr;
    a.fixed = fixed;
    a.allow_tc = true;
    a.lo_signed = p.lo_signed;
    a.err = err;
    ck(launch_matmul(a, st), "matmul kernel");
  });
}

int mmfree_cuda_kernel_status(void* stream) {
  return guard([&] {
    int dev = 0;
    ck(cudaGetDevice(&dev), "cudaGetDevice");
    need(dev >= 0 && dev < 64, "device index above 63");
    cudaStream_t st = as_stream(stream);
    uint32_t f = 0;
    char* arena = nullptr;
    {
      std::lock_guard<std::mutex> lock(g_scratch_mu);
      arena = static_cast<char*>(g_scratch[dev].base);
    }
    if (arena) f |= take_flags(reinterpret_cast<uint32_t*>(arena) + kAsyncFlagWord, st);
    if (char* head = noalloc_base_if_ready(dev)) f |= take_flags(reinterpret_cast<uint32_t*>(head), st);
    if (f & kErrTimeout)
      throw TimeoutError("a bounded wait inside a BitLinear kernel gave up: the outputs of the "
                         "kernel calls since the last status check are undefined");
    if (f) throw std::runtime_error("device error flag set");
  });
}

void mmfree_cuda_set_wait_limit(int64_t polls) { set_wait_limit(polls); }

int mmfree_cuda_bitlinear_cluster(float* const* outs, const float* x,
                                  const float* const* norm_weights,
                                  const void* const* wpacked, const float* scale_w, int k,
                                  size_t rows, size_t in_dim, size_t out_dim, float eps,
                                  int frac_bits, int32_t* acc_out, void* stream) {
  return guard([&] {
    need(k >= 1 && k <= 3, "cluster size k must be 1..3");
    need(outs && norm_weights && wpacked && scale_w, "null array");
    run_bitlinear(k, outs, x, norm_weights, wpacked, scale_w, rows, in_dim, out_dim, eps,
                  nullptr, true, frac_bits, acc_out, as_stream(stream));
  });
}

int mmfree_cuda_ternary_matmul(int32_t* acc, const int32_t* x, const void* wpacked, size_t N,
                               size_t M, size_t b, void* stream) {
  return guard([&] {
    check_dims(b, N, M);
    need(acc && x && wpacked, "null pointer");
    if (b == 0) return;
    const size_t kp = static_cast<size_t>(padded_k(static_cast<int64_t>(N)));
    char* base = scratch(a256(2 * b * kp) + a256(b * 4));
    auto* flags = reinterpret_cast<uint32_t*>(base);
    auto* planes = reinterpret_cast<int8_t*>(base + 256);
    auto* rowsum = reinterpret_cast<int32_t*>(base + 256 + a256(2 * b * kp));
    cudaStream_t st = as_stream(stream);
    ck(launch_codes_to_planes(planes, rowsum, x, static_cast<int>(b), static_cast<int>(N), flags,
                              st),
       "codes kernel");
    MatmulArgs a;
    a.w = wpacked;
    a.planes = planes;
    a.rowsum = rowsum;
    a.M = static_cast<int>(b);
    a.N = static_cast<int>(M);
    a.K = static_cast<int>(N);
    a.acc_out = acc;
    a.fixed = true;
    ck(launch_matmul(a, st), "matmul kernel");
    check_flags(flags, st);
  });
}

// ---- TernaryBackend seam over host buffers ------------------------------------------------
struct mmfree_cuda_seam {
  int device = 0;
  cudaStream_t st = nullptr;
  // packed weights per (host wq pointer, out_dim, in_dim), uploaded on first sight
  std::map<std::tuple<const int8_t*, size_t, size_t>, void*> packed;
  char* dev = nullptr;  // flags (256 B), x codes, planes, row sums, accumulators
  size_t dev_bytes = 0;
  int8_t* stage = nullptr;  // int8 upload buffer of the repack
  size_t stage_bytes = 0;
};

int mmfree_cuda_seam_open(int device, mmfree_cuda_seam** out) {
  return guard([&] {
    need(out != nullptr, "null pointer");
    *out = nullptr;
    int n = 0;
    ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    need(device >= 0 && device < n, "no such CUDA device");
    ck(cudaSetDevice(device), "cudaSetDevice");
    auto* s = new mmfree_cuda_seam;
    s->device = device;
    if (cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking) != cudaSuccess) {
      delete s;
      throw CudaError("cudaStreamCreate failed");
    }
    *out = s;
  });
}

void mmfree_cuda_seam_close(mmfree_cuda_seam* s) {
  if (!s) return;
  cudaSetDevice(s->device);
  cudaStreamSynchronize(s->st);
  for (auto& kv : s->packed) cudaFree(kv.second);
  cudaFree(s->dev);
  cudaFree(s->stage);
  cudaStreamDestroy(s->st);
  delete s;
}

int mmfree_cuda_seam_matmul(mmfree_cuda_seam* s, const int8_t* wq, size_t N, size_t M,
                            const int32_t* x, int32_t* acc, size_t b) {
  return guard([&] {
    need(s && wq && x && acc, "null pointer");
    check_dims(b, N, M);
    if (b == 0) return;
    ck(cudaSetDevice(s->device), "cudaSetDevice");
    cudaStream_t st = s->st;
    const size_t kp = static_cast<size_t>(padded_k(static_cast<int64_t>(N)));
    const size_t o_x = 256, o_pl = o_x + a256(4 * b * N), o_rs = o_pl + a256(2 * b * kp),
                 o_acc = o_rs + a256(4 * b), total = o_acc + a256(4 * b * M);
    if (total > s->dev_bytes) {
      ck(cudaStreamSynchronize(st), "cudaStreamSynchronize");
      cudaFree(s->dev);
      s->dev = nullptr;
      s->dev_bytes = 0;
      ck(cudaMalloc(&s->dev, total), "cudaMalloc(seam)");
      ck(cudaMemsetAsync(s->dev, 0, 256, st), "cudaMemsetAsync(seam flags)");
      s->dev_bytes = total;
    }
    auto* flags = reinterpret_cast<uint32_t*>(s->dev);
    const auto key = std::make_tuple(wq, M, N);
    auto it = s->packed.find(key);
    if (it == s->packed.end()) {
      if (M * N > s->stage_bytes) {
        ck(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        cudaFree(s->stage);
        s->stage = nullptr;
        s->stage_bytes = 0;
        ck(cudaMalloc(&s->stage, M * N), "cudaMalloc(seam staging)");
        s->stage_bytes = M * N;
      }
      void* p = nullptr;
      ck(cudaMalloc(&p, static_cast<size_t>(packed_bytes(M, N))), "cudaMalloc(seam weights)");
      ck(cudaMemcpyAsync(s->stage, wq, M * N, cudaMemcpyHostToDevice, st), "cudaMemcpyAsync(wq)");
      ck(launch_repack(p, s->stage, static_cast<int64_t>(M), static_cast<int64_t>(N), flags, st),
         "repack kernel");
      it = s->packed.emplace(key, p).first;
    }
    auto* dx = reinterpret_cast<int32_t*>(s->dev + o_x);
    auto* planes = reinterpret_cast<int8_t*>(s->dev + o_pl);
    auto* rowsum = reinterpret_cast<int32_t*>(s->dev + o_rs);
    auto* dacc = reinterpret_cast<int32_t*>(s->dev + o_acc);
    ck(cudaMemcpyAsync(dx, x, 4 * b * N, cudaMemcpyHostToDevice, st), "cudaMemcpyAsync(x)");
    ck(launch_codes_to_planes(planes, rowsum, dx, static_cast<int>(b), static_cast<int>(N), flags,
                              st),
       "codes kernel");
    MatmulArgs a;
    a.w = it->second;
    a.planes = planes;
    a.rowsum = rowsum;
    a.M = static_cast<int>(b);
    a.N = static_cast<int>(M);
    a.K = static_cast<int>(N);
    a.acc_out = dacc;
    a.fixed = true;
    ck(launch_matmul(a, st), "matmul kernel");
    ck(cudaMemcpyAsync(acc, dacc, 4 * b * M, cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync(acc)");
    check_flags(flags, st);  // synchronizes: acc is final on return
  });
}

int mmfree_cuda_rmsnorm(float* y, const float* x, const float* weight, size_t rows,
                        size_t cols, float eps, void* stream) {
  return guard([&] {
    need(y && x && weight, "null pointer");
    check_dims(rows, cols, 1);
    ck(launch_rmsnorm(y, x, weight, static_cast<int>(rows), static_cast<int>(cols), eps,
                      as_stream(stream)),
       "rmsnorm kernel");
  });
}

int mmfree_cuda_swiglu(float* out, const float* a, const float* b, size_t n, void* stream) {
  return guard([&] {
    need(out && a && b, "null pointer");
    ck(launch_swiglu(out, a, b, static_cast<int64_t>(n), as_stream(stream)), "swiglu kernel");
  });
}

int mmfree_cuda_hgrn_scan(float* out, const float* i, const float* f, size_t T, size_t D,
                          float* state_io, void* stream) {
  return guard([&] {
    need(out && i && f, "null pointer");
    need(T < (size_t(1) << 31) && D < (size_t(1) << 31), "dimension too large");
    ck(launch_scan(out, i, f, static_cast<int>(T), static_cast<int>(D), state_io,
                   as_stream(stream)),
       "scan kernel");
  });
}

int mmfree_cuda_rmsnorm_swishgate(float* out, const float* g, const float* o,
                                  const float* weight, size_t rows, size_t cols, float eps,
                                  void* stream) {
  return guard([&] {
    need(out && g && o && weight, "null pointer");
    check_dims(rows, cols, 1);
    ck(launch_swishgate(out, g, o, weight, static_cast<int>(rows), static_cast<int>(cols), eps,
                        as_stream(stream)),
       "swishgate kernel");
  });
}

// ---- model -------------------------------------------------------------------------------
int mmfree_cuda_model_open(const char* blob_path, int device, int act_quant, int frac_bits,
                           mmfree_cuda_model** out) {
  return guard([&] {
    need(blob_path && out, "null pointer");
    need(act_quant == MMFREE_ACT_FLOAT || act_quant == MMFREE_ACT_FIXED_Q510, "bad act_quant");
    need(frac_bits >= 0 && frac_bits <= 30, "frac_bits must be in [0, 30]");
    *out = nullptr;
    int n = 0;
    ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    need(device >= 0 && device < n, "no such CUDA device");
    auto* h = new mmfree_cuda_model{nullptr};
    try {
      h->impl = new Model(blob_path, device, act_quant == MMFREE_ACT_FIXED_Q510, frac_bits);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int mmfree_cuda_nccl_unique_id(unsigned char* out) {
  return guard([&] {
    need(out != nullptr, "null pointer");
    TpComm::unique_id(out);
  });
}

int mmfree_cuda_model_open_tp(const char* blob_path, int device, int act_quant, int frac_bits,
                              int rank, int world, const unsigned char* nccl_id,
                              mmfree_cuda_model** out) {
  return guard([&] {
    need(blob_path && out && nccl_id, "null pointer");
    need(act_quant == MMFREE_ACT_FLOAT || act_quant == MMFREE_ACT_FIXED_Q510, "bad act_quant");
    need(frac_bits >= 0 && frac_bits <= 30, "frac_bits must be in [0, 30]");
    need(world >= 1 && rank >= 0 && rank < world, "bad rank / world size");
    *out = nullptr;
    int n = 0;
    ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    need(device >= 0 && device < n, "no such CUDA device");
    TpSpec tp;
    tp.rank = rank;
    tp.world = world;
    tp.nccl_id = nccl_id;
    auto* h = new mmfree_cuda_model{nullptr};
    try {
      h->impl = new Model(blob_path, device, act_quant == MMFREE_ACT_FIXED_Q510, frac_bits, tp);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

void mmfree_cuda_model_close(mmfree_cuda_model* m) {
  if (!m) return;
  delete m->impl;
  delete m;
}

static void fill_config(const BlobConfig& c, mmfree_cuda_config* out) {
    out->vocab_size = c.vocab_size;
    out->hidden_size = c.hidden_size;
    out->num_hidden_layers = c.num_hidden_layers;
    out->num_heads = c.num_heads;
    out->expand_ratio = c.expand_ratio;
    out->intermediate_size = c.intermediate_size;
    out->use_lower_bound = c.use_lower_bound;
    out->use_short_conv = c.use_short_conv;
    out->rms_norm_eps = c.rms_norm_eps;
}

int mmfree_cuda_model_config(const mmfree_cuda_model* m, mmfree_cuda_config* out) {
  return guard([&] {
    need(m && out, "null pointer");
    fill_config(m->impl->config(), out);
  });
}

int mmfree_cuda_blob_config(const char* blob_path, mmfree_cuda_config* out) {
  return guard([&] {
    need(blob_path && out, "null pointer");
    Blob b(blob_path);
    fill_config(b.config(), out);
  });
}

size_t mmfree_cuda_model_weight_bytes(const mmfree_cuda_model* m) {
  return m ? m->impl->weight_bytes() : 0;
}

int mmfree_cuda_generate(mmfree_cuda_model* m, const int64_t* ids, size_t n,
                         size_t new_tokens, int64_t eos_id, float temperature, int top_k,
                         uint64_t seed, int64_t* out_ids, size_t out_cap, size_t* out_len) {
  return guard([&] {
    need(m && ids && out_ids && out_len, "null pointer");
    need(out_cap >= n + new_tokens, "out_cap < n + new_tokens");
    Sampling s{temperature, top_k, seed};
    auto st = m->impl->generate(ids, n, new_tokens, eos_id, s);
    std::memcpy(out_ids, st.data(), st.size() * 8);
    *out_len = st.size();
  });
}

int mmfree_cuda_generate_stream(mmfree_cuda_model* m, const int64_t* ids, size_t n,
                                size_t new_tokens, int64_t eos_id, float temperature, int top_k,
                                uint64_t seed, mmfree_cuda_token_fn on_token, void* ctx,
                                int64_t* out_ids, size_t out_cap, size_t* out_len) {
  return guard([&] {
    need(m && ids && out_ids && out_len, "null pointer");
    need(out_cap >= n + new_tokens, "out_cap < n + new_tokens");
    Sampling s{temperature, top_k, seed};
    std::function<void(int64_t)> cb = [&](int64_t id) {
      if (on_token) on_token(id, ctx);
    };
    auto st = m->impl->generate(ids, n, new_tokens, eos_id, s, &cb);
    std::memcpy(out_ids, st.data(), st.size() * 8);
    *out_len = st.size();
  });
}

int mmfree_cuda_forward(mmfree_cuda_model* m, const int64_t* ids, size_t T, float* logits) {
  return guard([&] {
    need(m && ids && logits, "null pointer");
    m->impl->forward(ids, T, logits, false);
  });
}

int mmfree_cuda_forward_last(mmfree_cuda_model* m, const int64_t* ids, size_t T,
                             float* logits) {
  return guard([&] {
    need(m && ids && logits, "null pointer");
    m->impl->forward(ids, T, logits, true);
  });
}

int mmfree_cuda_forward_trace(mmfree_cuda_model* m, const int64_t* ids, size_t T, float* logits,
                              float* trace) {
  return guard([&] {
    need(m && ids && logits && trace, "null pointer");
    m->impl->forward_trace(ids, T, logits, trace);
  });
}

static std::vector<std::vector<int64_t>> gather_prompts(size_t B, const int64_t* const* prompts,
                                                        const size_t* lens) {
  need(B > 0 && prompts && lens, "null prompts");
  std::vector<std::vector<int64_t>> ps(B);
  for (size_t b = 0; b < B; ++b) {
    need(prompts[b] != nullptr || lens[b] == 0, "null prompt pointer");
    ps[b].assign(prompts[b], prompts[b] + lens[b]);
  }
  return ps;
}

int mmfree_cuda_generate_serve(mmfree_cuda_model* m, size_t B, const int64_t* const* prompts,
                               const size_t* lens, size_t new_tokens, int64_t eos_id,
                               float temperature, int top_k, uint64_t seed, int64_t* out,
                               size_t out_stride, size_t* out_lens) {
  return guard([&] {
    need(m && out && out_lens, "null pointer");
    auto ps = gather_prompts(B, prompts, lens);
    for (size_t b = 0; b < B; ++b)
      need(out_stride >= lens[b] + (new_tokens > 0 ? new_tokens : 1), "out_stride too small");
    Sampling s{temperature, top_k, seed};
    auto st = m->impl->generate_serve(ps, new_tokens, eos_id, s);
    for (size_t b = 0; b < B; ++b) {
      std::memcpy(out + b * out_stride, st[b].data(), st[b].size() * 8);
      out_lens[b] = st[b].size();
    }
  });
}

int mmfree_cuda_serve_begin(mmfree_cuda_model* m, size_t B, const int64_t* const* prompts,
                            const size_t* lens, int64_t* first_ids) {
  return guard([&] {
    need(m && first_ids, "null pointer");
    m->impl->serve_begin(gather_prompts(B, prompts, lens), first_ids);
  });
}

int mmfree_cuda_serve_step(mmfree_cuda_model* m, const int64_t* in_ids, int64_t* out_ids) {
  return guard([&] {
    need(m && in_ids && out_ids, "null pointer");
    m->impl->serve_step(in_ids, out_ids);
  });
}

int mmfree_cuda_serve_run(mmfree_cuda_model* m, size_t steps, int64_t* out) {
  return guard([&] {
    need(m && out, "null pointer");
    m->impl->serve_run(steps, out);
  });
}

void* mmfree_cuda_model_stream(mmfree_cuda_model* m) {
  return m ? static_cast<void*>(m->impl->stream()) : nullptr;
}

int mmfree_cuda_serve_profile(mmfree_cuda_model* m, size_t steps, mmfree_cuda_kernel_stats* out,
                              int max_classes, int* n_classes) {
  return guard([&] {
    need(m && out && n_classes, "null pointer");
    auto st = m->impl->serve_profile(steps);
    int n = 0;
    for (int c = 0; c < static_cast<int>(st.size()) && n < max_classes; ++c, ++n) {
      out[n].name = Model::class_name(c);
      out[n].ms = st[c].ms;
      out[n].launches = st[c].launches;
      out[n].bytes = st[c].bytes;
      out[n].ops = st[c].ops;
    }
    *n_classes = n;
  });
}

int mmfree_cuda_serve_end(mmfree_cuda_model* m) {
  return guard([&] {
    need(m != nullptr, "null pointer");
    m->impl->serve_end();
  });
}

}  // extern "C"
