// kernels.cu -- the unfused mmfree CUDA kernels (any row count M).
//
// prep      one CTA per row: the exact AVX2-order RMSNorm chain(s), the row transform
//           (plain / rmsnorm / gated rmsnorm), the BitLinear norm and the Q5.10 quantisation
//           into high/low byte planes (fixed) or fp32 activations (float).
//           Restates bitlinear.cpp:79-95 (+ rmsnorm.cpp:11-22, rmsnorm_swishgate.cpp:13-30).
// matmul    ternary x activations over the tiled 2-bit weight format with dp4a (fixed) or
//           fp32 FMA (float), dequant and optional residual add in the epilogue.
//           Restates ternary_backend.hpp:96-103 + simd.hpp:191-206 (+ hgrn_model.cpp:161-166,
//           :189-194 for the residual).
// mixer    the HGRN token mixer (hgrn_model.cpp:109-150): gate + scan in one pass (a decode
//           step runs it inside the o_proj prep instead, unless MMFREE_MIX_IN_PREP=0).
// others    swiglu split (hgrn_model.cpp:171-185), embedding gather, greedy argmax.
#include "common.cuh"
#include "exact.cuh"
#include "kernels.h"

#include <atomic>
#include <cfloat>
#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

namespace mmfree_cuda {

namespace {
constexpr int kPrepThreads = 512;  // prep: 16 warps share a row's elementwise passes
constexpr int kPrepThreadsMany = 128;  // prep of many rows: several row CTAs per SM
constexpr int kPrepManyRows = 1024;
constexpr int kMatmulThreads = 128;
constexpr int kMaxDynSmem = 224 * 1024;  // below the 227 KB opt-in, leaving room for static smem
}  // namespace

// ------------------------------------------------------------------------------ repack
__global__ void repack_kernel(uint32_t* __restrict__ dst, const int8_t* __restrict__ wq, int64_t n,
                              int64_t k, int64_t kc, int64_t nwords, uint32_t* bad) {
  int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= nwords) return;
  const int w = static_cast<int>(idx & 3);
  int64_t t = idx >> 2;
  const int r = static_cast<int>(t & 31);
  t >>= 5;
  const int64_t c = t % kc, g = t / kc;
  const int64_t row = g * kRowsPerGroup + r, k0 = c * kChunkK + w * 16;
  uint32_t word = 0;
  bool nonternary = false;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int64_t kk = k0 + i;
    uint32_t u = 1;
    if (row < n && kk < k) {
      const int v = wq[row * k + kk];
      nonternary |= (v < -1 || v > 1);
      u = v > 0 ? 2u : (v < 0 ? 0u : 1u);
    }
    word |= u << (8 * (i & 3) + 2 * (i >> 2));
  }
  dst[idx] = word;
  if (nonternary && bad) atomicOr(bad, kErrNotTernary);
}

cudaError_t launch_repack(void* dst, const int8_t* wq, int64_t n, int64_t k, uint32_t* err,
                          cudaStream_t s) {
  const int64_t kc = packed_chunks(k);
  const int64_t nwords = packed_groups(n) * kc * kRowsPerGroup * 4;
  const int threads = 256;
  repack_kernel<<<static_cast<unsigned>(ceil_div(nwords, threads)), threads, 0, s>>>(
      static_cast<uint32_t*>(dst), wq, n, k, kc, nwords, err);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ prep
// Copies up to NA arrays of K floats (those with a non-null dst) from global into shared
// memory; every thread issues the loads of a whole batch (kBatch elements of each array)
// before its first store, so one memory latency covers the batch instead of one per element.
template <int kBatch, int NA>
__device__ __forceinline__ void stage_arrays(float* const (&dst)[NA], const float* const (&src)[NA],
                                             int K) {
  for (int c0 = threadIdx.x; c0 < K; c0 += kBatch * blockDim.x) {
    float v[NA][kBatch];
#pragma unroll
    for (int s = 0; s < NA; ++s)
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int c = c0 + i * static_cast<int>(blockDim.x);
        v[s][i] = (dst[s] != nullptr && c < K) ? __ldg(src[s] + c) : 0.0f;
      }
#pragma unroll
    for (int s = 0; s < NA; ++s)
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int c = c0 + i * static_cast<int>(blockDim.x);
        if (dst[s] != nullptr && c < K) dst[s][c] = v[s][i];
      }
  }
}

// Shared-memory floats of one prep CTA: the row, plus (when staged) every per-element input,
// each array padded to a multiple of 4 floats (16-byte aligned).
static int64_t prep_smem_floats(const PrepArgs& a, int mode, bool staged) {
  int arrays = 1;
  if (staged) arrays += (mode != kPrepPlain ? 1 : 0) + (mode == kPrepSwishgate ? 1 : 0) + a.nproj;
  return static_cast<int64_t>(arrays) * ((a.K + 3) & ~3);
}

// Polls of a row's bulk-copy wait before the prep gives up (kErrTimeout). Host code may lower
// it (set_wait_limit) to make the wait give up on purpose; the drain of a copy still in flight
// after giving up always uses the full limit.
constexpr uint32_t kRowSpin = 1u << 22;
static std::atomic<int64_t> g_row_polls{-1};

void set_wait_limit(int64_t polls) { g_row_polls.store(polls < 0 ? -1 : polls); }
static uint32_t row_polls() {
  const int64_t v = g_row_polls.load();
  return v < 0 ? kRowSpin : static_cast<uint32_t>(v > 0xffffffffLL ? 0xffffffffLL : v);
}

__device__ __forceinline__ uint32_t shared_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// bulk global -> shared copy of a row, completing on an mbarrier (no multicast)
__device__ __forceinline__ void row_bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          shared_addr(dst)),
      "l"(src), "r"(bytes), "r"(shared_addr(bar))
      : "memory");
}
__device__ __forceinline__ bool row_bar_done(uint64_t* bar) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(shared_addr(bar))
      : "memory");
  return ok != 0;
}

// 4 consecutive floats p[c0..c0+3] (0 past K): one 16-byte load when aligned and in range
__device__ __forceinline__ void load4(const float* p, int c0, int K, bool vec, float (&v)[4]) {
  if (vec && c0 + 3 < K) {
    const float4 t = *reinterpret_cast<const float4*>(p + c0);
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  } else {
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = c0 + u < K ? p[c0 + u] : 0.0f;
  }
}

__global__ void __launch_bounds__(kPrepThreads) prep_kernel(PrepArgs a, int mode, int staged) {
  extern __shared__ __align__(16) float sbuf[];
  float* srow = sbuf;  // the row being normalized, K floats
  __shared__ float s_rstd;
  __shared__ int s_red[3][kPrepThreads / 32];
  __shared__ __align__(8) uint64_t s_rowbar;
  const int m = blockIdx.x, K = a.K, tid = threadIdx.x;
  const int64_t Kp = padded_k(K);
  const int K4 = (K + 3) & ~3;  // staged arrays start 16-byte aligned
  const float* x = a.x + static_cast<int64_t>(m) * K;
  const float* orow = a.o ? a.o + static_cast<int64_t>(m) * K : nullptr;

  // stage the inputs: with `staged` every pass below reads shared memory only
  // (slots: row, row-transform weight, recurrence output, projection norm weights)
  const float* prew = a.prew;
  const float* nw[3] = {a.normw[0], a.normw[1], a.normw[2]};
  {
    const bool use1 = staged && mode != kPrepPlain, use2 = staged && mode == kPrepSwishgate;
    const bool copy2 = use2 && a.mix_i == nullptr;  // o is read (not computed here)
    // rows of a multiple of 4 floats at 16-byte aligned addresses arrive by one bulk copy each
    const bool bulk = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                      (!copy2 || (reinterpret_cast<uintptr_t>(a.o) & 15) == 0);
    if (bulk && tid == 0) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(shared_addr(&s_rowbar)));
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    float* p1 = sbuf + K4;
    float* p2 = p1 + (use1 ? K4 : 0);
    float* p3 = p2 + (use2 ? K4 : 0);
    // weights first: no earlier kernel writes them, so they load while the predecessor runs
    float* const dw[4] = {use1 ? p1 : nullptr, staged && a.nproj > 0 ? p3 : nullptr,
                          staged && a.nproj > 1 ? p3 + K4 : nullptr,
                          staged && a.nproj > 2 ? p3 + 2 * K4 : nullptr};
    const float* const sw[4] = {a.prew, a.normw[0], a.normw[1], a.normw[2]};
    stage_arrays<8>(dw, sw, K);
    if (bulk) __syncthreads();  // the barrier's initialisation, before anyone waits on it
    grid_dep_launch();
    grid_dep_wait();
    if (bulk) {
      if (tid == 0) {
        const uint32_t bytes = static_cast<uint32_t>(K) * 4u;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(shared_addr(&s_rowbar)),
                     "r"(copy2 ? 2 * bytes : bytes)
                     : "memory");
        row_bulk_copy(srow, x, bytes, &s_rowbar);
        if (copy2) row_bulk_copy(p2, orow, bytes, &s_rowbar);
      }
      bool done = false;
      for (uint32_t i = 0; i < a.row_polls && !done; ++i) done = row_bar_done(&s_rowbar);
      if (__syncthreads_or(!done)) {  // (uniform) report, let the copies land (bounded), and
                                      // leave the outputs unwritten
        if (tid == 0 && a.err) atomicOr(a.err, kErrTimeout);
        // the copy itself is still in flight: drain it with the full limit before leaving
        for (uint32_t i = 0; i < kRowSpin && !row_bar_done(&s_rowbar); ++i) {
        }
        return;
      }
    } else {
      float* const dr[2] = {srow, copy2 ? p2 : nullptr};
      const float* const sr[2] = {x, orow};
      // one memory latency per row: 12 loads per thread for rows longer than 8 per thread
      if (K > 8 * static_cast<int>(blockDim.x)) stage_arrays<12>(dr, sr, K);
      else stage_arrays<8>(dr, sr, K);
    }
    if (use1) prew = p1;
    if (use2) orow = p2;
    if (staged) {
      nw[0] = p3;
      nw[1] = p3 + K4;
      nw[2] = p3 + 2 * K4;
    }
  }
  __syncthreads();

  if (mode != kPrepPlain) {
    if (tid < 8) {
      const float r = rstd_of(sumsq_exact8(srow, K, 0xffu), static_cast<float>(K), a.eps);
      if (tid == 0) s_rstd = r;
    } else if (a.mix_i && tid >= 32) {
      // the fused token mixer of this row (warps 1.., while warp 0 runs the norm chain): per
      // lane the forget gate (sigmoid, lower bound), the SwiGLU scan input and one
      // recurrence step, as mixer_decode_kernel; the recurrence output goes to shared memory
      // (o of the swish gate), the new state and the output to global memory
      const int nt = static_cast<int>(blockDim.x) - 32;
      const int tail_from = K - static_cast<int>((static_cast<int64_t>(a.mix_seg_rows) * K) % 8);
      const bool last_row = (m + 1) % a.mix_seg_rows == 0;
      const int64_t rb = static_cast<int64_t>(m) * K;
      float* ob = const_cast<float*>(orow);  // the o slot in shared memory (staged)
      for (int c0 = 4 * (tid - 32); c0 < K; c0 += 4 * nt) {
        const float4 i4 = __ldcs(reinterpret_cast<const float4*>(a.mix_i + rb + c0));
        const float4 f4 = __ldcs(reinterpret_cast<const float4*>(a.mix_f + rb + c0));
        const float4 s4 = *reinterpret_cast<const float4*>(a.mix_state + rb + c0);
        const float4 l4 = a.mix_lb ? __ldg(reinterpret_cast<const float4*>(a.mix_lb + c0)) : make_float4(0, 0, 0, 0);
        const float iv[4] = {i4.x, i4.y, i4.z, i4.w}, fv[4] = {f4.x, f4.y, f4.z, f4.w};
        const float sv0[4] = {s4.x, s4.y, s4.z, s4.w}, lv[4] = {l4.x, l4.y, l4.z, l4.w};
        bool body[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) body[u] = !last_row || c0 + u < tail_from;
        float f[4], om[4], sw[4], st[4];
        sigmoid_n(fv, body, f);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (a.mix_lb) f[u] = lower_bound_x(f[u], lv[u]);
          om[u] = __fadd_rn(1.0f, -f[u]);
        }
        swiglu_n(iv, om, body, sw);
#pragma unroll
        for (int u = 0; u < 4; ++u) st[u] = hgrn_step_x(f[u], sv0[u], sw[u]);
        const float4 o4 = make_float4(st[0], st[1], st[2], st[3]);
        *reinterpret_cast<float4*>(ob + c0) = o4;
        *reinterpret_cast<float4*>(a.mix_state + rb + c0) = o4;
        if (a.mix_out) *reinterpret_cast<float4*>(a.mix_out + rb + c0) = o4;
      }
    }
    __syncthreads();
    const float r1 = s_rstd;
    const int nt = blockDim.x;
    for (int c0 = tid; c0 < K; c0 += 4 * nt) {
      float sg[4];
      if (mode == kPrepSwishgate) {  // four gates at a time (their divisions overlap)
        float xo[4];
        bool bd[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u * nt;
          xo[u] = c < K ? orow[c] : 0.0f;
          bd[u] = in_body(c, K);
        }
        silu_n(xo, bd, sg);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u * nt;
        if (c >= K) break;
        float t = norm_x(srow[c], r1, prew[c]);
        if (mode == kPrepSwishgate) t = __fmul_rn(t, sg[u]);
        srow[c] = t;
        if (a.pre_out) a.pre_out[static_cast<int64_t>(m) * K + c] = t;
      }
    }
    __syncthreads();
  }
  if (a.nproj == 0) return;

  if (tid < 8) {
    const float r = rstd_of(sumsq_exact8(srow, K, 0xffu), static_cast<float>(K), a.eps);
    if (tid == 0) s_rstd = r;
  }
  __syncthreads();
  const float r2 = s_rstd;

  // 4 consecutive elements per thread: 16-byte loads of the staged arrays, one 4-byte store
  // per byte plane (Kp is a multiple of 64) or one 16-byte store of fp32 activations
  int local[3] = {0, 0, 0};
  for (int c0 = 4 * tid; c0 < Kp; c0 += 4 * static_cast<int>(blockDim.x)) {
    float xv[4];
    load4(srow, c0, K, true, xv);
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (j >= a.nproj) break;
      float wv[4], y[4];
      load4(nw[j], c0, K, staged != 0, wv);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u;
        y[u] = c < K ? norm_x(xv[u], r2, wv[u]) : 0.0f;
        if (j == 0 && a.norm_out && c < K) a.norm_out[static_cast<int64_t>(m) * K + c] = y[u];
      }
      if (a.fixed) {
        uint32_t hi = 0, lo = 0;
        if (c0 + 3 < (K & ~7)) {  // 4 body elements
          quant4_body_planes(y, a.qs, a.lo_signed ? 0x80808080u : 0u, hi, lo, local[j]);
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c = c0 + u;
            const int32_t q = c < K ? quant_x(y[u], a.qs, in_body(c, K)) : 0;
            local[j] += q;
            hi |= static_cast<uint32_t>((q >> 8) & 0xff) << (8 * u);
            lo |= static_cast<uint32_t>((q & 0xff) ^ (a.lo_signed ? 0x80 : 0)) << (8 * u);
          }
        }
        *reinterpret_cast<uint32_t*>(a.planes[j] + static_cast<int64_t>(m) * Kp + c0) = hi;
        *reinterpret_cast<uint32_t*>(a.planes[j] + (static_cast<int64_t>(a.M) + m) * Kp + c0) = lo;
      } else if (a.bf16) {
        uint2 hi, lo;
        bf16_split4(y, hi, lo);
        *reinterpret_cast<uint2*>(a.planes[j] + 2 * (static_cast<int64_t>(m) * Kp + c0)) = hi;
        *reinterpret_cast<uint2*>(a.planes[j] + 2 * ((static_cast<int64_t>(a.M) + m) * Kp + c0)) = lo;
      } else {
        *reinterpret_cast<float4*>(a.yf[j] + static_cast<int64_t>(m) * Kp + c0) = make_float4(y[0], y[1], y[2], y[3]);
      }
    }
  }
  if (a.fixed) {  // row sums of the codes: warp reductions, then warp j sums projection j
    const int warp = tid >> 5, lane = tid & 31, nwarps = static_cast<int>(blockDim.x) >> 5;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (j >= a.nproj) break;
      const int v = __reduce_add_sync(0xffffffffu, local[j]);
      if (lane == 0) s_red[j][warp] = v;
    }
    __syncthreads();
    if (warp < a.nproj) {
      const int total = __reduce_add_sync(0xffffffffu, lane < nwarps ? s_red[warp][lane] : 0);
      if (lane == 0) a.rowsum[warp][m] = total;
    }
  }
}

// ------------------------------------------------------------------------------ prep, many rows
// Thousands of rows (prefill): R <= 8 rows per CTA instead of one, each staged by one bulk
// copy (with the gate operand in the gated mode). The norm weights are read through L1 -- every
// CTA reads the same ones -- instead of being staged per row, which dominated the per-row CTA.
// The flow per row is prep_kernel's: chain 1 (an 8-lane group per row, all R rows at once),
// the row transform by all threads, chain 2, then the projections' normalisation, Q5.10 planes
// (or Float activations) and row sums; the arithmetic is the same element by element.
// Two shapes: 128 threads with <= 42 KB of rows (five CTAs per SM, whose copy and chain phases
// overlap) for rows that fit at least twice, else 256 threads with <= 96 KB (long rows: one
// row per 128-thread CTA spent most of its time in the serial chain with the SM half idle)
constexpr int kRowsMax = 8, kRowsSmemSmall = 42 * 1024, kRowsSmemLarge = 96 * 1024;

// Floats from one staged row to the next: a multiple of 4 (rows 16-byte aligned) that is 8
// more than a multiple of 32, so that the 8-lane chain groups of the 4 rows of a warp read
// 4 different octets of banks.
__host__ __device__ inline int rows_stride(int K) {
  const int k4 = (K + 3) & ~3;
  return k4 + ((8 - (k4 & 31)) & 31);
}

// rows per CTA and its threads: as many rows as fit the shape's budget (at least 1, at most
// kRowsMax)
static int prep_rows_per_cta(int K, int mode, int* threads) {
  const int64_t per_row = static_cast<int64_t>(rows_stride(K)) * 4 * (mode == kPrepSwishgate ? 2 : 1);
  const bool small = 2 * per_row <= kRowsSmemSmall;
  *threads = small ? 128 : 256;
  const int64_t r = (small ? kRowsSmemSmall : kRowsSmemLarge) / per_row;
  return static_cast<int>(r < 1 ? 1 : (r > kRowsMax ? kRowsMax : r));
}

// NP: projections (a.nproj, 1 or 3); FX: FixedQ510 (a.fixed) -- compile-time, so that the
// unrolled per-element loops carry no runtime exits
template <int kRowsThreads, int NP, bool FX>
__global__ void __launch_bounds__(kRowsThreads, kRowsThreads == 128 ? (NP == 3 ? 4 : 5) : 2)
    prep_rows_kernel(PrepArgs a, int mode, int R) {
  extern __shared__ __align__(16) float sb[];
  __shared__ float s_r1[kRowsMax], s_r2[kRowsMax];
  __shared__ int s_red[NP][kRowsMax][kRowsThreads / 32];
  __shared__ __align__(8) uint64_t s_bar;
  const int K = a.K, tid = threadIdx.x, RS = rows_stride(K);
  const int64_t Kp = padded_k(K);
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * R;
  const int nr = static_cast<int>(a.M - m0 < R ? a.M - m0 : R);  // rows of this CTA
  const bool swish = mode == kPrepSwishgate;
  float* xs = sb;                                  // [R][RS]: x, then t in place
  float* os = sb + static_cast<int64_t>(R) * RS;   // [R][RS]: the gate operand (gated mode)
  const bool bulk = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                    (!swish || (reinterpret_cast<uintptr_t>(a.o) & 15) == 0);
  if (bulk && tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(shared_addr(&s_bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (bulk) __syncthreads();
  grid_dep_launch();
  grid_dep_wait();
  if (bulk) {
    if (tid == 0) {
      const uint32_t bytes = static_cast<uint32_t>(K) * 4u;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(shared_addr(&s_bar)),
                   "r"(bytes * static_cast<uint32_t>(nr) * (swish ? 2u : 1u))
                   : "memory");
      for (int r = 0; r < nr; ++r) {
        row_bulk_copy(xs + static_cast<int64_t>(r) * RS, a.x + (m0 + r) * K, bytes, &s_bar);
        if (swish) row_bulk_copy(os + static_cast<int64_t>(r) * RS, a.o + (m0 + r) * K, bytes, &s_bar);
      }
    }
    bool done = false;
    for (uint32_t i = 0; i < a.row_polls && !done; ++i) done = row_bar_done(&s_bar);
    if (__syncthreads_or(!done)) {  // (uniform) report, drain the copies, leave no output
      if (tid == 0 && a.err) atomicOr(a.err, kErrTimeout);
      for (uint32_t i = 0; i < kRowSpin && !row_bar_done(&s_bar); ++i) {
      }
      return;
    }
  } else {
    for (int64_t i = tid; i < static_cast<int64_t>(nr) * K; i += kRowsThreads) {
      const int r = static_cast<int>(i / K), c = static_cast<int>(i % K);
      xs[static_cast<int64_t>(r) * RS + c] = a.x[(m0 + r) * K + c];
      if (swish) os[static_cast<int64_t>(r) * RS + c] = a.o[(m0 + r) * K + c];
    }
    __syncthreads();
  }
  // the 8-lane groups of the chains: rows 0..nr-1 on threads 0..8 nr-1
  const int active = 8 * nr - 32 * (tid >> 5);
  const unsigned mask = active >= 32 ? 0xffffffffu : (active > 0 ? (1u << active) - 1u : 0u);
  const int cr = tid >> 3;  // the chain row of this thread (tid < 8 nr)
  if (mode != kPrepPlain) {
    if (tid < 8 * nr) {
      const float r = rstd_of(sumsq_exact8(xs + static_cast<int64_t>(cr) * RS, K, mask), static_cast<float>(K), a.eps);
      if ((tid & 7) == 0) s_r1[cr] = r;
    }
    __syncthreads();
    // t = rmsnorm(x) * prew (* silu(o)) in place, four columns per thread and step
    for (int r = 0; r < nr; ++r) {
      const float r1 = s_r1[r];
      float* xr = xs + static_cast<int64_t>(r) * RS;
      const float* orow = os + static_cast<int64_t>(r) * RS;
      for (int c0 = tid; c0 < K; c0 += 4 * kRowsThreads) {
        float sg[4] = {1.0f, 1.0f, 1.0f, 1.0f};
        if (swish) {
          float xo[4];
          bool bd[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c = c0 + u * kRowsThreads;
            xo[u] = c < K ? orow[c] : 0.0f;
            bd[u] = in_body(c, K);
          }
          silu_n(xo, bd, sg);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u * kRowsThreads;
          if (c >= K) break;
          float t = norm_x(xr[c], r1, __ldg(a.prew + c));
          if (swish) t = __fmul_rn(t, sg[u]);
          xr[c] = t;
          if (a.pre_out) a.pre_out[(m0 + r) * K + c] = t;
        }
      }
    }
    __syncthreads();
  }
  if (tid < 8 * nr) {
    const float r = rstd_of(sumsq_exact8(xs + static_cast<int64_t>(cr) * RS, K, mask), static_cast<float>(K), a.eps);
    if ((tid & 7) == 0) s_r2[cr] = r;
  }
  __syncthreads();
  int local[NP][kRowsMax] = {};
  const uint32_t lo_xor = a.lo_signed ? 0x80808080u : 0u;
  float* const norm_out = a.norm_out;
  bool nw16[NP];  // norm weights 16-byte aligned: 4 per load
#pragma unroll
  for (int j = 0; j < NP; ++j) nw16[j] = (reinterpret_cast<uintptr_t>(a.normw[j]) & 15) == 0;
  for (int c0 = 4 * tid; c0 < Kp; c0 += 4 * kRowsThreads) {
    const bool body4 = c0 + 3 < (K & ~7);  // 4 body elements
    const bool full4 = c0 + 3 < K;
    float nwv[NP][4];
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      if (full4 && nw16[j]) {
        const float4 w4 = __ldg(reinterpret_cast<const float4*>(a.normw[j] + c0));
        nwv[j][0] = w4.x;
        nwv[j][1] = w4.y;
        nwv[j][2] = w4.z;
        nwv[j][3] = w4.w;
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) nwv[j][u] = c0 + u < K ? __ldg(a.normw[j] + c0 + u) : 0.0f;
      }
    }
#pragma unroll
    for (int r = 0; r < kRowsMax; ++r) {
      if (r >= nr) break;
      const int64_t m = m0 + r;
      float t[4];
      load4(xs + static_cast<int64_t>(r) * RS, c0, K, true, t);
      const float r2 = s_r2[r];
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        float y[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u;
          y[u] = c < K ? norm_x(t[u], r2, nwv[j][u]) : 0.0f;
          if (j == 0 && norm_out && c < K) norm_out[m * K + c] = y[u];
        }
        if (FX) {
          uint32_t hi = 0, lo = 0;
          if (body4) {
            quant4_body_planes(y, a.qs, lo_xor, hi, lo, local[j][r]);
          } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int c = c0 + u;
              const int32_t q = c < K ? quant_x(y[u], a.qs, in_body(c, K)) : 0;
              local[j][r] += q;
              hi |= static_cast<uint32_t>((q >> 8) & 0xff) << (8 * u);
              lo |= static_cast<uint32_t>((q & 0xff) ^ (a.lo_signed ? 0x80 : 0)) << (8 * u);
            }
          }
          *reinterpret_cast<uint32_t*>(a.planes[j] + m * Kp + c0) = hi;
          *reinterpret_cast<uint32_t*>(a.planes[j] + (a.M + m) * Kp + c0) = lo;
        } else if (a.bf16) {
          uint2 hi, lo;
          bf16_split4(y, hi, lo);
          *reinterpret_cast<uint2*>(a.planes[j] + 2 * (m * Kp + c0)) = hi;
          *reinterpret_cast<uint2*>(a.planes[j] + 2 * ((a.M + m) * Kp + c0)) = lo;
        } else {
          *reinterpret_cast<float4*>(a.yf[j] + m * Kp + c0) = make_float4(y[0], y[1], y[2], y[3]);
        }
      }
    }
  }
  if (!FX) return;
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int j = 0; j < NP; ++j)
#pragma unroll
    for (int r = 0; r < kRowsMax; ++r) {
      const int v = __reduce_add_sync(0xffffffffu, local[j][r]);
      if (lane == 0) s_red[j][r][warp] = v;
    }
  __syncthreads();
  if (tid < NP * kRowsMax) {
    const int j = tid / kRowsMax, r = tid % kRowsMax;
    if (r < nr) {
      int total = 0;
#pragma unroll
      for (int w = 0; w < kRowsThreads / 32; ++w) total += s_red[j][r][w];
      a.rowsum[j][m0 + r] = total;
    }
  }
}

// Opts a kernel in to kMaxDynSmem of dynamic shared memory, once per (device, kernel).
static void raise_smem_limit(const void* fn) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.insert({dev, fn}).second)
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
}

cudaError_t launch_prep(const PrepArgs& a, cudaStream_t s) {
  if (a.M <= 0) return cudaSuccess;
  int mode = kPrepPlain;
  if (a.prew) mode = (a.o || a.mix_i) ? kPrepSwishgate : kPrepNorm;
  if (a.nproj < 0 || a.nproj > 3) return cudaErrorInvalidValue;
  int staged = 1;
  size_t smem = static_cast<size_t>(prep_smem_floats(a, mode, true)) * sizeof(float);
  if (smem > kMaxDynSmem) {  // very long rows: stage the row only
    staged = 0;
    smem = static_cast<size_t>(prep_smem_floats(a, mode, false)) * sizeof(float);
  }
  if (smem > kMaxDynSmem) return cudaErrorInvalidValue;
  if (a.mix_i) {  // fused token mixer: float4 lanes of staged rows
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (mode != kPrepSwishgate || !staged || a.o || a.K % 4 != 0 || a.K < 8 || a.mix_seg_rows < 1 ||
        !a.mix_f || !a.mix_state || !al16(a.mix_i) || !al16(a.mix_f) || !al16(a.mix_state) ||
        !al16(a.mix_lb) || !al16(a.mix_out))
      return cudaErrorInvalidValue;
  }
  if (a.M >= kPrepManyRows && !a.mix_i && (a.nproj == 1 || a.nproj == 3)) {  // many rows: several per CTA
    int threads = 128;
    const int R = prep_rows_per_cta(a.K, mode, &threads);
    const size_t rsmem = static_cast<size_t>(R) * rows_stride(a.K) * 4 * (mode == kPrepSwishgate ? 2 : 1);
    if (rsmem <= kMaxDynSmem) {
      PrepArgs q = a;
      q.row_polls = row_polls();
      const dim3 grid(static_cast<unsigned>(ceil_div(int64_t(a.M), R)));
      auto go = [&](auto kern, int nt) {
        if (rsmem > 48 * 1024) raise_smem_limit(reinterpret_cast<const void*>(kern));
        return launch_k(kern, grid, dim3(nt), rsmem, s, a.pdl, q, mode, R);
      };
      const bool three = a.nproj == 3;
      if (threads == 128) {
        if (a.fixed) return three ? go(prep_rows_kernel<128, 3, true>, 128) : go(prep_rows_kernel<128, 1, true>, 128);
        return three ? go(prep_rows_kernel<128, 3, false>, 128) : go(prep_rows_kernel<128, 1, false>, 128);
      }
      if (a.fixed) return three ? go(prep_rows_kernel<256, 3, true>, 256) : go(prep_rows_kernel<256, 1, true>, 256);
      return three ? go(prep_rows_kernel<256, 3, false>, 256) : go(prep_rows_kernel<256, 1, false>, 256);
    }
  }
  if (smem > 48 * 1024) raise_smem_limit(reinterpret_cast<const void*>(prep_kernel));
  PrepArgs q = a;
  q.row_polls = row_polls();
  // few rows: latency-bound, 512 threads per row; many rows: throughput-bound, 128 threads
  // per row so that registers allow several row CTAs per SM
  const int threads = a.M >= kPrepManyRows ? kPrepThreadsMany : kPrepThreads;
  return launch_k(prep_kernel, dim3(a.M), dim3(threads), smem, s, a.pdl, q, mode, staged);
}

__device__ __forceinline__ int block_sum_int(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int t = 0;
  if (threadIdx.x == 0)
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kPrepThreads) codes_kernel(int8_t* __restrict__ planes,
                                                            int32_t* __restrict__ rowsum,
                                                            const int32_t* __restrict__ x, int M,
                                                            int K, uint32_t* err) {
  __shared__ int s_red[kPrepThreads / 32];
  const int m = blockIdx.x;
  const int64_t Kp = padded_k(K);
  int local = 0;
  bool bad = false;
  for (int c = threadIdx.x; c < Kp; c += blockDim.x) {
    int32_t q = c < K ? x[static_cast<int64_t>(m) * K + c] : 0;
    if (q < -32768 || q > 32767) {
      bad = true;
      q = 0;
    }
    local += q;
    planes[static_cast<int64_t>(m) * Kp + c] = static_cast<int8_t>(q >> 8);
    planes[(static_cast<int64_t>(M) + m) * Kp + c] = static_cast<int8_t>(q & 0xff);
  }
  if (bad && err) atomicOr(err, kErrRange);
  const int total = block_sum_int(local, s_red);
  if (threadIdx.x == 0) rowsum[m] = total;
}

cudaError_t launch_codes_to_planes(int8_t* planes, int32_t* rowsum, const int32_t* x, int M,
                                   int K, uint32_t* err, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  codes_kernel<<<M, kPrepThreads, 0, s>>>(planes, rowsum, x, M, K, err);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ matmul
// CTA = one 32-row group of the packed weights x MT activation rows; its 4 warps split the
// k-chunks round robin and reduce through shared memory. Lane r owns output row 32g + r.
template <int MT>
__global__ void __launch_bounds__(kMatmulThreads) matmul_fixed_kernel(MatmulArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  const int g = blockIdx.x, m0 = blockIdx.y * MT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t kc = packed_chunks(a.K), kp = kc * kChunkK;
  const uint4* wp = static_cast<const uint4*>(a.w) + static_cast<int64_t>(g) * kc * 32 + lane;
  int acc_hi[MT][4], acc_lo[MT][4];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc_hi[mi][q] = acc_lo[mi][q] = 0;

  for (int64_t c = warp; c < kc; c += kMatmulThreads / 32) {
    const uint4 wv = __ldg(wp + c * 32);
    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
      const int m = min(m0 + mi, a.M - 1);  // rows past M repeat row M-1; never stored
      const uint4* hp = reinterpret_cast<const uint4*>(a.planes + static_cast<int64_t>(m) * kp + c * kChunkK);
      const uint4* lp = reinterpret_cast<const uint4*>(a.planes + (static_cast<int64_t>(a.M) + m) * kp + c * kChunkK);
#pragma unroll
      for (int w4 = 0; w4 < 4; ++w4) {
        const uint4 h = __ldg(hp + w4), l = __ldg(lp + w4);
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t mw = wd[w4] & (0x03030303u << (2 * q));
          acc_hi[mi][q] = dp4a_us(mw, hw[q], acc_hi[mi][q]);
          acc_lo[mi][q] = dp4a_uu(mw, lw[q], acc_lo[mi][q]);
        }
      }
    }
  }

  __shared__ uint32_t red[kMatmulThreads / 32][MT][32];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi) {
    uint32_t t = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      t += static_cast<uint32_t>(acc_hi[mi][q] >> (2 * q)) << 8;
      t += static_cast<uint32_t>(acc_lo[mi][q] >> (2 * q));
    }
    red[warp][mi][lane] = t;
  }
  __syncthreads();
  const int n = g * kRowsPerGroup + lane;
  for (int mi = warp; mi < MT; mi += kMatmulThreads / 32) {
    const int m = m0 + mi;
    if (m >= a.M || n >= a.N) continue;
    uint32_t t = 0;
#pragma unroll
    for (int w = 0; w < kMatmulThreads / 32; ++w) t += red[w][mi][lane];
    const int32_t acc = static_cast<int32_t>(t - static_cast<uint32_t>(a.rowsum[m]));
    if (a.acc_out) a.acc_out[static_cast<int64_t>(m) * a.N + n] = acc;
    if (!a.out) continue;
    float v = __fmul_rn(__int2float_rn(acc), a.scale);
    if (a.resid) v = __fadd_rn(a.resid[static_cast<int64_t>(m) * a.ldr + n], v);
    a.out[static_cast<int64_t>(m) * a.ldo + n] = v;
  }
}

template <int MT>
__global__ void __launch_bounds__(kMatmulThreads) matmul_float_kernel(MatmulArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  const int g = blockIdx.x, m0 = blockIdx.y * MT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t kc = packed_chunks(a.K), kp = kc * kChunkK;
  const uint4* wp = static_cast<const uint4*>(a.w) + static_cast<int64_t>(g) * kc * 32 + lane;
  float acc[MT];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi) acc[mi] = 0.0f;
  for (int64_t c = warp; c < kc; c += kMatmulThreads / 32) {
    const uint4 wv = __ldg(wp + c * 32);
    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
      const int m = min(m0 + mi, a.M - 1);
      const float4* yp = reinterpret_cast<const float4*>(a.yf + static_cast<int64_t>(m) * kp + c * kChunkK);
#pragma unroll
      for (int w4 = 0; w4 < 4; ++w4) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 y = __ldg(yp + 4 * w4 + q4);
          const float yv[4] = {y.x, y.y, y.z, y.w};
          const uint32_t m = (wd[w4] >> (2 * q4)) & 0x03030303u;  // byte e: weight 4 q4 + e
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[mi] = __fmaf_rn(ternary_f32(m, e), yv[e], acc[mi]);
        }
      }
    }
  }
  __shared__ float red[kMatmulThreads / 32][MT][32];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi) red[warp][mi][lane] = acc[mi];
  __syncthreads();
  const int n = g * kRowsPerGroup + lane;
  for (int mi = warp; mi < MT; mi += kMatmulThreads / 32) {
    const int m = m0 + mi;
    if (m >= a.M || n >= a.N) continue;
    float t = red[0][mi][lane];
#pragma unroll
    for (int w = 1; w < kMatmulThreads / 32; ++w) t = __fadd_rn(t, red[w][mi][lane]);
    float v = __fmul_rn(t, a.scale);
    if (a.resid) v = __fadd_rn(a.resid[static_cast<int64_t>(m) * a.ldr + n], v);
    a.out[static_cast<int64_t>(m) * a.ldo + n] = v;
  }
}

template <int MT>
static cudaError_t launch_matmul_mt(const MatmulArgs& a, cudaStream_t s) {
  dim3 grid(static_cast<unsigned>(packed_groups(a.N)), static_cast<unsigned>(ceil_div(a.M, MT)));
  if (a.fixed) return launch_k(matmul_fixed_kernel<MT>, grid, dim3(kMatmulThreads), 0, s, a.pdl, a);
  return launch_k(matmul_float_kernel<MT>, grid, dim3(kMatmulThreads), 0, s, a.pdl, a);
}

static int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& c = cached[dev & 63];
  if (c == 0) cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
  return c > 0 ? c : 148;
}

cudaError_t launch_matmul(const MatmulArgs& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return cudaSuccess;
  if (matmul_uses_tc(a)) {
    if (a.fixed && !a.lo_signed) return cudaErrorInvalidValue;  // planes in the wrong form
    return launch_matmul_tc(a, tc_splits(a, sm_count()), sm_count(), s);
  }
  if (a.M == 1) return launch_matmul_mt<1>(a, s);
  if (a.M == 2) return launch_matmul_mt<2>(a, s);
  if (a.M <= 4) return launch_matmul_mt<4>(a, s);
  return launch_matmul_mt<8>(a, s);
}

// ------------------------------------------------------------------------------ mixer
// The scan alone (the C-ABI hgrn_scan, hgrn_scan.cpp:11-19): state = fma(f, state, s) along
// t for each of nseq x H lanes; x layout [nseq][T][H], state [nseq][H] (nullable: zero
// start, not written back).
// The serial chain is one FMA per step; the loads of the next kScanAhead steps are issued
// before the chain consumes the current batch, so one memory latency covers a whole batch
// (few lanes run per SM: each must keep many loads in flight).
constexpr int kScanAhead = 32;
__global__ void scan_kernel(float* __restrict__ out, const float* __restrict__ s,
                            const float* __restrict__ f, float* __restrict__ state, int nseq,
                            int T, int H) {
  grid_dep_launch();
  grid_dep_wait();
  const int64_t lane = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (lane >= static_cast<int64_t>(nseq) * H) return;
  const int64_t q = lane / H, c = lane % H;
  const int64_t base = q * T * H + c;
  float st = state ? state[lane] : 0.0f;
  float fa[kScanAhead], sa[kScanAhead];
#pragma unroll
  for (int u = 0; u < kScanAhead; ++u) {
    const int64_t e = base + static_cast<int64_t>(u) * H;
    fa[u] = u < T ? __ldcs(f + e) : 0.0f;
    sa[u] = u < T ? __ldcs(s + e) : 0.0f;
  }
  for (int t0 = 0; t0 < T; t0 += kScanAhead) {
    float fn[kScanAhead], sn[kScanAhead];
#pragma unroll
    for (int u = 0; u < kScanAhead; ++u) {  // the next batch, in flight during this one
      const int t = t0 + kScanAhead + u;
      const int64_t e = base + static_cast<int64_t>(t) * H;
      fn[u] = t < T ? __ldcs(f + e) : 0.0f;
      sn[u] = t < T ? __ldcs(s + e) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kScanAhead; ++u) {
      if (t0 + u >= T) break;
      st = hgrn_step_x(fa[u], st, sa[u]);
      __stcs(out + base + static_cast<int64_t>(t0 + u) * H, st);
    }
#pragma unroll
    for (int u = 0; u < kScanAhead; ++u) {
      fa[u] = fn[u];
      sa[u] = sn[u];
    }
  }
  if (state) state[lane] = st;
}

// The gates of a prefill, element-parallel (hgrn_model.cpp:109-134): f = sigmoid(fraw), lower
// bounded, and the scan input swiglu(i, 1 - f), written in place over fraw and i. Element e of
// [nseq][T][H] is in the SIMD body of its reference vector call (seg elements) unless it is
// among the call's last seg % 8 elements. Four consecutive elements per thread.
__global__ void gates_kernel(float* __restrict__ iv, float* __restrict__ fv,
                             const float* __restrict__ lb, int64_t n, int H, int64_t seg) {
  grid_dep_launch();
  grid_dep_wait();
  const int64_t e0 = 4 * (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x);
  if (e0 >= n) return;
  const int64_t body_n = seg & ~int64_t(7);
  float a[4], b[4], l[4];
  bool body[4];
  const bool vec = e0 + 3 < n;
  const bool al = ((reinterpret_cast<uintptr_t>(iv) | reinterpret_cast<uintptr_t>(fv)) & 15) == 0;
  if (vec && al && H % 4 == 0) {
    // the 4 elements share a row (H and seg multiples of 4): one remainder each, 16-byte loads
    const int c0 = static_cast<int>(e0 % H);
    const int64_t s0 = e0 % seg;
    const float4 a4 = __ldcs(reinterpret_cast<const float4*>(iv + e0));
    const float4 b4 = __ldcs(reinterpret_cast<const float4*>(fv + e0));
    a[0] = a4.x; a[1] = a4.y; a[2] = a4.z; a[3] = a4.w;
    b[0] = b4.x; b[1] = b4.y; b[2] = b4.z; b[3] = b4.w;
    if (lb && (reinterpret_cast<uintptr_t>(lb) & 15) == 0) {
      const float4 l4 = __ldg(reinterpret_cast<const float4*>(lb + c0));
      l[0] = l4.x; l[1] = l4.y; l[2] = l4.z; l[3] = l4.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) l[u] = lb ? __ldg(lb + c0 + u) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) body[u] = s0 + u < body_n;
  } else {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t e = e0 + u;
      a[u] = (vec || e < n) ? __ldcs(iv + e) : 0.0f;
      b[u] = (vec || e < n) ? __ldcs(fv + e) : 0.0f;
      l[u] = lb ? __ldg(lb + e % H) : 0.0f;
      body[u] = e % seg < body_n;
    }
  }
  float f[4], om[4], x[4];
  sigmoid_n(b, body, f);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (lb) f[u] = lower_bound_x(f[u], l[u]);
    om[u] = __fadd_rn(1.0f, -f[u]);
  }
  swiglu_n(a, om, body, x);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (e0 + u >= n) break;
    fv[e0 + u] = f[u];
    iv[e0 + u] = x[u];
  }
}

// Chunked parallel scan (Float mode): the recurrence h_t = f_t h_{t-1} + x_t over chunks of
// kChunkT steps. Pass 1, one thread per (sequence, chunk, channel): the chunk's scan from a
// zero state (written to out) and its summary (prod f, end state). Pass 2, one thread per
// lane: carries in chunk order. Pass 3, one thread per (sequence, chunk, channel): out_t +=
// (prod_{s <= t} f_s) * carry-in. Sums are re-associated, which the Float tolerance allows.
constexpr int kChunkT = 64;
__global__ void chunk_scan_kernel(float* __restrict__ out, float2* __restrict__ summ,
                                  const float* __restrict__ x, const float* __restrict__ f,
                                  int nseq, int T, int H, int nch) {
  grid_dep_launch();
  grid_dep_wait();
  const int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (id >= static_cast<int64_t>(nseq) * nch * H) return;
  const int c = static_cast<int>(id % H);
  const int64_t qk = id / H;
  const int k = static_cast<int>(qk % nch), q = static_cast<int>(qk / nch);
  const int t0 = k * kChunkT, t1 = min(T, t0 + kChunkT);
  const int64_t base = static_cast<int64_t>(q) * T * H + c;
  float st = 0.0f, pr = 1.0f;
  for (int t = t0; t < t1; ++t) {
    const int64_t e = base + static_cast<int64_t>(t) * H;
    const float ft = f[e];
    st = __fmaf_rn(ft, st, x[e]);
    pr = __fmul_rn(pr, ft);
    out[e] = st;
  }
  summ[id] = make_float2(pr, st);
}

__global__ void chunk_carry_kernel(float2* __restrict__ summ, float* __restrict__ state, int nseq,
                                   int H, int nch) {
  const int64_t lane = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (lane >= static_cast<int64_t>(nseq) * H) return;
  const int c = static_cast<int>(lane % H);
  const int64_t q = lane / H;
  float carry = state ? state[lane] : 0.0f;
  for (int k = 0; k < nch; ++k) {
    const int64_t id = (q * nch + k) * H + c;
    const float2 s = summ[id];
    summ[id].y = carry;  // becomes this chunk's carry-in
    carry = __fmaf_rn(s.x, carry, s.y);
  }
  if (state) state[lane] = carry;
}

__global__ void chunk_fix_kernel(float* __restrict__ out, const float2* __restrict__ summ,
                                 const float* __restrict__ f, int nseq, int T, int H, int nch) {
  const int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (id >= static_cast<int64_t>(nseq) * nch * H) return;
  const int c = static_cast<int>(id % H);
  const int64_t qk = id / H;
  const int k = static_cast<int>(qk % nch), q = static_cast<int>(qk / nch);
  const float carry = summ[id].y;
  if (carry == 0.0f) return;
  const int t0 = k * kChunkT, t1 = min(T, t0 + kChunkT);
  const int64_t base = static_cast<int64_t>(q) * T * H + c;
  float pr = 1.0f;
  for (int t = t0; t < t1; ++t) {
    const int64_t e = base + static_cast<int64_t>(t) * H;
    pr = __fmul_rn(pr, f[e]);
    out[e] = __fmaf_rn(pr, carry, out[e]);
  }
}

// The token mixer of one decode step (one position per lane, H >= 8): a grid of about one
// 512-thread CTA per SM, each thread taking kMixLanes lanes per round with their loads and
// their divisions batched (all CTAs start as soon as the previous kernel's CTAs leave).
constexpr int kMixLanes = 2, kMixDecThreads = 512;
__global__ void __launch_bounds__(kMixDecThreads) mixer_decode_kernel(
    float* __restrict__ out, const float* __restrict__ iv, const float* __restrict__ fv,
    float* __restrict__ state, const float* __restrict__ lb, int nseq, int H, int64_t seg) {
  grid_dep_launch();
  grid_dep_wait();
  const int64_t total = static_cast<int64_t>(nseq) * H, stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // lane l = (q, c) is in the scalar tail of its segment (seg = seg_rows * H elements) only
  // in the segment's last row q, at columns c >= tail_from; (q, c) advance by counters
  const int64_t seg_rows = seg / H;
  const int tail_from = H - static_cast<int>(seg % 8);
  int64_t l0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  int64_t q = l0 / H;
  int c = static_cast<int>(l0 % H);
  const int64_t dq = stride / H;
  const int dc = static_cast<int>(stride % H);
  for (; l0 < total; l0 += kMixLanes * stride) {
    float a[kMixLanes], b[kMixLanes], s0[kMixLanes], lv[kMixLanes];
    bool body[kMixLanes];
#pragma unroll
    for (int u = 0; u < kMixLanes; ++u) {  // all loads of the round first
      const int64_t l = l0 + u * stride;
      const bool ok = l < total;
      a[u] = ok ? __ldcs(iv + l) : 0.0f;
      b[u] = ok ? __ldcs(fv + l) : 0.0f;
      s0[u] = (ok && state) ? state[l] : 0.0f;
      lv[u] = (ok && lb) ? __ldg(lb + c) : 0.0f;
      body[u] = c < tail_from || (q + 1) % seg_rows != 0;
      c += dc;
      q += dq;
      if (c >= H) {
        c -= H;
        ++q;
      }
    }
    float f[kMixLanes], om[kMixLanes], sv[kMixLanes];
    sigmoid_n(b, body, f);
#pragma unroll
    for (int u = 0; u < kMixLanes; ++u) {
      if (lb) f[u] = lower_bound_x(f[u], lv[u]);
      om[u] = __fadd_rn(1.0f, -f[u]);
    }
    swiglu_n(a, om, body, sv);
#pragma unroll
    for (int u = 0; u < kMixLanes; ++u) {
      const int64_t l = l0 + u * stride;  // element index = lane (T = 1)
      if (l >= total) break;
      const float st = hgrn_step_x(f[u], s0[u], sv[u]);
      out[l] = st;
      if (state) state[l] = st;
    }
  }
}

// The whole token mixer in one pass, one thread per (sequence, channel) lane: per step the
// forget gate (sigmoid, lower bound), the SwiGLU scan input and the recurrence step, i.e.
// the reference's gate loop (hgrn_model.cpp:109-134) followed by its scan (hgrn_scan.cpp:11-19)
// without the intermediate arrays. Loads run kMixAhead steps ahead of the serial recurrence.
constexpr int kMixAhead = 16;
__global__ void __launch_bounds__(128) mixer_kernel(float* __restrict__ out, const float* __restrict__ iv,
                                                    const float* __restrict__ fv, float* __restrict__ state,
                                                    const float* __restrict__ lb, int nseq, int T, int H,
                                                    int64_t seg) {
  grid_dep_launch();
  grid_dep_wait();
  const int64_t lane = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (lane >= static_cast<int64_t>(nseq) * H) return;
  const int64_t q = lane / H, c = lane % H;
  const int64_t base = q * T * H + c;
  const float lbc = lb ? __ldg(lb + c) : 0.0f;
  const int64_t body_n = seg & ~int64_t(7);
  int64_t es = base % seg;  // element index within its reference vector call (seg >= H)
  float st = state ? state[lane] : 0.0f;
  for (int t0 = 0; t0 < T; t0 += kMixAhead) {
    float a[kMixAhead], b[kMixAhead];
#pragma unroll
    for (int u = 0; u < kMixAhead; ++u) {
      const int64_t e = base + static_cast<int64_t>(t0 + u) * H;
      a[u] = t0 + u < T ? __ldcs(iv + e) : 0.0f;
      b[u] = t0 + u < T ? __ldcs(fv + e) : 0.0f;
    }
    // gates and scan inputs of the batch first (independent of the recurrence)
    bool body[kMixAhead];
#pragma unroll
    for (int u = 0; u < kMixAhead; ++u) {
      body[u] = es < body_n;
      es += H;
      if (es >= seg) es -= seg;
    }
    float f[kMixAhead], om[kMixAhead], sv[kMixAhead];
    sigmoid_n(b, body, f);
#pragma unroll
    for (int u = 0; u < kMixAhead; ++u) {
      if (lb) f[u] = lower_bound_x(f[u], lbc);
      om[u] = __fadd_rn(1.0f, -f[u]);
    }
    swiglu_n(a, om, body, sv);
#pragma unroll
    for (int u = 0; u < kMixAhead; ++u) {
      if (t0 + u >= T) break;
      const int64_t e = base + static_cast<int64_t>(t0 + u) * H;
      st = hgrn_step_x(f[u], st, sv[u]);
      out[e] = st;
    }
  }
  if (state) state[lane] = st;
}

cudaError_t launch_mixer(float* i, float* f, float* recur, float* state, const float* lb,
                         int nseq, int len, int H, int seg_rows, cudaStream_t s, bool pdl,
                         void* chunk_ws) {
  const int64_t lanes = static_cast<int64_t>(nseq) * H;
  if (lanes == 0 || len == 0) return cudaSuccess;
  if (len == 1 && H >= 8) {
    const int64_t ctas = std::min<int64_t>(ceil_div(lanes, kMixDecThreads * kMixLanes), sm_count());
    return launch_k(mixer_decode_kernel, dim3(static_cast<unsigned>(ctas)), dim3(kMixDecThreads), 0, s,
                    pdl, recur, static_cast<const float*>(i), static_cast<const float*>(f), state, lb,
                    nseq, H, static_cast<int64_t>(seg_rows) * H);
  }
  static const bool fused = [] {
    const char* e = std::getenv("MMFREE_MIXER_FUSED");
    return e && e[0] == '1';
  }();
  if (fused && !chunk_ws) {  // one pass, one thread per lane (gates and chain in one thread)
    const int64_t ctas = ceil_div(lanes, 128);
    return launch_k(mixer_kernel, dim3(static_cast<unsigned>(ctas)), dim3(128), 0, s, pdl,
                    recur, static_cast<const float*>(i), static_cast<const float*>(f), state, lb, nseq,
                    len, H, static_cast<int64_t>(seg_rows) * H);
  }
  // the gates element-parallel, then the scan: the exact serial chain per lane, or (Float, with
  // chunk_ws) the chunked parallel scan
  const int64_t n = lanes * len;
  cudaError_t e = launch_k(gates_kernel, dim3(static_cast<unsigned>(ceil_div(n, 4 * 256))), dim3(256),
                           0, s, pdl, i, f, lb, n, H, static_cast<int64_t>(seg_rows) * H);
  if (e != cudaSuccess) return e;
  if (!chunk_ws) {
    return launch_k(scan_kernel, dim3(static_cast<unsigned>(ceil_div(lanes, 128))), dim3(128), 0, s,
                    pdl, recur, static_cast<const float*>(i), static_cast<const float*>(f), state, nseq,
                    len, H);
  }
  const int nch = static_cast<int>(ceil_div(len, kChunkT));
  auto* summ = static_cast<float2*>(chunk_ws);
  const int64_t items = static_cast<int64_t>(nseq) * nch * H;
  chunk_scan_kernel<<<static_cast<unsigned>(ceil_div(items, 256)), 256, 0, s>>>(recur, summ, i, f, nseq,
                                                                                len, H, nch);
  chunk_carry_kernel<<<static_cast<unsigned>(ceil_div(lanes, 128)), 128, 0, s>>>(summ, state, nseq, H, nch);
  chunk_fix_kernel<<<static_cast<unsigned>(ceil_div(items, 256)), 256, 0, s>>>(recur, summ, f, nseq, len,
                                                                               H, nch);
  return cudaGetLastError();
}

size_t mixer_chunk_bytes(int nseq, int len, int H) {
  return static_cast<size_t>(nseq) * static_cast<size_t>(ceil_div(len, kChunkT)) * H * sizeof(float2);
}

cudaError_t launch_scan(float* out, const float* i, const float* f, int T, int D, float* state,
                        cudaStream_t s) {
  if (T == 0 || D == 0) return cudaSuccess;
  scan_kernel<<<static_cast<unsigned>(ceil_div(D, 128)), 128, 0, s>>>(out, i, f, state, 1, T, D);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ swiglu
__global__ void swiglu_split_kernel(float* __restrict__ z, const float* __restrict__ y,
                                    int64_t n, int64_t seg, int I) {
  grid_dep_launch();
  grid_dep_wait();
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (e >= n) return;
  const int64_t t = e / I, c = e % I;
  const float* yr = y + t * 2 * I;
  z[e] = swiglu_x(yr[c], yr[I + c], in_body(e % seg, seg));
}

cudaError_t launch_swiglu_split(float* z, const float* y, int rows, int I, int seg_rows,
                                cudaStream_t s, bool pdl) {
  const int64_t n = static_cast<int64_t>(rows) * I;
  if (n == 0) return cudaSuccess;
  return launch_k(swiglu_split_kernel, dim3(static_cast<unsigned>(ceil_div(n, 256))), dim3(256), 0, s,
                  pdl, z, y, n, static_cast<int64_t>(seg_rows) * I, I);
}

__global__ void swiglu_kernel(float* __restrict__ out, const float* __restrict__ a,
                              const float* __restrict__ b, int64_t n) {
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (e < n) out[e] = swiglu_x(a[e], b[e], in_body(e, n));
}

cudaError_t launch_swiglu(float* out, const float* a, const float* b, int64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  swiglu_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, s>>>(out, a, b, n);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(float* y, const float* x, const float* w, int rows, int cols,
                           float eps, cudaStream_t s) {
  PrepArgs a;
  a.x = x;
  a.prew = w;
  a.pre_out = y;
  a.nproj = 0;
  a.M = rows;
  a.K = cols;
  a.eps = eps;
  return launch_prep(a, s);
}

cudaError_t launch_swishgate(float* out, const float* g, const float* o, const float* w, int rows,
                             int cols, float eps, cudaStream_t s) {
  PrepArgs a;
  a.x = g;
  a.o = o;
  a.prew = w;
  a.pre_out = out;
  a.nproj = 0;
  a.M = rows;
  a.K = cols;
  a.eps = eps;
  return launch_prep(a, s);
}

// ------------------------------------------------------------------------------ embed
__global__ void embed_kernel(float* __restrict__ h, const float* __restrict__ emb,
                             const int64_t* __restrict__ ids, int H, int V, uint32_t* err) {
  const int t = blockIdx.x;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && err) atomicOr(err, kErrBadToken);
  const float4* src = reinterpret_cast<const float4*>(emb + (ok ? id : 0) * static_cast<int64_t>(H));
  float* dst = h + static_cast<int64_t>(t) * H;
  if ((H & 3) == 0) {
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x)
      reinterpret_cast<float4*>(dst)[c] = ok ? __ldg(src + c) : make_float4(0, 0, 0, 0);
  } else {
    const float* s1 = emb + (ok ? id : 0) * static_cast<int64_t>(H);
    for (int c = threadIdx.x; c < H; c += blockDim.x) dst[c] = ok ? s1[c] : 0.0f;
  }
}

cudaError_t launch_embed(float* h, const float* emb, const int64_t* ids, int T, int H, int V,
                         uint32_t* err, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  embed_kernel<<<T, 256, 0, s>>>(h, emb, ids, H, V, err);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ argmax
// First index of the maximum; NaN never wins, and a NaN at index 0 wins outright, exactly
// like the reference's sequential `if (l[v] > l[chosen]) chosen = v` scan. Whole block.
__device__ int block_argmax(const float* __restrict__ l, int V) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ int result;
  const float first = l[0];
  if (isnan(first)) return 0;
  float bv = first;
  int bi = 0;
  // each thread visits v = tid, tid + blockDim, ... in increasing order; the loads of 8 such
  // elements are issued before their compares (one memory latency per 8, not per element);
  // a padding NaN never wins
  constexpr int kArgBatch = 8;
  for (int v0 = threadIdx.x; v0 < V; v0 += kArgBatch * blockDim.x) {
    float x[kArgBatch];
#pragma unroll
    for (int u = 0; u < kArgBatch; ++u) {
      const int v = v0 + u * static_cast<int>(blockDim.x);
      x[u] = v < V ? l[v] : __int_as_float(0x7fc00000);
    }
#pragma unroll
    for (int u = 0; u < kArgBatch; ++u)
      if (x[u] > bv) {
        bv = x[u];
        bi = v0 + u * static_cast<int>(blockDim.x);
      }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : first;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) result = bi;
  }
  __syncthreads();
  return result;
}

__global__ void argmax_kernel(int64_t* __restrict__ ids, const float* __restrict__ logits, int V,
                              int ld) {
  const int best = block_argmax(logits + static_cast<int64_t>(blockIdx.x) * ld, V);
  if (threadIdx.x == 0) ids[blockIdx.x] = best;
}

cudaError_t launch_argmax(int64_t* ids, const float* logits, int M, int V, int ld,
                          cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  argmax_kernel<<<M, 1024, 0, s>>>(ids, logits, V, ld);
  return cudaGetLastError();
}

__global__ void argmax_at_kernel(int64_t* __restrict__ ids, int64_t stride, int64_t* pos,
                                 unsigned* done, const float* __restrict__ logits, int V, int ld) {
  grid_dep_launch();
  grid_dep_wait();
  const int b = blockIdx.x;
  const int best = block_argmax(logits + static_cast<int64_t>(b) * ld, V);
  if (threadIdx.x == 0) {
    const int64_t p = *pos;
    ids[b * stride + p + 1] = best;
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {  // last block: advance the position
      *done = 0;
      *pos = p + 1;
    }
  }
}

cudaError_t launch_argmax_at(int64_t* ids, int64_t stride, int64_t* pos, unsigned* done,
                             const float* logits, int B, int V, int ld, cudaStream_t s, bool pdl) {
  if (B == 0) return cudaSuccess;
  return launch_k(argmax_at_kernel, dim3(B), dim3(1024), 0, s, pdl, ids, stride, pos, done, logits, V, ld);
}

// ------------------------------------------------------------------------------ sampling
// Temperature / top-k sampling of one logits row per CTA (hgrn_model.cpp:274-300, :382-405):
// the k highest logits are the candidates (ties at the k-th value go to the lower index),
// p_j = exp((l_j - max) / temperature) in float (computed as a double exp rounded to float),
// summed in double, and the first candidate in ascending index order whose running sum
// reaches u * sum is drawn, u being the stream's uniform for this position (drawn on the host
// from the stream's mt19937_64, as the reference draws it). With k = V the candidates are in
// the reference's own order (all of them, ascending), so the draw is the reference's.
constexpr int kSampleThreads = 1024;

__device__ __forceinline__ uint32_t order_key(float v) {  // monotone in v; NaN lowest
  if (isnan(v)) return 0u;
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <class T>
__device__ __forceinline__ T block_excl_scan(T v, T* sh, T& total) {  // 1024 threads
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T w = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sh[lane] = w;
  }
  __syncthreads();
  total = sh[31];
  const T before = warp ? sh[warp - 1] : T(0);
  __syncthreads();
  return before + x - v;
}

__global__ void __launch_bounds__(kSampleThreads) sample_at_kernel(
    int64_t* __restrict__ ids, int64_t stride, int64_t* pos, unsigned* done, int advance, int row0,
    const float* __restrict__ logits, int V, int ld, const double* __restrict__ uni,
    int64_t ustride, float temperature, int top_k) {
  grid_dep_launch();
  grid_dep_wait();
  extern __shared__ __align__(16) float s_l[];  // the row, V floats
  __shared__ uint32_t s_hist[256];
  __shared__ double s_d[32];
  __shared__ int s_i[32];
  __shared__ uint32_t s_u[4];
  __shared__ int s_pick;
  const int tid = threadIdx.x, b = row0 + blockIdx.x;
  const float* lg = logits + static_cast<int64_t>(blockIdx.x) * ld;
  for (int j = tid; j < V; j += kSampleThreads) s_l[j] = lg[j];
  if (tid == 0) s_pick = 0x7fffffff;
  __syncthreads();
  // candidates: keys above the k-th largest key, plus the first (k - above) equal to it
  const int k = (top_k > 0 && top_k < V) ? top_k : V;
  uint32_t kth = 0;  // every key >= 0: all candidates when k == V
  int above = 0;
  if (k < V) {
    uint32_t prefix = 0, mask = 0;
    int want = k;  // rank (1-based, from the top) of the k-th largest within the prefix class
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += kSampleThreads) s_hist[i] = 0;
      __syncthreads();
      for (int j = tid; j < V; j += kSampleThreads) {
        const uint32_t key = order_key(s_l[j]);
        if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t acc = 0;
        int d = 255;
        for (; d > 0; --d) {
          if (acc + s_hist[d] >= static_cast<uint32_t>(want)) break;
          acc += s_hist[d];
        }
        s_u[0] = static_cast<uint32_t>(d);
        s_u[1] = acc;
      }
      __syncthreads();
      prefix |= s_u[0] << shift;
      mask |= 255u << shift;
      want -= static_cast<int>(s_u[1]);
      above += static_cast<int>(s_u[1]);
      __syncthreads();
    }
    kth = prefix;
  }
  const int need_eq = k - above;  // equal keys to take, lowest indices first
  // maximum over the candidates = the maximum of the row (the top element is a candidate)
  float mx = -INFINITY;
  for (int j = tid; j < V; j += kSampleThreads) mx = fmaxf(mx, s_l[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) s_d[tid >> 5] = mx;
  __syncthreads();
  if (tid < 32) {
    float m = static_cast<float>(s_d[tid]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (tid == 0) s_d[0] = m;
  }
  __syncthreads();
  const float maxl = static_cast<float>(s_d[0]);
  __syncthreads();
  // each thread owns a contiguous chunk of indices: ranks of equal keys, then p and sums
  const int per = (V + kSampleThreads - 1) / kSampleThreads;
  const int j0 = tid * per, j1 = min(V, j0 + per);
  int eq_local = 0;
  for (int j = j0; j < j1; ++j) eq_local += order_key(s_l[j]) == kth;
  int eq_total;
  int eq_before = block_excl_scan<int>(eq_local, s_i, eq_total);
  double part = 0.0;
  for (int j = j0; j < j1; ++j) {
    const uint32_t key = order_key(s_l[j]);
    bool cand = key > kth;
    if (key == kth) cand = eq_before++ < need_eq;
    float p = 0.0f;
    if (cand) p = __double2float_rn(exp(static_cast<double>(__fdiv_rn(__fsub_rn(s_l[j], maxl), temperature))));
    s_l[j] = cand ? p : -1.0f;  // candidate weights (p >= 0), -1 marks the others
    part += static_cast<double>(p);
  }
  __syncthreads();
  double sum;
  const double before = block_excl_scan<double>(part, s_d, sum);
  const double r = uni[static_cast<int64_t>(b) * ustride + (*pos + 1)] * sum;
  // first candidate whose running sum reaches r; else the last candidate
  double acc = before;
  int last_cand = -1;
  for (int j = j0; j < j1; ++j) {
    const float p = s_l[j];
    if (p < 0.0f) continue;
    last_cand = j;
    acc += static_cast<double>(p);
    if (r <= acc) {
      atomicMin(&s_pick, j);
      break;
    }
  }
  __syncthreads();
  int lc = last_cand;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lc = max(lc, __shfl_xor_sync(0xffffffffu, lc, o));
  if ((tid & 31) == 0) s_i[tid >> 5] = lc;
  __syncthreads();
  if (tid == 0) {
    int l = -1;
    for (int w = 0; w < kSampleThreads / 32; ++w) l = max(l, s_i[w]);
    const int chosen = s_pick != 0x7fffffff ? s_pick : max(l, 0);
    const int64_t p = *pos;
    ids[b * stride + p + 1] = chosen;
    if (advance) {
      __threadfence();
      if (atomicAdd(done, 1u) == gridDim.x - 1) {  // last block: advance the position
        *done = 0;
        *pos = p + 1;
      }
    }
  }
}

cudaError_t launch_sample_at(int64_t* ids, int64_t stride, int64_t* pos, unsigned* done,
                             bool advance, int row0, const float* logits, int B, int V, int ld,
                             const double* uni, int64_t ustride, float temperature, int top_k,
                             cudaStream_t s, bool pdl) {
  if (B == 0) return cudaSuccess;
  const size_t smem = static_cast<size_t>(V) * sizeof(float);
  if (smem > kMaxDynSmem || !(temperature > 0.0f)) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) raise_smem_limit(reinterpret_cast<const void*>(sample_at_kernel));
  return launch_k(sample_at_kernel, dim3(B), dim3(kSampleThreads), smem, s, pdl, ids, stride, pos,
                  done, advance ? 1 : 0, row0, logits, V, ld, uni, ustride, temperature, top_k);
}

__global__ void embed_at_kernel(float* __restrict__ h, const float* __restrict__ emb,
                                const int64_t* __restrict__ ids, int64_t stride,
                                const int64_t* pos, int H, int V, uint32_t* err) {
  grid_dep_launch();
  grid_dep_wait();
  const int b = blockIdx.x;
  const int64_t id = ids[b * stride + *pos];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && err) atomicOr(err, kErrBadToken);
  const float* src = emb + (ok ? id : 0) * static_cast<int64_t>(H);
  float* dst = h + static_cast<int64_t>(b) * H;
  // 8 loads per thread issued before their stores (one memory latency per 8 elements)
  constexpr int kEmbBatch = 8;
  for (int c0 = threadIdx.x; c0 < H; c0 += kEmbBatch * blockDim.x) {
    float v[kEmbBatch];
#pragma unroll
    for (int u = 0; u < kEmbBatch; ++u) {
      const int c = c0 + u * static_cast<int>(blockDim.x);
      v[u] = (ok && c < H) ? __ldg(src + c) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kEmbBatch; ++u) {
      const int c = c0 + u * static_cast<int>(blockDim.x);
      if (c < H) dst[c] = v[u];
    }
  }
}

cudaError_t launch_embed_at(float* h, const float* emb, const int64_t* ids, int64_t stride,
                            const int64_t* pos, int B, int H, int V, uint32_t* err,
                            cudaStream_t s, bool pdl) {
  if (B == 0) return cudaSuccess;
  return launch_k(embed_at_kernel, dim3(B), dim3(256), 0, s, pdl, h, emb, ids, stride, pos, H, V, err);
}

}  // namespace mmfree_cuda
