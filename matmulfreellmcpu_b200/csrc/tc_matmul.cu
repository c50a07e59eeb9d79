// tc_matmul.cu -- FixedQ510 BitLinear matmul on the 5th-generation tensor cores (tcgen05).
//
// out[t, n] = dequant(sum_k w[n, k] * q[t, k]) for M activation rows (tokens) t and N output
// rows n, the same integer result as matmul_fixed_kernel (kernels.cu) and the reference's
// CpuBackend (ternary_backend.hpp:96-103), so every output is bit-identical.
//
// Per CTA: a tile of 128 weight rows x BN tokens, K in blocks of 128.
//   A (weights)  tiled 2-bit codes u = w + 1 are loaded by the 128 threads (thread = row,
//                16 B per 64-k chunk, a warp reads one contiguous 512-B line), expanded to u8
//                in registers and written to TENSOR MEMORY with tcgen05.st (row = TMEM lane,
//                4 codes per 32-bit column). The 4x-expanded operand never uses shared
//                memory bandwidth.
//   B (acts)     the high-byte (s8) and low-byte (u8) planes of the Q5.10 codes, BN rows x
//                128 B per k-block, copied with cp.async into shared memory in the
//                128-byte-swizzled K-major layout the MMA descriptor names.
//   MMA          one thread issues tcgen05.mma.cta_group::1.kind::i8 with A from TMEM:
//                D_hi += u x hi (u8 x s8), D_lo += u x lo (u8 x u8), M=128, N=BN, K=32 per
//                instruction, int32 accumulators in TMEM; tcgen05.commit signals an mbarrier
//                per pipeline stage.
//   epilogue     tcgen05.ld of D_hi/D_lo; acc = 256*D_hi + D_lo - sum_k q[t, k] (exact in
//                int32); split-K partials are combined with integer atomics (exact, order
//                free) and the last CTA of a tile applies dequant (+ residual).
// Every wait on an mbarrier is bounded; on timeout the CTA sets an error flag, stops issuing
// work, waits (bounded) for its own MMAs and still frees its tensor memory.
#include "common.cuh"
#include "kernels.h"

#include <cstdint>

namespace mmfree_cuda {

namespace {

constexpr int kTcThreads = 128;
constexpr int kStages = 4;           // pipeline depth (A in TMEM, B in shared memory)
constexpr int kPrefetch = 2;         // B k-blocks in flight ahead of the current one
constexpr int kKBlock = 128;         // k per pipeline stage (2 packed chunks)
constexpr uint32_t kSpinLimit = 1u << 26;  // bounded mbarrier waits

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// true when the phase with the given parity has completed
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bounded wait; returns false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes <- 16 registers per thread
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 consecutive TMEM columns of this warp's 32 lanes -> 16 registers per thread
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address (16-B units)
  d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused, K-major SW)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset: next 8 rows
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                  // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::i8: D s32, A u8 (K-major), B u8/s8 (K-major), M=128, N=bn.
__host__ __device__ constexpr uint32_t idesc_i8(bool b_signed, int bn) {
  return (2u << 4) | (0u << 7) | ((b_signed ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(bn >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

}  // namespace

struct TcArgs {
  MatmulArgs m;
  uint32_t* accum;    // split-K: [M, N] int32 partial sums (zero on entry, left zero on exit)
  uint32_t* tiles;    // split-K: one arrival counter per (weight tile, token tile), left zero
  uint32_t* err;      // bit kErrTimeout on a timed-out wait
  int splits;         // k-block ranges per tile (grid.z)
};

template <int BN>
__global__ void __launch_bounds__(kTcThreads, 1) tc_matmul_kernel(TcArgs p) {
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 64, "BN must be 16..64, a multiple of 16");
  constexpr int kCols = kStages * 32 + 2 * BN;                 // A stages + D_hi + D_lo
  constexpr int kAllocCols = kCols <= 128 ? 128 : (kCols <= 256 ? 256 : 512);
  static_assert(kAllocCols <= 256, "two CTAs per SM must fit in the 512 TMEM columns");
  constexpr int kBStage = BN * 128;                            // bytes of one plane per stage

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // align the B stages to the 1024-byte swizzle atom
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* b_hi = smem;                                  // [kStages][BN][128]
  unsigned char* b_lo = smem + kStages * kBStage;              // [kStages][BN][128]
  __shared__ uint64_t bars[kStages + 1];  // one per stage + a drain barrier
  __shared__ uint32_t tmem_base_sh;
  __shared__ uint32_t s_fail;
  __shared__ uint32_t s_last;

  const MatmulArgs& a = p.m;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * 128, t0 = blockIdx.y * BN;
  const int64_t kc = packed_chunks(a.K), kp = kc * kChunkK;
  const int nkb = static_cast<int>((kc + 1) / 2);
  const int kb0 = static_cast<int>(static_cast<int64_t>(nkb) * blockIdx.z / p.splits);
  const int kb1 = static_cast<int>(static_cast<int64_t>(nkb) * (blockIdx.z + 1) / p.splits);
  const int nk = kb1 - kb0;

  if (tid == 0) {
    for (int s = 0; s <= kStages; ++s) mbar_init(&bars[s], 1);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"(kAllocCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t tmem_a = tmem;                          // columns [0, 32*kStages)
  const uint32_t tmem_dhi = tmem + kStages * 32;         // BN columns
  const uint32_t tmem_dlo = tmem_dhi + BN;               // BN columns
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

  // this thread's weight row and its packed row pointer (16 B per 64-k chunk)
  const int wrow_group = (n0 >> 5) + warp;
  const bool wrow_ok = wrow_group < packed_groups(a.N);
  const uint4* wrow = static_cast<const uint4*>(a.w) + static_cast<int64_t>(wrow_group) * kc * 32 + lane;

  // B copy: each k-block needs 2 planes x BN rows x 8 chunks of 16 B
  auto issue_b = [&](int kb, int s) {
    constexpr int kChunks = 2 * BN * 8;
    for (int i = tid; i < kChunks; i += kTcThreads) {
      const int plane = i / (BN * 8), rem = i % (BN * 8), r = rem >> 3, c = rem & 7;
      const int trow = min(t0 + r, a.M - 1);  // rows past M repeat row M-1 (never stored)
      const int64_t kbyte = static_cast<int64_t>(kb) * kKBlock + c * 16;
      const int8_t* src = a.planes + (static_cast<int64_t>(plane) * a.M + trow) * kp +
                          (kbyte < kp ? kbyte : 0);
      unsigned char* dst = (plane ? b_lo : b_hi) + s * kBStage + r * 128 + ((c ^ (r & 7)) << 4);
      cp_async16(dst, src, kbyte < kp ? 16u : 0u);  // zero-fill past the padded row end
    }
  };

  bool fail = false;
  // prologue: B for the first kPrefetch k-blocks
  for (int j = 0; j < kPrefetch; ++j) {
    if (j < nk) issue_b(kb0 + j, j % kStages);
    cp_async_commit();
  }
  uint4 wnext[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  auto load_w = [&](int kb, uint4 (&w)[2]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t c = static_cast<int64_t>(kb) * 2 + h;
      w[h] = (wrow_ok && c < kc) ? __ldg(wrow + c * 32) : make_uint4(0x55555555u, 0x55555555u,
                                                                       0x55555555u, 0x55555555u);
    }
  };
  if (nk > 0) load_w(kb0, wnext);

  for (int i = 0; i < nk && !fail; ++i) {
    const int kb = kb0 + i, s = i % kStages;
    uint4 wcur[2] = {wnext[0], wnext[1]};
    if (i + 1 < nk) load_w(kb + 1, wnext);
    // refill B stage of k-block i + kPrefetch once the MMAs that read it (i + kPrefetch -
    // kStages) are done
    const int ip = i + kPrefetch;
    if (ip < nk) {
      const int used = ip - kStages;
      if (used >= 0 && !mbar_wait(&bars[used % kStages], (used / kStages) & 1)) fail = true;
      issue_b(kb0 + ip, ip % kStages);
    }
    cp_async_commit();
    // A stage s was read by the MMAs of k-block i - kStages
    if (i >= kStages && !mbar_wait(&bars[s], ((i - kStages) / kStages) & 1)) fail = true;
    tc_fence_after();
    // expand 2 x 64 codes to u8 and store them to TMEM columns s*32 + [0, 32)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t wd[4] = {wcur[h].x, wcur[h].y, wcur[h].z, wcur[h].w};
      uint32_t r[16];
#pragma unroll
      for (int w4 = 0; w4 < 4; ++w4)
#pragma unroll
        for (int q = 0; q < 4; ++q) r[4 * w4 + q] = (wd[w4] >> (2 * q)) & 0x03030303u;
      tmem_st16(tmem_a + lane_base + static_cast<uint32_t>(s * 32 + h * 16), r);
    }
    tmem_st_wait();
    cp_async_wait<kPrefetch>();  // this k-block's B copies have landed
    fence_proxy_async();          // make them visible to the tensor core (async proxy)
    if (fail) s_fail = 1;
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && s_fail == 0) {
      tc_fence_after();
      const uint32_t hi_base = smem_u32(b_hi + s * kBStage);
      const uint32_t lo_base = smem_u32(b_lo + s * kBStage);
#pragma unroll
      for (int j = 0; j < kKBlock / 32; ++j) {
        const uint32_t acc = (i > 0 || j > 0) ? 1u : 0u;
        const uint32_t a_addr = tmem_a + static_cast<uint32_t>(s * 32 + j * 8);
        mma_i8_ts(tmem_dhi, a_addr, smem_desc_sw128(hi_base + j * 32), idesc_i8(true, BN), acc);
        mma_i8_ts(tmem_dlo, a_addr, smem_desc_sw128(lo_base + j * 32), idesc_i8(false, BN), acc);
      }
      mma_commit(&bars[s]);
    }
    __syncthreads();
    fail = s_fail != 0;
  }
  cp_async_wait<0>();

  // wait for the last MMAs (their commit covers every earlier MMA of this thread)
  if (nk > 0 && !fail) {
    const int last = nk - 1;
    if (!mbar_wait(&bars[last % kStages], (last / kStages) & 1)) fail = true;
  }
  // one decision for the whole CTA: the epilogue's tcgen05.ld is warp-collective
  fail = __syncthreads_or(fail) != 0;
  tc_fence_after();
  if (fail) {
    if (tid == 0) {
      if (p.err) atomicOr(p.err, kErrTimeout);
      // drain: a commit arrives once every MMA this thread issued has finished
      mma_commit(&bars[kStages]);
      mbar_wait(&bars[kStages], 0);
    }
  } else if (nk > 0) {
    // epilogue: thread = weight row n, columns = tokens
    const int n = n0 + tid;
    const bool n_ok = n < a.N;
#pragma unroll
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t dh[16], dl[16];
      tmem_ld16(tmem_dhi + lane_base + c0, dh);
      tmem_ld16(tmem_dlo + lane_base + c0, dl);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = t0 + c0 + j;
        if (!n_ok || t >= a.M) continue;
        const uint32_t part = (dh[j] << 8) + dl[j];  // 256*D_hi + D_lo, wrapping like int32
        if (p.splits == 1) {
          const int32_t acc = static_cast<int32_t>(part - static_cast<uint32_t>(a.rowsum[t]));
          if (a.acc_out) a.acc_out[static_cast<int64_t>(t) * a.N + n] = acc;
          if (a.out) {
            float v = __fmul_rn(__int2float_rn(acc), a.scale);
            if (a.resid) v = __fadd_rn(a.resid[static_cast<int64_t>(t) * a.ldr + n], v);
            a.out[static_cast<int64_t>(t) * a.ldo + n] = v;
          }
        } else {
          atomicAdd(p.accum + static_cast<int64_t>(t) * a.N + n, part);
        }
      }
    }
    if (p.splits > 1) {
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
        s_last = atomicAdd(p.tiles + tile, 1u) == static_cast<uint32_t>(p.splits - 1);
        if (s_last) p.tiles[tile] = 0;
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
        for (int j = 0; j < BN; ++j) {
          const int t = t0 + j;
          if (!n_ok || t >= a.M) continue;
          uint32_t* cell = p.accum + static_cast<int64_t>(t) * a.N + n;
          const uint32_t sum = __ldcg(cell);
          *cell = 0;  // leave the workspace zeroed for the next launch
          const int32_t acc = static_cast<int32_t>(sum - static_cast<uint32_t>(a.rowsum[t]));
          if (a.acc_out) a.acc_out[static_cast<int64_t>(t) * a.N + n] = acc;
          if (a.out) {
            float v = __fmul_rn(__int2float_rn(acc), a.scale);
            if (a.resid) v = __fadd_rn(a.resid[static_cast<int64_t>(t) * a.ldr + n], v);
            a.out[static_cast<int64_t>(t) * a.ldo + n] = v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kAllocCols)
                 : "memory");
  }
}

// At least 80 KB per CTA, so that no more than two CTAs (2 x 256 TMEM columns) share an SM
// and tcgen05.alloc never waits for another CTA's columns.
template <int BN>
static size_t tc_smem_bytes() {
  const size_t need = 1024 + 2 * kStages * BN * 128;
  return need < 80 * 1024 ? 80 * 1024 : need;
}

template <int BN>
static cudaError_t launch_tc_bn(const TcArgs& p, cudaStream_t s) {
  const size_t smem = tc_smem_bytes<BN>();
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(tc_matmul_kernel<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  dim3 grid(static_cast<unsigned>(ceil_div(p.m.N, 128)), static_cast<unsigned>(ceil_div(p.m.M, BN)),
            static_cast<unsigned>(p.splits));
  tc_matmul_kernel<BN><<<grid, kTcThreads, smem, s>>>(p);
  return cudaGetLastError();
}

int tc_token_tile(int M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

int tc_splits(const MatmulArgs& a, int sm_count) {
  // enough CTAs to cover the SMs; every split keeps >= 2 k-blocks
  const int64_t tiles = ceil_div(a.N, 128) * ceil_div(a.M, tc_token_tile(a.M));
  const int nkb = static_cast<int>((packed_chunks(a.K) + 1) / 2);
  int splits = 1;
  while (tiles * splits * 2 <= sm_count && nkb / (splits * 2) >= 2) splits *= 2;
  return splits;
}

cudaError_t launch_matmul_tc(const MatmulArgs& a, uint32_t* accum, uint32_t* tiles, int splits,
                             uint32_t* err, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return cudaSuccess;
  TcArgs p{a, accum, tiles, err, splits};
  switch (tc_token_tile(a.M)) {
    case 16: return launch_tc_bn<16>(p, s);
    case 32: return launch_tc_bn<32>(p, s);
    default: return launch_tc_bn<64>(p, s);
  }
}

}  // namespace mmfree_cuda
