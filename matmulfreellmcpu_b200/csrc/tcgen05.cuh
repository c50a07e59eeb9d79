// tcgen05.cuh -- device helpers shared by the tensor-core BitLinear kernels (tc_matmul.cu,
// tc_rows.cu): mbarriers, bulk and TMA copies, tensor-memory loads and stores, shared-memory
// matrix and instruction descriptors, and the launch argument blocks.
#pragma once
#include "common.cuh"
#include "kernels.h"

#include <cuda.h>
#include <cstdint>

namespace mmfree_cuda {

namespace {

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

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// arrive and add `bytes` to the transaction count the phase waits for
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// L2 policy for data read once per launch (the weights): evict first, so that the stream
// does not displace activations and kernel code
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// L2 policy for weights that several token tiles of one launch read (prefill): evict last
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// bulk global -> shared copy completing on an mbarrier (no multicast), with an L2 policy
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// 2-D tiled TMA load (no multicast) with an L2 policy; x * element size is a multiple of 16 B
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                                 uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// 3-D tiled TMA load (no multicast); x * element size is a multiple of 16 B
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// 2-D tiled TMA load (no multicast); x is a multiple of 128 bytes
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// all threads of all CTAs of the cluster (release / acquire of shared memory)
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// address of the same shared-memory location in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// 16-byte load from a peer's shared memory (no memory clobber: callers read peer data
// written before a cluster barrier, whose asm orders it; without the clobber a batch of
// these loads is issued before its first use)
__device__ __forceinline__ void ld_cluster_v4(uint32_t addr, uint32_t* v) {
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(addr));
}
// the same from this CTA's own shared memory
__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint32_t* v) {
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(addr));
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

// Instruction descriptor of kind::f16 for the Float path: D f32, A and B both bf16 (the same
// type, as the kind requires), both K-major, M=128, N=bn.
__host__ __device__ constexpr uint32_t idesc_bf16(int bn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(bn >> 3) << 17) |
         (static_cast<uint32_t>(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Two ternary codes (u = w + 1 in the low 2 bits of bytes b and b + 1 of m) as a pair of bf16
// weights w in {-1, 0, +1} (0xBF80, 0, 0x3F80): the low and high bytes of each bf16 are looked
// up by byte_perm in the tables 0x00800080 (lows) and 0x003F00BF (highs), indexed by u.
__device__ __forceinline__ uint32_t ternary_bf16x2(uint32_t m, int b) {
  const uint32_t u0 = (m >> (8 * b)) & 3u, u1 = (m >> (8 * b + 8)) & 3u;
  return __byte_perm(0x003F00BFu, 0x00800080u, (4u + u0) | (u0 << 4) | ((4u + u1) << 8) | (u1 << 12));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}


__device__ __forceinline__ bool cta_failed(const uint32_t* f) {
  return *reinterpret_cast<const volatile uint32_t*>(f) != 0;
}

// bounded wait that gives up early once another role of the CTA has failed
__device__ __forceinline__ bool role_wait(uint64_t* bar, uint32_t parity, uint32_t* s_fail) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && cta_failed(s_fail)) return false;
  }
  return false;
}

}  // namespace

// One projection of a launch (i/f/g share a launch; they differ only in these).
struct TcProj {
  const void* w;           // packed weights
  const int32_t* rowsum;   // [M] code sums of the projection's activation rows
  float* out;              // [M, ldo]
  float scale;             // 1 / (2^f * scale_w)
};

struct TcArgs {
  MatmulArgs m;       // shape, residual and raw-accumulator output (single projection)
  TcProj pj[3];
  int nproj;          // grid.z = nproj * splits
  int pair;           // SwiGLU gate_proj: I/32, the first group of the up rows; 0 otherwise
  int seg_rows;       // SwiGLU: token rows of one reference vector call (SIMD tails) ...
  int tail_from;      // ... whose last row's columns >= tail_from are its scalar tail
  uint32_t* err;      // bit kErrTimeout on a timed-out wait
  int splits;         // k-block ranges per tile = cluster size along z (1, 2, 4 or 8)
  int vec;            // outputs, residual and raw accumulators allow 16-byte accesses
};

struct TcMaps {
  CUtensorMap m[3];   // activation planes of each projection
  CUtensorMap w[3];   // packed weights of each projection (FixedQ510: a k-block of a tile's
                      // 4 groups, or 2 + 2 for a SwiGLU pair tile, per copy)
};

// The activation planes [2][M][Kp] as one 2-D tensor map of 2M rows (u8, or bf16 for the Float
// path); a box is bn rows x 128 B, written to shared memory with the 128-byte swizzle.
cudaError_t planes_map(CUtensorMap* map, const int8_t* planes, int M, int64_t kp, int bn, bool bf16);
// The u8 planes as a 3-D tensor {Kp, M, 2}: a box of 128 B x bn rows x 2 planes (a k-block of
// both planes in one copy), 128-byte swizzle.
cudaError_t planes_map3(CUtensorMap* map, const int8_t* planes, int M, int64_t kp, int bn);
// Packed ternary weights as a 2-D tensor of 32-bit words (a row per 32-row group); a box is one
// 128-k block (two chunks, 1 KB) of `rows` consecutive groups.
cudaError_t weights_map(CUtensorMap* map, const void* w, int64_t n, int64_t k, int rows);

// The persistent large-M kernel (tc_rows.cu): whether it is enabled (MMFREE_TC_ROWS=0 turns it
// off), its tile count for a launch (0: it does not apply) and the launch itself.
bool tc_rows_enabled();
int64_t tc_rows_tiles(const MatmulArgs& a, int nproj, int pair);
cudaError_t launch_tc_rows(const TcArgs& p, const MatmulArgs* a, int sm_count, cudaStream_t s);

}  // namespace mmfree_cuda
