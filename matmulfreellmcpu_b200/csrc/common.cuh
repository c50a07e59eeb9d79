// common.cuh -- shared definitions for the mmfree CUDA kernels (sm_100a).
//
// Packed ternary weight layout ("tiled 2-bit"), the HBM format of every BitLinear weight:
//
//   A [N, K] ternary matrix (nn.Linear layout, N = out features, K = in features) is
//   stored as Ng = ceil(N/32) row groups x Kc = ceil(K/64) k-chunks of 512 bytes. Chunk
//   (g, c) holds rows 32g..32g+31, 16 bytes per row (row r of the group at byte 16r), so a
//   warp whose lane r loads 16 bytes reads one contiguous 512-byte line.
//   Each 16-byte row piece is 4 little-endian u32 words; word w holds the 16 weights
//   k = 64c + 16w + 4g' + j (g' = 0..3, j = 0..3) as 2-bit codes u = w_ternary + 1 in
//   {0, 1, 2} at bit 8j + 2g'. Masking with 0x03030303 << 2g' therefore yields 4 bytes
//   u * 4^g' whose byte j lines up with activation k = 64c + 16w + 4g' + j: one dp4a per
//   4 weights and activation plane. Padding rows and columns hold u = 1 (weight 0).
//
// Accumulation identity used by every integer kernel:
//   sum_k w_k q_k = sum_k u_k q_k - sum_k q_k,
// with q_k = 256 * hi_k + lo_k split into a signed high byte and an unsigned low byte
// (the Q5.10 codes are int16). Both sides are exact in int32 for K <= 65536.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mmfree_cuda {

constexpr int kRowsPerGroup = 32;
constexpr int kChunkK = 64;
constexpr int kChunkBytes = kRowsPerGroup * 16;
constexpr int kMaxK = 65536;

__host__ __device__ constexpr int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ constexpr int64_t packed_groups(int64_t n) { return ceil_div(n, kRowsPerGroup); }
__host__ __device__ constexpr int64_t packed_chunks(int64_t k) { return ceil_div(k, kChunkK); }
__host__ __device__ constexpr int64_t packed_bytes(int64_t n, int64_t k) {
  return packed_groups(n) * packed_chunks(k) * kChunkBytes;
}
// K padded to whole chunks: the row length of every activation plane.
__host__ __device__ constexpr int64_t padded_k(int64_t k) { return packed_chunks(k) * kChunkK; }

// Byte offset of the 2-bit code of weight (n, k) and its bit position.
__host__ __device__ inline int64_t packed_word_offset(int64_t n, int64_t k, int64_t kc) {
  int64_t g = n / kRowsPerGroup, r = n % kRowsPerGroup, c = k / kChunkK, w = (k % kChunkK) / 16;
  return ((g * kc + c) * kRowsPerGroup + r) * 16 + 4 * w;
}
__host__ __device__ inline int packed_bit(int64_t k) {
  int i = static_cast<int>(k % 16);
  return 8 * (i & 3) + 2 * (i >> 2);
}

// dp4a with explicit signedness: weights are unsigned bytes, activation planes are signed
// (high bytes) or unsigned (low bytes).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// The ternary weight (code - 1) of byte jj of m (codes 0..2 in the low bits of each byte) as
// an exact float, without an int-to-float conversion: the byte is placed in the mantissa of
// 2^23 (bits 0x4B0000cc = 2^23 + code), and 2^23 + 1 is subtracted.
__device__ __forceinline__ float ternary_f32(uint32_t m, int jj) {
  const float f = __uint_as_float(__byte_perm(m, 0x4B000000u, 0x7540u | static_cast<unsigned>(jj)));
  return __fadd_rn(f, -8388609.0f);
}

// Float-mode activations for the tensor cores: y = hi + lo + e with hi = bf16(y),
// lo = bf16(y - hi) (the difference is exact in fp32) and |e| <= 2^-17 |y|. Four values per
// call, packed as two 64-bit words of bf16 (element u in bits 16u..16u+15).
__device__ __forceinline__ void bf16_split4(const float (&y)[4], uint2& hi, uint2& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const __nv_bfloat16 hb = __float2bfloat16_rn(y[u]);
    const __nv_bfloat16 lb = __float2bfloat16_rn(__fsub_rn(y[u], __bfloat162float(hb)));
    h[u] = __bfloat16_as_ushort(hb);
    l[u] = __bfloat16_as_ushort(lb);
  }
  hi = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
  lo = make_uint2(l[0] | (l[1] << 16), l[2] | (l[3] << 16));
}

// Device-side error flags (bitmask), raised by kernels instead of trapping.
enum : uint32_t {
  kErrBadToken = 1u,     // a token id outside [0, vocab)
  kErrNotTernary = 2u,   // a weight outside {-1, 0, +1} given to the repack kernel
  kErrRange = 4u,        // an activation code outside int16 given to the ternary matmul
  kErrTimeout = 8u,      // a bounded wait inside a kernel gave up
};

// Programmatic dependent launch. A kernel launched with launch_k(..., pdl = true) may start
// while its predecessor in the stream still runs: before grid_dep_wait() it may only read
// data no earlier kernel writes (weights, norm weights) and write nothing global; after it,
// every earlier kernel has finished and its writes are visible. grid_dep_launch() lets the
// next kernel start its own prologue.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t s, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Epilogue selectors of the BitLinear matmul kernels.
enum Epilogue : int {
  kEpiStore = 0,   // out[m, n] = acc * scale
  kEpiResid = 1,   // out[m, n] = resid[m, n] + acc * scale
};

}  // namespace mmfree_cuda
