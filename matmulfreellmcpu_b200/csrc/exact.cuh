// exact.cuh -- device arithmetic that reproduces the reference CPU engine bit for bit.
//
// The reference (matmulfreellmCPU) defines its numerics by its x86 build: AVX2 primitives in
// cpp/include/mmfree/simd.hpp compiled by g++ -O2 -mavx2 -mfma with GCC's default FP
// contraction. Every operation below is an explicitly rounded intrinsic (__fmul_rn,
// __fadd_rn, __fdiv_rn, __fsqrt_rn, __fmaf_rn), so nvcc cannot contract or reorder it, and
// each mul+add pair that the reference build fuses is written as one __fmaf_rn:
//   * hgrn_step:          state = fma(f, state, in)              (simd.hpp:340, :354)
//   * lower bound:        f = fma(1 - lb, f, lb)                 (hgrn_model.cpp:121)
//   * expf_poly tail:     the GCC-fused form of simd.hpp:215-224
// The sumsq tail (simd.hpp:87) stays unfused, as in the reference build.
#pragma once

#include <cstdint>

namespace mmfree_cuda {

// Cephes single-precision exp (S. L. Moshier, Cephes Math Library expf.c): log2(e), ln(2)
// split hi/lo and the degree-6 minimax polynomial, in the form the reference writes it
// (simd.hpp:208-249).
constexpr float kExpHi = 88.3762626647949f;
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693359375f;
constexpr float kLn2Lo = -2.12194440e-4f;
constexpr float kP0 = 1.9875691500E-4f;
constexpr float kP1 = 1.3981999507E-3f;
constexpr float kP2 = 8.3334519073E-3f;
constexpr float kP3 = 4.1665795894E-2f;
constexpr float kP4 = 1.6666665459E-1f;
constexpr float kP5 = 5.0000001201E-1f;

__device__ __forceinline__ float pow2_of(float fx) {
  // fx is integral in [-127, 128]; build the exponent field directly (simd.hpp:246-248).
  uint32_t e = static_cast<uint32_t>(__float2int_rz(fx) + 127) << 23;
  return __uint_as_float(e);
}

// Element e of an n-element vector op is in the 8-wide SIMD body iff e < 8*floor(n/8);
// the rest is the scalar tail, whose exp differs (exp_neg).
__device__ __forceinline__ bool in_body(uint64_t e, uint64_t n) { return e < (n & ~uint64_t(7)); }

// exp(-x) as the vector exp of the SIMD body computes it (simd.hpp:232-249) or, !body, as
// the scalar-tail exp of the compiled reference (simd.hpp:212-229), without a branch: the
// two differ only in how a NaN is clamped (vmaxps/vminps select the bound; the tail's
// compares keep the NaN) and in how the last polynomial step adds 1 (the tail's form is
// fused by the build).
__device__ __forceinline__ float exp_neg(float x, bool body) {
  x = -x;
  float xv = (x > -kExpHi) ? x : -kExpHi;
  xv = (xv < kExpHi) ? xv : kExpHi;
  const float xt = (x > kExpHi) ? kExpHi : ((x < -kExpHi) ? -kExpHi : x);
  x = body ? xv : xt;
  const float fx = floorf(__fmaf_rn(x, kLog2e, 0.5f));
  float r = __fmaf_rn(-fx, kLn2Hi, x);
  r = __fmaf_rn(-fx, kLn2Lo, r);
  float p = kP0;
  p = __fmaf_rn(p, r, kP1);
  p = __fmaf_rn(p, r, kP2);
  p = __fmaf_rn(p, r, kP3);
  p = __fmaf_rn(p, r, kP4);
  p = __fmaf_rn(p, r, kP5);
  const float rr = __fmul_rn(r, r);
  const float pv = __fmaf_rn(p, rr, __fadd_rn(r, 1.0f));
  const float pt = __fadd_rn(__fmaf_rn(p, rr, r), 1.0f);
  return __fmul_rn(body ? pv : pt, pow2_of(fx));
}

// simd::sigmoid / silu / swiglu (simd.hpp:270-330), one element.
__device__ __forceinline__ float sigmoid_x(float x, bool body) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_neg(x, body)));
}
__device__ __forceinline__ float silu_x(float x, bool body) {
  return __fdiv_rn(x, __fadd_rn(1.0f, exp_neg(x, body)));
}
__device__ __forceinline__ float swiglu_x(float a, float b, bool body) {
  return __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, exp_neg(a, body))), b);
}

// The same for N elements at a time: the branch-free exps of all N first, then the divisions.
template <int N>
__device__ __forceinline__ void sigmoid_n(const float (&x)[N], const bool (&body)[N], float (&out)[N]) {
  float d[N];
#pragma unroll
  for (int i = 0; i < N; ++i) d[i] = __fadd_rn(1.0f, exp_neg(x[i], body[i]));
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __fdiv_rn(1.0f, d[i]);
}
template <int N>
__device__ __forceinline__ void silu_n(const float (&x)[N], const bool (&body)[N], float (&out)[N]) {
  float d[N];
#pragma unroll
  for (int i = 0; i < N; ++i) d[i] = __fadd_rn(1.0f, exp_neg(x[i], body[i]));
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __fdiv_rn(x[i], d[i]);
}
template <int N>
__device__ __forceinline__ void swiglu_n(const float (&a)[N], const float (&b)[N], const bool (&body)[N],
                                         float (&out)[N]) {
  float d[N];
#pragma unroll
  for (int i = 0; i < N; ++i) d[i] = __fadd_rn(1.0f, exp_neg(a[i], body[i]));
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __fmul_rn(__fdiv_rn(a[i], d[i]), b[i]);
}

// rstd = 1 / sqrt(sumsq / n + eps)  (rmsnorm.cpp:18, bitlinear.cpp:86).
__device__ __forceinline__ float rstd_of(float sumsq, float n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, n), eps)));
}

// y = x * rstd * w, left to right (rmsnorm.cpp:19).
__device__ __forceinline__ float norm_x(float x, float rstd, float w) {
  return __fmul_rn(__fmul_rn(x, rstd), w);
}

// simd::quant_q510 (simd.hpp:162-187), one element. In the SIMD body the float->int
// conversion is cvtps2dq (round half to even, NaN / out-of-range -> INT32_MIN) followed by
// an integer clamp; in the scalar tail the clamp is in float and the cast truncates (NaN ->
// INT32_MIN). Both forms are evaluated with selects (no branches in unrolled loops).
__device__ __forceinline__ int32_t quant_x(float y, float qs, bool body) {
  const float q = __fmul_rn(y, qs);
  const int32_t cv = __float2int_rn(q);
  const int32_t vb = fabsf(q) < 2147483648.0f ? cv : INT32_MIN;  // false for NaN too
  const int32_t bq = vb < -32768 ? -32768 : (vb > 32767 ? 32767 : vb);
  float r = rintf(q);
  r = r > 32767.0f ? 32767.0f : (r < -32768.0f ? -32768.0f : r);
  const int32_t tq = isnan(q) ? INT32_MIN : static_cast<int32_t>(r);
  return body ? bq : tq;
}

// quant_x's SIMD-body form for 4 elements of the body, straight into the two byte-plane words
// (byte u = element u) plus their code sum, without a float->int conversion: clamping before
// rounding equals rounding before clamping (integer bounds); NaN and q <= -2^31 clamp to
// -32768 like cvtps2dq's INT32_MIN does, q >= 2^31 is selected to it; the clamped value is
// rounded half to even by one round-to-nearest add of 1.5 * 2^23 (the sum lies in [2^23,
// 2^24), where the float spacing is 1), after which its low 16 bits hold the code in two's
// complement. `lo_xor` is 0x80808080 for the signed low plane, else 0.
__device__ __forceinline__ void quant4_body_planes(const float (&y)[4], float qs, uint32_t lo_xor,
                                                   uint32_t& hi, uint32_t& lo, int32_t& sum) {
  uint32_t b[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float q = __fmul_rn(y[u], qs);
    float c = fminf(fmaxf(q, -32768.0f), 32767.0f);  // fmaxf(NaN, v) = v
    c = q >= 2147483648.0f ? -32768.0f : c;
    b[u] = __float_as_uint(__fadd_rn(c, 12582912.0f));
    sum += static_cast<int32_t>(b[u] - 0x4B400000u);
  }
  const uint32_t t01 = __byte_perm(b[0], b[1], 0x5140);  // [lo0, lo1, hi0, hi1]
  const uint32_t t23 = __byte_perm(b[2], b[3], 0x5140);  // [lo2, lo3, hi2, hi3]
  lo = __byte_perm(t01, t23, 0x5410) ^ lo_xor;
  hi = __byte_perm(t01, t23, 0x7632);
}

// Lower-bounded forget gate of layers > 0 (hgrn_model.cpp:116-124), as fused by the build.
__device__ __forceinline__ float lower_bound_x(float f, float lb) {
  return __fmaf_rn(__fadd_rn(1.0f, -lb), f, lb);
}

// One recurrence step (simd.hpp:335-357), as fused by the build.
__device__ __forceinline__ float hgrn_step_x(float f, float state, float in) {
  return __fmaf_rn(f, state, in);
}

// The AVX2 horizontal sum of 8 lane partials (simd.hpp:48-57), for lanes held by 8
// consecutive threads of a warp (lane j of the group holds partial j). Every thread of the
// 8-lane group receives the sum.
__device__ __forceinline__ float hsum8_lanes(float v, unsigned mask = 0xffffffffu) {
  const int j = threadIdx.x & 7;
  float hi = __shfl_down_sync(mask, v, 4, 8);    // lanes 0..3 get v[j+4]
  float b = __fadd_rn(v, hi);                    // b_j = v_j + v_{j+4}
  float b1 = __shfl_down_sync(mask, b, 1, 8);    // lane 0 gets b1, lane 2 gets b3
  float c = __fadd_rn(b, b1);                    // c0 = b0+b1, c2 = b2+b3
  float c2 = __shfl_down_sync(mask, c, 2, 8);    // lane 0 gets c2
  float s = __fadd_rn(c, c2);
  (void)j;
  return __shfl_sync(mask, s, 0, 8);
}

// Lane j (= threadIdx.x & 7) of an 8-lane group runs chain j of the AVX2 sum of squares
// (simd.hpp:69-89) over s[0..K): acc_j = fma(s[8i+j], s[8i+j], acc_j) for i < K/8, in order.
// Whole batches of 8 are loaded unconditionally one batch ahead of their FMAs, so the serial
// chain waits only on the FMA latency; a remainder of K/8 mod 8 steps follows.
__device__ __forceinline__ float sumsq_chain_lane(const float* s, int K) {
  const float* p = s + (threadIdx.x & 7);
  const int n8 = K >> 3, nb = n8 >> 3;
  float acc = 0.0f;
  if (nb > 0) {
    float cur[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) cur[u] = p[8 * u];
    for (int b = 1; b < nb; ++b) {
      float nxt[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) nxt[u] = p[64 * b + 8 * u];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fmaf_rn(cur[u], cur[u], acc);
#pragma unroll
      for (int u = 0; u < 8; ++u) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fmaf_rn(cur[u], cur[u], acc);
  }
  for (int i = nb * 8; i < n8; ++i) {
    const float v = p[8 * i];
    acc = __fmaf_rn(v, v, acc);
  }
  return acc;
}

// Full reference sum of squares of s[0..K) for the 8-lane group (every lane gets it).
__device__ __forceinline__ float sumsq_exact8(const float* s, int K, unsigned mask) {
  float sum = hsum8_lanes(sumsq_chain_lane(s, K), mask);
  for (int c = (K >> 3) * 8; c < K; ++c) sum = __fadd_rn(sum, __fmul_rn(s[c], s[c]));
  return sum;
}

}  // namespace mmfree_cuda
