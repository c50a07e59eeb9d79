// decode.cu -- fused BitLinear kernels for few-row decode steps (M <= 4 rows: b=1 decode, or
// a handful of lockstep streams).
//
// One layer of the reference block (hgrn_model.cpp:80-195) becomes four launches:
//   K1  i/f/g projections   prologue rmsnorm(h)*attn_norm, then the exact BitLinear norm of
//                           each projection; epilogue: forget gate, lower bound, swiglu scan
//                           input and one recurrence step (hgrn_model.cpp:109-150) per column
//   K2  o_proj              prologue g_norm(g)*silu(recurrence) (rmsnorm_swishgate.cpp:13-30)
//                           then the BitLinear norm; epilogue resid = h + o
//   K3  gate_proj           prologue rmsnorm(resid)*mlp_norm; a CTA owns output columns c
//                           and I + c, so the epilogue writes z = silu(y[c]) * y[I + c]
//   K4  down_proj           prologue plain BitLinear norm of z; epilogue h = resid + down
// and the head is one more (final norm + lm_head with the greedy argmax fused in).
//
// Every CTA recomputes the prologue for its rows (the serial AVX2-order sum of squares is
// 8 FMA chains of K/8, the same in every CTA), so no separate normalisation kernel and no
// grid-wide synchronisation is needed. The arithmetic is that of exact.cuh / kernels.cu
// (bit-identical to the reference in FixedQ510).
//
// Launches use programmatic dependent launch: a kernel first asks L2 to prefetch its weight
// rows (one bulk prefetch per contiguous range), then waits for its predecessor
// (griddepcontrol.wait) before reading activations, and lets its own dependent launch early
// (griddepcontrol.launch_dependents). Weight streaming of layer l+1 thus overlaps layer l.
#include "common.cuh"
#include "exact.cuh"
#include "kernels.h"

#include <cfloat>

namespace mmfree_cuda {

namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;

__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// sum of squares of s[0..K) in the reference order, for the row handled by this 8-lane
// group of warp 0 (all 32 lanes participate; every 8-lane group gets its own row's sum)
__device__ __forceinline__ float chain8(const float* s, int K) {
  const int j = threadIdx.x & 7;
  const int n8 = K >> 3;
  float acc = 0.0f;
#pragma unroll 8
  for (int i = 0; i < n8; ++i) {
    const float v = s[8 * i + j];
    acc = __fmaf_rn(v, v, acc);
  }
  float sum = hsum8_lanes(acc, 0xffffffffu);
  for (int c = n8 * 8; c < K; ++c) sum = __fadd_rn(sum, __fmul_rn(s[c], s[c]));
  return sum;
}

}  // namespace

template <int MT, int NP, int NW, int PRO, int EPI>
__global__ void __launch_bounds__(kDecThreads) dec_kernel(DecArgs a) {
  extern __shared__ __align__(16) unsigned char dsm[];
  const int K = a.K, M = a.M, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t kc = packed_chunks(K), kp = kc * kChunkK;
  const int K4 = (K + 3) & ~3;
  float* xs = reinterpret_cast<float*>(dsm);                                   // [MT][K4]
  int8_t* pl = reinterpret_cast<int8_t*>(dsm + static_cast<size_t>(MT) * K4 * 4);  // [NP][MT][2][kp]
  uint32_t* red = reinterpret_cast<uint32_t*>(pl + static_cast<size_t>(NP) * MT * 2 * kp);
  __shared__ float s_r[MT];
  __shared__ int s_rowsum[NP][MT];
  __shared__ int s_red[kDecWarps];

  // ---- units of this CTA: a 32-row group, or for SwiGLU the pair (g, g + I/32)
  const int ngroups = static_cast<int>(packed_groups(a.N));
  const int units = EPI == kDecEpiSwiglu ? ngroups / 2 : ngroups;
  const int half = ngroups / 2;  // SwiGLU: I/32 (the launcher requires I % 32 == 0)

  // ---- 1. warm L2 with this CTA's weights (independent of the predecessor kernel)
  if (tid == 0) {
    const uint32_t gbytes = static_cast<uint32_t>(kc * kChunkBytes);
    for (int u = blockIdx.x; u < units; u += gridDim.x)
      for (int j = 0; j < NW; ++j) {
        const int g = EPI == kDecEpiSwiglu ? u + j * half : u;
        const void* wj = EPI == kDecEpiSwiglu ? a.w[0] : a.w[j];
        prefetch_l2(static_cast<const unsigned char*>(wj) + static_cast<int64_t>(g) * gbytes, gbytes);
      }
  }
  // ---- 2. the predecessor's outputs are needed from here on
  grid_dep_wait();
  grid_dep_launch();

  // ---- 3. prologue: rows into shared memory, exact norms, Q5.10 byte planes
  for (int t = 0; t < MT; ++t) {
    const int tr = t < M ? t : M - 1;
    for (int c = tid; c < K; c += kDecThreads) xs[t * K4 + c] = a.x[static_cast<int64_t>(tr) * K + c];
  }
  __syncthreads();
  const int myrow = (lane >> 3) < MT ? (lane >> 3) : MT - 1;  // warp 0: 8 lanes per row
  if (PRO != kDecProPlain) {
    if (warp == 0) {
      const float r = rstd_of(chain8(xs + myrow * K4, K), static_cast<float>(K), a.eps);
      if ((lane & 7) == 0 && (lane >> 3) < MT) s_r[lane >> 3] = r;
    }
    __syncthreads();
    for (int t = 0; t < MT; ++t) {
      const float r1 = s_r[t];
      const int tr = t < M ? t : M - 1;
      for (int c = tid; c < K; c += kDecThreads) {
        float v = norm_x(xs[t * K4 + c], r1, a.prew[c]);
        if (PRO == kDecProSwish) v = __fmul_rn(v, silu_x(a.o[static_cast<int64_t>(tr) * K + c], in_body(c, K)));
        xs[t * K4 + c] = v;
      }
    }
    __syncthreads();
  }
  if (warp == 0) {
    const float r = rstd_of(chain8(xs + myrow * K4, K), static_cast<float>(K), a.eps);
    if ((lane & 7) == 0 && (lane >> 3) < MT) s_r[lane >> 3] = r;
  }
  __syncthreads();
  for (int j = 0; j < NP; ++j)
    for (int t = 0; t < MT; ++t) {
      const float r2 = s_r[t];
      int local = 0;
      int8_t* hi = pl + (static_cast<int64_t>(j) * MT + t) * 2 * kp;
      int8_t* lo = hi + kp;
      for (int c = tid; c < kp; c += kDecThreads) {
        int32_t q = 0;
        if (c < K) q = quant_x(norm_x(xs[t * K4 + c], r2, a.normw[j][c]), a.qs, in_body(c, K));
        local += q;
        hi[c] = static_cast<int8_t>(q >> 8);
        lo[c] = static_cast<int8_t>(q & 0xff);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
      if (lane == 0) s_red[warp] = local;
      __syncthreads();
      if (tid == 0) {
        int tot = 0;
        for (int w = 0; w < kDecWarps; ++w) tot += s_red[w];
        s_rowsum[j][t] = tot;
      }
      __syncthreads();
    }

  // ---- 4. matmul over this CTA's units; lane = output row, warps split the k-chunks
  float best_v[MT];
  int best_i[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) { best_v[t] = -FLT_MAX; best_i[t] = 0x7fffffff; }

  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    int acc_hi[NW][MT][4], acc_lo[NW][MT][4];
#pragma unroll
    for (int j = 0; j < NW; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc_hi[j][t][q] = acc_lo[j][t][q] = 0;
    for (int64_t c = warp; c < kc; c += kDecWarps) {
      uint4 wv[NW];
#pragma unroll
      for (int j = 0; j < NW; ++j) {
        const int g = EPI == kDecEpiSwiglu ? u + j * half : u;
        const void* wj = EPI == kDecEpiSwiglu ? a.w[0] : a.w[j];
        wv[j] = __ldg(static_cast<const uint4*>(wj) + (static_cast<int64_t>(g) * kc + c) * 32 + lane);
      }
#pragma unroll
      for (int j = 0; j < NW; ++j) {
        const int pj = NP == 1 ? 0 : j;
        const uint32_t wd[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const uint4* hp = reinterpret_cast<const uint4*>(pl + ((static_cast<int64_t>(pj) * MT + t) * 2) * kp + c * kChunkK);
          const uint4* lp = reinterpret_cast<const uint4*>(reinterpret_cast<const int8_t*>(hp) + kp);
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            const uint4 h = hp[w4], l = lp[w4];
            const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t mw = wd[w4] & (0x03030303u << (2 * q));
              acc_hi[j][t][q] = dp4a_us(mw, hw[q], acc_hi[j][t][q]);
              acc_lo[j][t][q] = dp4a_uu(mw, lw[q], acc_lo[j][t][q]);
            }
          }
        }
      }
    }
    // combine the 4 byte-shift groups, then the warps, in shared memory
#pragma unroll
    for (int j = 0; j < NW; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        uint32_t v = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v += static_cast<uint32_t>(acc_hi[j][t][q] >> (2 * q)) << 8;
          v += static_cast<uint32_t>(acc_lo[j][t][q] >> (2 * q));
        }
        red[((warp * NW + j) * MT + t) * 32 + lane] = v;
      }
    __syncthreads();
    if (warp == 0) {
      int32_t acc[NW][MT];
#pragma unroll
      for (int j = 0; j < NW; ++j)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          uint32_t v = 0;
          for (int w = 0; w < kDecWarps; ++w) v += red[((w * NW + j) * MT + t) * 32 + lane];
          acc[j][t] = static_cast<int32_t>(v - static_cast<uint32_t>(s_rowsum[NP == 1 ? 0 : j][t]));
        }
      const int n = u * 32 + lane;  // output column (first group of the unit)
      for (int t = 0; t < M && t < MT; ++t) {
        if (EPI == kDecEpiMixer) {
          if (n < a.N) {
            const float iv = __fmul_rn(__int2float_rn(acc[0][t]), a.scale[0]);
            const float fr = __fmul_rn(__int2float_rn(acc[NW > 1 ? 1 : 0][t]), a.scale[NW > 1 ? 1 : 0]);
            const float gv = __fmul_rn(__int2float_rn(acc[NW > 2 ? 2 : 0][t]), a.scale[NW > 2 ? 2 : 0]);
            const int64_t e = static_cast<int64_t>(t) * a.N + n;
            const bool body = in_body(e % a.seg, a.seg);
            float fv = sigmoid_x(fr, body);
            if (a.lb) fv = lower_bound_x(fv, a.lb[n]);
            const float sv = swiglu_x(iv, __fadd_rn(1.0f, -fv), body);
            const float st = hgrn_step_x(fv, a.state[e], sv);
            a.state[e] = st;
            a.out[0][e] = st;  // recurrence output
            a.out[1][e] = gv;  // g_proj output (normed by K2)
          }
        } else if (EPI == kDecEpiResid) {
          if (n < a.N) {
            const int64_t e = static_cast<int64_t>(t) * a.N + n;
            a.out[0][e] = __fadd_rn(a.resid[e], __fmul_rn(__int2float_rn(acc[0][t]), a.scale[0]));
          }
        } else if (EPI == kDecEpiSwiglu) {
          const int I = a.N / 2;
          if (n < I) {
            const float ya = __fmul_rn(__int2float_rn(acc[0][t]), a.scale[0]);
            const float yb = __fmul_rn(__int2float_rn(acc[NW > 1 ? 1 : 0][t]), a.scale[0]);
            const int64_t e = static_cast<int64_t>(t) * I + n;
            a.out[0][e] = swiglu_x(ya, yb, in_body(e % a.seg, a.seg));
          }
        } else {  // logits (+ greedy argmax)
          if (n < a.N) {
            const float v = __fmul_rn(__int2float_rn(acc[0][t]), a.scale[0]);
            if (a.out[0]) a.out[0][static_cast<int64_t>(t) * a.N + n] = v;
            if (v > best_v[t] || (v == best_v[t] && n < best_i[t])) { best_v[t] = v; best_i[t] = n; }
          }
        }
      }
    }
    __syncthreads();
  }

  if (EPI == kDecEpiLogits && a.ids) {
    // CTA partial argmax (warp 0 holds the candidates), then the last CTA reduces them all
    __shared__ unsigned s_last;
    if (warp == 0) {
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        float bv = best_v[t];
        int bi = best_i[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
          a.part_v[static_cast<int64_t>(blockIdx.x) * MT + t] = bv;
          a.part_i[static_cast<int64_t>(blockIdx.x) * MT + t] = bi;
        }
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_last && warp == 0) {
      __threadfence();
      const int64_t p = *a.pos;
      for (int t = 0; t < M && t < MT; ++t) {
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;
        for (int c = lane; c < static_cast<int>(gridDim.x); c += 32) {
          const float ov = __ldcg(a.part_v + static_cast<int64_t>(c) * MT + t);
          const int oi = __ldcg(a.part_i + static_cast<int64_t>(c) * MT + t);
          if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        // the reference scan (hgrn_model.cpp:271-273) starts from index 0 and never moves
        // away from a NaN there; NaNs elsewhere never win (NaN comparisons are false)
        const float l0 = __ldcg(a.out[0] + static_cast<int64_t>(t) * a.N);
        if (lane == 0) a.ids[t * a.stride + p + 1] = isnan(l0) ? 0 : (bv == -FLT_MAX && bi == 0x7fffffff ? 0 : bi);
      }
      if (lane == 0) {
        *a.done = 0;
        *a.pos = p + 1;
      }
    }
  }
}

template <int MT, int NP, int NW, int PRO, int EPI>
static cudaError_t launch_dec_t(const DecArgs& a, int grid, cudaStream_t s, bool pdl) {
  const int64_t kp = padded_k(a.K);
  const int K4 = (a.K + 3) & ~3;
  const size_t smem = static_cast<size_t>(MT) * K4 * 4 + static_cast<size_t>(NP) * MT * 2 * kp +
                      static_cast<size_t>(kDecWarps) * NW * MT * 32 * 4;
  if (smem > 224 * 1024) return cudaErrorInvalidValue;
  // the opt-in limit covers static + dynamic shared memory: raise it to what this launch needs
  static size_t attr[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && smem > attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(dec_kernel<MT, NP, NW, PRO, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr[dev & 63] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, dec_kernel<MT, NP, NW, PRO, EPI>, a);
}

// units of work and a grid of at most two CTAs per SM
int dec_units(const DecArgs& a, int epi) {
  const int ng = static_cast<int>(packed_groups(a.N));
  return epi == kDecEpiSwiglu ? ng / 2 : ng;
}

template <int MT>
static cudaError_t launch_dec_mt(const DecArgs& a, int pro, int epi, int grid, cudaStream_t s,
                                 bool pdl) {
  if (epi == kDecEpiMixer) return launch_dec_t<MT, 3, 3, kDecProNorm2, kDecEpiMixer>(a, grid, s, pdl);
  if (epi == kDecEpiSwiglu) return launch_dec_t<MT, 1, 2, kDecProNorm2, kDecEpiSwiglu>(a, grid, s, pdl);
  if (epi == kDecEpiLogits) return launch_dec_t<MT, 1, 1, kDecProNorm2, kDecEpiLogits>(a, grid, s, pdl);
  if (pro == kDecProSwish) return launch_dec_t<MT, 1, 1, kDecProSwish, kDecEpiResid>(a, grid, s, pdl);
  return launch_dec_t<MT, 1, 1, kDecProPlain, kDecEpiResid>(a, grid, s, pdl);
}

cudaError_t launch_dec(const DecArgs& a, int pro, int epi, int grid, cudaStream_t s, bool pdl) {
  if (a.M <= 0) return cudaSuccess;
  if (a.M == 1) return launch_dec_mt<1>(a, pro, epi, grid, s, pdl);
  if (a.M == 2) return launch_dec_mt<2>(a, pro, epi, grid, s, pdl);
  if (a.M <= 4) return launch_dec_mt<4>(a, pro, epi, grid, s, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace mmfree_cuda
