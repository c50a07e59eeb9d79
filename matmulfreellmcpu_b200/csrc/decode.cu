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
// Two drivers run the same phase body (dec_body):
//   dec_kernel          one launch per phase, as a programmatic dependent of the previous
//                       launch. Everything a phase needs that its predecessor does not produce
//                       -- the weights of its first unit (bulk-copied into shared memory), its
//                       norm weights, the lower bounds and recurrent state of its columns, an L2
//                       prefetch of its other weights -- is fetched before griddepcontrol.wait;
//                       after the wait only the activation rows are read.
//   dec_persist_kernel  the whole decode step (every layer's four phases and the head) in one
//                       cooperative launch of one CTA per SM. Between phases a split grid
//                       barrier: a CTA arrives when its part of phase p is written and waits
//                       for all arrivals only after staging phase p+1's weights, so the staging
//                       overlaps the other CTAs' tail of phase p. Each phase also starts an L2
//                       prefetch of the next phase's weights. Data written inside the launch is
//                       read through L2 only (ld.global.cg): the L1 caches of other SMs are not
//                       coherent with it.
#include "common.cuh"
#include "exact.cuh"
#include "kernels.h"

#include <cfloat>

namespace mmfree_cuda {

namespace {

// threads per CTA: one stream keeps few registers per thread, so it gets twice the warps for
// the elementwise prologue and the k-split of the matmul
__host__ __device__ constexpr int dec_threads(int MT) { return MT == 1 ? 512 : 256; }

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

constexpr uint32_t kStageSpin = 1u << 24;  // bounded wait for the staged weights
constexpr uint32_t kBarSpin = 1u << 22;    // bounded wait at a grid barrier (a phase takes microseconds)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// bulk global -> shared copy completing on an mbarrier (no multicast)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Copies NA float arrays of K elements (those with a non-null source) from global into
// shared memory. Each thread issues the loads of a whole batch (kB elements of every array)
// before its first store, so one memory latency covers the batch. CG: read through L2 only
// (data written earlier in the same launch); otherwise the read-only path (constants).
template <int kB, int NA, bool CG, int kThr>
__device__ __forceinline__ void load_arrays(float* const (&dst)[NA], const float* const (&src)[NA], int K) {
  for (int c0 = threadIdx.x; c0 < K; c0 += kB * kThr) {
    float v[NA][kB];
#pragma unroll
    for (int s = 0; s < NA; ++s)
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int c = c0 + i * kThr;
        v[s][i] = (src[s] != nullptr && c < K) ? (CG ? __ldcg(src[s] + c) : __ldg(src[s] + c)) : 0.0f;
      }
#pragma unroll
    for (int s = 0; s < NA; ++s)
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int c = c0 + i * kThr;
        if (src[s] != nullptr && c < K) dst[s][c] = v[s][i];
      }
  }
}

}  // namespace

// L2 prefetch of the weights a CTA will read in phase n
__device__ __forceinline__ void prefetch_phase(const DecArgs& n, int cta, int ncta) {
  const int64_t kc = packed_chunks(n.K);
  const uint32_t gbytes = static_cast<uint32_t>(kc * kChunkBytes);
  const int ngroups = static_cast<int>(packed_groups(n.N));
  const bool pair = n.epi == kDecEpiSwiglu;
  const int units = pair ? ngroups / 2 : ngroups;
  const int nw = n.epi == kDecEpiMixer ? 3 : (pair ? 2 : 1);
  for (int u = cta; u < units; u += ncta)
    for (int j = 0; j < nw; ++j) {
      const int g = pair ? u + j * (ngroups / 2) : u;
      const void* wj = pair ? n.w[0] : n.w[j];
      prefetch_l2(static_cast<const unsigned char*>(wj) + static_cast<int64_t>(g) * gbytes, gbytes);
    }
}

// One phase for CTA `cta` of `ncta`: units cta, cta + ncta, ... `wait` is called by every
// thread once the phase's constants are staged; it returns false when the step must stop.
// Returns false when it stopped.
template <int MT, int NP, int NW, int PRO, int EPI, bool FL, class Wait>
__device__ __forceinline__ bool dec_body(const DecArgs& a, int cta, int ncta, unsigned char* dsm,
                                         const DecArgs* next, Wait&& wait) {
  constexpr int kDecThreads = dec_threads(MT), kDecWarps = kDecThreads / 32;
  const int K = a.K, M = a.M, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t kc = packed_chunks(K), kp = kc * kChunkK;
  const int K4 = (K + 3) & ~3;
  constexpr int kNorms = (PRO == kDecProPlain ? 0 : 1) + NP;  // prew + projection norms
  constexpr int kRows = PRO == kDecProSwish ? 2 * MT : MT;    // x rows (+ gate operand rows)
  float* xs = reinterpret_cast<float*>(dsm);                              // [MT][K4]
  float* os = xs + static_cast<size_t>(MT) * K4;                          // [MT][K4] (Swish)
  float* nws = xs + static_cast<size_t>(kRows) * K4;                      // [kNorms][K4]
  // FixedQ510: Q5.10 byte planes [NP][MT][2][kp]; Float: normalised activations [NP][MT][kp]
  int8_t* pl = reinterpret_cast<int8_t*>(nws + static_cast<size_t>(kNorms) * K4);
  float* yf = reinterpret_cast<float*>(pl);
  uint32_t* red = reinterpret_cast<uint32_t*>(pl + static_cast<size_t>(NP) * MT * (FL ? 4 : 2) * kp);
  __shared__ float s_r[MT];
  __shared__ int s_rowsum[NP][MT];

  // units of this CTA: a 32-row group, or for SwiGLU the pair (g, g + I/32)
  const int ngroups = static_cast<int>(packed_groups(a.N));
  const int units = EPI == kDecEpiSwiglu ? ngroups / 2 : ngroups;
  const int half = ngroups / 2;  // SwiGLU: I/32 (the launcher requires I % 32 == 0)
  auto wrow = [&](int u, int j) -> const uint4* {
    const int g = EPI == kDecEpiSwiglu ? u + j * half : u;
    const void* wj = EPI == kDecEpiSwiglu ? a.w[0] : a.w[j];
    return static_cast<const uint4*>(wj) + static_cast<int64_t>(g) * kc * 32 + lane;
  };

  // ---- 1. independent of the predecessor: first-unit weights (bulk copy into shared memory),
  //         L2 prefetch of the other units, norm weights, lower bounds and state
  const int u0 = cta;
  const bool stage = a.stage && u0 < units;
  uint4* wst = reinterpret_cast<uint4*>(red + kDecWarps * NW * MT * 32);  // [NW][kc][32] uint4
  __shared__ __align__(8) uint64_t s_bar;
  if (tid == 0) {
    const uint32_t gbytes = static_cast<uint32_t>(kc * kChunkBytes);
    if (stage) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&s_bar)));
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&s_bar)),
                   "r"(gbytes * NW)
                   : "memory");
      for (int j = 0; j < NW; ++j) bulk_g2s(wst + j * kc * 32, wrow(u0, j) - lane, gbytes, &s_bar);
    } else if (u0 < units) {
      for (int j = 0; j < NW; ++j) prefetch_l2(wrow(u0, j) - lane, gbytes);
    }
    for (int u = u0 + ncta; u < units; u += ncta)
      for (int j = 0; j < NW; ++j) prefetch_l2(wrow(u, j) - lane, gbytes);
    if (next) prefetch_phase(*next, cta, ncta);
  }
  {  // norm weights (one batch of loads)
    constexpr int s0 = PRO == kDecProPlain ? 0 : 1;
    float* const dst[4] = {nws, nws + s0 * K4, nws + (s0 + 1) * K4, nws + (s0 + 2) * K4};
    const float* const src[4] = {PRO == kDecProPlain ? nullptr : a.prew, a.normw[0],
                                 NP > 1 ? a.normw[1] : nullptr, NP > 2 ? a.normw[2] : nullptr};
    if (PRO == kDecProPlain) {
      float* const d1[4] = {dst[1], nullptr, nullptr, nullptr};
      const float* const s1[4] = {a.normw[0], nullptr, nullptr, nullptr};
      load_arrays<8, 4, false, kDecThreads>(d1, s1, K);
    } else {
      load_arrays<8, 4, false, kDecThreads>(dst, src, K);
    }
  }
  float lb_pre = 0.0f, st_pre[MT];
  if (EPI == kDecEpiMixer && warp == 0 && u0 < units) {
    const int n = u0 * 32 + lane;
    if (n < a.N) {
      if (a.lb) lb_pre = __ldg(a.lb + n);
#pragma unroll
      for (int t = 0; t < MT; ++t) st_pre[t] = t < M ? __ldcg(a.state + static_cast<int64_t>(t) * a.N + n) : 0.0f;
    }
  }

  // ---- 2. the predecessor's outputs are needed from here on
  if (!wait()) {
    if (stage)  // let the staged copy land before the CTA moves on
      for (uint32_t i = 0; i < kStageSpin && !mbar_test(&s_bar, 0); ++i) {
      }
    return false;
  }

  // ---- 3. prologue: rows into shared memory (or gathered from the embedding table), exact
  //         norms, Q5.10 byte planes
  {
    float* dst[2 * MT];
    const float* src[2 * MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int tr = t < M ? t : M - 1;
      const float* xr = a.x + static_cast<int64_t>(tr) * K;
      if (a.xids) {  // the step's first phase: x = embedding row of the current token
        const int64_t id = a.xids[tr * a.xstride + *a.xpos];
        const bool ok = id >= 0 && id < a.V;
        if (!ok && tid == 0 && a.err) atomicOr(a.err, kErrBadToken);
        xr = ok ? a.x + id * K : nullptr;
      }
      dst[t] = xs + t * K4;
      src[t] = xr;
      dst[MT + t] = os + t * K4;
      src[MT + t] = PRO == kDecProSwish ? a.o + static_cast<int64_t>(tr) * K : nullptr;
    }
    load_arrays<MT == 1 ? 16 : 8, 2 * MT, true, kDecThreads>(dst, src, K);
#pragma unroll
    for (int t = 0; t < MT; ++t)  // a bad id gives a zero row
      if (src[t] == nullptr)
        for (int c = tid; c < K; c += kDecThreads) xs[t * K4 + c] = 0.0f;
  }
  __syncthreads();
  if (a.xcopy && cta == 0)
    for (int t = 0; t < M && t < MT; ++t)
      for (int c = tid; c < K; c += kDecThreads) a.xcopy[static_cast<int64_t>(t) * K + c] = xs[t * K4 + c];
  const int myrow = (lane >> 3) < MT ? (lane >> 3) : MT - 1;  // warp 0: 8 lanes per row
  const float* nproj = nws + (PRO == kDecProPlain ? 0 : K4);    // projection norm weights
  // rstd of every row into s_r (a __syncthreads must follow): FixedQ510 in the reference's
  // serial 8-chain order on warp 0 (bit-exact); Float as a block-parallel sum, which
  // re-associates the row's sum of squares within the Float tolerance
  __shared__ float s_part[kDecWarps][MT];
  auto row_rstd = [&] {
    if (FL) {
      float part[MT];
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        part[t] = 0.0f;
        for (int c = tid; c < K; c += kDecThreads) part[t] = __fmaf_rn(xs[t * K4 + c], xs[t * K4 + c], part[t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part[t] += __shfl_xor_sync(0xffffffffu, part[t], o);
        if (lane == 0) s_part[warp][t] = part[t];
      }
      __syncthreads();
      if (tid < MT) {
        float s = 0.0f;
        for (int w = 0; w < kDecWarps; ++w) s += s_part[w][tid];
        s_r[tid] = rstd_of(s, static_cast<float>(K), a.eps);
      }
    } else if (warp == 0) {
      const float r = rstd_of(sumsq_exact8(xs + myrow * K4, K, 0xffffffffu), static_cast<float>(K), a.eps);
      if ((lane & 7) == 0 && (lane >> 3) < MT) s_r[lane >> 3] = r;
    }
  };
  if (PRO != kDecProPlain) {
    row_rstd();
    __syncthreads();
    for (int t = 0; t < MT; ++t) {
      const float r1 = s_r[t];
      for (int c = tid; c < K; c += kDecThreads) {
        float v = norm_x(xs[t * K4 + c], r1, nws[c]);
        if (PRO == kDecProSwish) v = __fmul_rn(v, silu_x(os[t * K4 + c], in_body(c, K)));
        xs[t * K4 + c] = v;
      }
    }
    __syncthreads();
  }
  row_rstd();
  __syncthreads();
  {
    int local[NP][MT];
#pragma unroll
    for (int j = 0; j < NP; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t) local[j][t] = 0;
    // 4 consecutive k per step: vector loads, one 4-byte store per plane
    for (int c4 = tid * 4; FL && c4 < kp; c4 += kDecThreads * 4) {  // Float: y in fp32 (bitlinear.cpp:95-105)
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const float4 xv4 = c4 < K ? *reinterpret_cast<const float4*>(xs + t * K4 + c4) : make_float4(0, 0, 0, 0);
        const float xv[4] = {xv4.x, xv4.y, xv4.z, xv4.w};
        const float r2 = s_r[t];
#pragma unroll
        for (int j = 0; j < NP; ++j) {
          const float4 w4 = c4 < K ? *reinterpret_cast<const float4*>(nproj + j * K4 + c4) : make_float4(0, 0, 0, 0);
          const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
          float y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) y[e] = c4 + e < K ? norm_x(xv[e], r2, wv[e]) : 0.0f;
          *reinterpret_cast<float4*>(yf + (static_cast<int64_t>(j) * MT + t) * kp + c4) =
              make_float4(y[0], y[1], y[2], y[3]);
        }
      }
    }
    for (int c4 = tid * 4; !FL && c4 < kp; c4 += kDecThreads * 4) {
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const float4 xv4 = c4 < K ? *reinterpret_cast<const float4*>(xs + t * K4 + c4) : make_float4(0, 0, 0, 0);
        const float xv[4] = {xv4.x, xv4.y, xv4.z, xv4.w};
        const float r2 = s_r[t];
#pragma unroll
        for (int j = 0; j < NP; ++j) {
          const float4 w4 = c4 < K ? *reinterpret_cast<const float4*>(nproj + j * K4 + c4) : make_float4(0, 0, 0, 0);
          const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
          uint32_t hw = 0, lw = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = c4 + e;
            const int32_t q = c < K ? quant_x(norm_x(xv[e], r2, wv[e]), a.qs, in_body(c, K)) : 0;
            local[j][t] += q;
            hw |= static_cast<uint32_t>((q >> 8) & 0xff) << (8 * e);
            lw |= static_cast<uint32_t>(q & 0xff) << (8 * e);
          }
          int8_t* hi = pl + (static_cast<int64_t>(j) * MT + t) * 2 * kp;
          *reinterpret_cast<uint32_t*>(hi + c4) = hw;
          *reinterpret_cast<uint32_t*>(hi + kp + c4) = lw;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NP; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        int v = local[j][t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[(j * MT + t) * kDecWarps + warp] = static_cast<uint32_t>(v);
      }
    __syncthreads();
    if (tid < NP * MT) {
      int tot = 0;
      for (int w = 0; w < kDecWarps; ++w) tot += static_cast<int>(red[tid * kDecWarps + w]);
      s_rowsum[tid / MT][tid % MT] = tot;
    }
    __syncthreads();
  }

  // ---- 4. matmul over this CTA's units; lane = output row, warps split the k-chunks
  float best_v[MT];
  int best_i[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) { best_v[t] = -FLT_MAX; best_i[t] = 0x7fffffff; }

  for (int u = u0; u < units; u += ncta) {
    int acc_hi[NW][MT][4], acc_lo[NW][MT][4];
    float accf[NW][MT];  // Float: sum of y * w (order free within the mode's tolerance)
#pragma unroll
    for (int j = 0; j < NW; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        accf[j][t] = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) acc_hi[j][t][q] = acc_lo[j][t][q] = 0;
      }
    auto chunk = [&](const uint4 (&wv)[NW], int64_t c) {
#pragma unroll
      for (int j = 0; FL && j < NW; ++j) {
        const int pj = NP == 1 ? 0 : j;
        const uint32_t wd[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const float4* yp = reinterpret_cast<const float4*>(yf + (static_cast<int64_t>(pj) * MT + t) * kp + c * kChunkK);
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {  // k = 64c + 16 w4 + 4 g + jj at bit 8 jj + 2 g
            const float4 y0 = yp[4 * w4], y1 = yp[4 * w4 + 1], y2 = yp[4 * w4 + 2], y3 = yp[4 * w4 + 3];
            const float yv[16] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w,
                                  y2.x, y2.y, y2.z, y2.w, y3.x, y3.y, y3.z, y3.w};
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const uint32_t m = (wd[w4] >> (2 * g)) & 0x03030303u;  // byte jj: code of k 4g + jj
#pragma unroll
              for (int jj = 0; jj < 4; ++jj)
                accf[j][t] = __fmaf_rn(yv[4 * g + jj], ternary_f32(m, jj), accf[j][t]);
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; !FL && j < NW; ++j) {
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
    };
    bool from_smem = false;
    if (stage && u == u0) {  // the staged first unit (bounded wait; global loads if it times out)
      for (uint32_t i = 0; i < kStageSpin && !from_smem; ++i) from_smem = mbar_test(&s_bar, 0);
    }
    for (int64_t c = warp; c < kc; c += kDecWarps) {
      uint4 wv[NW];
#pragma unroll
      for (int j = 0; j < NW; ++j) wv[j] = from_smem ? wst[(j * kc + c) * 32 + lane] : __ldg(wrow(u, j) + c * 32);
      chunk(wv, c);
    }
    // combine the 4 byte-shift groups (FixedQ510), then the warps, in shared memory
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
        red[((warp * NW + j) * MT + t) * 32 + lane] = FL ? __float_as_uint(accf[j][t]) : v;
      }
    __syncthreads();
    if (warp == 0) {
      // dequantised outputs: acc * scale (FixedQ510: 1/(2^f scale_w), exact int32 acc;
      // Float: 1/scale_w); a SwiGLU unit's two halves share projection 0's scale
      float val[NW][MT];
#pragma unroll
      for (int j = 0; j < NW; ++j)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const float sc = a.scale[EPI == kDecEpiSwiglu ? 0 : j];
          if (FL) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kDecWarps; ++w) v += __uint_as_float(red[((w * NW + j) * MT + t) * 32 + lane]);
            val[j][t] = __fmul_rn(v, sc);
          } else {
            uint32_t v = 0;
#pragma unroll
            for (int w = 0; w < kDecWarps; ++w) v += red[((w * NW + j) * MT + t) * 32 + lane];
            val[j][t] = __fmul_rn(__int2float_rn(static_cast<int32_t>(v - static_cast<uint32_t>(
                                      s_rowsum[NP == 1 ? 0 : j][t]))), sc);
          }
        }
      const int n = u * 32 + lane;  // output column (first group of the unit)
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        if (t >= M) break;
        if (EPI == kDecEpiMixer) {
          if (n < a.N) {
            const float iv = val[0][t];
            const float fr = val[NW > 1 ? 1 : 0][t];
            const float gv = val[NW > 2 ? 2 : 0][t];
            const int64_t e = static_cast<int64_t>(t) * a.N + n;
            // seg is a whole number of N-element rows: only columns n >= N - seg % 8 of a
            // segment's last row are in the tail (the division runs for those alone)
            const bool body = n < a.N - static_cast<int>(a.seg & 7) || in_body(e % a.seg, a.seg);
            const bool first = u == u0;
            float fv = sigmoid_x(fr, body);
            if (a.lb) fv = lower_bound_x(fv, first ? lb_pre : __ldg(a.lb + n));
            const float sv = swiglu_x(iv, __fadd_rn(1.0f, -fv), body);
            const float st = hgrn_step_x(fv, first ? st_pre[t] : __ldcg(a.state + e), sv);
            a.state[e] = st;
            a.out[0][e] = st;  // recurrence output
            a.out[1][e] = gv;  // g_proj output (normed by K2)
          }
        } else if (EPI == kDecEpiResid) {
          if (n < a.N) {
            const int64_t e = static_cast<int64_t>(t) * a.N + n;
            a.out[0][e] = a.resid ? __fadd_rn(__ldcg(a.resid + e), val[0][t]) : val[0][t];
          }
        } else if (EPI == kDecEpiSwiglu) {
          const int I = a.N / 2;
          if (n < I) {
            const float ya = val[0][t];
            const float yb = val[NW > 1 ? 1 : 0][t];
            const int64_t e = static_cast<int64_t>(t) * I + n;
            const bool body = n < I - static_cast<int>(a.seg & 7) || in_body(e % a.seg, a.seg);  // (as above)
            a.out[0][e] = swiglu_x(ya, yb, body);
          }
        } else {  // logits (+ greedy argmax)
          if (n < a.N) {
            const float v = val[0][t];
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
          a.part_v[static_cast<int64_t>(cta) * MT + t] = bv;
          a.part_i[static_cast<int64_t>(cta) * MT + t] = bi;
        }
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.done, 1u) == static_cast<unsigned>(ncta) - 1;
    __syncthreads();
    if (s_last && warp == 0) {
      __threadfence();
      const int64_t p = *a.pos;
      for (int t = 0; t < M && t < MT; ++t) {
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;
        for (int c = lane; c < ncta; c += 32) {
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
        if (lane == 0)
          a.ids[t * a.stride + p + 1] = isnan(l0) ? 0 : (bi == 0x7fffffff ? 0 : bi);
      }
      if (lane == 0) {
        *a.done = 0;
        *a.pos = p + 1;
      }
    }
  }
  return true;
}

template <int MT, int NP, int NW, int PRO, int EPI, bool FL>
__global__ void __launch_bounds__(dec_threads(MT)) dec_kernel(DecArgs a) {
  extern __shared__ __align__(16) unsigned char dsm[];
  dec_body<MT, NP, NW, PRO, EPI, FL>(a, blockIdx.x, gridDim.x, dsm, nullptr, [] {
    grid_dep_wait();
    grid_dep_launch();
    return true;
  });
}

// The whole decode step in one cooperative launch (phase table in device memory).
template <int MT>
__global__ void __launch_bounds__(dec_threads(MT), 1) dec_persist_kernel(const DecArgs* __restrict__ phases,
                                                                     int nphases, unsigned* bar,
                                                                     uint32_t* err) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ unsigned s_ok;
  __shared__ DecArgs s_args[2];  // this phase's descriptor and the next one (copied ahead)
  constexpr int kWords = sizeof(DecArgs) / 16;
  const int cta = blockIdx.x, ncta = gridDim.x;
  auto fetch = [&](int ph) {  // asynchronous 16-byte copies, completed before the next phase
    if (threadIdx.x < kWords)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(
                       reinterpret_cast<const char*>(&s_args[ph & 1]) + 16 * threadIdx.x)),
                   "l"(reinterpret_cast<const char*>(phases + ph) + 16 * threadIdx.x)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  fetch(0);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  for (int ph = 0; ph < nphases; ++ph) {
    if (ph + 1 < nphases) fetch(ph + 1);
    const DecArgs& a = s_args[ph & 1];
    const DecArgs* next = ph + 1 < nphases ? &phases[ph + 1] : nullptr;
    // phase ph may start once every CTA has finished phase ph - 1
    auto wait = [&]() -> bool {
      if (ph == 0) return true;  // inputs come from earlier launches
      if (threadIdx.x == 0) {
        const unsigned target = static_cast<unsigned>(ncta) * static_cast<unsigned>(ph);
        unsigned v = 0;
        for (uint32_t i = 0; i < kBarSpin; ++i) {
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
          if (v >= target) break;
        }
        s_ok = v >= target;
        if (!s_ok && err) atomicOr(err, kErrTimeout);
        __threadfence();
      }
      __syncthreads();
      return s_ok != 0;
    };
    bool ok;
    if (a.epi == kDecEpiMixer)
      ok = dec_body<MT, 3, 3, kDecProNorm2, kDecEpiMixer, false>(a, cta, ncta, dsm, next, wait);
    else if (a.epi == kDecEpiSwiglu)
      ok = dec_body<MT, 1, 2, kDecProNorm2, kDecEpiSwiglu, false>(a, cta, ncta, dsm, next, wait);
    else if (a.epi == kDecEpiLogits)
      ok = dec_body<MT, 1, 1, kDecProNorm2, kDecEpiLogits, false>(a, cta, ncta, dsm, next, wait);
    else if (a.pro == kDecProSwish)
      ok = dec_body<MT, 1, 1, kDecProSwish, kDecEpiResid, false>(a, cta, ncta, dsm, next, wait);
    else
      ok = dec_body<MT, 1, 1, kDecProPlain, kDecEpiResid, false>(a, cta, ncta, dsm, next, wait);
    asm volatile("cp.async.wait_all;" ::: "memory");  // the next descriptor has landed
    if (!ok) return;  // a barrier timed out (error flag set): every CTA stops
    // arrive: this CTA's part of phase ph is written
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(bar, 1u);
    }
  }
}

constexpr size_t kDecSmemMax = 224 * 1024;

// Shared memory of one phase (rows, norm weights, planes, reduction) and of its staged unit.
struct DecSmem {
  size_t base, staged;
};
static DecSmem dec_smem(int K, int MT, int NP, int NW, int PRO, bool FL = false) {
  const int64_t kp = padded_k(K);
  const int K4 = (K + 3) & ~3;
  const int norms = (PRO == kDecProPlain ? 0 : 1) + NP;
  const int rows = PRO == kDecProSwish ? 2 * MT : MT;
  DecSmem d;
  d.base = static_cast<size_t>(rows + norms) * K4 * 4 + static_cast<size_t>(NP) * MT * (FL ? 4 : 2) * kp +
           static_cast<size_t>(dec_threads(MT) / 32) * NW * MT * 32 * 4;
  d.staged = static_cast<size_t>(NW) * kp / kChunkK * kChunkBytes;
  return d;
}
static void dec_shape(int pro, int epi, int* np, int* nw, int* pr) {
  if (epi == kDecEpiMixer) { *np = 3; *nw = 3; *pr = kDecProNorm2; }
  else if (epi == kDecEpiSwiglu) { *np = 1; *nw = 2; *pr = kDecProNorm2; }
  else if (epi == kDecEpiLogits) { *np = 1; *nw = 1; *pr = kDecProNorm2; }
  else { *np = 1; *nw = 1; *pr = pro == kDecProSwish ? kDecProSwish : kDecProPlain; }
}
static int dec_mt(int M) { return M == 1 ? 1 : (M == 2 ? 2 : 4); }

// raise a kernel's dynamic shared memory limit to `smem` (once per device and size)
template <class K>
static cudaError_t dec_smem_attr(K kernel, size_t smem, size_t (&cache)[64]) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && smem > cache[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cache[dev & 63] = smem;
  }
  return cudaSuccess;
}

template <int MT, int NP, int NW, int PRO, int EPI, bool FL>
static cudaError_t launch_dec_t(const DecArgs& a, int grid, cudaStream_t s, bool pdl) {
  const DecSmem d = dec_smem(a.K, MT, NP, NW, PRO, FL);
  if (d.base > kDecSmemMax) return cudaErrorInvalidValue;
  // stage the first unit's weights in shared memory when they fit
  DecArgs b = a;
  b.pro = PRO;
  b.epi = EPI;
  b.stage = d.base + d.staged <= kDecSmemMax ? 1 : 0;
  const size_t smem = d.base + (b.stage ? d.staged : 0);
  static size_t cache[64] = {0};
  cudaError_t e = dec_smem_attr(dec_kernel<MT, NP, NW, PRO, EPI, FL>, smem, cache);
  if (e != cudaSuccess) return e;
  return launch_k(dec_kernel<MT, NP, NW, PRO, EPI, FL>, dim3(static_cast<unsigned>(grid)), dim3(dec_threads(MT)),
                  smem, s, pdl, b);
}

// units of work (the launcher uses at most two CTAs per SM)
int dec_units(const DecArgs& a, int epi) {
  const int ng = static_cast<int>(packed_groups(a.N));
  return epi == kDecEpiSwiglu ? ng / 2 : ng;
}

template <int MT, bool FL>
static cudaError_t launch_dec_mf(const DecArgs& a, int pro, int epi, int grid, cudaStream_t s,
                                 bool pdl) {
  if (epi == kDecEpiMixer) return launch_dec_t<MT, 3, 3, kDecProNorm2, kDecEpiMixer, FL>(a, grid, s, pdl);
  if (epi == kDecEpiSwiglu) return launch_dec_t<MT, 1, 2, kDecProNorm2, kDecEpiSwiglu, FL>(a, grid, s, pdl);
  if (epi == kDecEpiLogits) return launch_dec_t<MT, 1, 1, kDecProNorm2, kDecEpiLogits, FL>(a, grid, s, pdl);
  if (pro == kDecProSwish) return launch_dec_t<MT, 1, 1, kDecProSwish, kDecEpiResid, FL>(a, grid, s, pdl);
  return launch_dec_t<MT, 1, 1, kDecProPlain, kDecEpiResid, FL>(a, grid, s, pdl);
}

template <int MT>
static cudaError_t launch_dec_mt(const DecArgs& a, int pro, int epi, int grid, cudaStream_t s,
                                 bool pdl) {
  return a.fl ? launch_dec_mf<MT, true>(a, pro, epi, grid, s, pdl)
              : launch_dec_mf<MT, false>(a, pro, epi, grid, s, pdl);
}

cudaError_t launch_dec(const DecArgs& a, int pro, int epi, int grid, cudaStream_t s, bool pdl) {
  if (a.M <= 0) return cudaSuccess;
  if (a.M == 1) return launch_dec_mt<1>(a, pro, epi, grid, s, pdl);
  if (a.M == 2) return launch_dec_mt<2>(a, pro, epi, grid, s, pdl);
  if (a.M <= 4) return launch_dec_mt<4>(a, pro, epi, grid, s, pdl);
  return cudaErrorInvalidValue;
}

// ---- persistent decode step

size_t dec_persist_plan(DecArgs* phases, int n) {
  if (n <= 0 || phases[0].fl) return 0;  // the persistent step is FixedQ510 only
  const int MT = dec_mt(phases[0].M);
  size_t need = 0;
  for (int i = 0; i < n; ++i) {  // rows, norms, planes of every phase must fit
    int np, nw, pr;
    dec_shape(phases[i].pro, phases[i].epi, &np, &nw, &pr);
    phases[i].pro = pr;
    const DecSmem d = dec_smem(phases[i].K, MT, np, nw, pr);
    if (d.base > kDecSmemMax || phases[i].M != phases[0].M) return 0;
    need = d.base > need ? d.base : need;
  }
  size_t smem = need;
  for (int i = 0; i < n; ++i) {  // stage first units where the largest phase leaves room
    int np, nw, pr;
    dec_shape(phases[i].pro, phases[i].epi, &np, &nw, &pr);
    const DecSmem d = dec_smem(phases[i].K, MT, np, nw, pr);
    phases[i].stage = d.base + d.staged <= kDecSmemMax ? 1 : 0;
    if (phases[i].stage && d.base + d.staged > smem) smem = d.base + d.staged;
  }
  return smem;
}

template <int MT>
static cudaError_t persist_mt(const DecArgs* dev_phases, int n, unsigned* bar, uint32_t* err,
                              size_t smem, int* grid, bool launch, cudaStream_t s) {
  static size_t cache[64] = {0};
  cudaError_t e = dec_smem_attr(dec_persist_kernel<MT>, smem, cache);
  if (e != cudaSuccess) return e;
  if (!launch) {  // one CTA per SM, all co-resident (the CTAs wait on one another)
    int dev = 0, sms = 0, coop = 0, per_sm = 0;
    cudaGetDevice(&dev);
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dec_persist_kernel<MT>, dec_threads(MT),
                                                           smem)) != cudaSuccess)
      return e;
    *grid = coop && per_sm >= 1 ? sms : 0;
    return cudaSuccess;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(*grid));
  cfg.blockDim = dim3(dec_threads(MT));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, dec_persist_kernel<MT>, dev_phases, n, bar, err);
}

static cudaError_t persist_dispatch(int M, const DecArgs* dev_phases, int n, unsigned* bar,
                                    uint32_t* err, size_t smem, int* grid, bool launch, cudaStream_t s) {
  switch (dec_mt(M)) {
    case 1: return persist_mt<1>(dev_phases, n, bar, err, smem, grid, launch, s);
    case 2: return persist_mt<2>(dev_phases, n, bar, err, smem, grid, launch, s);
    default: return persist_mt<4>(dev_phases, n, bar, err, smem, grid, launch, s);
  }
}

int dec_persist_grid(int M, size_t smem) {
  if (M < 1 || M > kDecMaxRows || smem == 0) return 0;
  int grid = 0;
  if (persist_dispatch(M, nullptr, 0, nullptr, nullptr, smem, &grid, false, nullptr) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return grid;
}

cudaError_t launch_dec_persist(const DecArgs* dev_phases, int nphases, int M, unsigned* bar,
                               uint32_t* err, size_t smem, int grid, cudaStream_t s) {
  if (grid <= 0 || nphases <= 0) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(bar, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return e;
  return persist_dispatch(M, dev_phases, nphases, bar, err, smem, &grid, true, s);
}

}  // namespace mmfree_cuda
