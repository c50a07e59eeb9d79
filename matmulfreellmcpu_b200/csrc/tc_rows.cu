// tc_rows.cu -- FixedQ510 BitLinear for thousands of token rows (prefill) on the tcgen05 tensor
// cores: a persistent kernel, one CTA per SM, that walks output tiles of 128 weight rows x 128
// tokens. The integer result is the one tc_matmul.cu and the reference's CpuBackend
// (ternary_backend.hpp:96-103) compute, so every output is bit-identical.
//
// Why a second kernel: with one 128 x 64 tile per CTA (tc_matmul.cu) a prefill BitLinear
// spends most of each CTA's life outside the MMAs (start-up, the epilogue, and half the SM's
// tensor memory idle while it drains). Here the epilogue of tile i overlaps the MMAs of tile
// i + 1 (two tensor-memory accumulators), and each expanded weight k-block feeds MMAs of
// N = 256 (128 tokens x both planes).
//
// Roles (20 warps):
//   warp 0      weight producer     one TMA copy per 128-k block of the tile's 4 packed 32-row
//                                   groups (two for a SwiGLU pair tile: 2 gate groups and their
//                                   2 up groups; L2 evict-last: every token tile reads them
//                                   again), 4-stage ring
//   warp 1      activation producer one TMA copy per 128-k block of both byte planes (high, and
//                                   low stored as lo - 128) of the 128 tokens, 4-stage ring
//   warp 2      MMA issuer          per 32 k one tcgen05.mma.kind::i8, A (u8 codes u = w + 1,
//                                   M = 128) and B (both planes, N = 256) from shared memory
//   warps 4-11  expanders           2-bit codes -> u8 rows of the A operand in shared memory
//                                   (K-major, 128-byte swizzle; a warp writes one chunk, 64 k,
//                                   of 32 rows) and the rows' code sums
//   warps 12-19 epilogue            tcgen05.ld of the finished accumulator, then
//                                   acc = 256*D_hi + D_lo' + 128*sum_k u - sum_k q (mod 2^32),
//                                   dequant and the residual, or the SwiGLU of a gate row with
//                                   its up row (a gate_proj tile's gate row i and up row i are
//                                   A rows 2i and 2i + 1, so neighbouring lanes hold a pair and
//                                   exchange by one shuffle)
// Every wait is bounded; on a timeout the CTA sets an error flag, the roles stop, producers
// wait (bounded) for their copies in flight, the MMAs are drained before tensor memory is freed.
#include "exact.cuh"
#include "tcgen05.cuh"

#include <cstdlib>

namespace mmfree_cuda {

namespace {

constexpr int kRThreads = 640;
constexpr int kRWWarp = 0, kRBWarp = 1, kRMmaWarp = 2, kRExp0 = 4, kREpi0 = 12;
constexpr int kRTok = 128;                           // tokens per tile
constexpr int kRWStages = 4, kRAStages = 3, kRBStages = 4;
constexpr int kRWBlock = 4 * 2 * kChunkBytes;        // 4 groups x 128 k of 2-bit codes: 4 KB
constexpr int kRAStage = 128 * 128;                  // the M = 128 operand, 128 k of u8: 16 KB
constexpr int kRBPlane = kRTok * 128;                // one plane, 128 tokens x 128 k
constexpr int kRBStage = 2 * kRBPlane;
constexpr int kRAOff = 0;
constexpr int kRBOff = kRAOff + kRAStages * kRAStage;
constexpr int kRWOff = kRBOff + kRBStages * kRBStage;
constexpr int kRBytes = kRWOff + kRWStages * kRWBlock;
constexpr int kRDyn = kRBytes + 1024;                // + alignment of the base to 1024 bytes
static_assert(kRDyn + 4096 <= 227 * 1024, "shared memory of one CTA");
// tensor memory: 2 accumulators x (128 high-plane token columns, then 128 low-plane ones)
constexpr int kRCols = 512;

// tcgen05.mma kind::i8 with both operands in shared memory
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// 8 TMEM columns of this warp's lanes, without the wait
__device__ __forceinline__ void tmem_ld8_nw(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// generic-proxy shared-memory writes -> visible to the tensor cores (async proxy)
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// tensor maps of a launch: the activation planes (3-D, both planes per box) and the packed
// weights (4-group boxes, or 2-group boxes for a SwiGLU pair) of each projection
struct RowsMaps {
  CUtensorMap act[3];
  CUtensorMap w[3];
};

struct RowsTiles {
  int ntn, nproj, ntok;
  __device__ int count() const { return ntn * nproj * ntok; }
};

}  // namespace

__global__ void __launch_bounds__(kRThreads, 1)
    tc_rows_kernel(const __grid_constant__ RowsMaps maps, const __grid_constant__ TcArgs p, RowsTiles T) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* ast = smem + kRAOff;  // [kRAStages][128 rows][128 B], swizzled
  unsigned char* bst = smem + kRBOff;  // [kRBStages][2 planes][128 rows][128 B], swizzled
  unsigned char* wst = smem + kRWOff;  // [kRWStages][4 groups][2 chunks][512 B]
  __shared__ uint64_t wfull[kRWStages], wempty[kRWStages], afull[kRAStages], aempty[kRAStages];
  __shared__ uint64_t bfull[kRBStages], bempty[kRBStages], dfull[2], dempty[2], sufull[2], mdone;
  __shared__ uint32_t s_su[2][2][128];  // code sums of the tile's 128 rows, per chunk half
  __shared__ uint32_t tmem_base_sh;
  __shared__ uint32_t s_fail;

  const MatmulArgs& a = p.m;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t kc = packed_chunks(a.K);
  const int nkb = static_cast<int>((kc + 1) / 2);
  const int ntiles = T.count();
  // tile t: token tile t / (nproj * ntn) (consecutive CTAs share activations in L2), then
  // projection and weight tile
  auto decode = [&](int t, int& tok0, int& proj, int& tn) {
    const int per = T.nproj * T.ntn;
    tok0 = (t / per) * kRTok;
    proj = (t % per) / T.ntn;
    tn = t % T.ntn;
  };

  if (tid == 0) {
    for (int s = 0; s < kRWStages; ++s) { mbar_init(&wfull[s], 1); mbar_init(&wempty[s], 8); }
    for (int s = 0; s < kRAStages; ++s) { mbar_init(&afull[s], 8); mbar_init(&aempty[s], 1); }
    for (int s = 0; s < kRBStages; ++s) { mbar_init(&bfull[s], 1); mbar_init(&bempty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&dfull[b], 1); mbar_init(&dempty[b], 8); mbar_init(&sufull[b], 8); }
    mbar_init(&mdone, 1);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // (no griddepcontrol.launch_dependents: see the launch below)
  }
  if (warp == kRMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"(kRCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kRBWarp && lane < T.nproj) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.act[lane])) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.w[lane])) : "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == kRWWarp) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_last();
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int tok0, proj, tn;
        decode(t, tok0, proj, tn);
        const CUtensorMap* wmap = &maps.w[proj];
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kRWStages;
          if (it == kRWStages) grid_dep_wait();  // the bounded waits exclude the predecessor
          if (it >= kRWStages && !role_wait(&wempty[s], ((it / kRWStages) - 1) & 1, &s_fail)) {
            ok = false;
            break;
          }
          // (groups past the rows and chunks past Kp arrive as zeros; whole boxes are counted)
          mbar_arrive_tx(&wfull[s], static_cast<uint32_t>(kRWBlock));
          unsigned char* dst = wst + s * kRWBlock;
          const int x = kb * (2 * kChunkBytes / 4);  // 32-bit words
          if (p.pair) {  // 2 gate groups, then their 2 up groups
            tma_load_2d_hint(dst, wmap, x, 2 * tn, &wfull[s], pol);
            tma_load_2d_hint(dst + 2 * 2 * kChunkBytes, wmap, x, p.pair + 2 * tn, &wfull[s], pol);
          } else {
            tma_load_2d_hint(dst, wmap, x, 4 * tn, &wfull[s], pol);
          }
        }
      }
      if (!ok) {  // note it, then let the copies already issued land
        atomicOr(&s_fail, 1u);
        for (int j = it - kRWStages > 0 ? it - kRWStages : 0; j < it; ++j)
          mbar_wait(&wfull[j % kRWStages], (j / kRWStages) & 1);
      }
    }
  } else if (warp == kRBWarp) {
    if (lane == 0) {
      grid_dep_wait();
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int tok0, proj, tn;
        decode(t, tok0, proj, tn);
        const CUtensorMap* bmap = &maps.act[proj];
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kRBStages;
          if (it >= kRBStages && !role_wait(&bempty[s], ((it / kRBStages) - 1) & 1, &s_fail)) {
            ok = false;
            break;
          }
          mbar_arrive_tx(&bfull[s], static_cast<uint32_t>(kRBStage));
          tma_load_3d(bst + s * kRBStage, bmap, kb * 128, tok0, 0, &bfull[s]);  // high rows, low rows
        }
      }
      if (!ok) {
        atomicOr(&s_fail, 1u);
        for (int j = it - kRBStages > 0 ? it - kRBStages : 0; j < it; ++j)
          mbar_wait(&bfull[j % kRBStages], (j / kRBStages) & 1);
      }
    }
  } else if (warp == kRMmaWarp) {
    if (lane == 0) {
      grid_dep_wait();
      constexpr uint32_t idesc = idesc_i8(true, 256);  // N = 128 high + 128 low token columns
      int it = 0, ti = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++ti) {
        const int b = ti & 1;
        if (ti >= 2 && !role_wait(&dempty[b], ((ti >> 1) - 1) & 1, &s_fail)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + static_cast<uint32_t>(b * 256);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int sa = it % kRAStages, sb = it % kRBStages;
          if (!role_wait(&afull[sa], (it / kRAStages) & 1, &s_fail) ||
              !role_wait(&bfull[sb], (it / kRBStages) & 1, &s_fail)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(ast + sa * kRAStage), b_base = smem_u32(bst + sb * kRBStage);
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // 32 k per MMA
            const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
            mma_i8_ss(d0, smem_desc_sw128(a_base + j * 32), smem_desc_sw128(b_base + j * 32), idesc, acc);
          }
          mma_commit(&aempty[sa]);
          mma_commit(&bempty[sb]);
        }
        if (ok) mma_commit(&dfull[b]);
      }
      if (!ok) atomicOr(&s_fail, 1u);
      // every MMA issued above has completed once this arrives
      mma_commit(&mdone);
      mbar_wait(&mdone, 0);
    }
  } else if (warp >= kRExp0 && warp < kREpi0) {
    // ---- expanders: warp 4 + 4h + e writes chunk h (k = 64h .. 64h + 63 of the block) of
    //      staged weight row 32e + lane (group e), as A row r: the same row, or in a SwiGLU
    //      pair tile (groups 0-1 gate rows i, groups 2-3 up rows i) row 2i resp. 2i + 1. Every
    //      decision is warp-uniform (the warp-wide syncs below need every lane)
    const int e8 = warp - kRExp0, hc = e8 >> 2, wr = 32 * (e8 & 3) + lane;
    const int r = p.pair ? 2 * (wr & 63) + (wr >> 6) : wr;
    int it = 0, ti = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++ti) {
      uint32_t su = 0u;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int sw = it % kRWStages, sa = it % kRAStages;
        if (!__all_sync(0xffffffffu, role_wait(&wfull[sw], (it / kRWStages) & 1, &s_fail))) {
          ok = false;
          break;
        }
        const uint4 wv =
            reinterpret_cast<const uint4*>(wst + sw * kRWBlock + (e8 & 3) * 2 * kChunkBytes + hc * kChunkBytes)[lane];
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[sw]);
        // code sums of the chunk when below Kp (past Kp the copy brought zeros: codes u = 0
        // there, where the activations are 0 too)
        if (2 * static_cast<int64_t>(kb) + hc < kc) {
          const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) su += __popc(wd[w4] & 0x55555555u) + 2u * __popc(wd[w4] & 0xAAAAAAAAu);
        }
        if (it >= kRAStages &&
            !__all_sync(0xffffffffu, role_wait(&aempty[sa], ((it / kRAStages) - 1) & 1, &s_fail))) {
          ok = false;
          break;
        }
        // row r: 16-byte piece q = 4 hc + w (k = 16q .. 16q + 15, word w of the chunk) at
        // (q ^ (r & 7)) * 16 in the row's 128 bytes (128-byte swizzle)
        {
          unsigned char* row = ast + sa * kRAStage + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t x = w == 0 ? wv.x : (w == 1 ? wv.y : (w == 2 ? wv.z : wv.w));
            const uint4 codes = make_uint4(x & 0x03030303u, (x >> 2) & 0x03030303u, (x >> 4) & 0x03030303u,
                                           (x >> 6) & 0x03030303u);
            *reinterpret_cast<uint4*>(row + (((4 * hc + w) ^ (r & 7)) << 4)) = codes;
          }
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[sa]);
      }
      if (!ok) break;
      // the tile's code sums (per chunk half); buffer ti & 1 was last read by the epilogue of
      // tile ti - 2, which released its accumulator before the MMAs of this tile began (at
      // least kRAStages + 1 k-blocks per tile, so the aempty waits above ordered this after that)
      const int b = ti & 1;
      s_su[b][hc][r] = su;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sufull[b]);
    }
    if (!ok) atomicOr(&s_fail, 1u);
  } else if (warp >= kREpi0) {
    // ---- epilogue: warp 12 + w reads TMEM lanes 32 (w % 4) .. + 31 (A rows; a warp reaches
    //      the lane quarter of its warp index mod 4) for tokens 64 (w / 4) .. + 63 of the tile,
    //      8 at a time. In a SwiGLU pair tile lane 2i holds gate row i and lane 2i + 1 its up
    //      row: the two swap values by one shuffle, the even lane finishes tokens 0-3 of the 8
    //      and the odd lane tokens 4-7.
    const int ew = warp - kREpi0, lq = ew & 3, half = ew >> 2;
    const int c = 32 * lq + lane;  // A row = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(32 * lq) << 16;
    const int I = p.pair * 32;
    const int side = c & 1;  // pair tiles: 0 gate, 1 up
    grid_dep_wait();  // row sums and residuals come from earlier kernels
    int ti = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++ti) {
      int tok0, proj, tn;
      decode(t, tok0, proj, tn);
      const TcProj& P = p.pj[proj];
      const int b = ti & 1;
      // (warp-uniform: tcgen05.ld is a warp-wide instruction)
      if (!__all_sync(0xffffffffu, role_wait(&dfull[b], (ti >> 1) & 1, &s_fail) &&
                                       role_wait(&sufull[b], (ti >> 1) & 1, &s_fail))) {
        atomicOr(&s_fail, 1u);
        break;
      }
      tc_fence_after();
      const uint32_t su = s_su[b][0][c] + s_su[b][1][c];
      // this thread's weight row: the output column (gate or plain row) and its raw index
      int64_t n, col;
      bool okn;
      if (p.pair) {
        col = 64 * static_cast<int64_t>(tn) + (c >> 1);  // gate row index = output column
        n = side ? I + col : col;
        okn = col < I;
      } else {
        n = col = 128 * static_cast<int64_t>(tn) + c;
        okn = n < a.N;
      }
      const bool tail_col = p.pair && col >= p.tail_from;
      const uint32_t dcol = tmem + static_cast<uint32_t>(b * 256) + lane_base;
#pragma unroll 1
      for (int g = 0; g < 8; ++g) {  // 8 tokens at a time
        const int j0 = 64 * half + 8 * g;
        const int64_t t0 = tok0 + j0;
        uint32_t v[8];
        {
          uint32_t hh[8], ll[8];
          tmem_ld8_nw(dcol + j0, hh);
          tmem_ld8_nw(dcol + 128 + j0, ll);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = (hh[j] << 8) + ll[j] + (su << 7);
        }
        if (g == 7) {  // the accumulator is free for the MMAs of tile ti + 2
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dempty[b]);
        }
        // every load of the group before its first store (an output may alias a residual)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] -= t0 + j < a.M ? static_cast<uint32_t>(__ldg(P.rowsum + t0 + j)) : 0u;
        if (a.acc_out) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (t0 + j < a.M && okn) a.acc_out[(t0 + j) * a.N + n] = static_cast<int32_t>(v[j]);
        }
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(__int2float_rn(static_cast<int32_t>(v[j])), P.scale);
        if (p.pair) {
          // the even lane keeps tokens 0-3 and sends 4-7; the odd lane keeps 4-7 and sends 0-3
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float send = side ? y[jj] : y[4 + jj];
            const float mine = side ? y[4 + jj] : y[jj];
            const float other = __shfl_xor_sync(0xffffffffu, send, 1);
            const int64_t tk = t0 + 4 * side + jj;
            const float gv = side ? other : mine, uv = side ? mine : other;
            // element (tk, col) is in the scalar tail of its segment only in the segment's last
            // row, at columns >= tail_from
            const bool body = !tail_col || (tk + 1) % p.seg_rows != 0;
            const float z = swiglu_x(gv, uv, body);
            if (tk < a.M && okn && P.out) P.out[tk * a.ldo + col] = z;
          }
        } else {
          float rv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) rv[j] = (a.resid && okn && t0 + j < a.M) ? a.resid[(t0 + j) * a.ldr + n] : 0.0f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (t0 + j >= a.M || !okn || !P.out) continue;
            P.out[(t0 + j) * a.ldo + n] = a.resid ? __fadd_rn(rv[j], y[j]) : y[j];
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (s_fail != 0 && tid == 0 && p.err) atomicOr(p.err, kErrTimeout);
  if (warp == kRMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kRCols) : "memory");
  }
}

// ---- host side

bool tc_rows_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("MMFREE_TC_ROWS");
    return !(e && std::atoi(e) == 0);
  }();
  return on;
}

// Tiles of the persistent kernel for this launch, or 0 where it does not apply: FixedQ510 and
// at least kRAStages + 1 k-blocks (128 k each) per tile
int64_t tc_rows_tiles(const MatmulArgs& a, int nproj, int pair) {
  if (!a.fixed || a.M <= 0) return 0;
  const int64_t nkb = (packed_chunks(a.K) + 1) / 2;
  if (nkb < kRAStages + 1) return 0;
  const int64_t ntn = pair ? ceil_div(static_cast<int64_t>(pair), 2) : ceil_div(a.N, 128);
  return ntn * nproj * ceil_div(a.M, kRTok);
}

cudaError_t launch_tc_rows(const TcArgs& p, const MatmulArgs* a, int sm_count, cudaStream_t s) {
  const MatmulArgs& m = p.m;
  const int64_t tiles = tc_rows_tiles(m, p.nproj, p.pair);
  if (tiles <= 0 || tiles > INT32_MAX || p.splits != 1 || sm_count < 1) return cudaErrorInvalidValue;
  RowsMaps maps;
  for (int j = 0; j < p.nproj; ++j) {
    cudaError_t e = planes_map3(&maps.act[j], a[j].planes, a[j].M, padded_k(a[j].K), kRTok);
    if (e == cudaSuccess) e = weights_map(&maps.w[j], a[j].w, a[j].N, a[j].K, p.pair ? 2 : 4);
    if (e != cudaSuccess) return e;
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(tc_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRDyn);
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  RowsTiles T;
  T.ntn = static_cast<int>(p.pair ? ceil_div(static_cast<int64_t>(p.pair), 2) : ceil_div(m.N, 128));
  T.nproj = p.nproj;
  T.ntok = static_cast<int>(ceil_div(m.M, kRTok));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tiles < sm_count ? tiles : sm_count));
  cfg.blockDim = dim3(kRThreads);
  cfg.dynamicSmemBytes = kRDyn;
  cfg.stream = s;
  // launched in plain stream order, not as a programmatic dependent, and launching none: its
  // CTAs all start after the previous kernel ends and the next kernel starts after it ends.
  // (Overlapping the neighbours' tails gave wrong ids in a few of 64 streams in some runs of a
  // prefill followed by decoding; the overlap is worth microseconds against a millisecond.)
  return cudaLaunchKernelEx(&cfg, tc_rows_kernel, maps, p, T);
}

}  // namespace mmfree_cuda
