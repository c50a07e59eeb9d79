// tc_matmul.cu -- FixedQ510 BitLinear matmul on the 5th-generation tensor cores (tcgen05).
//
// out[t, n] = dequant(sum_k w[n, k] * q[t, k]) for M activation rows (tokens) t and N output
// rows n, the same integer result as matmul_fixed_kernel (kernels.cu) and the reference's
// CpuBackend (ternary_backend.hpp:96-103), so every output is bit-identical.
//
// Per CTA: a tile of 128 weight rows (4 packed 32-row groups) x BN tokens, K in blocks of
// 128, split-K over blockIdx.z (the S CTAs of a tile form one thread-block cluster).
// Warp-specialised, every hand-off through an mbarrier ring:
//   warp 4  weight producer    one bulk async copy per group and k-block (the packed format
//                              keeps a group's chunks contiguous) into an 8-stage ring; the
//                              weights depend on no earlier kernel, so this runs ahead of
//                              griddepcontrol.wait and overlaps the predecessor kernel
//   warp 5  activation producer after griddepcontrol.wait, TMA (cp.async.bulk.tensor.2d)
//                              loads of the high-byte planes and the low-byte planes stored
//                              as lo - 128 (both s8) of the Q5.10 codes, BN rows x 128 B each
//                              per k-block, back to back: one 2*BN-row operand written with
//                              the 128-byte swizzle the MMA descriptor names
//   warps 0-3 expanders        warp w expands group w's 2-bit codes u = w + 1 to u8 and
//                              writes them to TENSOR MEMORY (lane = weight row, 4 codes per
//                              32-bit column) with tcgen05.st (a 4-stage TMEM ring), and
//                              sums its row's codes (popcount) for the low-plane offset
//   warp 6  MMA issuer         tcgen05.mma.cta_group::1.kind::i8 with A from TMEM, one
//                              instruction per 32 k for both planes: D[:, 0:BN] += u x hi,
//                              D[:, BN:2BN] += u x (lo - 128) (u8 x s8, M=128, N=2*BN),
//                              int32 accumulators in TMEM; tcgen05.commit releases the rings
//   epilogue (warps 0-3)       tcgen05.ld of D; acc = 256*D_hi + D_lo' + 128*sum_k u - sum_k q
//                              (exact modulo 2^32, hence in int32); with split-K each CTA
//                              leaves its partial tile in shared memory, and after a cluster
//                              barrier CTA r sums its BN/S tokens from every peer over
//                              distributed shared memory (integer sums: exact, order free) and
//                              applies dequant (+ residual, or the SwiGLU pair); a second
//                              barrier keeps the partials alive until every peer has read them.
// Every wait on an mbarrier is bounded; on timeout the CTA sets an error flag, the other roles
// stop, producers wait (bounded) for their copies in flight, the MMA issuer's final commit
// covers its MMAs, and the tensor memory is freed.
#include "exact.cuh"
#include "tcgen05.cuh"

#include <type_traits>
#include <cstdlib>

namespace mmfree_cuda {

namespace {

constexpr int kTcThreads = 224;      // 7 warps (roles above)
constexpr int kWWarp = 4, kBWarp = 5, kMmaWarp = 6;
constexpr int kWStages = 8;          // weight k-blocks in shared memory
constexpr int kBStages1 = 4;         // activation k-blocks in shared memory (one token tile)
constexpr int kAStages = 4;          // expanded weight k-blocks in tensor memory (32 columns)
constexpr int kKBlock = 128;         // k per pipeline stage (2 packed chunks)
constexpr int kWBlock = 4 * 2 * kChunkBytes;  // bytes of one weight k-block (4 groups)

// Smem layout of one CTA (offsets from a 1024-byte aligned base): the activation ring first
// (1024-aligned stages, as the 128-byte swizzle wants), then the weight ring.
// TT token tiles of BN rows share each expanded weight k-block (TT > 1: large M, one CTA
// per SM, all 512 TMEM columns).
template <int BN, int TT>
struct TcLayout {
  static constexpr int kBStages = TT == 1 ? kBStages1 : 3;
  static constexpr int kBPlane = BN * 128;               // one plane of one token tile
  static constexpr int kBTile = 2 * kBPlane;             // high + low plane of one token tile
  static constexpr int kBStage = TT * kBTile;            // one k-block of every token tile
  static constexpr int kWOff = kBStages * kBStage;
  static constexpr int kBytes = kWOff + kWStages * kWBlock;
  // TT == 1: at least 80 KB, so that no more than two CTAs (2 x 256 TMEM columns) share an
  // SM and tcgen05.alloc never waits for a CTA of this kernel; TT > 1 needs more than half
  // of the SM's shared memory anyway (one CTA per SM, 512 columns)
  static constexpr int kDyn = (kBytes + 1024) < 80 * 1024 ? 80 * 1024 : (kBytes + 1024);
  static_assert(TT == 1 || kDyn > 114 * 1024, "TT > 1 must keep one CTA per SM");
};


}  // namespace

// FL (Float mode): the activation planes are bf16 hi / lo splits of the fp32 activations, the
// weights are expanded to bf16 {-1, 0, +1} (two per TMEM column) and the MMA is kind::f16 with
// an f32 accumulator; a k-block is then 64 k (one packed chunk), which keeps every shared- and
// tensor-memory geometry of the integer path: a 128-byte activation row per plane and k-block,
// 32 TMEM columns of A per stage, 4 MMAs per stage. D = D_hi + D_lo, dequantised by 1/scale_w.
template <int BN, int TT, bool FL>
__global__ void __launch_bounds__(kTcThreads, 2)
    tc_matmul_kernel(const __grid_constant__ TcMaps maps, const __grid_constant__ TcArgs p) {
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 64, "BN must be 16..64, a multiple of 16");
  constexpr int kKB = FL ? kChunkK : kKBlock;  // k per pipeline stage
  constexpr int kCols = kAStages * 32 + TT * 2 * BN;  // A stages + TT x (D_hi, D_lo)
  constexpr int kAllocCols = kCols <= 128 ? 128 : (kCols <= 256 ? 256 : 512);
  static_assert(kCols <= 512 && (TT > 1 || kAllocCols <= 256),
                "two CTAs per SM must fit in the 512 TMEM columns");
  using L = TcLayout<BN, TT>;
  constexpr int kBStages = L::kBStages;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* bst = smem;             // [kBStages][2][BN][128], 128-byte swizzled rows
  unsigned char* wst = smem + L::kWOff;  // [kWStages][4 groups][2 chunks][512]
  __shared__ uint64_t wfull[kWStages], wempty[kWStages], bfull[kBStages], bempty[kBStages];
  __shared__ uint64_t afull[kAStages], aempty[kAStages], dfull;
  __shared__ uint32_t tmem_base_sh;
  __shared__ uint32_t s_fail;
  __shared__ int s_rowsum[BN];

  const MatmulArgs& a = p.m;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * 128, tb = blockIdx.y * BN * TT;  // first token of the CTA
  int t0 = tb;  // first token of the tile the epilogue works on
  const int proj = blockIdx.z / p.splits, split = blockIdx.z % p.splits;
  const TcProj& P = p.pj[proj];
  const CUtensorMap* bmap = &maps.m[proj];
  // weight row group of row block g (0..3): 4 consecutive groups, or for a SwiGLU pair the
  // gate groups 2x, 2x+1 and the up groups pair + 2x, pair + 2x + 1
  auto tile_group = [&](int g) -> int64_t {
    return p.pair ? (g < 2 ? 2 * blockIdx.x + g : p.pair + 2 * blockIdx.x + g - 2) : (n0 >> 5) + g;
  };
  const int64_t kc = packed_chunks(a.K);
  const int nkb = static_cast<int>(FL ? kc : (kc + 1) / 2);
  const int kb0 = static_cast<int>(static_cast<int64_t>(nkb) * split / p.splits);
  const int kb1 = static_cast<int>(static_cast<int64_t>(nkb) * (split + 1) / p.splits);
  const int nk = kb1 - kb0;

  if (tid == 0) {
    for (int s = 0; s < kWStages; ++s) { mbar_init(&wfull[s], 1); mbar_init(&wempty[s], 4); }
    for (int s = 0; s < kBStages; ++s) { mbar_init(&bfull[s], 1); mbar_init(&bempty[s], 1); }
    for (int s = 0; s < kAStages; ++s) { mbar_init(&afull[s], 4); mbar_init(&aempty[s], 1); }
    mbar_init(&dfull, 1);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // the next kernel may start its own weight streaming now (it reads no output of ours
    // before its griddepcontrol.wait)
    grid_dep_launch();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"(kAllocCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kBWarp && lane == 0)
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(bmap)) : "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t tmem_a = tmem;                   // columns [0, 32*kAStages)
  const uint32_t tmem_dhi = tmem + kAStages * 32; // BN columns
  const uint32_t tmem_dlo = tmem_dhi + BN;        // BN columns

  // ---- epilogue helpers (epilogue warps 0-3; thread = TMEM lane = weight row n)
  const int n = p.pair ? (tid < 64 ? 64 * blockIdx.x + tid : p.pair * 32 + 64 * blockIdx.x + tid - 64)
                       : n0 + tid;
  const bool n_ok = tid < 128 && n < a.N;
  uint32_t* xtile = reinterpret_cast<uint32_t*>(bst);                 // [BN][128] split-K partials
  float* xch = reinterpret_cast<float*>(bst + BN * 128 * 4);          // [8][128] SwiGLU exchange
  const bool add_resid = a.resid && P.out;
  auto load16 = [&](int c0, float (&r)[16], int cnt = 16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int t = t0 + c0 + j;
      r[j] = (add_resid && n_ok && j < cnt && t < a.M) ? a.resid[static_cast<int64_t>(t) * a.ldr + n] : 0.0f;
    }
  };
  // dequant (+ residual) of 16 finished int32 accumulators of tokens t0 + c0 + [0, 16);
  // a SwiGLU pair then combines gate row c (thread c) with up row I + c (thread 64 + c).
  // Called by all 128 epilogue threads alike (the pair exchange synchronises them).
  auto emit16 = [&](int c0, const uint32_t (&v)[16], const float (&r)[16], int cnt = 16) {
    float o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int t = t0 + c0 + j;
      if (FL) {  // v: the float sum D_hi + D_lo
        o[j] = __fmul_rn(__uint_as_float(v[j]), P.scale);
      } else {
        const int32_t acc = static_cast<int32_t>(v[j] - static_cast<uint32_t>(s_rowsum[(c0 + j) & (BN - 1)]));
        if (a.acc_out && n_ok && j < cnt && t < a.M) a.acc_out[static_cast<int64_t>(t) * a.N + n] = acc;
        o[j] = __fmul_rn(__int2float_rn(acc), P.scale);
      }
      if (a.resid) o[j] = __fadd_rn(r[j], o[j]);
    }
    if (!p.pair) {
      if (P.out)
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (n_ok && j < cnt && t0 + c0 + j < a.M) P.out[static_cast<int64_t>(t0 + c0 + j) * a.ldo + n] = o[j];
      return;
    }
    named_sync(1, 128);  // the previous group has been read
    // gate threads (tid < 64) pass up tokens 8..15 of their row, up threads tokens 0..7 of
    // theirs, so that all 128 threads then combine 8 tokens of gate row c with up row I + c
    const int c = tid & 63;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) xch[jj * 128 + tid] = tid < 64 ? o[8 + jj] : o[jj];
    named_sync(1, 128);
    // element (t, col) is in the scalar tail of its segment only in the segment's last row, at
    // columns >= tail_from (fewer than 8 columns, so the division is rare)
    const int col = 64 * blockIdx.x + c;
    const bool tail_col = col >= p.tail_from;
    const int jb = tid < 64 ? 0 : 8;
    float g[8], u[8], z[8];
    bool body[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      g[jj] = tid < 64 ? o[jj] : xch[jj * 128 + c];
      u[jj] = tid < 64 ? xch[jj * 128 + 64 + c] : o[8 + jj];
      body[jj] = !tail_col || (t0 + c0 + jb + jj + 1) % p.seg_rows != 0;
    }
    swiglu_n(g, u, body, z);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int t = t0 + c0 + jb + jj;
      if (jb + jj < cnt && t < a.M && col < p.pair * 32) P.out[static_cast<int64_t>(t) * a.ldo + col] = z[jj];
    }
  };

  if (warp == kWWarp) {
    // ---- weight producer: 4 groups x (1 or 2) chunks per k-block, contiguous per group
    if (lane == 0) {
      const int64_t ngroups = packed_groups(a.N);
      const unsigned char* wbase = static_cast<const unsigned char*>(P.w);
      // one token tile: the weights are read once (decode); more: every token tile re-reads
      // them, so they stay in L2 (prefill)
      const uint64_t pol = a.M > BN * TT ? l2_evict_last() : l2_evict_first();
      int i = 0;
      for (; i < nk; ++i) {
        const int s = i % kWStages;
        // from here on progress depends on the activations: wait for the predecessor first,
        // so that the bounded waits never include its run time
        if (i == kWStages) grid_dep_wait();
        if (i >= kWStages && !role_wait(&wempty[s], ((i / kWStages) - 1) & 1, &s_fail)) break;
        const int64_t c0 = (FL ? 1 : 2) * static_cast<int64_t>(kb0 + i);  // first chunk
        if (!FL) {
          // one tensor copy of the k-block's 4 groups (2 + 2 for a pair tile); groups past the
          // rows and a chunk past Kp arrive as zeros, whole boxes counted
          mbar_arrive_tx(&wfull[s], static_cast<uint32_t>(kWBlock));
          const CUtensorMap* wmap = &maps.w[proj];
          const int x = static_cast<int>(c0) * (kChunkBytes / 4);  // 32-bit words
          if (p.pair) {
            tma_load_2d_hint(wst + s * kWBlock, wmap, x, static_cast<int>(tile_group(0)), &wfull[s], pol);
            tma_load_2d_hint(wst + s * kWBlock + 2 * 2 * kChunkBytes, wmap, x, static_cast<int>(tile_group(2)),
                             &wfull[s], pol);
          } else {
            tma_load_2d_hint(wst + s * kWBlock, wmap, x, static_cast<int>(tile_group(0)), &wfull[s], pol);
          }
          continue;
        }
        const uint32_t bytes = kChunkBytes;
        uint32_t total = 0;
        for (int g = 0; g < 4; ++g)
          if (tile_group(g) < ngroups) total += bytes;
        mbar_arrive_tx(&wfull[s], total);
        for (int g = 0; g < 4; ++g) {
          const int64_t gg = tile_group(g);
          if (gg < ngroups)
            bulk_g2s(wst + s * kWBlock + g * 2 * kChunkBytes, wbase + (gg * kc + c0) * kChunkBytes,
                     bytes, &wfull[s], pol);
        }
      }
      if (i < nk) {  // failed: note it, then let the copies already issued land
        atomicOr(&s_fail, 1u);
        for (int j = i - kWStages > 0 ? i - kWStages : 0; j < i; ++j)
          mbar_wait(&wfull[j % kWStages], (j / kWStages) & 1);
      }
    }
  } else if (warp == kBWarp) {
    // ---- activation producer: TMA loads of the high / low byte planes (after the
    //      predecessor kernel has written them)
    if (lane == 0) {
      grid_dep_wait();
      int i = 0;
      for (; i < nk; ++i) {
        const int s = i % kBStages;
        if (i >= kBStages && !role_wait(&bempty[s], ((i / kBStages) - 1) & 1, &s_fail)) break;
        const int x = (kb0 + i) * kKB;  // elements: 128 bytes of either plane type
        unsigned char* dst = bst + s * L::kBStage;
        mbar_arrive_tx(&bfull[s], static_cast<uint32_t>(L::kBStage));
#pragma unroll
        for (int tt = 0; tt < TT; ++tt) {
          const int tr = tb + tt * BN;
          tma_load_2d(dst + tt * L::kBTile, bmap, x, tr, &bfull[s]);                   // high rows
          tma_load_2d(dst + tt * L::kBTile + L::kBPlane, bmap, x, a.M + tr, &bfull[s]);  // low rows
        }
      }
      if (i < nk) {
        atomicOr(&s_fail, 1u);
        for (int j = i - kBStages > 0 ? i - kBStages : 0; j < i; ++j)
          mbar_wait(&bfull[j % kBStages], (j / kBStages) & 1);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---- MMA issuer: per k-block 4 k-steps x (high, low) planes
    if (lane == 0) {
      grid_dep_wait();
      for (int i = 0; i < nk; ++i) {
        const int sa = i % kAStages, sb = i % kBStages;
        if (!role_wait(&afull[sa], (i / kAStages) & 1, &s_fail) ||
            !role_wait(&bfull[sb], (i / kBStages) & 1, &s_fail)) {
          atomicOr(&s_fail, 1u);
          break;
        }
        tc_fence_after();
        const uint32_t b_base = smem_u32(bst + sb * L::kBStage);
        // both planes in one instruction: B rows [0, BN) are the high bytes, [BN, 2BN) the
        // low bytes - 128 (both s8, one 128-byte-swizzled tile), D columns likewise; the
        // same A (weight) columns serve every token tile
        // per MMA: 32 bytes of K from the activation rows and 8 TMEM columns of weights
        // (32 u8 or 16 bf16 k), 4 per stage either way
#pragma unroll
        for (int tt = 0; tt < TT; ++tt)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t acc = (i > 0 || j > 0) ? 1u : 0u;
            const uint32_t a_addr = tmem_a + static_cast<uint32_t>(sa * 32 + j * 8);
            const uint64_t bd = smem_desc_sw128(b_base + tt * L::kBTile + j * 32);
            if (FL) mma_bf16_ts(tmem_dhi + tt * 2 * BN, a_addr, bd, idesc_bf16(2 * BN), acc);
            else mma_i8_ts(tmem_dhi + tt * 2 * BN, a_addr, bd, idesc_i8(true, 2 * BN), acc);
          }
        mma_commit(&aempty[sa]);
        mma_commit(&bempty[sb]);
      }
      // arrives once every MMA issued above has completed (also on failure)
      mma_commit(&dfull);
    }
    __syncwarp();
  } else {
    // ---- warps 0-3: expand the 2-bit codes of group `warp` (TMEM lanes 32*warp..+31) into
    //      u8 TMEM columns, then the epilogue
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    bool ok = true;
    uint32_t su = 0;  // sum of this row's codes u over the k-blocks of this CTA (k < Kp)
    for (int i = 0; i < nk; ++i) {
      const int sw = i % kWStages, sa = i % kAStages;
      if (!role_wait(&wfull[sw], (i / kWStages) & 1, &s_fail)) { ok = false; break; }
      const uint4* src = reinterpret_cast<const uint4*>(wst + sw * kWBlock + warp * 2 * kChunkBytes) + lane;
      const uint4 wv[2] = {src[0], FL ? src[0] : src[kChunkBytes / 16]};
      const int nch = 2 * static_cast<int64_t>(kb0 + i) + 1 < kc ? 2 : 1;  // chunks below Kp
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (FL || h >= nch) break;  // (the Float combine needs no code sums)
        const uint32_t wd[4] = {wv[h].x, wv[h].y, wv[h].z, wv[h].w};
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4)
          su += __popc(wd[w4] & 0x55555555u) + 2u * __popc(wd[w4] & 0xAAAAAAAAu);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[sw]);
      if (i == kAStages) grid_dep_wait();  // later stages wait on MMAs that need activations
      if (i >= kAStages && !role_wait(&aempty[sa], ((i / kAStages) - 1) & 1, &s_fail)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t r[16];
        if (FL) {
          // one chunk: column 16h + c holds k = 32h + 2c, 2c + 1 as bf16 weights; word w4 of
          // the chunk holds k = 16 w4 + 4q + j (j = 0..3) in byte j of (word >> 2q)
          const uint32_t wd[4] = {wv[0].x, wv[0].y, wv[0].z, wv[0].w};
#pragma unroll
          for (int w = 0; w < 2; ++w)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t m = (wd[2 * h + w] >> (2 * q)) & 0x03030303u;
              r[8 * w + 2 * q] = ternary_bf16x2(m, 0);
              r[8 * w + 2 * q + 1] = ternary_bf16x2(m, 2);
            }
        } else {
          const uint32_t wd[4] = {wv[h].x, wv[h].y, wv[h].z, wv[h].w};
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4)
#pragma unroll
            for (int q = 0; q < 4; ++q) r[4 * w4 + q] = (wd[w4] >> (2 * q)) & 0x03030303u;
        }
        tmem_st16(tmem_a + lane_base + static_cast<uint32_t>(sa * 32 + h * 16), r);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[sa]);
    }
    if (!ok) atomicOr(&s_fail, 1u);
    // epilogue: row sums and residuals belong to earlier kernels. The code runs once per
    // CTA, so every instruction is a cold instruction-cache miss: the loops over 16-token
    // groups stay rolled. Loads of a group are issued before its stores (a store may alias
    // them) and the next group's residuals are fetched while the current group is written.
    grid_dep_wait();
    if (tid < BN) s_rowsum[tid] = (!FL && t0 + tid < a.M) ? P.rowsum[t0 + tid] : 0;
    const bool done = mbar_wait(&dfull, 0);
    tc_fence_after();
    if (!done) atomicOr(&s_fail, 1u);
    named_sync(1, 128);  // row sums staged; the decision below is uniform over the 4 warps
    if (s_fail != 0) {
      if (tid == 0 && p.err) atomicOr(p.err, kErrTimeout);
    } else if (nk > 0) {
      // 256*D_hi + D_lo, with D_lo = D_lo' + 128*sum(u) for the low plane stored as lo - 128
      auto part16 = [&](int tt, int c0, uint32_t (&v)[16]) {
        uint32_t dh[16], dl[16];
        tmem_ld16(tmem_dhi + tt * 2 * BN + lane_base + c0, dh);
        tmem_ld16(tmem_dlo + tt * 2 * BN + lane_base + c0, dl);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          v[j] = FL ? __float_as_uint(__fadd_rn(__uint_as_float(dh[j]), __uint_as_float(dl[j])))
                    : (dh[j] << 8) + dl[j] + (su << 7);  // mod 2^32
      };
      if (p.splits == 1) {
#pragma unroll 1
        for (int tt = 0; tt < TT; ++tt) {
          if (tt > 0) {  // next token tile: its row sums (uniform over the 128 threads)
            t0 = tb + tt * BN;
            if (t0 >= a.M) break;
            named_sync(1, 128);
            if (tid < BN) s_rowsum[tid] = (!FL && t0 + tid < a.M) ? P.rowsum[t0 + tid] : 0;
            named_sync(1, 128);
          }
          float rv[16];
          load16(0, rv);
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            uint32_t v[16];
            part16(tt, c0, v);
            float rn[16];
            if (c0 + 16 < BN) load16(c0 + 16, rn);
            emit16(c0, v, rv);
#pragma unroll
            for (int j = 0; j < 16; ++j) rv[j] = rn[j];
          }
        }
      } else {
        // split-K: leave this CTA's partial tile in shared memory for the cluster leader
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t v[16];
          part16(0, c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) xtile[(c0 + j) * 128 + tid] = v[j];
        }
      }
    }
  }

  __syncwarp();
  if (p.splits > 1) {
    // split-K over the cluster (the CTAs of one output tile): after the first barrier every
    // partial tile is in its CTA's shared memory ([token][row]); CTA r then sums its BN / S
    // tokens from every peer over distributed shared memory and writes them; the second
    // barrier keeps each CTA's shared memory alive until its peers have read it. Every CTA
    // reaches both barriers, on the error paths too.
    cluster_sync();
    if (warp < 4 && s_fail == 0 && nk > 0) {
      // a thread takes 4 consecutive rows of a token: one warp reads a whole token row
      // (512 contiguous bytes) per 16-byte load, and stores 4 consecutive outputs. All loads
      // of a thread (<= 64 words) are issued before the first sum.
      const uint32_t xbase = smem_u32(xtile);
      auto reduce = [&](auto S_) {
        constexpr int S = decltype(S_)::value, G = BN / S;
        uint32_t pb[S];
#pragma unroll
        for (int r = 0; r < S; ++r) pb[r] = cluster_map(xbase, r);
        const int tok0 = split * G;  // first token (within the tile) of this CTA
        if (!p.pair) {
          constexpr int NI = (G + 3) / 4;
          const int q = tid & 31, w = tid >> 5;
          const int nq = n0 + 4 * q;
          const bool full = p.vec && nq + 3 < a.N;
          // residuals and partials of token j (zeros for j >= G): the own partial from local
          // shared memory
          auto fetch = [&](int j, float (&fr)[4], uint32_t (&fp)[S][4]) {
            const int t = t0 + tok0 + j;
#pragma unroll
            for (int e = 0; e < 4; ++e) fr[e] = 0.0f;
            if (add_resid && j < G && t < a.M) {
              const float* rp = a.resid + static_cast<int64_t>(t) * a.ldr + nq;
              if (full) {
                const float4 v4 = *reinterpret_cast<const float4*>(rp);
                fr[0] = v4.x; fr[1] = v4.y; fr[2] = v4.z; fr[3] = v4.w;
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) fr[e] = nq + e < a.N ? rp[e] : 0.0f;
              }
            }
            const uint32_t off = 4u * static_cast<uint32_t>((tok0 + j) * 128 + 4 * q);
#pragma unroll
            for (int r = 0; r < S; ++r) {
              if (j >= G) fp[r][0] = fp[r][1] = fp[r][2] = fp[r][3] = 0u;
              else if (r == split) ld_shared_v4(xbase + off, fp[r]);
              else ld_cluster_v4(pb[r] + off, fp[r]);
            }
          };
          // one token per iteration, rolled (cold instruction cache); the next token's loads
          // are issued before this one is combined
          float rv[4];
          uint32_t part[S][4];
          fetch(w, rv, part);
#pragma unroll 1
          for (int i = 0; i < NI; ++i) {
            const int j = w + 4 * i, t = t0 + tok0 + j;
            float nr[4];
            uint32_t np[S][4];
            fetch(i + 1 < NI ? j + 4 : G, nr, np);
            if (j < G && t < a.M) {
              const uint32_t rs = static_cast<uint32_t>(s_rowsum[tok0 + j]);
              float o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                if (FL) {  // float partials, summed in split order
                  float vs = 0.0f;
#pragma unroll
                  for (int r = 0; r < S; ++r) vs = __fadd_rn(vs, __uint_as_float(part[r][e]));
                  o[e] = __fmul_rn(vs, P.scale);
                } else {
                  uint32_t v = 0;
#pragma unroll
                  for (int r = 0; r < S; ++r) v += part[r][e];
                  const int32_t acc = static_cast<int32_t>(v - rs);
                  if (a.acc_out && nq + e < a.N) a.acc_out[static_cast<int64_t>(t) * a.N + nq + e] = acc;
                  o[e] = __fmul_rn(__int2float_rn(acc), P.scale);
                }
                if (a.resid) o[e] = __fadd_rn(rv[e], o[e]);
              }
              if (P.out) {
                float* op = P.out + static_cast<int64_t>(t) * a.ldo + nq;
                if (full) {
                  *reinterpret_cast<float4*>(op) = make_float4(o[0], o[1], o[2], o[3]);
                } else {
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    if (nq + e < a.N) op[e] = o[e];
                }
              }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              rv[e] = nr[e];
#pragma unroll
              for (int r = 0; r < S; ++r) part[r][e] = np[r][e];
            }
          }
        } else {
          // SwiGLU pair: tile rows [0, 64) are gate rows, [64, 128) the matching up rows; a
          // thread combines 4 gate rows with their 4 up rows for its tokens
          constexpr int NI = (G + 7) / 8;
          const int q = tid & 15, w = tid >> 4;
          const int col = 64 * blockIdx.x + 4 * q;  // output column of gate row 4q
          const int I = p.pair * 32;
          // partials of token j (zeros for j >= G): the own one from local shared memory
          auto fetch = [&](int j, uint32_t (&fg)[S][4], uint32_t (&fu)[S][4]) {
            const uint32_t off = 4u * static_cast<uint32_t>((tok0 + j) * 128 + 4 * q);
#pragma unroll
            for (int r = 0; r < S; ++r) {
              if (j < G && r == split) {
                ld_shared_v4(xbase + off, fg[r]);
                ld_shared_v4(xbase + off + 4u * 64u, fu[r]);
              } else if (j < G) {
                ld_cluster_v4(pb[r] + off, fg[r]);
                ld_cluster_v4(pb[r] + off + 4u * 64u, fu[r]);
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) fg[r][e] = fu[r][e] = 0u;
              }
            }
          };
          // one token per iteration, rolled (this code runs once per CTA, from a cold
          // instruction cache); the next token's partials load while this one is combined
          uint32_t pg[S][4], pu[S][4];
          fetch(w, pg, pu);
#pragma unroll 1
          for (int i = 0; i < NI; ++i) {
            const int j = w + 8 * i, t = t0 + tok0 + j;
            uint32_t ng[S][4], nu[S][4];
            fetch(i + 1 < NI ? j + 8 : G, ng, nu);
            if (j < G && t < a.M) {
              const uint32_t rs = static_cast<uint32_t>(s_rowsum[tok0 + j]);
              float g[4], u[4], z[4];
              bool body[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                if (FL) {
                  float sg = 0.0f, sv = 0.0f;
#pragma unroll
                  for (int r = 0; r < S; ++r) {
                    sg = __fadd_rn(sg, __uint_as_float(pg[r][e]));
                    sv = __fadd_rn(sv, __uint_as_float(pu[r][e]));
                  }
                  g[e] = __fmul_rn(sg, P.scale);
                  u[e] = __fmul_rn(sv, P.scale);
                } else {
                  uint32_t vg = 0, vu = 0;
#pragma unroll
                  for (int r = 0; r < S; ++r) {
                    vg += pg[r][e];
                    vu += pu[r][e];
                  }
                  const int32_t ag = static_cast<int32_t>(vg - rs), au = static_cast<int32_t>(vu - rs);
                  if (a.acc_out) {
                    a.acc_out[static_cast<int64_t>(t) * a.N + col + e] = ag;
                    a.acc_out[static_cast<int64_t>(t) * a.N + I + col + e] = au;
                  }
                  g[e] = __fmul_rn(__int2float_rn(ag), P.scale);
                  u[e] = __fmul_rn(__int2float_rn(au), P.scale);
                }
                // element (t, col) is in the scalar tail of its segment only in the segment's
                // last row, at columns >= tail_from (fewer than 8, so the division is rare)
                body[e] = col + e < p.tail_from || (t + 1) % p.seg_rows != 0;
              }
              swiglu_n(g, u, body, z);
              float* op = P.out + static_cast<int64_t>(t) * a.ldo + col;
              if (p.vec) {
                *reinterpret_cast<float4*>(op) = make_float4(z[0], z[1], z[2], z[3]);
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) op[e] = z[e];
              }
            }
#pragma unroll
            for (int r = 0; r < S; ++r)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                pg[r][e] = ng[r][e];
                pu[r][e] = nu[r][e];
              }
          }
        }
      };
      if (p.splits == 2) reduce(std::integral_constant<int, 2>{});
      else if (p.splits == 4) reduce(std::integral_constant<int, 4>{});
      else reduce(std::integral_constant<int, 8>{});
    }
    cluster_sync();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kAllocCols)
                 : "memory");
  }
}

// ---- host side

namespace {

// cuTensorMapEncodeTiled, resolved through the runtime (no link against the driver library)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

}  // namespace

// The planes [2][M][Kp] as one 2-D tensor of 2M rows x Kp elements (u8, or bf16 for the Float
// path); a box is BN rows x 128 B (one k-block), written to shared memory with the 128-byte
// swizzle; reads past row 2M or column Kp return zeros.
cudaError_t planes_map(CUtensorMap* map, const int8_t* planes, int M, int64_t kp, int bn, bool bf16) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(planes) & 15) != 0) return cudaErrorMisalignedAddress;
  const cuuint64_t esize = bf16 ? 2 : 1;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kp), 2 * static_cast<cuuint64_t>(M)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kp) * esize};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esize), static_cast<cuuint32_t>(bn)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                   const_cast<int8_t*>(planes), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// The same planes as a 3-D tensor {Kp, M, 2} (u8): one box of 128 B x bn rows x both planes
// is a whole activation k-block (high rows, then low rows) in one copy; rows past M read 0.
cudaError_t planes_map3(CUtensorMap* map, const int8_t* planes, int M, int64_t kp, int bn) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(planes) & 15) != 0) return cudaErrorMisalignedAddress;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kp), static_cast<cuuint64_t>(M), 2};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kp), static_cast<cuuint64_t>(kp) * static_cast<cuuint64_t>(M)};
  const cuuint32_t box[3] = {128, static_cast<cuuint32_t>(bn), 2};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(planes), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Packed ternary weights [groups][chunks][512 B] as a 2-D tensor of 32-bit words, one row per
// 32-row group (kc * 128 words); a box is 256 words (two chunks, 128 k) x `rows` groups, so
// one copy brings a k-block of several groups; groups past N and chunks past Kp read 0.
cudaError_t weights_map(CUtensorMap* map, const void* w, int64_t n, int64_t k, int rows) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(w) & 15) != 0) return cudaErrorMisalignedAddress;
  const int64_t kc = packed_chunks(k);
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kc) * (kChunkBytes / 4), static_cast<cuuint64_t>(packed_groups(n))};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kc) * kChunkBytes};
  const cuuint32_t box[2] = {2 * kChunkBytes / 4, static_cast<cuuint32_t>(rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}


template <int BN, int TT, bool FL>
static cudaError_t launch_tc_bn(const TcArgs& p, const MatmulArgs* a, bool pdl, cudaStream_t s) {
  using L = TcLayout<BN, TT>;
  TcMaps maps;
  for (int j = 0; j < p.nproj; ++j) {
    cudaError_t e = planes_map(&maps.m[j], a[j].planes, a[j].M, padded_k(a[j].K), BN, FL);
    if (e == cudaSuccess && !FL) e = weights_map(&maps.w[j], a[j].w, a[j].N, a[j].K, p.pair ? 2 : 4);
    if (e != cudaSuccess) return e;
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(tc_matmul_kernel<BN, TT, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kDyn);
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ceil_div(p.m.N, 128)), static_cast<unsigned>(ceil_div(p.m.M, BN * TT)),
                     static_cast<unsigned>(p.nproj * p.splits));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = L::kDyn;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (p.splits > 1) {  // the k-splits of one output tile form a cluster (reduced over DSMEM)
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = 1;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = static_cast<unsigned>(p.splits);
    ++na;
  }
  if (pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, tc_matmul_kernel<BN, TT, FL>, maps, p);
}

// k-blocks of a reduction over K: 128 k per block for the integer path, 64 for Float
static int tc_kblocks(const MatmulArgs& a) {
  const int64_t kc = packed_chunks(a.K);
  return static_cast<int>(a.fixed ? (kc + 1) / 2 : kc);
}

int tc_token_tile(int M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

int tc_splits(const MatmulArgs& a, int sm_count, int nproj) {
  // up to two CTAs per SM, the residency the kernel is built for (MMFREE_TC_CTAS_PER_SM=1:
  // one, for comparison): at 64 tokens splitting a long reduction over more CTAs costs less
  // in the cluster reduction than it saves in the k-loop; every split keeps >= 2 k-blocks; a
  // cluster holds <= 8 CTAs
  static const int per_sm = [] {
    const char* e = std::getenv("MMFREE_TC_CTAS_PER_SM");
    return (e && std::atoi(e) == 1) ? 1 : 2;
  }();
  const int64_t tiles = ceil_div(a.N, 128) * ceil_div(a.M, tc_token_tile(a.M)) * nproj;
  const int nkb = tc_kblocks(a);
  int splits = 1;
  while (splits < 8 && tiles * splits * 2 <= per_sm * sm_count && nkb / (splits * 2) >= 2) splits *= 2;
  return splits;
}

// nproj projections of one shape in one launch; pair > 0: a SwiGLU gate_proj (N = 2I,
// pair = I / 32, out = z [M, I], tails per seg)
static cudaError_t launch_tc(const MatmulArgs* a, int nproj, int pair, int64_t seg, int splits,
                             int sm_count, cudaStream_t s) {
  const MatmulArgs& m = a[0];
  if (m.M <= 0 || m.N <= 0) return cudaSuccess;
  const int nkb = tc_kblocks(m);
  if (nproj < 1 || nproj > 3 || splits < 1 || splits > 8 || (splits & (splits - 1)) || splits > nkb)
    return cudaErrorInvalidValue;
  if (pair && (nproj != 1 || m.N != 64 * pair)) return cudaErrorInvalidValue;
  // FixedQ510: low planes stored lo - 128; Float: bf16 planes (no raw accumulators)
  for (int j = 0; j < nproj; ++j)
    if (a[j].M != m.M || a[j].N != m.N || a[j].K != m.K || a[j].fixed != m.fixed ||
        (m.fixed ? !a[j].lo_signed : (!a[j].bf16 || a[j].acc_out)))
      return cudaErrorInvalidValue;
  TcArgs p{};
  p.m = m;
  p.nproj = nproj;
  p.pair = pair;
  if (pair) {  // seg = seg_rows * I elements, I = 32 * pair >= 64
    const int64_t I = 32 * static_cast<int64_t>(pair);
    if (seg <= 0 || seg % I != 0 || seg / I > INT32_MAX) return cudaErrorInvalidValue;
    p.seg_rows = static_cast<int>(seg / I);
    p.tail_from = static_cast<int>(I - seg % 8);
  } else {
    p.seg_rows = 1;
    p.tail_from = INT32_MAX;
  }
  p.err = m.err;
  p.splits = splits;
  {
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    bool vec = m.ldo % 4 == 0 && (!m.resid || (al16(m.resid) && m.ldr % 4 == 0)) &&
               (!m.acc_out || (al16(m.acc_out) && m.N % 4 == 0));
    for (int j = 0; j < nproj; ++j) vec = vec && (!a[j].out || al16(a[j].out));
    p.vec = vec ? 1 : 0;
  }
  for (int j = 0; j < nproj; ++j) p.pj[j] = TcProj{a[j].w, a[j].rowsum, a[j].out, a[j].scale};
  // thousands of rows: the persistent kernel, once every SM gets two tiles or more
  if (m.fixed && tc_rows_enabled() && tc_rows_tiles(m, nproj, pair) >= 2 * static_cast<int64_t>(sm_count)) {
    p.splits = 1;
    return launch_tc_rows(p, a, sm_count, s);
  }
  if (pair % 2 != 0) return cudaErrorInvalidValue;  // 64-row pair tiles below
  const int bn = tc_token_tile(m.M);
  // (three 64-row token tiles per CTA sharing each expanded weight k-block, TT = 3, were
  // measured 1.3x slower on the 2.7B prefill than two one-tile CTAs per SM)
  if (!m.fixed) {
    if (bn == 16) return launch_tc_bn<16, 1, true>(p, a, m.pdl, s);
    if (bn == 32) return launch_tc_bn<32, 1, true>(p, a, m.pdl, s);
    return launch_tc_bn<64, 1, true>(p, a, m.pdl, s);
  }
  if (bn == 16) return launch_tc_bn<16, 1, false>(p, a, m.pdl, s);
  if (bn == 32) return launch_tc_bn<32, 1, false>(p, a, m.pdl, s);
  return launch_tc_bn<64, 1, false>(p, a, m.pdl, s);
}

cudaError_t launch_matmul_tc(const MatmulArgs& a, int splits, int sm_count, cudaStream_t s) {
  return launch_tc(&a, 1, 0, 1, splits, sm_count, s);
}

cudaError_t launch_matmul_tc_group(const MatmulArgs* a, int nproj, int swiglu_I, int64_t seg,
                                   int sm_count, cudaStream_t s) {
  return launch_tc(a, nproj, swiglu_I > 0 ? swiglu_I / 32 : 0, seg, tc_splits(a[0], sm_count, nproj),
                   sm_count, s);
}

}  // namespace mmfree_cuda
