// kernels.h -- host-side launch wrappers of the mmfree CUDA kernels (internal C++ API).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mmfree_cuda {

// How a prep row transform builds the projection input t from its inputs.
enum PrepMode : int {
  kPrepPlain = 0,      // t = x
  kPrepNorm = 1,       // t = rmsnorm(x) * prew                    (attn_norm, mlp_norm, final norm)
  kPrepSwishgate = 2,  // t = rmsnorm(x) * prew * silu(o)          (g_norm over g_proj, recurrence)
};

struct PrepArgs {
  const float* x = nullptr;      // [M, K] rows
  const float* o = nullptr;      // [M, K] recurrence output (kPrepSwishgate)
  const float* prew = nullptr;   // [K] weight of the row transform
  float* pre_out = nullptr;      // optional [M, K]: t
  int nproj = 1;                 // projections sharing t (1..3)
  const float* normw[3] = {};    // per projection BitLinear norm weight [K]
  float* norm_out = nullptr;     // optional [M, K]: normalized input of projection 0
  int8_t* planes[3] = {};        // fixed: [2][M][Kp] high bytes then low bytes of Q5.10 codes
  bool lo_signed = false;        // fixed: low plane stored as (lo ^ 0x80) = lo - 128 (s8), the
                                 // form the tensor-core matmul reads (matmul_uses_tc)
  int32_t* rowsum[3] = {};       // fixed: [M] sum of codes
  float* yf[3] = {};             // float: [M][Kp] normalized activations (zero padded)
  bool bf16 = false;             // float: write planes[j] as bf16 [2][M][Kp] (hi = bf16(y),
                                 // lo = bf16(y - hi)) for the tensor-core matmul, not yf
  int M = 0, K = 0;
  float eps = 1e-6f;
  float qs = 1024.0f;            // 2^frac_bits
  bool fixed = true;
  bool pdl = false;              // launch as a programmatic dependent of the previous kernel
  uint32_t* err = nullptr;       // optional: bit kErrTimeout on a timed-out wait
  uint32_t row_polls = 0;        // set by launch_prep: polls of the row-staging wait
  // kPrepSwishgate of one decode step with the token mixer fused in: o is not read but
  // computed here from the i / f projections and the recurrent state (which is updated), as
  // launch_mixer does for len 1; needs K % 4 == 0, 16-byte aligned rows and K >= 8
  const float* mix_i = nullptr;  // [M, K]
  const float* mix_f = nullptr;  // [M, K]
  float* mix_state = nullptr;    // [M, K] in / out
  const float* mix_lb = nullptr; // [K] lower bound (nullable)
  float* mix_out = nullptr;      // [M, K] recurrence output (nullable)
  int mix_seg_rows = 1;          // rows of one reference vector call (SIMD tails)
};

struct MatmulArgs {
  const void* w = nullptr;        // packed ternary weights
  const int8_t* planes = nullptr; // fixed: [2][M][Kp]
  const int32_t* rowsum = nullptr;
  const float* yf = nullptr;      // float: [M][Kp]
  int M = 0, N = 0, K = 0;
  float scale = 1.0f;             // fixed: 1/(2^f * scale_w); float: 1/scale_w
  float* out = nullptr;           // [M, ldo] (nullable: accumulators only)
  int ldo = 0;
  const float* resid = nullptr;   // optional [M, ldr]: out = resid + dequant
  int ldr = 0;
  int32_t* acc_out = nullptr;     // optional [M, N] raw int32 accumulators (fixed)
  bool fixed = true;
  // tensor-core path (FixedQ510, M >= kTcMinRows): opt-in, plus a device error word
  // (split-K partials are reduced inside a thread-block cluster: no workspace)
  bool allow_tc = false;
  uint32_t* err = nullptr;
  bool pdl = false;               // launch as a programmatic dependent of the previous kernel
  bool lo_signed = false;         // planes hold lo - 128 (required by the tensor-core path)
  bool bf16 = false;              // float: planes hold bf16 hi / lo activations [2][M][Kp]
                                  // (PrepArgs::bf16); the tensor-core path reads them
};

constexpr int kTcMinRows = 16;
// Does launch_matmul take the tensor-core path (FixedQ510 planes lo_signed, or Float bf16
// planes)?
inline bool matmul_uses_tc(const MatmulArgs& a) {
  return a.allow_tc && a.M >= kTcMinRows && (a.fixed || a.bf16);
}

// ---- fused few-row decode kernels (decode.cu)
enum DecPro : int {
  kDecProNorm2 = 0,  // rmsnorm(x) * prew, then each projection's BitLinear norm
  kDecProSwish = 1,  // rmsnorm(x) * prew * silu(o), then the BitLinear norm
  kDecProPlain = 2,  // the BitLinear norm of x
};
enum DecEpi : int {
  kDecEpiMixer = 0,   // i/f/g -> gate, lower bound, scan input, one recurrence step
  kDecEpiResid = 1,   // out = resid + dequant
  kDecEpiSwiglu = 2,  // gate_proj: out[c] = silu(y[c]) * y[I + c]
  kDecEpiLogits = 3,  // lm_head logits, greedy argmax into ids[t*stride + *pos + 1]
};
constexpr int kDecMaxRows = 4;

struct alignas(16) DecArgs {
  const float* x = nullptr;       // [M, K] (or the embedding table [V, K] when xids is set)
  const float* o = nullptr;       // [M, K] recurrence output (kDecProSwish)
  const float* prew = nullptr;    // [K] first norm weight
  const float* normw[3] = {};     // projection norm weights [K]
  const void* w[3] = {};          // packed weights (N x K each)
  float scale[3] = {1.0f, 1.0f, 1.0f};
  int M = 0, K = 0, N = 0;
  float eps = 1e-6f, qs = 1024.0f;
  float* out[2] = {};             // mixer: recurrence, g; resid/swiglu/logits: out[0]
  const float* resid = nullptr;   // [M, N]
  float* state = nullptr;         // [M, N] recurrent state (mixer)
  const float* lb = nullptr;      // [N] lower bound or nullptr (mixer)
  int64_t seg = 1;                // element count of one reference vector call (tails)
  int64_t* ids = nullptr;         // logits: token ids [M][stride], position *pos
  int64_t stride = 0;
  int64_t* pos = nullptr;
  unsigned* done = nullptr;
  float* part_v = nullptr;        // logits: per-CTA partial maxima [grid][kDecMaxRows]
  int* part_i = nullptr;
  // x gathered from the embedding table: row t is x[xids[t * xstride + *xpos]]; CTA 0 also
  // writes the rows to xcopy. Ids outside [0, V) set kErrBadToken in *err (zero row).
  const int64_t* xids = nullptr;
  int64_t xstride = 0;
  const int64_t* xpos = nullptr;
  float* xcopy = nullptr;
  int V = 0;
  uint32_t* err = nullptr;
  int pro = 0, epi = 0;           // phase kind (DecPro, DecEpi)
  int fl = 0;                     // Float activations (scale = 1/scale_w) instead of FixedQ510
  int stage = 0;                  // set by the launcher: first unit staged in shared memory
};
int dec_units(const DecArgs& a, int epi);
cudaError_t launch_dec(const DecArgs& a, int pro, int epi, int grid, cudaStream_t s, bool pdl);
// The persistent decode step: a table of phases (pro/epi set) run by one cooperative launch.
// dec_persist_plan sets each phase's staging flag and returns the dynamic shared memory
// (0: some phase does not fit); dec_persist_grid returns the CTA count (one per SM, 0 when a
// cooperative launch of that size is impossible). The barrier word is zeroed by the launcher.
size_t dec_persist_plan(DecArgs* phases, int n);
int dec_persist_grid(int M, size_t smem);
cudaError_t launch_dec_persist(const DecArgs* dev_phases, int nphases, int M, unsigned* bar,
                               uint32_t* err, size_t smem, int grid, cudaStream_t s);

// tcgen05 BitLinear matmul (tc_matmul.cu)
int tc_token_tile(int M);
int tc_splits(const MatmulArgs& a, int sm_count, int nproj = 1);
cudaError_t launch_matmul_tc(const MatmulArgs& a, int splits, int sm_count, cudaStream_t s);
// Several tensor-core BitLinears in one launch: nproj (1..3) projections of one shape (the
// i/f/g cluster; a[0] carries the error word and the launch mode), or with
// swiglu_I > 0 (I % 64 == 0, nproj 1) a gate_proj of N = 2I whose epilogue writes
// a[0].out = z [M, I] = silu(y[:, :I]) * y[:, I:] with SIMD tails per seg elements.
cudaError_t launch_matmul_tc_group(const MatmulArgs* a, int nproj, int swiglu_I, int64_t seg,
                                   int sm_count, cudaStream_t s);

// int8 ternary [n, k] (nn.Linear layout) -> tiled 2-bit format; entries outside {-1,0,1}
// set bit 2 (kErrNotTernary) of *err (nullable) and are packed by sign.
cudaError_t launch_repack(void* dst, const int8_t* wq, int64_t n, int64_t k, uint32_t* err,
                          cudaStream_t s);
cudaError_t launch_prep(const PrepArgs& a, cudaStream_t s);
// Polls of the prep's row-staging wait before it gives up and raises kErrTimeout, for the
// launches that follow (negative: the default limit). A diagnostic switch: 0 makes every
// staged wait give up at once, which exercises the error path without a fault.
void set_wait_limit(int64_t polls);
// int32 activation codes [M, K] (int16 range) -> high/low byte planes [2][M][Kp] + row sums;
// codes outside int16 set kErrRange in *err.
cudaError_t launch_codes_to_planes(int8_t* planes, int32_t* rowsum, const int32_t* x, int M,
                                   int K, uint32_t* err, cudaStream_t s);
cudaError_t launch_matmul(const MatmulArgs& a, cudaStream_t s);

// HGRN token mixer (hgrn_model.cpp:109-150) over rows = nseq * len rows laid out
// [nseq][len][H]: f = sigmoid(fraw) (lower-bounded when lb != nullptr), scan input
// silu(i) * (1 - f) (both in place in f and i), then the recurrence of each of the nseq
// sequences from state [nseq][H] (nullable: zero start, not written back). The reference's
// SIMD body/tail split is taken over segments of seg_rows * H elements: the rows of one
// reference block() call.
// For len > 1 the gates run element-parallel, then the scan: the reference's serial chain per
// lane (bit-exact), or with chunk_ws (mixer_chunk_bytes of device memory; Float mode) a
// chunked parallel scan over time that re-associates the recurrence.
cudaError_t launch_mixer(float* i, float* f, float* recur, float* state, const float* lb,
                         int nseq, int len, int H, int seg_rows, cudaStream_t s, bool pdl = false,
                         void* chunk_ws = nullptr);
size_t mixer_chunk_bytes(int nseq, int len, int H);
// z[t, c] = silu(y[t, c]) * y[t, I + c]  (hgrn_model.cpp:171-185), tails per seg_rows rows.
cudaError_t launch_swiglu_split(float* z, const float* y, int rows, int I, int seg_rows,
                                cudaStream_t s, bool pdl = false);
// out[n] = silu(a[n]) * b[n]  (activations.cpp:9-15)
cudaError_t launch_swiglu(float* out, const float* a, const float* b, int64_t n, cudaStream_t s);
// rmsnorm rows (rmsnorm.cpp:11-22)
cudaError_t launch_rmsnorm(float* y, const float* x, const float* w, int rows, int cols,
                           float eps, cudaStream_t s);
// rmsnorm_swishgate rows (rmsnorm_swishgate.cpp:13-30)
cudaError_t launch_swishgate(float* out, const float* g, const float* o, const float* w, int rows,
                             int cols, float eps, cudaStream_t s);
// sequential scan over T (hgrn_scan.cpp:11-19); state nullable (zero start)
cudaError_t launch_scan(float* out, const float* i, const float* f, int T, int D, float* state,
                        cudaStream_t s);
// h[t] = emb[ids[t]]; ids outside [0, V) raise kErrBadToken and give a zero row.
cudaError_t launch_embed(float* h, const float* emb, const int64_t* ids, int T, int H, int V,
                         uint32_t* err, cudaStream_t s);
// ids[m] = first index of the maximum of logits[m, :V] (hgrn_model.cpp:271-273).
cudaError_t launch_argmax(int64_t* ids, const float* logits, int M, int V, int ld,
                          cudaStream_t s);

// Temperature / top-k sampling (hgrn_model.cpp:274-300): row i of logits [B][ld] (V used)
// draws for stream row0 + i into ids[(row0 + i) * stride + *pos + 1] with the uniform
// uni[(row0 + i) * ustride + *pos + 1]; with `advance`, the last block advances *pos. The k
// highest logits are the candidates (ties to the lower index), walked in ascending index
// order; temperature > 0.
cudaError_t launch_sample_at(int64_t* ids, int64_t stride, int64_t* pos, unsigned* done,
                             bool advance, int row0, const float* logits, int B, int V, int ld,
                             const double* uni, int64_t ustride, float temperature, int top_k,
                             cudaStream_t s, bool pdl = false);

// Device-resident decode loop helpers. Stream b's token at position *pos lives at
// ids[b * stride + *pos]. embed_at gathers those B rows; argmax_at writes the greedy pick of
// logits row b to ids[b * stride + *pos + 1] and the last block to finish advances *pos.
cudaError_t launch_embed_at(float* h, const float* emb, const int64_t* ids, int64_t stride,
                            const int64_t* pos, int B, int H, int V, uint32_t* err,
                            cudaStream_t s, bool pdl = false);
cudaError_t launch_argmax_at(int64_t* ids, int64_t stride, int64_t* pos, unsigned* done,
                             const float* logits, int B, int V, int ld, cudaStream_t s,
                             bool pdl = false);

}  // namespace mmfree_cuda
