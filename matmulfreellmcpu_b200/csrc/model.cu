// model.cu -- device-resident HGRN-Bit forward, generate and lockstep serving.
//
// Control flow restates matmulfreellmCPU cpp/src/model/hgrn_model.cpp:
//   block()            :80-195   -> Model::layers (prep / matmul / mixer kernels)
//   layers_and_norm()  :220-237  -> Model::forward
//   generate()         :249-347  -> Model::generate (greedy: CUDA-graph decode loop)
//   generate_serve()   :349-454  -> Model::generate_serve (lockstep, one launch per projection)
// Sampling (temperature > 0) follows the reference's host algorithm (:263-303, :368-406) on
// logits copied back, so the same seed draws the same tokens.
#include "model.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"
#include "tp.h"

namespace mmfree_cuda {

namespace {

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("cuda: ") + what + ": " + cudaGetErrorString(e));
}
#define CK(call) ck((call), #call)

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

const char* kProjTags[6] = {"i_proj", "f_proj", "g_proj", "o_proj", "gate_proj", "down_proj"};

}  // namespace

Model::Model(const std::string& blob_path, int device, bool fixed, int frac_bits, const TpSpec& tp)
    : device_(device), fixed_(fixed) {
  if (frac_bits < 0 || frac_bits > 30) throw std::runtime_error("frac_bits must be in [0, 30]");
  qs_ = static_cast<float>(1u << frac_bits);
  CK(cudaSetDevice(device));
  Blob blob(blob_path);
  cfg_ = blob.config();
  H_ = static_cast<int>(cfg_.hidden_size);
  I_ = static_cast<int>(cfg_.intermediate_size);
  V_ = static_cast<int>(cfg_.vocab_size);
  L_ = static_cast<int>(cfg_.num_hidden_layers);
  eps_ = cfg_.rms_norm_eps;
  if (H_ <= 0 || I_ <= 0 || V_ <= 0 || L_ <= 0) throw std::runtime_error("weights: bad config");
  if (tp.world > 1) {
    // shards of whole 32-row weight groups, and no SIMD tails inside a shard (H, I multiples
    // of 8 keep every elementwise call of the reference free of tails)
    if (tp.rank < 0 || tp.rank >= tp.world || !tp.nccl_id)
      throw std::invalid_argument("tensor parallel: bad rank, world size or NCCL id");
    if (H_ % (32 * tp.world) != 0 || I_ % (32 * tp.world) != 0)
      throw std::invalid_argument("tensor parallel: hidden and intermediate sizes must be "
                                  "multiples of 32 x world size");
    tp_rank_ = tp.rank;
    tp_world_ = tp.world;
    Hs_ = H_ / tp.world;
    Is_ = I_ / tp.world;
  } else {
    Hs_ = H_;
    Is_ = I_;
  }
  if (padded_k(std::max(H_, I_)) * 4 > 227 * 1024)
    throw std::runtime_error("hidden/intermediate size too large for the prep kernel");
  CK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  CK(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, device));
  {
    const char* env = std::getenv("MMFREE_FUSED_DECODE");
    fused_ok_ = !(env && env[0] == '0');
    const char* penv = std::getenv("MMFREE_PDL");
    pdl_ = !(penv && penv[0] == '0');
    const char* cenv = std::getenv("MMFREE_PERSIST");
    persist_ok_ = cenv && cenv[0] == '1';
    const char* menv = std::getenv("MMFREE_MIX_IN_PREP");
    mix_prep_ok_ = !(menv && menv[0] == '0');
    const char* senv = std::getenv("MMFREE_HOST_SAMPLING");
    host_sampling_ = senv && senv[0] == '1';
    const char* fenv = std::getenv("MMFREE_FLOAT_TC");
    float_tc_ = !(fenv && fenv[0] == '0');
  }
  CK(cudaMalloc(&dec_part_v_, sizeof(float) * kDecMaxRows * 2 * 1024));
  CK(cudaMalloc(&dec_part_i_, sizeof(int) * kDecMaxRows * 2 * 1024));
  CK(cudaMalloc(&err_, 64));
  CK(cudaMemsetAsync(err_, 0, 64, stream_));
  pos_ = reinterpret_cast<int64_t*>(reinterpret_cast<char*>(err_) + 8);
  done_ = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(err_) + 16);
  persist_bar_ = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(err_) + 24);

  // ---- fp32 tensors: one arena
  struct FpItem { std::string name; size_t n; const float** dst; };
  std::vector<FpItem> fps;
  layers_.resize(L_);
  const size_t H = H_, I = I_, V = V_;
  auto expect = [&](const std::string& name, std::vector<size_t> shape, bool i8) {
    const BlobTensor& t = blob.get(name);
    if (t.is_int8 != i8 || t.numel() != [&] { size_t n = 1; for (auto s : shape) n *= s; return n; }())
      throw std::runtime_error("weights: unexpected dtype/shape for " + name);
    return &t;
  };
  expect("model.embeddings", {V, H}, false);
  fps.push_back({"model.embeddings", V * H, &emb_});
  expect("model.norm.w", {H}, false);
  fps.push_back({"model.norm.w", H, &final_norm_});
  expect("lm_head.normw", {H}, false);
  fps.push_back({"lm_head.normw", H, &lm_head_.normw});
  const bool use_lb = cfg_.use_lower_bound && blob.has("lower_bounds");
  if (cfg_.use_lower_bound) expect("lower_bounds", {size_t(L_), H}, false);
  const float* lb_base = nullptr;
  if (use_lb) fps.push_back({"lower_bounds", size_t(L_) * H, &lb_base});
  for (int l = 0; l < L_; ++l) {
    const std::string p = "model.layers." + std::to_string(l);
    Layer& ly = layers_[l];
    fps.push_back({p + ".attn_norm.w", H, &ly.attn_norm});
    fps.push_back({p + ".mlp_norm.w", H, &ly.mlp_norm});
    fps.push_back({p + ".g_norm.w", H, &ly.g_norm});
    for (int j = 0; j < 6; ++j) {
      const size_t in = j == kDown ? I : H;
      fps.push_back({p + "." + kProjTags[j] + ".normw", in, &ly.p[j].normw});
    }
  }
  size_t fp_total = 0;
  for (auto& f : fps) {
    expect(f.name, {f.n}, false);
    fp_total += align256(f.n * 4);
  }
  CK(cudaMalloc(&fp_arena_, fp_total));
  {
    char* cur = reinterpret_cast<char*>(fp_arena_);
    for (auto& f : fps) {
      const BlobTensor& t = blob.get(f.name);
      // stream-ordered: a blocking cudaMemcpy from pageable memory may return before its
      // DMA lands, and nothing orders the legacy stream before this non-blocking stream
      CK(cudaMemcpyAsync(cur, blob.data(t), f.n * 4, cudaMemcpyHostToDevice, stream_));
      *f.dst = reinterpret_cast<const float*>(cur);
      cur += align256(f.n * 4);
    }
  }
  for (int l = 0; l < L_; ++l) layers_[l].lb = (use_lb && l > 0) ? lb_base + size_t(l) * H : nullptr;

  // ---- ternary weights: upload int8, repack to the tiled 2-bit format. With tensor
  // parallelism a projection holds this rank's shard: whole (lm_head), a block of output rows
  // (column-parallel), the two row blocks of a SwiGLU pair (gate_proj), or a block of input
  // columns (row-parallel o/down in Float).
  enum ShardKind { kWhole = 0, kRows, kGatePair, kCols };
  struct WItem { std::string tag; size_t out, in; Proj* p; int kind; size_t sout, sin, off; };
  std::vector<WItem> ws;
  const size_t Hs = Hs_, Is = Is_, r = tp_rank_;
  ws.push_back({"lm_head", V, H, &lm_head_, kWhole, V, H, 0});
  for (int l = 0; l < L_; ++l) {
    const std::string p = "model.layers." + std::to_string(l);
    for (int j = 0; j < 6; ++j) {
      size_t out = H, in = H;
      if (j == kGate) out = 2 * I;
      if (j == kDown) in = I;
      WItem w{p + "." + kProjTags[j], out, in, &layers_[l].p[j], kWhole, out, in, 0};
      if (tp_world_ > 1) {
        if (j == kGate) w = {w.tag, out, in, w.p, kGatePair, 2 * Is, in, r * Is};
        else if (j == kDown && !fixed_) w = {w.tag, out, in, w.p, kCols, H, Is, r * Is};
        else if (j == kO && !fixed_) w = {w.tag, out, in, w.p, kCols, H, Hs, r * Hs};
        else w = {w.tag, out, in, w.p, kRows, Hs, in, r * Hs};
      }
      ws.push_back(w);
    }
  }
  size_t max_i8 = 0;
  packed_bytes_ = 0;
  for (auto& w : ws) {
    const BlobTensor& t = blob.get(w.tag + ".wq");
    if (!(t.is_int8 || t.is_packed) || t.shape.size() != 2 || t.shape[0] != w.out || t.shape[1] != w.in)
      throw std::runtime_error("weights: unexpected dtype/shape for " + w.tag + ".wq");
    if (t.is_packed && w.kind != kWhole)
      throw std::invalid_argument("tensor parallel: needs the int8 model.mmfree blob, not model.mmfree2");
    expect(w.tag + ".scale_w", {1}, false);
    if (!t.is_packed) max_i8 = std::max(max_i8, w.sout * w.sin);
    packed_bytes_ += static_cast<size_t>(packed_bytes(w.sout, w.sin));
  }
  CK(cudaMalloc(&arena_, packed_bytes_));
  int8_t* staging = nullptr;  // int8 upload buffer of the repack (none for model.mmfree2)
  if (max_i8) CK(cudaMalloc(&staging, max_i8));
  {
    char* cur = static_cast<char*>(arena_);
    for (auto& w : ws) {
      const BlobTensor& t = blob.get(w.tag + ".wq");
      const auto* src = static_cast<const int8_t*>(blob.data(t));
      if (t.is_packed) {  // model.mmfree2: already in the device format
        CK(cudaMemcpyAsync(cur, src, packed_bytes(w.out, w.in), cudaMemcpyHostToDevice, stream_));
      } else {
        switch (w.kind) {
          case kWhole:
            CK(cudaMemcpyAsync(staging, src, w.out * w.in, cudaMemcpyHostToDevice, stream_));
            break;
          case kRows:
            CK(cudaMemcpyAsync(staging, src + w.off * w.in, w.sout * w.in, cudaMemcpyHostToDevice, stream_));
            break;
          case kGatePair: {  // gate rows [off, off + Is) then up rows [I + off, I + off + Is)
            const size_t half = w.sout / 2 * w.in;
            CK(cudaMemcpyAsync(staging, src + w.off * w.in, half, cudaMemcpyHostToDevice, stream_));
            CK(cudaMemcpyAsync(staging + half, src + (I + w.off) * w.in, half, cudaMemcpyHostToDevice,
                               stream_));
            break;
          }
          case kCols:
            CK(cudaMemcpy2DAsync(staging, w.sin, src + w.off, w.in, w.sin, w.sout,
                                 cudaMemcpyHostToDevice, stream_));
            break;
        }
        CK(launch_repack(cur, staging, w.sout, w.sin, err_, stream_));
      }
      float s;
      std::memcpy(&s, blob.data(blob.get(w.tag + ".scale_w")), 4);
      w.p->w = cur;
      w.p->scale_w = s;
      w.p->in = static_cast<int>(w.sin);
      w.p->out = static_cast<int>(w.sout);
      cur += packed_bytes(w.sout, w.sin);
    }
  }
  uint32_t err = 0;
  CK(cudaMemcpyAsync(&err, err_, 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  cudaFree(staging);
  if (err & kErrNotTernary) throw std::runtime_error("weights: a wq entry is outside {-1,0,1}");
  // every rank reaches this point: the communicator's set-up is collective
  if (tp_world_ > 1) tp_ = std::make_unique<TpComm>(tp.nccl_id, tp.rank, tp.world);
}

Model::~Model() {
  cudaSetDevice(device_);
  drop_graph();
  for (cudaEvent_t e : ev_free_) cudaEventDestroy(e);
  if (stream_) cudaStreamSynchronize(stream_);
  cudaFree(arena_);
  cudaFree(fp_arena_);
  cudaFree(ws_);
  cudaFree(state_);
  cudaFree(loop_ids_);
  cudaFree(err_);
  cudaFree(dec_part_v_);
  cudaFree(dec_part_i_);
  cudaFree(persist_tab_);
  cudaFree(tp_ws_);
  cudaFree(chunk_ws_);
  cudaFree(uni_);
  tp_.reset();
  if (pinned_) cudaFreeHost(pinned_);
  if (stream_) cudaStreamDestroy(stream_);
}

void Model::drop_graph() {
  if (graph_) cudaGraphExecDestroy(graph_);
  graph_ = nullptr;
  graph_b_ = 0;
  graph_stride_ = 0;
  persist_b_ = 0;  // the persistent phase table holds buffer pointers: rebuild it
  persist_stride_ = -1;
}

void Model::ensure_ws(size_t rows) {
  if (rows <= ws_rows_) return;
  drop_graph();
  CK(cudaStreamSynchronize(stream_));
  cudaFree(ws_);
  ws_ = nullptr;
  const size_t H = H_, I = I_, V = V_;
  const size_t Kp = static_cast<size_t>(padded_k(std::max(H_, I_)));
  size_t sz = 0;
  auto carve = [&](size_t bytes) { size_t o = sz; sz += align256(bytes); return o; };
  size_t o_h = carve(rows * H * 4), o_resid = carve(rows * H * 4), o_ib = carve(rows * H * 4),
         o_fb = carve(rows * H * 4), o_gb = carve(rows * H * 4), o_recur = carve(rows * H * 4),
         o_y = carve(rows * 2 * I * 4), o_z = carve(rows * I * 4), o_lg = carve(rows * V * 4),
         o_hl = carve(rows * H * 4), o_ids = carve(rows * 8);
  size_t o_pl[3], o_rs[3], o_yf[3];
  for (int j = 0; j < 3; ++j) {
    o_pl[j] = carve((fixed_ ? 2 : 4) * rows * Kp);  // u8 planes, or Float's bf16 hi / lo planes
    o_rs[j] = carve(rows * 4);
    o_yf[j] = fixed_ ? 0 : carve(rows * Kp * 4);
  }
  CK(cudaMalloc(&ws_, sz));
  char* b = static_cast<char*>(ws_);
  h_ = reinterpret_cast<float*>(b + o_h);
  resid_ = reinterpret_cast<float*>(b + o_resid);
  ib_ = reinterpret_cast<float*>(b + o_ib);
  fb_ = reinterpret_cast<float*>(b + o_fb);
  gb_ = reinterpret_cast<float*>(b + o_gb);
  recur_ = reinterpret_cast<float*>(b + o_recur);
  y_ = reinterpret_cast<float*>(b + o_y);
  z_ = reinterpret_cast<float*>(b + o_z);
  logits_ = reinterpret_cast<float*>(b + o_lg);
  hl_ = reinterpret_cast<float*>(b + o_hl);
  ids_ = reinterpret_cast<int64_t*>(b + o_ids);
  for (int j = 0; j < 3; ++j) {
    planes_[j] = reinterpret_cast<int8_t*>(b + o_pl[j]);
    rowsum_[j] = reinterpret_cast<int32_t*>(b + o_rs[j]);
    yf_[j] = fixed_ ? nullptr : reinterpret_cast<float*>(b + o_yf[j]);
  }
  ws_rows_ = rows;
}

void* Model::chunk_ws(int nseq, int len, int H) {
  if (fixed_ || len <= 1) return nullptr;  // FixedQ510 keeps the reference's serial order
  const size_t need = mixer_chunk_bytes(nseq, len, H);
  if (need > chunk_bytes_) {
    CK(cudaStreamSynchronize(stream_));
    cudaFree(chunk_ws_);
    chunk_ws_ = nullptr;
    chunk_bytes_ = 0;
    CK(cudaMalloc(&chunk_ws_, need));
    chunk_bytes_ = need;
  }
  return chunk_ws_;
}

void Model::float_state(size_t elems) {
  if (elems > state_elems_) {
    drop_graph();
    CK(cudaStreamSynchronize(stream_));
    cudaFree(state_);
    state_ = nullptr;
    CK(cudaMalloc(&state_, elems * 4));
    state_elems_ = elems;
  }
  CK(cudaMemsetAsync(state_, 0, elems * 4, stream_));
}

void Model::loop_ids(size_t elems) {
  if (elems <= loop_ids_elems_) return;
  drop_graph();
  CK(cudaStreamSynchronize(stream_));
  cudaFree(loop_ids_);
  loop_ids_ = nullptr;
  CK(cudaMalloc(&loop_ids_, elems * 8));
  loop_ids_elems_ = elems;
}

void Model::pinned(size_t elems) {
  if (elems <= pinned_elems_) return;
  CK(cudaStreamSynchronize(stream_));
  if (pinned_) cudaFreeHost(pinned_);
  pinned_ = nullptr;
  CK(cudaMallocHost(&pinned_, elems * 8));
  pinned_elems_ = elems;
}

void Model::check_errors() {
  uint32_t err = 0;
  CK(cudaMemcpyAsync(&err, err_, 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  if (err) {
    CK(cudaMemsetAsync(err_, 0, 4, stream_));
    CK(cudaStreamSynchronize(stream_));
    if (err & kErrBadToken) throw std::out_of_range("token id outside [0, vocab_size)");
    throw std::runtime_error("device error flag set");
  }
}

template <class F>
void Model::timed(int cls, double bytes, double ops, F&& launch) {
  if (!prof_on_) {
    launch();
    return;
  }
  auto take = [&] {
    if (ev_free_.empty()) {
      cudaEvent_t e;
      CK(cudaEventCreate(&e));
      return e;
    }
    cudaEvent_t e = ev_free_.back();
    ev_free_.pop_back();
    return e;
  };
  Mark m{cls, take(), take(), bytes, ops};
  CK(cudaEventRecord(m.a, stream_));
  launch();
  CK(cudaEventRecord(m.b, stream_));
  marks_.push_back(m);
}

void Model::prep(const PrepArgs& p) {
  // algorithmic bytes: the row in (+ the gate operand), weights, planes/activations out
  const double rows = p.M, K = p.K;
  const double out_row = p.fixed ? 2.0 * padded_k(p.K) + 4 : 4.0 * padded_k(p.K);
  const double bytes = rows * K * 4 * (p.o ? 2 : 1) + K * 4 * (p.nproj + (p.prew ? 1 : 0)) +
                       rows * out_row * p.nproj;
  PrepArgs q = p;
  q.pdl = pdl_;
  q.err = err_;
  // the BitLinear of these rows runs on the tensor cores: FixedQ510 low planes as lo - 128,
  // Float activations as bf16 hi / lo planes
  q.lo_signed = fixed_ && tc_rows(q.M);
  q.bf16 = !fixed_ && tc_rows(q.M);
  timed(kClsPrep, bytes, 0, [&] { CK(launch_prep(q, stream_)); });
}

const char* Model::class_name(int c) {
  static const char* n[kNumClasses] = {"prep", "bitlinear_matmul", "lm_head_matmul", "mixer",
                                       "swiglu", "embed", "argmax", "decode_step"};
  return (c >= 0 && c < kNumClasses) ? n[c] : "?";
}

MatmulArgs Model::mm_args(const Proj& p, int plane, float* out, int M, const float* resid) const {
  MatmulArgs a;
  a.w = p.w;
  a.planes = planes_[plane];
  a.rowsum = rowsum_[plane];
  a.yf = yf_[plane];
  a.M = M;
  a.N = p.out;
  a.K = p.in;
  a.scale = fixed_ ? 1.0f / (qs_ * p.scale_w) : 1.0f / p.scale_w;
  a.out = out;
  a.ldo = p.out;
  a.resid = resid;
  a.ldr = p.out;
  a.fixed = fixed_;
  a.allow_tc = true;
  a.err = err_;
  a.pdl = pdl_;
  a.lo_signed = fixed_ && tc_rows(M);
  a.bf16 = !fixed_ && tc_rows(M);
  return a;
}

void Model::bitlinear(const Proj& p, int plane, float* out, int M, const float* resid) {
  const MatmulArgs a = mm_args(p, plane, out, M, resid);
  // algorithmic bytes (2-bit weights, activations in, outputs out) and 2*M*K*N ops
  const double K = p.in, N = p.out;
  const double bytes = K * N / 4 + 4.0 * M * K + 4.0 * M * N * (resid ? 2 : 1);
  timed(&p == &lm_head_ ? kClsLmHead : kClsMatmul, bytes, 2.0 * M * K * N,
        [&] { CK(launch_matmul(a, stream_)); });
}

bool Model::tc_rows(int M) const { return M >= kTcMinRows && (fixed_ || float_tc_); }

void Model::bitlinear_ifg(const Layer& ly, int M) {
  if (!tc_rows(M)) {
    bitlinear(ly.p[kI], 0, ib_, M, nullptr);
    bitlinear(ly.p[kF], 1, fb_, M, nullptr);
    bitlinear(ly.p[kG], 2, gb_, M, nullptr);
    return;
  }
  const MatmulArgs a[3] = {mm_args(ly.p[kI], 0, ib_, M, nullptr), mm_args(ly.p[kF], 1, fb_, M, nullptr),
                           mm_args(ly.p[kG], 2, gb_, M, nullptr)};
  const double K = H_, N = H_;
  const double bytes = 3 * (K * N / 4 + 4.0 * M * K + 4.0 * M * N);
  timed(kClsMatmul, bytes, 6.0 * M * K * N,
        [&] { CK(launch_matmul_tc_group(a, 3, 0, 0, sms_, stream_)); });
}

void Model::bitlinear_gate_swiglu(const Layer& ly, int M, int seg_rows) {
  if (!tc_rows(M) || I_ % 64 != 0) {
    bitlinear(ly.p[kGate], 0, y_, M, nullptr);
    timed(kClsSwiglu, 12.0 * M * I_, 0,
          [&] { CK(launch_swiglu_split(z_, y_, M, I_, seg_rows, stream_, pdl_)); });
    return;
  }
  MatmulArgs a = mm_args(ly.p[kGate], 0, z_, M, nullptr);
  a.ldo = I_;
  const double K = H_, N = 2.0 * I_;
  const double bytes = K * N / 4 + 4.0 * M * K + 4.0 * M * I_;
  timed(kClsMatmul, bytes, 2.0 * M * K * N, [&] {
    CK(launch_matmul_tc_group(&a, 1, I_, static_cast<int64_t>(seg_rows) * I_, sms_, stream_));
  });
}

template <class StateFn>
void Model::layers(int nseq, int len, int seg_rows, StateFn state) {
  if (tp_) {
    layers_tp(nseq, len, seg_rows);
    return;
  }
  const int rows = nseq * len;
  for (int l = 0; l < L_; ++l) {
    const Layer& ly = layers_[l];
    PrepArgs p;
    p.fixed = fixed_;
    p.qs = qs_;
    p.eps = eps_;
    p.M = rows;
    for (int j = 0; j < 3; ++j) {
      p.planes[j] = planes_[j];
      p.rowsum[j] = rowsum_[j];
      p.yf[j] = yf_[j];
    }
    // attention: hs = rmsnorm(h) * attn_norm; i/f/g BitLinear cluster on hs
    p.x = h_;
    p.prew = ly.attn_norm;
    p.K = H_;
    p.nproj = 3;
    p.normw[0] = ly.p[kI].normw;
    p.normw[1] = ly.p[kF].normw;
    p.normw[2] = ly.p[kG].normw;
    prep(p);
    bitlinear_ifg(ly, rows);
    // one decode step: the token mixer runs inside the o_proj prep (while its norm chain runs)
    const bool mix_in_prep = mix_prep_ok_ && len == 1 && H_ % 4 == 0 && H_ >= 8;
    if (!mix_in_prep)
      timed(kClsMixer, 4.0 * rows * H_ * 5 + 8.0 * nseq * H_, 0, [&] {
        CK(launch_mixer(ib_, fb_, recur_, state(l), ly.lb, nseq, len, H_, seg_rows, stream_, pdl_,
                        chunk_ws(nseq, len, H_)));
      });
    // o_proj on g_norm(g) * silu(recurrence); resid = h + o
    p.x = gb_;
    p.o = mix_in_prep ? nullptr : recur_;
    p.prew = ly.g_norm;
    p.nproj = 1;
    p.normw[0] = ly.p[kO].normw;
    if (mix_in_prep) {
      p.mix_i = ib_;
      p.mix_f = fb_;
      p.mix_state = state(l);
      p.mix_lb = ly.lb;
      p.mix_out = recur_;
      p.mix_seg_rows = seg_rows;
    }
    prep(p);
    p.mix_i = p.mix_f = p.mix_lb = nullptr;
    p.mix_state = p.mix_out = nullptr;
    bitlinear(ly.p[kO], 0, resid_, rows, h_);
    // mlp: gate_proj on rmsnorm(resid) * mlp_norm, swiglu, down_proj; h = resid + down
    p.x = resid_;
    p.o = nullptr;
    p.prew = ly.mlp_norm;
    p.normw[0] = ly.p[kGate].normw;
    prep(p);
    bitlinear_gate_swiglu(ly, rows, seg_rows);
    p.x = z_;
    p.prew = nullptr;
    p.K = I_;
    p.normw[0] = ly.p[kDown].normw;
    prep(p);
    bitlinear(ly.p[kDown], 0, h_, rows, resid_);
    if (trace_) {  // recurrence output, residual after o_proj, layer output
      const size_t th = static_cast<size_t>(rows) * H_;
      float* tr = trace_ + th * (1 + 3 * static_cast<size_t>(l));
      CK(cudaMemcpyAsync(tr, recur_, th * 4, cudaMemcpyDeviceToHost, stream_));
      CK(cudaMemcpyAsync(tr + th, resid_, th * 4, cudaMemcpyDeviceToHost, stream_));
      CK(cudaMemcpyAsync(tr + 2 * th, h_, th * 4, cudaMemcpyDeviceToHost, stream_));
    }
  }
}

void Model::tp_only_prefill(const char* what) const {
  if (tp_)
    throw std::logic_error(std::string(what) + ": a tensor-parallel handle runs prefills only "
                                               "(forward, forward_last, serve_begin)");
}

void Model::ensure_tp_ws(size_t rows) {
  if (rows <= tp_rows_) return;
  CK(cudaStreamSynchronize(stream_));
  cudaFree(tp_ws_);
  tp_ws_ = nullptr;
  const size_t H = H_, I = I_, Hs = Hs_, Is = Is_;
  size_t sz = 0;
  auto carve = [&](size_t floats) { size_t o = sz; sz += align256(floats * 4); return o; };
  const size_t o_g = carve(rows * H), o_rec = carve(rows * H), o_st = carve(rows * std::max(H, I)),
               o_rs = carve(rows * Hs), o_zs = carve(rows * Is), o_hs = carve(rows * Hs),
               o_ts = carve(rows * Hs), o_ss = carve(rows * 4);
  CK(cudaMalloc(&tp_ws_, sz));
  char* b = static_cast<char*>(tp_ws_);
  tp_g_ = reinterpret_cast<float*>(b + o_g);
  tp_rec_ = reinterpret_cast<float*>(b + o_rec);
  tp_stage_ = reinterpret_cast<float*>(b + o_st);
  tp_rs_ = reinterpret_cast<float*>(b + o_rs);
  tp_zs_ = reinterpret_cast<float*>(b + o_zs);
  tp_hs_ = reinterpret_cast<float*>(b + o_hs);
  tp_ts_ = reinterpret_cast<float*>(b + o_ts);
  tp_ss_ = reinterpret_cast<float*>(b + o_ss);
  tp_rows_ = rows;
}

void Model::tp_gather(float* full, const float* slice, int rows, int n) {
  tp_->all_gather(slice, tp_stage_, static_cast<size_t>(rows) * n * 4, stream_);
  CK(launch_interleave(full, tp_stage_, tp_world_, rows, n, stream_));
}

// One prefill over this rank's shards (hgrn_model.cpp:80-195 split as tp.h describes). The
// row transforms and exact norms run on whole rows (replicated on every rank); h, the residual
// and z are whole on every rank between the exchanges.
void Model::layers_tp(int nseq, int len, int seg_rows) {
  const int rows = nseq * len;
  ensure_tp_ws(static_cast<size_t>(rows));
  const int H = H_, Hs = Hs_, Is = Is_;
  const size_t hoff = static_cast<size_t>(tp_rank_) * Hs, ioff = static_cast<size_t>(tp_rank_) * Is;
  float* ss_a = tp_ss_;          // [rows] sums of squares
  float* ss_b = tp_ss_ + rows;
  auto prep_full = [&](const float* x, const float* o, const float* prew, int K, int nproj,
                       const float* nw0, const float* nw1, const float* nw2) {
    PrepArgs p;
    p.fixed = fixed_;
    p.qs = qs_;
    p.eps = eps_;
    p.M = rows;
    p.x = x;
    p.o = o;
    p.prew = prew;
    p.K = K;
    p.nproj = nproj;
    p.normw[0] = nw0;
    p.normw[1] = nw1;
    p.normw[2] = nw2;
    for (int j = 0; j < 3; ++j) {
      p.planes[j] = planes_[j];
      p.rowsum[j] = rowsum_[j];
      p.yf[j] = yf_[j];
    }
    prep(p);
  };
  // a shard's BitLinear into out (row stride ldo), optionally + resid (row stride ldr);
  // from_yf: Float row-parallel inputs written as fp32 activations by launch_norm_slice (below
  // the tensor-core row count: the CUDA-core kernel reads them)
  auto shard_mm = [&](const Proj& pj, int plane, float* out, int ldo, const float* resid, int ldr,
                      bool from_yf = false) {
    MatmulArgs a = mm_args(pj, plane, out, rows, resid);
    a.ldo = ldo;
    a.ldr = ldr;
    if (from_yf) a.allow_tc = false;
    timed(kClsMatmul, 0, 2.0 * rows * pj.in * pj.out, [&] { CK(launch_matmul(a, stream_)); });
  };
  for (int l = 0; l < L_; ++l) {
    const Layer& ly = layers_[l];
    const float* lb = ly.lb ? ly.lb + hoff : nullptr;
    // i/f/g column shards on whole rows of rmsnorm(h) * attn_norm
    prep_full(h_, nullptr, ly.attn_norm, H, 3, ly.p[kI].normw, ly.p[kF].normw, ly.p[kG].normw);
    bitlinear_ifg(ly, rows);  // shards: N = Hs each, into ib_ / fb_ / gb_ [rows][Hs]
    CK(launch_mixer(ib_, fb_, recur_, nullptr, lb, nseq, len, Hs, seg_rows, stream_, pdl_,
                    chunk_ws(nseq, len, Hs)));
    if (fixed_) {
      // whole rows of g and the recurrence for the exact g_norm chain, then o_proj columns
      tp_gather(tp_g_, gb_, rows, Hs);
      tp_gather(tp_rec_, recur_, rows, Hs);
      prep_full(tp_g_, tp_rec_, ly.g_norm, H, 1, ly.p[kO].normw, nullptr, nullptr);
      shard_mm(ly.p[kO], 0, tp_rs_, Hs, h_ + hoff, H);
      tp_gather(resid_, tp_rs_, rows, Hs);
    } else {
      // g_norm and o_proj's norm from all-reduced partial sums of squares; o_proj rows
      CK(launch_row_sumsq(ss_a, gb_, rows, Hs, Hs, stream_));
      tp_->all_reduce_f32(ss_a, rows, stream_);
      CK(launch_gate_slice(tp_ts_, ss_b, gb_, recur_, ss_a, ly.g_norm + hoff, rows, Hs, H, eps_,
                           stream_));
      tp_->all_reduce_f32(ss_b, rows, stream_);
      const int kp = static_cast<int>(padded_k(Hs));
      if (tc_rows(rows)) {  // bf16 planes for the tensor cores
        CK(launch_norm_slice_planes(planes_[0], tp_ts_, ss_b, ly.p[kO].normw + hoff, rows, Hs, kp, H, eps_,
                                    stream_));
        shard_mm(ly.p[kO], 0, resid_, H, nullptr, 0);  // partial [rows][H]
      } else {
        CK(launch_norm_slice(yf_[0], tp_ts_, ss_b, ly.p[kO].normw + hoff, rows, Hs, kp, H, eps_, stream_));
        shard_mm(ly.p[kO], 0, resid_, H, nullptr, 0, true);
      }
      tp_->all_reduce_f32(resid_, static_cast<size_t>(rows) * H, stream_);
      CK(launch_add(resid_, h_, resid_, static_cast<int64_t>(rows) * H, stream_));
    }
    // gate_proj SwiGLU pairs of this rank's Is columns of z
    prep_full(resid_, nullptr, ly.mlp_norm, H, 1, ly.p[kGate].normw, nullptr, nullptr);
    if (tc_rows(rows) && Is % 64 == 0) {
      MatmulArgs a = mm_args(ly.p[kGate], 0, tp_zs_, rows, nullptr);
      a.ldo = Is;
      timed(kClsMatmul, 0, 2.0 * rows * H * 2.0 * Is, [&] {
        CK(launch_matmul_tc_group(&a, 1, Is, static_cast<int64_t>(seg_rows) * Is, sms_, stream_));
      });
    } else {
      shard_mm(ly.p[kGate], 0, y_, 2 * Is, nullptr, 0);
      CK(launch_swiglu_split(tp_zs_, y_, rows, Is, seg_rows, stream_, pdl_));
    }
    if (fixed_) {
      // whole rows of z for the exact down_proj norm, then down_proj columns; h whole again
      tp_gather(z_, tp_zs_, rows, Is);
      prep_full(z_, nullptr, nullptr, I_, 1, ly.p[kDown].normw, nullptr, nullptr);
      shard_mm(ly.p[kDown], 0, tp_hs_, Hs, resid_ + hoff, H);
      tp_gather(h_, tp_hs_, rows, Hs);
    } else {
      CK(launch_row_sumsq(ss_a, tp_zs_, rows, Is, Is, stream_));
      tp_->all_reduce_f32(ss_a, rows, stream_);
      const int kp = static_cast<int>(padded_k(Is));
      if (tc_rows(rows)) {
        CK(launch_norm_slice_planes(planes_[0], tp_zs_, ss_a, ly.p[kDown].normw + ioff, rows, Is, kp, I_,
                                    eps_, stream_));
        shard_mm(ly.p[kDown], 0, h_, H, nullptr, 0);  // partial [rows][H]
      } else {
        CK(launch_norm_slice(yf_[0], tp_zs_, ss_a, ly.p[kDown].normw + ioff, rows, Is, kp, I_, eps_,
                             stream_));
        shard_mm(ly.p[kDown], 0, h_, H, nullptr, 0, true);
      }
      tp_->all_reduce_f32(h_, static_cast<size_t>(rows) * H, stream_);
      CK(launch_add(h_, resid_, h_, static_cast<int64_t>(rows) * H, stream_));
    }
  }
}

void Model::forward_trace(const int64_t* ids, size_t T, float* logits, float* trace) {
  tp_only_prefill("forward_trace");
  CK(cudaSetDevice(device_));
  if (T == 0) throw std::invalid_argument("forward: empty input");
  for (size_t t = 0; t < T; ++t)
    if (ids[t] < 0 || ids[t] >= V_) throw std::out_of_range("token id outside [0, vocab_size)");
  ensure_ws(T);
  CK(cudaMemcpyAsync(ids_, ids, T * 8, cudaMemcpyHostToDevice, stream_));
  CK(launch_embed(h_, emb_, ids_, static_cast<int>(T), H_, V_, err_, stream_));
  CK(cudaMemcpyAsync(trace, h_, T * H_ * 4, cudaMemcpyDeviceToHost, stream_));
  trace_ = trace;
  try {
    layers(1, static_cast<int>(T), static_cast<int>(T), [](int) { return static_cast<float*>(nullptr); });
  } catch (...) {
    trace_ = nullptr;
    throw;
  }
  trace_ = nullptr;
  head(h_, static_cast<int>(T));
  CK(cudaMemcpyAsync(logits, logits_, T * V_ * 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  check_errors();
}

void Model::head(const float* rows, int M) {
  PrepArgs p;
  p.fixed = fixed_;
  p.qs = qs_;
  p.eps = eps_;
  p.M = M;
  p.x = rows;
  p.prew = final_norm_;
  p.K = H_;
  p.nproj = 1;
  p.normw[0] = lm_head_.normw;
  p.planes[0] = planes_[0];
  p.rowsum[0] = rowsum_[0];
  p.yf[0] = yf_[0];
  prep(p);
  bitlinear(lm_head_, 0, logits_, M, nullptr);
}

void Model::decode_graph_step(int B, int64_t stride) {
  auto pick = [&] {  // the next token of every stream: sampled, or the greedy argmax
    if (samp_) {
      timed(kClsArgmax, 4.0 * B * V_, 0, [&] {
        CK(launch_sample_at(loop_ids_, stride, pos_, done_, true, 0, logits_, B, V_, V_, uni_, stride,
                            samp_->temperature, samp_->top_k, stream_, pdl_));
      });
    } else {
      timed(kClsArgmax, 4.0 * B * V_, 0, [&] {
        CK(launch_argmax_at(loop_ids_, stride, pos_, done_, logits_, B, V_, V_, stream_, pdl_));
      });
    }
  };
  if (!samp_ && fused_decode(B) && persist_ok_ && persist_b_ == B && persist_stride_ == stride &&
      persist_grid_ > 0) {
    // the whole step in one cooperative launch (table prepared by persist_ready)
    timed(kClsStep, static_cast<double>(packed_bytes_), 0, [&] {
      CK(launch_dec_persist(persist_tab_, persist_n_, B, persist_bar_, err_, persist_smem_,
                            persist_grid_, stream_));
    });
    return;
  }
  timed(kClsEmbed, 8.0 * B * H_, 0, [&] {
    CK(launch_embed_at(h_, emb_, loop_ids_, stride, pos_, B, H_, V_, err_, stream_, pdl_));
  });
  if (fused_decode(B)) {
    fused_step(B, stride);  // with samp_ its head phase writes logits only
    if (samp_) pick();
    return;
  }
  layers(B, 1, B, [&](int l) { return state_ + static_cast<size_t>(l) * B * H_; });
  head(h_, B);
  pick();
}

bool Model::fused_decode(int B) const {
  return fused_ok_ && B <= kDecMaxRows && I_ % 32 == 0;
}

std::vector<DecArgs> Model::dec_phases(int B, int64_t stride) {
  std::vector<DecArgs> ph;
  auto base = [&](DecArgs& a, int pro, int epi) {
    a.M = B;
    a.eps = eps_;
    a.qs = qs_;
    a.pro = pro;
    a.epi = epi;
    a.fl = fixed_ ? 0 : 1;
  };
  // dequant scale: FixedQ510 1/(2^f scale_w) (bitlinear.cpp:89-94), Float 1/scale_w (:113-116)
  auto scale = [&](float scale_w) { return fixed_ ? 1.0f / (qs_ * scale_w) : 1.0f / scale_w; };
  const size_t BH = static_cast<size_t>(B) * H_;
  for (int l = 0; l < L_; ++l) {
    const Layer& ly = layers_[l];
    DecArgs k1;  // i/f/g + mixer: attn rmsnorm, recurrence step (hgrn_model.cpp:95-150)
    base(k1, kDecProNorm2, kDecEpiMixer);
    k1.x = h_;
    k1.prew = ly.attn_norm;
    for (int j = 0; j < 3; ++j) {
      k1.normw[j] = ly.p[j].normw;
      k1.w[j] = ly.p[j].w;
      k1.scale[j] = scale(ly.p[j].scale_w);
    }
    k1.K = H_;
    k1.N = H_;
    k1.out[0] = recur_;
    k1.out[1] = gb_;
    k1.state = state_ + static_cast<size_t>(l) * BH;
    k1.lb = ly.lb;
    k1.seg = static_cast<int64_t>(BH);
    ph.push_back(k1);

    DecArgs k2;  // o_proj on g_norm(g) * silu(recurrence); resid = h + o (:152-166)
    base(k2, kDecProSwish, kDecEpiResid);
    k2.x = gb_;
    k2.o = recur_;
    k2.prew = ly.g_norm;
    k2.normw[0] = ly.p[kO].normw;
    k2.w[0] = ly.p[kO].w;
    k2.scale[0] = scale(ly.p[kO].scale_w);
    k2.K = H_;
    k2.N = H_;
    k2.out[0] = resid_;
    k2.resid = h_;
    ph.push_back(k2);

    DecArgs k3;  // gate_proj on mlp rmsnorm(resid), swiglu (:168-185)
    base(k3, kDecProNorm2, kDecEpiSwiglu);
    k3.x = resid_;
    k3.prew = ly.mlp_norm;
    k3.normw[0] = ly.p[kGate].normw;
    k3.w[0] = ly.p[kGate].w;
    k3.scale[0] = scale(ly.p[kGate].scale_w);
    k3.K = H_;
    k3.N = 2 * I_;
    k3.out[0] = z_;
    k3.seg = static_cast<int64_t>(B) * I_;
    ph.push_back(k3);

    DecArgs k4;  // down_proj; h = resid + down (:187-194)
    base(k4, kDecProPlain, kDecEpiResid);
    k4.x = z_;
    k4.normw[0] = ly.p[kDown].normw;
    k4.w[0] = ly.p[kDown].w;
    k4.scale[0] = scale(ly.p[kDown].scale_w);
    k4.K = I_;
    k4.N = H_;
    k4.out[0] = h_;
    k4.resid = resid_;
    ph.push_back(k4);
  }
  DecArgs hd;  // final norm + lm_head + greedy argmax (:304-310, :269-273)
  base(hd, kDecProNorm2, kDecEpiLogits);
  hd.x = h_;
  hd.prew = final_norm_;
  hd.normw[0] = lm_head_.normw;
  hd.w[0] = lm_head_.w;
  hd.scale[0] = scale(lm_head_.scale_w);
  hd.K = H_;
  hd.N = V_;
  hd.out[0] = logits_;
  hd.ids = samp_ ? nullptr : loop_ids_;  // sampled steps: logits only, sample_at follows
  hd.stride = stride;
  hd.pos = pos_;
  hd.done = done_;
  hd.part_v = dec_part_v_;
  hd.part_i = dec_part_i_;
  ph.push_back(hd);
  return ph;
}

bool Model::persist_ready(int B, int64_t stride) {
  if (!fused_decode(B) || !persist_ok_ || samp_) return false;
  if (persist_b_ == B && persist_stride_ == stride) return persist_grid_ > 0;
  std::vector<DecArgs> ph = dec_phases(B, stride);
  // the first phase gathers its rows from the embedding table (and writes h for o_proj)
  ph[0].x = emb_;
  ph[0].xids = loop_ids_;
  ph[0].xstride = stride;
  ph[0].xpos = pos_;
  ph[0].xcopy = h_;
  ph[0].V = V_;
  ph[0].err = err_;
  const size_t smem = dec_persist_plan(ph.data(), static_cast<int>(ph.size()));
  const int grid = smem ? dec_persist_grid(B, smem) : 0;
  if (grid > 2 * 1024) throw std::logic_error("persistent decode: grid above the partials buffer");
  CK(cudaStreamSynchronize(stream_));
  cudaFree(persist_tab_);
  persist_tab_ = nullptr;
  if (grid > 0) {
    CK(cudaMalloc(&persist_tab_, ph.size() * sizeof(DecArgs)));
    CK(cudaMemcpy(persist_tab_, ph.data(), ph.size() * sizeof(DecArgs), cudaMemcpyHostToDevice));
  }
  persist_n_ = static_cast<int>(ph.size());
  persist_smem_ = smem;
  persist_grid_ = grid;
  persist_b_ = B;
  persist_stride_ = stride;
  return grid > 0;
}

// One decode step of B <= 4 streams with the fused kernels of decode.cu, one launch per
// phase, each launched as a programmatic dependent of the previous one.
void Model::fused_step(int B, int64_t stride) {
  for (DecArgs& a : dec_phases(B, stride)) {
    const int units = dec_units(a, a.epi);
    const int grid = std::max(1, std::min(units, 2 * sms_));
    const double wbytes = static_cast<double>(packed_bytes(a.N, a.K)) * (a.epi == kDecEpiMixer ? 3 : 1);
    const double bytes = wbytes + 4.0 * B * a.K * (a.pro == kDecProSwish ? 2 : 1) + 4.0 * B * a.N;
    const double ops = 2.0 * B * a.K * a.N * (a.epi == kDecEpiMixer ? 3 : 1);
    timed(a.epi == kDecEpiLogits ? kClsLmHead : kClsMatmul, bytes, ops,
          [&] { CK(launch_dec(a, a.pro, a.epi, grid, stream_, true)); });
  }
}

std::vector<Model::ClassStats> Model::serve_profile(size_t steps) {
  tp_only_prefill("serve_profile");
  if (serve_b_ == 0) throw std::logic_error("serve_profile without serve_begin");
  const int B = serve_b_;
  const int64_t stride = static_cast<int64_t>(steps) + 1;
  loop_ids(static_cast<size_t>(stride) * B);
  const int64_t zero = 0;
  CK(cudaMemcpy2DAsync(loop_ids_, stride * 8, serve_last_.data(), 8, 8, B, cudaMemcpyHostToDevice,
                       stream_));
  CK(cudaMemcpyAsync(pos_, &zero, 8, cudaMemcpyHostToDevice, stream_));
  marks_.clear();
  persist_ready(B, stride);
  prof_on_ = true;
  try {
    for (size_t s = 0; s < steps; ++s) decode_graph_step(B, stride);
  } catch (...) {
    prof_on_ = false;
    throw;
  }
  prof_on_ = false;
  CK(cudaStreamSynchronize(stream_));
  std::vector<ClassStats> out(kNumClasses);
  for (const Mark& m : marks_) {
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, m.a, m.b));
    ClassStats& c = out[m.cls];
    c.ms += ms;
    c.launches += 1;
    c.bytes += m.bytes;
    c.ops += m.ops;
    ev_free_.push_back(m.a);
    ev_free_.push_back(m.b);
  }
  marks_.clear();
  pinned(static_cast<size_t>(stride) * B);
  CK(cudaMemcpyAsync(pinned_, loop_ids_, static_cast<size_t>(stride) * B * 8, cudaMemcpyDeviceToHost,
                     stream_));
  CK(cudaStreamSynchronize(stream_));
  for (int b = 0; b < B; ++b) serve_last_[b] = pinned_[static_cast<size_t>(b) * stride + steps];
  check_errors();
  return out;
}

namespace {
struct Sampler {
  const Sampling& s;
  size_t V;
  int64_t operator()(const float* lg, std::mt19937_64& rng) const {
    std::uniform_real_distribution<double> uni(0.0, 1.0);
    std::vector<size_t> cand(V);
    std::iota(cand.begin(), cand.end(), size_t(0));
    auto hotter = [&](size_t a, size_t b) { return lg[a] > lg[b]; };
    const size_t k = (s.top_k > 0 && static_cast<size_t>(s.top_k) < V) ? static_cast<size_t>(s.top_k) : V;
    if (k < V) {
      std::nth_element(cand.begin(), cand.begin() + static_cast<std::ptrdiff_t>(k), cand.end(), hotter);
      cand.resize(k);
    }
    float maxl = lg[cand[0]];
    for (size_t j = 1; j < cand.size(); ++j) maxl = std::max(maxl, lg[cand[j]]);
    double sum = 0.0;
    std::vector<double> p(cand.size());
    for (size_t j = 0; j < cand.size(); ++j) {
      p[j] = std::exp((lg[cand[j]] - maxl) / s.temperature);
      sum += p[j];
    }
    const double r = uni(rng) * sum;
    double acc = 0.0;
    for (size_t j = 0; j < cand.size(); ++j) {
      acc += p[j];
      if (r <= acc) return static_cast<int64_t>(cand[j]);
    }
    return static_cast<int64_t>(cand.back());
  }
};
}  // namespace

std::vector<int64_t> Model::generate(const int64_t* ids, size_t n, size_t new_tokens,
                                     int64_t eos_id, const Sampling& samp,
                                     const std::function<void(int64_t)>* on_token) {
  tp_only_prefill("generate");
  CK(cudaSetDevice(device_));
  if (n == 0) throw std::invalid_argument("generate: empty prompt");
  for (size_t t = 0; t < n; ++t)
    if (ids[t] < 0 || ids[t] >= V_) throw std::out_of_range("token id outside [0, vocab_size)");
  std::vector<int64_t> stream(ids, ids + n);
  if (new_tokens == 0) return stream;  // the prefill result is not observable
  ensure_ws(std::max<size_t>(n, 1));
  float_state(static_cast<size_t>(L_) * H_);
  CK(cudaMemcpyAsync(ids_, ids, n * 8, cudaMemcpyHostToDevice, stream_));
  CK(launch_embed(h_, emb_, ids_, static_cast<int>(n), H_, V_, err_, stream_));
  layers(1, static_cast<int>(n), static_cast<int>(n),
         [&](int l) { return state_ + static_cast<size_t>(l) * H_; });
  head(h_ + (n - 1) * H_, 1);

  const int64_t stride = static_cast<int64_t>(new_tokens);
  loop_ids(new_tokens);
  if (samp.temperature > 0.0f && !host_sampling_) {
    // Sampling on the device: the uniforms the reference's emit() draws, one per token
    // (hgrn_model.cpp:263-264, :292), made here up front and uploaded once.
    std::mt19937_64 rng(samp.seed);
    std::uniform_real_distribution<double> uni(0.0, 1.0);
    std::vector<double> u(new_tokens);
    for (double& v : u) v = uni(rng);
    upload_uniforms(u);
    SampScope scope(this, &samp);
    const int64_t minus1 = -1;
    CK(cudaMemcpyAsync(pos_, &minus1, 8, cudaMemcpyHostToDevice, stream_));
    sample_first(1, 0, stride, false);
    int64_t first = 0;
    CK(cudaMemcpyAsync(&first, loop_ids_, 8, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    check_errors();
    std::vector<std::vector<int64_t>> st = {stream};
    st[0].push_back(first);
    if (on_token) (*on_token)(first);
    if (first != eos_id && new_tokens > 1)
      sampled_loop(1, stride, new_tokens - 1, eos_id, st, on_token);
    return st[0];
  }
  if (samp.temperature > 0.0f) {
    // Host sampling: one logits row back per step, same draws as the reference.
    std::mt19937_64 rng(samp.seed);
    Sampler pick{samp, static_cast<size_t>(V_)};
    std::vector<float> lg(V_);
    for (size_t step = 0; step < new_tokens; ++step) {
      if (step > 0) {
        CK(cudaMemcpyAsync(ids_, &stream.back(), 8, cudaMemcpyHostToDevice, stream_));
        CK(launch_embed(h_, emb_, ids_, 1, H_, V_, err_, stream_));
        layers(1, 1, 1, [&](int l) { return state_ + static_cast<size_t>(l) * H_; });
        head(h_, 1);
      }
      CK(cudaMemcpyAsync(lg.data(), logits_, V_ * 4, cudaMemcpyDeviceToHost, stream_));
      CK(cudaStreamSynchronize(stream_));
      const int64_t t = pick(lg.data(), rng);
      stream.push_back(t);
      if (on_token) (*on_token)(t);
      if (t == eos_id) break;
    }
    check_errors();
    return stream;
  }

  // Greedy: first token from the prefill logits, then graph replays.
  const int64_t zero = -1;
  CK(cudaMemcpyAsync(pos_, &zero, 8, cudaMemcpyHostToDevice, stream_));
  CK(launch_argmax_at(loop_ids_, stride, pos_, done_, logits_, 1, V_, V_, stream_));
  if (!graph_ || graph_b_ != 1 || graph_stride_ != stride) {
    drop_graph();
    CK(cudaStreamSynchronize(stream_));
    cudaGraph_t g;
    persist_ready(1, stride);
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    decode_graph_step(1, stride);
    CK(cudaStreamEndCapture(stream_, &g));
    CK(cudaGraphInstantiate(&graph_, g, 0));
    cudaGraphDestroy(g);
    graph_b_ = 1;
    graph_stride_ = stride;
  }
  pinned(new_tokens);
  if (eos_id < 0) {
    for (size_t step = 1; step < new_tokens; ++step) CK(cudaGraphLaunch(graph_, stream_));
    CK(cudaMemcpyAsync(pinned_, loop_ids_, new_tokens * 8, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    check_errors();
    stream.insert(stream.end(), pinned_, pinned_ + new_tokens);
    if (on_token)
      for (size_t i = 0; i < new_tokens; ++i) (*on_token)(pinned_[i]);
    return stream;
  }
  for (size_t step = 0; step < new_tokens; ++step) {
    if (step > 0) CK(cudaGraphLaunch(graph_, stream_));
    CK(cudaMemcpyAsync(pinned_, loop_ids_ + step, 8, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    const int64_t t = pinned_[0];
    stream.push_back(t);
    if (on_token) (*on_token)(t);
    if (t == eos_id) break;
  }
  check_errors();
  return stream;
}

void Model::forward(const int64_t* ids, size_t T, float* logits, bool last_row_only) {
  CK(cudaSetDevice(device_));
  if (T == 0) throw std::invalid_argument("forward: empty input");
  for (size_t t = 0; t < T; ++t)
    if (ids[t] < 0 || ids[t] >= V_) throw std::out_of_range("token id outside [0, vocab_size)");
  ensure_ws(T);
  CK(cudaMemcpyAsync(ids_, ids, T * 8, cudaMemcpyHostToDevice, stream_));
  CK(launch_embed(h_, emb_, ids_, static_cast<int>(T), H_, V_, err_, stream_));
  layers(1, static_cast<int>(T), static_cast<int>(T), [](int) { return static_cast<float*>(nullptr); });
  if (last_row_only) {
    head(h_ + (T - 1) * H_, 1);
    CK(cudaMemcpyAsync(logits, logits_, static_cast<size_t>(V_) * 4, cudaMemcpyDeviceToHost, stream_));
  } else {
    head(h_, static_cast<int>(T));
    CK(cudaMemcpyAsync(logits, logits_, T * V_ * 4, cudaMemcpyDeviceToHost, stream_));
  }
  CK(cudaStreamSynchronize(stream_));
  check_errors();
}

void Model::serve_begin(const std::vector<std::vector<int64_t>>& prompts, int64_t* first_ids) {
  prefill_runs(prompts, first_ids, 0);
  const size_t B = prompts.size();
  serve_b_ = static_cast<int>(B);
  serve_last_.assign(first_ids, first_ids + B);
}

void Model::prefill_runs(const std::vector<std::vector<int64_t>>& prompts, int64_t* first_ids,
                         int64_t stride) {
  CK(cudaSetDevice(device_));
  const size_t B = prompts.size();
  if (B == 0) throw std::invalid_argument("serve: no prompts");
  size_t max_rows = B;
  for (const auto& p : prompts) {
    if (p.empty()) throw std::invalid_argument("serve: empty prompt");
    for (int64_t t : p)
      if (t < 0 || t >= V_) throw std::out_of_range("token id outside [0, vocab_size)");
  }
  // prefill runs of consecutive streams with equal prompt length as one batch
  std::vector<std::pair<size_t, size_t>> runs;  // (first stream, count)
  for (size_t b = 0; b < B;) {
    size_t e = b + 1;
    while (e < B && prompts[e].size() == prompts[b].size()) ++e;
    runs.push_back({b, e - b});
    max_rows = std::max(max_rows, (e - b) * prompts[b].size());
    b = e;
  }
  ensure_ws(max_rows);
  float_state(static_cast<size_t>(L_) * B * H_);
  pinned(std::max(max_rows, B));
  for (const auto& run : runs) {
    const size_t b0 = run.first, G = run.second;
    const size_t T0 = prompts[b0].size();
    for (size_t g = 0; g < G; ++g) std::memcpy(pinned_ + g * T0, prompts[b0 + g].data(), T0 * 8);
    CK(cudaMemcpyAsync(ids_, pinned_, G * T0 * 8, cudaMemcpyHostToDevice, stream_));
    CK(launch_embed(h_, emb_, ids_, static_cast<int>(G * T0), H_, V_, err_, stream_));
    const size_t Bsz = B;
    layers(static_cast<int>(G), static_cast<int>(T0), static_cast<int>(T0), [&](int l) {
      return state_ + (static_cast<size_t>(l) * Bsz + b0) * H_;
    });
    // last row of every stream in the run -> hl_ [G][H]
    CK(cudaMemcpy2DAsync(hl_, H_ * 4, h_ + (T0 - 1) * H_, T0 * H_ * 4, H_ * 4, G,
                         cudaMemcpyDeviceToDevice, stream_));
    head(hl_, static_cast<int>(G));
    if (samp_) {
      sample_first(static_cast<int>(G), static_cast<int>(b0), stride, false);
      continue;
    }
    CK(launch_argmax(ids_, logits_, static_cast<int>(G), V_, V_, stream_));
    CK(cudaMemcpyAsync(first_ids + b0, ids_, G * 8, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
  }
  check_errors();
}

void Model::upload_uniforms(const std::vector<double>& u) {
  if (u.size() > uni_elems_) {
    CK(cudaStreamSynchronize(stream_));
    cudaFree(uni_);
    uni_ = nullptr;
    uni_elems_ = 0;
    CK(cudaMalloc(&uni_, u.size() * sizeof(double)));
    uni_elems_ = u.size();
  }
  CK(cudaMemcpyAsync(uni_, u.data(), u.size() * sizeof(double), cudaMemcpyHostToDevice, stream_));
  CK(cudaStreamSynchronize(stream_));  // u is a host vector that the caller may release
}

// The sampled first token of streams row0 .. row0 + B - 1 from logits_ rows 0 .. B - 1,
// written at loop_ids_[b * stride + *pos_ + 1] (*pos_ is -1 here).
void Model::sample_first(int B, int row0, int64_t stride, bool advance) {
  CK(launch_sample_at(loop_ids_, stride, pos_, done_, advance, row0, logits_, B, V_, V_, uni_, stride,
                      samp_->temperature, samp_->top_k, stream_));
}

// `steps` sampled lockstep steps of B streams from the tokens at position 0 of loop_ids_,
// graph-replayed on the device; ids are read back every 32 steps to stop once every stream
// has emitted eos_id (a finished stream keeps its slot; its later ids are dropped, as the
// reference drops them, hgrn_model.cpp:432-452).
void Model::sampled_loop(int B, int64_t stride, size_t steps, int64_t eos_id,
                         std::vector<std::vector<int64_t>>& streams,
                         const std::function<void(int64_t)>* on_token) {
  const int64_t zero = 0;
  CK(cudaMemcpyAsync(pos_, &zero, 8, cudaMemcpyHostToDevice, stream_));
  drop_graph();  // the graph bakes the sampling parameters: capture one for this call
  CK(cudaStreamSynchronize(stream_));
  cudaGraph_t g;
  CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
  decode_graph_step(B, stride);
  CK(cudaStreamEndCapture(stream_, &g));
  CK(cudaGraphInstantiate(&graph_, g, 0));
  cudaGraphDestroy(g);
  graph_b_ = B;
  graph_stride_ = -stride;  // never matches a greedy call's key
  pinned(static_cast<size_t>(stride) * B);
  std::vector<char> done(B, 0);
  for (int b = 0; b < B; ++b) done[b] = streams[b].back() == eos_id;
  size_t s = 0;
  const size_t chunk = eos_id < 0 ? steps : 32;
  while (s < steps) {
    const size_t n = std::min(chunk, steps - s);
    for (size_t i = 0; i < n; ++i) CK(cudaGraphLaunch(graph_, stream_));
    CK(cudaMemcpyAsync(pinned_, loop_ids_, static_cast<size_t>(stride) * B * 8, cudaMemcpyDeviceToHost,
                       stream_));
    CK(cudaStreamSynchronize(stream_));
    bool all_done = true;
    for (int b = 0; b < B; ++b) {
      for (size_t t = s + 1; t <= s + n && !done[b]; ++t) {
        const int64_t id = pinned_[static_cast<size_t>(b) * stride + t];
        streams[b].push_back(id);
        if (b == 0 && on_token) (*on_token)(id);
        if (id == eos_id) done[b] = 1;
      }
      all_done = all_done && done[b];
    }
    s += n;
    if (all_done) break;
  }
  check_errors();
  drop_graph();
}

void Model::serve_step(const int64_t* in_ids, int64_t* out_ids) {
  tp_only_prefill("serve_step");
  if (serve_b_ == 0) throw std::logic_error("serve_step without serve_begin");
  const int B = serve_b_;
  // one lockstep step: ids [B][2], position 0 holds the inputs
  loop_ids(static_cast<size_t>(2) * B);
  if (!graph_ || graph_b_ != B || graph_stride_ != 2) {
    drop_graph();
    CK(cudaStreamSynchronize(stream_));
    cudaGraph_t g;
    persist_ready(B, 2);
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    decode_graph_step(B, 2);
    CK(cudaStreamEndCapture(stream_, &g));
    CK(cudaGraphInstantiate(&graph_, g, 0));
    cudaGraphDestroy(g);
    graph_b_ = B;
    graph_stride_ = 2;
  }
  pinned(static_cast<size_t>(2) * B + 1);
  for (int b = 0; b < B; ++b) pinned_[2 * b] = in_ids[b];
  pinned_[2 * B] = 0;  // position
  CK(cudaMemcpyAsync(loop_ids_, pinned_, static_cast<size_t>(2) * B * 8, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(pos_, pinned_ + 2 * B, 8, cudaMemcpyHostToDevice, stream_));
  CK(cudaGraphLaunch(graph_, stream_));
  CK(cudaMemcpy2DAsync(out_ids, 8, loop_ids_ + 1, 16, 8, B, cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  serve_last_.assign(out_ids, out_ids + B);
}

void Model::serve_run(size_t steps, int64_t* out) {
  tp_only_prefill("serve_run");
  if (serve_b_ == 0) throw std::logic_error("serve_run without serve_begin");
  const int B = serve_b_;
  int64_t stride = static_cast<int64_t>(steps) + 1;
  // the stride is only the row pitch of the id buffer: a graph captured for a longer run
  // serves a shorter one too (no re-capture)
  if (graph_ && graph_b_ == B && graph_stride_ >= stride) stride = graph_stride_;
  loop_ids(static_cast<size_t>(stride) * B);
  if (!graph_ || graph_b_ != B || graph_stride_ != stride) {
    drop_graph();
    CK(cudaStreamSynchronize(stream_));
    cudaGraph_t g;
    persist_ready(B, stride);
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    decode_graph_step(B, stride);
    CK(cudaStreamEndCapture(stream_, &g));
    CK(cudaGraphInstantiate(&graph_, g, 0));
    cudaGraphDestroy(g);
    graph_b_ = B;
    graph_stride_ = stride;
  }
  pinned(static_cast<size_t>(stride) * B + 1);
  const int64_t zero = 0;
  CK(cudaMemcpy2DAsync(loop_ids_, stride * 8, serve_last_.data(), 8, 8, B, cudaMemcpyHostToDevice,
                       stream_));
  CK(cudaMemcpyAsync(pos_, &zero, 8, cudaMemcpyHostToDevice, stream_));
  for (size_t s = 0; s < steps; ++s) CK(cudaGraphLaunch(graph_, stream_));
  CK(cudaMemcpyAsync(pinned_, loop_ids_, static_cast<size_t>(stride) * B * 8, cudaMemcpyDeviceToHost,
                     stream_));
  CK(cudaStreamSynchronize(stream_));
  check_errors();
  for (int b = 0; b < B; ++b) {
    std::memcpy(out + static_cast<size_t>(b) * steps, pinned_ + static_cast<size_t>(b) * stride + 1,
                steps * 8);
    serve_last_[b] = pinned_[static_cast<size_t>(b) * stride + steps];
  }
}

void Model::serve_end() { serve_b_ = 0; }

std::vector<std::vector<int64_t>> Model::generate_serve(
    const std::vector<std::vector<int64_t>>& prompts, size_t new_tokens, int64_t eos_id,
    const Sampling& samp) {
  tp_only_prefill("generate_serve");
  const size_t B = prompts.size();
  std::vector<std::vector<int64_t>> streams = prompts;
  if (B == 0) return streams;
  std::vector<int64_t> first(B);
  if (samp.temperature > 0.0f && !host_sampling_) {
    // device-sampled lockstep loop: stream b's uniforms come from its mt19937_64 seeded
    // seed + b (hgrn_model.cpp:368-373), one per token, made up front
    const int64_t stride = static_cast<int64_t>(std::max<size_t>(new_tokens, 1));
    std::vector<double> u(B * static_cast<size_t>(stride));
    std::uniform_real_distribution<double> uni(0.0, 1.0);
    for (size_t b = 0; b < B; ++b) {
      std::mt19937_64 rng(samp.seed + b);
      for (int64_t t = 0; t < stride; ++t) u[b * stride + t] = uni(rng);
    }
    upload_uniforms(u);
    loop_ids(B * static_cast<size_t>(stride));
    SampScope scope(this, &samp);
    const int64_t minus1 = -1;
    CK(cudaMemcpyAsync(pos_, &minus1, 8, cudaMemcpyHostToDevice, stream_));
    prefill_runs(prompts, nullptr, stride);  // first tokens sampled into loop_ids_[b * stride]
    CK(cudaMemcpy2DAsync(first.data(), 8, loop_ids_, stride * 8, 8, B, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    for (size_t b = 0; b < B; ++b) streams[b].push_back(first[b]);
    if (new_tokens > 1) sampled_loop(static_cast<int>(B), stride, new_tokens - 1, eos_id, streams);
    return streams;
  }
  if (samp.temperature > 0.0f) {
    // host-sampled lockstep loop (hgrn_model.cpp:368-406): per-stream RNG seeded seed + b,
    // prefill stream by stream, then one batched step per token.
    CK(cudaSetDevice(device_));
    size_t max_t = B;
    for (const auto& p : prompts) {
      if (p.empty()) throw std::invalid_argument("serve: empty prompt");
      for (int64_t t : p)
        if (t < 0 || t >= V_) throw std::out_of_range("token id outside [0, vocab_size)");
      max_t = std::max(max_t, p.size());
    }
    std::vector<std::mt19937_64> rng;
    rng.reserve(B);
    for (size_t b = 0; b < B; ++b) rng.emplace_back(samp.seed + b);
    Sampler pick{samp, static_cast<size_t>(V_)};
    std::vector<char> done(B, 0);
    std::vector<float> lg(static_cast<size_t>(V_) * B);
    ensure_ws(max_t);
    float_state(static_cast<size_t>(L_) * B * H_);
    for (size_t b = 0; b < B; ++b) {
      const size_t T0 = prompts[b].size();
      CK(cudaMemcpyAsync(ids_, prompts[b].data(), T0 * 8, cudaMemcpyHostToDevice, stream_));
      CK(launch_embed(h_, emb_, ids_, static_cast<int>(T0), H_, V_, err_, stream_));
      layers(1, static_cast<int>(T0), static_cast<int>(T0),
             [&](int l) { return state_ + (static_cast<size_t>(l) * B + b) * H_; });
      head(h_ + (T0 - 1) * H_, 1);
      CK(cudaMemcpyAsync(lg.data(), logits_, V_ * 4, cudaMemcpyDeviceToHost, stream_));
      CK(cudaStreamSynchronize(stream_));
      const int64_t t0 = pick(lg.data(), rng[b]);
      streams[b].push_back(t0);
      if (t0 == eos_id) done[b] = 1;
    }
    std::vector<int64_t> last(B);
    for (size_t step = 1; step < new_tokens; ++step) {
      for (size_t b = 0; b < B; ++b) last[b] = streams[b].back();
      CK(cudaMemcpyAsync(ids_, last.data(), B * 8, cudaMemcpyHostToDevice, stream_));
      CK(launch_embed(h_, emb_, ids_, static_cast<int>(B), H_, V_, err_, stream_));
      layers(static_cast<int>(B), 1, static_cast<int>(B),
             [&](int l) { return state_ + static_cast<size_t>(l) * B * H_; });
      head(h_, static_cast<int>(B));
      CK(cudaMemcpyAsync(lg.data(), logits_, B * V_ * 4, cudaMemcpyDeviceToHost, stream_));
      CK(cudaStreamSynchronize(stream_));
      bool all_done = true;
      for (size_t b = 0; b < B; ++b) {
        if (done[b]) continue;
        const int64_t t = pick(lg.data() + b * V_, rng[b]);
        streams[b].push_back(t);
        if (t == eos_id) done[b] = 1;
        else all_done = false;
      }
      if (all_done) break;
    }
    check_errors();
    return streams;
  }

  serve_begin(prompts, first.data());
  std::vector<char> done(B, 0);
  for (size_t b = 0; b < B; ++b) {
    streams[b].push_back(first[b]);
    if (first[b] == eos_id) done[b] = 1;
  }
  if (new_tokens > 1) {
    const size_t steps = new_tokens - 1;
    std::vector<int64_t> out(B * steps);
    if (eos_id < 0) {
      serve_run(steps, out.data());
      for (size_t b = 0; b < B; ++b)
        streams[b].insert(streams[b].end(), out.begin() + b * steps, out.begin() + (b + 1) * steps);
    } else {
      // a finished stream keeps its slot (its outputs are dropped), as in the reference
      std::vector<int64_t> step_ids(B);
      for (size_t s = 0; s < steps; ++s) {
        serve_run(1, step_ids.data());
        bool all_done = true;
        for (size_t b = 0; b < B; ++b) {
          if (done[b]) continue;
          streams[b].push_back(step_ids[b]);
          if (step_ids[b] == eos_id) done[b] = 1;
          else all_done = false;
        }
        if (all_done) break;
      }
    }
  }
  serve_end();
  return streams;
}

}  // namespace mmfree_cuda
