// model.h -- device-resident HGRN-Bit forward (the CUDA counterpart of mmfree::Model,
// matmulfreellmCPU cpp/include/mmfree/model.hpp:33-120).
//
// Weights are uploaded once from the model.mmfree blob; every BitLinear weight is repacked
// on the device into the tiled 2-bit format (common.cuh). Activations, the recurrent state
// [L][B][H] and the token ids stay in HBM across steps; the per-token decode step is
// captured in a CUDA graph and replayed with a device-side position counter, so a greedy
// generation needs no host round trip until the ids are copied back.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "blob.h"
#include "kernels.h"

namespace mmfree_cuda {

struct Sampling {  // model.hpp:27-31
  float temperature = 0.0f;
  int top_k = 0;
  uint64_t seed = 0;
};

// Tensor-parallel prefill: this handle is rank `rank` of `world`, all sharing the NCCL unique
// id (TpComm::unique_id on one rank, distributed by the caller). world = 1: no parallelism.
struct TpSpec {
  int rank = 0, world = 1;
  const unsigned char* nccl_id = nullptr;
};

class TpComm;

class Model {
 public:
  Model(const std::string& blob_path, int device, bool fixed, int frac_bits,
        const TpSpec& tp = TpSpec());
  ~Model();
  Model(const Model&) = delete;
  Model& operator=(const Model&) = delete;

  const BlobConfig& config() const { return cfg_; }
  int device() const { return device_; }
  int tp_world() const { return tp_world_; }
  cudaStream_t stream() const { return stream_; }
  size_t weight_bytes() const { return packed_bytes_; }

  // model.hpp:36-50 / hgrn_model.cpp:249-347.
  // on_token (nullable, model.hpp:44-50) is called with every generated id, in order, as soon
  // as the host has it: per step when eos_id >= 0 (the step's id is read back to test it),
  // otherwise once the device loop is done.
  std::vector<int64_t> generate(const int64_t* ids, size_t n, size_t new_tokens, int64_t eos_id,
                                const Sampling& samp,
                                const std::function<void(int64_t)>* on_token = nullptr);
  // model.hpp:34 / hgrn_model.cpp:239-247: logits [T, V] (host), or only the last row.
  void forward(const int64_t* ids, size_t T, float* logits, bool last_row_only);
  // forward plus a host trace of (1 + 3L) x [T, H]: embeddings, then per layer the
  // recurrence output, the residual after o_proj and the layer output (debugging parity,
  // like the reference's capture hooks, tools/reference.py:108-117).
  void forward_trace(const int64_t* ids, size_t T, float* logits, float* trace);
  // model.hpp:52-70 / hgrn_model.cpp:349-454.
  std::vector<std::vector<int64_t>> generate_serve(const std::vector<std::vector<int64_t>>& prompts,
                                                   size_t new_tokens, int64_t eos_id,
                                                   const Sampling& samp);

  // Serving session, one lockstep decode step per call (host ids in, host ids out). begin
  // prefills every prompt and returns each stream's first greedy token.
  void serve_begin(const std::vector<std::vector<int64_t>>& prompts, int64_t* first_ids);
  void serve_step(const int64_t* in_ids, int64_t* out_ids);
  void serve_end();
  int serve_batch() const { return serve_b_; }

  // Greedy decode steps of a serving session with no host round trip: `steps` lockstep
  // steps starting from the session's last tokens, ids written to out [B][steps] (host).
  void serve_run(size_t steps, int64_t* out);

  // Kernel classes of a decode step, for serve_profile.
  enum KernelClass { kClsPrep = 0, kClsMatmul, kClsLmHead, kClsMixer, kClsSwiglu, kClsEmbed,
                     kClsArgmax, kClsStep, kNumClasses };  // kClsStep: a persistent whole step
  struct ClassStats {
    double ms = 0;        // summed device time of the class's launches
    int64_t launches = 0;
    double bytes = 0;     // algorithmic bytes moved by those launches
    double ops = 0;       // algorithmic integer/float ops (2*M*K*N per BitLinear)
  };
  static const char* class_name(int c);
  // `steps` greedy decode steps like serve_run (same kernels, not graph-captured), with a
  // CUDA event pair around every launch; returns per-class totals.
  std::vector<ClassStats> serve_profile(size_t steps);
  // the stream every kernel of this model is launched on

 private:
  struct Proj {
    const void* w = nullptr;
    const float* normw = nullptr;
    float scale_w = 1.0f;
    int in = 0, out = 0;
  };
  struct Layer {
    const float* attn_norm = nullptr;
    const float* mlp_norm = nullptr;
    const float* g_norm = nullptr;
    const float* lb = nullptr;  // lower bound row of this layer (nullptr for layer 0)
    Proj p[6];                  // i, f, g, o, gate, down
  };
  enum { kI = 0, kF, kG, kO, kGate, kDown };

  void ensure_ws(size_t rows);
  void prep(const PrepArgs& p);
  template <class F>
  void timed(int cls, double bytes, double ops, F&& launch);
  MatmulArgs mm_args(const Proj& p, int plane, float* out, int M, const float* resid) const;
  void bitlinear(const Proj& p, int plane, float* out, int M, const float* resid);
  bool tc_rows(int M) const;                          // tensor-core BitLinear for M rows?
  void bitlinear_ifg(const Layer& ly, int M);         // i/f/g (one launch on tensor cores)
  void bitlinear_gate_swiglu(const Layer& ly, int M, int seg_rows);  // z = swiglu(gate_proj)
  // All layers over `rows` = nseq * len rows of h_ ([nseq][len][H]); state(l) gives the
  // layer's state base ([nseq][H]) or nullptr; seg_rows = rows of one reference block call.
  template <class StateFn>
  void layers(int nseq, int len, int seg_rows, StateFn state);
  // The same over this rank's shards (no recurrent state is kept: prefill only).
  void layers_tp(int nseq, int len, int seg_rows);
  void ensure_tp_ws(size_t rows);
  void tp_gather(float* full, const float* slice, int rows, int n);  // all-gather of columns
  void tp_only_prefill(const char* what) const;  // throws for calls a TP handle cannot serve
  void head(const float* rows, int M);  // final norm + lm_head into logits_
  void check_errors();
  void decode_graph_step(int B, int64_t stride);  // embed_at, layers (streams), head, argmax_at
  bool fused_decode(int B) const;                 // use the fused kernels of decode.cu?
  void fused_step(int B, int64_t stride);
  // The fused step's phases: per layer mixer, o_proj, gate_proj + swiglu, down_proj; then
  // the head. The first phase gathers its rows from the embedding table at *pos_.
  std::vector<DecArgs> dec_phases(int B, int64_t stride);
  // Plans and uploads the persistent step's phase table for (B, stride); false when the
  // step cannot run as one cooperative launch. Not callable during stream capture.
  bool persist_ready(int B, int64_t stride);
  int sms_ = 148;
  bool fused_ok_ = true;           // MMFREE_FUSED_DECODE=0 selects the unfused decode step
  bool pdl_ = true;                // MMFREE_PDL=0: plain stream order between kernels
  bool persist_ok_ = false;        // MMFREE_PERSIST=1: the whole fused step in one launch
  bool mix_prep_ok_ = true;        // MMFREE_MIX_IN_PREP=0: the decode mixer as its own kernel
  bool float_tc_ = true;           // MMFREE_FLOAT_TC=0: Float BitLinears of >= 16 rows on the
                                   // CUDA cores instead of the bf16 tensor-core path
  DecArgs* persist_tab_ = nullptr; // device copy of the persistent step's phase table
  int persist_n_ = 0, persist_grid_ = 0, persist_b_ = 0;
  int64_t persist_stride_ = -1;
  size_t persist_smem_ = 0;
  unsigned* persist_bar_ = nullptr;  // grid barrier word of the persistent step
  float* dec_part_v_ = nullptr;    // fused head: per-CTA argmax partials
  int* dec_part_i_ = nullptr;

  BlobConfig cfg_;
  int device_ = 0;
  bool fixed_ = true;
  float qs_ = 1024.0f;
  int H_ = 0, I_ = 0, V_ = 0, L_ = 0;
  float eps_ = 1e-6f;
  cudaStream_t stream_ = nullptr;

  // weights
  void* arena_ = nullptr;          // packed ternary weights of every projection
  size_t packed_bytes_ = 0;
  float* fp_arena_ = nullptr;      // embeddings, norms, lower bounds
  const float* emb_ = nullptr;
  const float* final_norm_ = nullptr;
  Proj lm_head_;
  std::vector<Layer> layers_;

  // workspace (rows = capacity)
  size_t ws_rows_ = 0;
  void* ws_ = nullptr;
  float *h_ = nullptr, *resid_ = nullptr, *ib_ = nullptr, *fb_ = nullptr, *gb_ = nullptr;
  float *recur_ = nullptr, *y_ = nullptr, *z_ = nullptr, *logits_ = nullptr, *hl_ = nullptr;
  int8_t* planes_[3] = {};
  int32_t* rowsum_[3] = {};
  float* yf_[3] = {};
  int64_t* ids_ = nullptr;

  // state and decode loop
  float* state_ = nullptr;
  size_t state_elems_ = 0;
  int64_t* loop_ids_ = nullptr;    // [B][stride]
  size_t loop_ids_elems_ = 0;
  int64_t* pos_ = nullptr;         // device position counter
  unsigned* done_ = nullptr;       // argmax_at completion counter
  uint32_t* err_ = nullptr;        // device error flags
  int64_t* pinned_ = nullptr;      // pinned staging for ids
  size_t pinned_elems_ = 0;

  cudaGraphExec_t graph_ = nullptr;  // captured decode step
  int graph_b_ = 0;
  int64_t graph_stride_ = 0;

  float* trace_ = nullptr;         // forward_trace destination (host), else nullptr
  bool prof_on_ = false;
  struct Mark { int cls; cudaEvent_t a, b; double bytes, ops; };
  std::vector<Mark> marks_;
  std::vector<cudaEvent_t> ev_free_;

  int serve_b_ = 0;                // active serving session batch (0 = none)
  std::vector<int64_t> serve_last_;

  // Sampled decoding on the device: while samp_ is set, decode steps end in sample_at instead
  // of the greedy argmax, drawing with the per-stream uniforms uni_ [B][stride] (drawn on the
  // host from each stream's mt19937_64). MMFREE_HOST_SAMPLING=1 keeps the host sampler.
  const Sampling* samp_ = nullptr;
  bool host_sampling_ = false;
  struct SampScope {  // samp_ for one sampled call; its decode graph is dropped on the way out
    Model* m;
    SampScope(Model* mm, const Sampling* s) : m(mm) {
      m->drop_graph();
      m->samp_ = s;
    }
    ~SampScope() {
      m->samp_ = nullptr;
      m->drop_graph();
    }
  };
  double* uni_ = nullptr;
  size_t uni_elems_ = 0;
  void upload_uniforms(const std::vector<double>& u);
  void sample_first(int B, int row0, int64_t stride, bool advance);  // from logits_ rows
  // prefill of every prompt (runs of equal length batched); first tokens greedy into ids_
  // (first_ids on the host) or, with samp_, sampled into loop_ids_[b * stride]
  void prefill_runs(const std::vector<std::vector<int64_t>>& prompts, int64_t* first_ids,
                    int64_t stride);
  void sampled_loop(int B, int64_t stride, size_t steps, int64_t eos_id,
                    std::vector<std::vector<int64_t>>& streams,
                    const std::function<void(int64_t)>* on_token = nullptr);  // stream 0's ids
  // Float-mode prefill: workspace of the chunked scan (nullptr: the exact serial scan)
  void* chunk_ws(int nseq, int len, int H);
  void* chunk_ws_ = nullptr;
  size_t chunk_bytes_ = 0;
  void float_state(size_t elems);
  void loop_ids(size_t elems);
  void pinned(size_t elems);
  void drop_graph();

  // tensor parallelism (tp_ == nullptr: one GPU). Shard widths Hs = H / P, Is = I / P; the
  // projections in layers_ hold this rank's shards (column shards of i/f/g/gate, and of o/down
  // in FixedQ510; row shards of o/down in Float), lm_head is whole on every rank.
  std::unique_ptr<TpComm> tp_;
  int tp_rank_ = 0, tp_world_ = 1, Hs_ = 0, Is_ = 0;
  size_t tp_rows_ = 0;
  void* tp_ws_ = nullptr;
  float *tp_g_ = nullptr, *tp_rec_ = nullptr, *tp_stage_ = nullptr, *tp_rs_ = nullptr;
  float *tp_zs_ = nullptr, *tp_hs_ = nullptr, *tp_ts_ = nullptr, *tp_ss_ = nullptr;
};

}  // namespace mmfree_cuda
