// ref_ops.cpp -- TEST INFRASTRUCTURE ONLY: a C-ABI driver over the reference engine's own
// public C++ API, so Python tests and the CPU-baseline leg of bench.py can call the
// unmodified reference code path (compiled from its sources by oracle/Makefile).
//
// Every function here forwards to the reference:
//   kernels      mmfree::bitlinear / bitlinear_cluster / rmsnorm / swiglu / hgrn_scan /
//                rmsnorm_swishgate                         (cpp/include/mmfree/kernels.hpp:29-68)
//   primitives   mmfree::simd::*                           (cpp/include/mmfree/simd.hpp:69-357)
//   model        mmfree::Weights + mmfree::Model           (cpp/include/mmfree/model.hpp:33-80)
// The only added logic is RecordingBackend, a TernaryBackend that computes exactly what
// CpuBackend computes (cpp/include/mmfree/ternary_backend.hpp:96-103) and also copies the
// int32 accumulators out, so tests can compare them bit for bit.
#include "mmfree/kernels.hpp"
#include "mmfree/model.hpp"
#include "mmfree/simd.hpp"
#include "mmfree/ternary_backend.hpp"
#include "mmfree/weights.hpp"

#include <chrono>
#include <random>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

thread_local std::string g_err;

// CpuBackend arithmetic + a copy of every accumulator row, in call order.
struct RecordingBackend final : mmfree::TernaryBackend {
  std::int32_t* sink = nullptr;
  std::size_t cursor = 0;
  void matmul(int, const std::int32_t* x, std::int32_t* acc, const std::int8_t* wq,
              std::size_t N, std::size_t M) override {
#pragma omp parallel for schedule(static)
    for (std::size_t o = 0; o < M; ++o) acc[o] = mmfree::simd::ternary_dot_i32(x, wq + o * N, N);
    if (sink) {
      std::memcpy(sink + cursor, acc, M * sizeof(std::int32_t));
      cursor += M;
    }
  }
};

struct ModelHandle {
  std::unique_ptr<mmfree::Weights> w;
  std::unique_ptr<mmfree::Model> m;
};

mmfree::ActQuant aq_of(int aq) {
  return aq == 1 ? mmfree::ActQuant::FixedQ510 : mmfree::ActQuant::Float;
}

using clk = std::chrono::steady_clock;
double secs(clk::duration d) { return std::chrono::duration<double>(d).count(); }

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

int ref_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void ref_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

// ---- kernels (kernels.hpp) -------------------------------------------------------------
void ref_bitlinear(float* out, const float* x, const float* nw, const std::int8_t* wq,
                   float scale_w, std::size_t rows, std::size_t in_dim, std::size_t out_dim,
                   float eps, float* norm_out, int aq, int frac, std::int32_t* acc_out) {
  RecordingBackend be;
  be.sink = acc_out;
  mmfree::bitlinear(out, x, nw, wq, scale_w, rows, in_dim, out_dim, eps, norm_out, aq_of(aq),
                    frac, acc_out ? &be : nullptr, -1);
}

void ref_bitlinear_cluster(float* const* outs, const float* x, const float* const* nws,
                           const std::int8_t* const* wqs, const float* scales, int k,
                           std::size_t rows, std::size_t in_dim, std::size_t out_dim, float eps,
                           int frac, std::int32_t* acc_out) {
  RecordingBackend be;
  be.sink = acc_out;
  std::vector<int> ids(k, -1);
  mmfree::bitlinear_cluster(outs, x, nws, wqs, scales, k, rows, in_dim, out_dim, eps, frac,
                            acc_out ? &be : nullptr, ids.data());
}

void ref_rmsnorm(float* y, const float* x, const float* w, std::size_t rows, std::size_t cols,
                 float eps) {
  mmfree::rmsnorm(y, x, w, rows, cols, eps);
}

void ref_swiglu(float* out, const float* a, const float* b, std::size_t n) {
  mmfree::swiglu(out, a, b, n);
}

void ref_hgrn_scan(float* out, const float* i, const float* f, std::size_t T, std::size_t D,
                   float* state_io) {
  mmfree::hgrn_scan(out, i, f, T, D, state_io);
}

void ref_rmsnorm_swishgate(float* out, const float* g, const float* o, const float* w,
                           std::size_t rows, std::size_t cols, float eps) {
  mmfree::rmsnorm_swishgate(out, g, o, w, rows, cols, eps);
}

// ---- primitives (simd.hpp) -------------------------------------------------------------
float ref_sumsq(const float* x, std::size_t n) { return mmfree::simd::sumsq(x, n); }
void ref_quant_q510(std::int32_t* yq, const float* y, float qs, std::size_t n) {
  mmfree::simd::quant_q510(yq, y, qs, n);
}
void ref_dequant_scale(float* out, const std::int32_t* acc, float s, std::size_t n) {
  mmfree::simd::dequant_scale(out, acc, s, n);
}
void ref_sigmoid(float* out, const float* x, std::size_t n) { mmfree::simd::sigmoid(out, x, n); }
void ref_silu(float* out, const float* x, std::size_t n) { mmfree::simd::silu(out, x, n); }
void ref_hgrn_step(float* state, float* out, const float* f, const float* in, std::size_t D) {
  mmfree::simd::hgrn_step(state, out, f, in, D);
}
float ref_expf_poly(float x) { return mmfree::simd::expf_poly(x); }
float ref_ternary_dot_f32(const float* y, const std::int8_t* w, std::size_t n) {
  return mmfree::simd::ternary_dot_f32(y, w, n);
}

// ---- model (model.hpp) -----------------------------------------------------------------
void* ref_model_open(const char* blob, int aq, int frac) {
  try {
    auto h = std::make_unique<ModelHandle>();
    h->w = std::make_unique<mmfree::Weights>(blob);
    h->m = std::make_unique<mmfree::Model>(*h->w, aq_of(aq), frac);
    return h.release();
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void ref_model_close(void* h) { delete static_cast<ModelHandle*>(h); }

int ref_model_config(void* h, std::size_t* out6) {
  const auto& c = static_cast<ModelHandle*>(h)->m->config();
  out6[0] = c.vocab_size;
  out6[1] = c.hidden_size;
  out6[2] = c.num_hidden_layers;
  out6[3] = c.intermediate_size;
  out6[4] = c.use_lower_bound;
  out6[5] = c.num_heads;
  return 0;
}

int ref_model_generate(void* hp, const std::int64_t* ids, std::size_t n, std::size_t gen,
                       std::int64_t eos, float temp, int top_k, std::uint64_t seed,
                       std::int64_t* out, std::size_t cap, std::size_t* out_n) {
  try {
    auto* h = static_cast<ModelHandle*>(hp);
    mmfree::Sampling s;
    s.temperature = temp;
    s.top_k = top_k;
    s.seed = seed;
    std::vector<std::int64_t> in(ids, ids + n);
    auto st = h->m->generate(in, gen, eos, s);
    if (st.size() > cap) { g_err = "output capacity too small"; return -1; }
    std::memcpy(out, st.data(), st.size() * sizeof(std::int64_t));
    *out_n = st.size();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

int ref_model_forward(void* hp, const std::int64_t* ids, std::size_t T, float* logits) {
  try {
    auto* h = static_cast<ModelHandle*>(hp);
    std::vector<float> lg;
    h->m->forward(ids, T, lg);
    std::memcpy(logits, lg.data(), lg.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// prompts: B pointers; out: B rows of out_stride ids; out_lens[b] = stream length.
int ref_model_generate_serve(void* hp, std::size_t B, const std::int64_t* const* prompts,
                             const std::size_t* lens, std::size_t gen, std::int64_t eos,
                             float temp, int top_k, std::uint64_t seed, std::int64_t* out,
                             std::size_t out_stride, std::size_t* out_lens) {
  try {
    auto* h = static_cast<ModelHandle*>(hp);
    std::vector<std::vector<std::int64_t>> ps(B);
    for (std::size_t b = 0; b < B; ++b) ps[b].assign(prompts[b], prompts[b] + lens[b]);
    mmfree::Sampling s;
    s.temperature = temp;
    s.top_k = top_k;
    s.seed = seed;
    auto st = h->m->generate_serve(ps, gen, eos, s);
    for (std::size_t b = 0; b < B; ++b) {
      if (st[b].size() > out_stride) { g_err = "output stride too small"; return -1; }
      std::memcpy(out + b * out_stride, st[b].data(), st[b].size() * sizeof(std::int64_t));
      out_lens[b] = st[b].size();
    }
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// Timed greedy generate with the reference bench's own split (cpp/src/util/bench.cpp:51-66):
// prefill = t(first token) - t0, decode = t(last token) - t(first token) over n-1 tokens.
int ref_model_bench_generate(void* hp, const std::int64_t* ids, std::size_t n, std::size_t gen,
                             double* prefill_s, double* decode_s, std::size_t* emitted) {
  try {
    auto* h = static_cast<ModelHandle*>(hp);
    std::vector<std::int64_t> in(ids, ids + n);
    clk::time_point t0 = clk::now(), t_first = t0, t_last = t0;
    bool got = false;
    std::size_t cnt = 0;
    h->m->generate(in, gen, -1, mmfree::Sampling{}, [&](std::int64_t) {
      auto now = clk::now();
      if (!got) { t_first = now; got = true; }
      t_last = now;
      ++cnt;
    });
    *prefill_s = secs(t_first - t0);
    *decode_s = cnt > 1 ? secs(t_last - t_first) : 0.0;
    *emitted = cnt;
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// Timed greedy generate_serve: decode = from the last prefill token callback to the last
// decode callback; decode_tokens = callbacks fired in that window.
int ref_model_bench_serve(void* hp, std::size_t B, const std::int64_t* const* prompts,
                          const std::size_t* lens, std::size_t gen, double* prefill_s,
                          double* decode_s, std::size_t* decode_tokens) {
  try {
    auto* h = static_cast<ModelHandle*>(hp);
    std::vector<std::vector<std::int64_t>> ps(B);
    for (std::size_t b = 0; b < B; ++b) ps[b].assign(prompts[b], prompts[b] + lens[b]);
    clk::time_point t0 = clk::now(), t_pref = t0, t_last = t0;
    std::size_t seen = 0, dec = 0;
    h->m->generate_serve(ps, gen, -1, mmfree::Sampling{}, [&](std::size_t, std::int64_t) {
      auto now = clk::now();
      ++seen;
      if (seen <= B) t_pref = now;  // the B prefill tokens arrive first, stream by stream
      else ++dec;
      t_last = now;
    });
    *prefill_s = secs(t_pref - t0);
    *decode_s = dec ? secs(t_last - t_pref) : 0.0;
    *decode_tokens = dec;
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// The uniforms the reference's sampler draws for a stream seeded `seed`, in order
// (std::mt19937_64 + std::uniform_real_distribution<double>(0, 1), hgrn_model.cpp:263-264,
// :292), from the same C++ library the reference is built with.
void ref_uniforms(std::uint64_t seed, std::size_t n, double* out) {
  std::mt19937_64 rng(seed);
  std::uniform_real_distribution<double> uni(0.0, 1.0);
  for (std::size_t i = 0; i < n; ++i) out[i] = uni(rng);
}

}  // extern "C"
