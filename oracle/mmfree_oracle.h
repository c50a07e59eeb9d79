/* mmfree_oracle.h -- TEST INFRASTRUCTURE ONLY (CPU checker for the CUDA path).
 *
 * A plain-C restatement of the HGRN-Bit forward numerics of the reference engine
 * (matmulfreellmCPU, built for x86 with AVX2+FMA and GCC's default FP contraction).
 * Each function cites the reference file:line it restates. Only tests/, the smoke check
 * and the CPU-baseline leg of bench.py may call it; the product never does.
 */
#ifndef MMFREE_ORACLE_H
#define MMFREE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- primitives (cpp/include/mmfree/simd.hpp) ---- */
float orc_sumsq(const float* x, size_t n);
void orc_quant_q510(int32_t* yq, const float* y, float qs, size_t n);
float orc_exp8_lane(float x);
float orc_expf_tail(float x);
void orc_sigmoid(float* out, const float* x, size_t n);
void orc_silu(float* out, const float* x, size_t n);
void orc_swiglu(float* out, const float* a, const float* b, size_t n);
void orc_hgrn_step(float* state, float* out, const float* f, const float* in, size_t d);
float orc_ternary_dot_f32(const float* y, const int8_t* w, size_t n);
int32_t orc_ternary_dot_i32(const int32_t* yq, const int8_t* w, size_t n);

/* ---- kernels (cpp/include/mmfree/kernels.hpp) ---- */
void orc_rmsnorm(float* y, const float* x, const float* w, size_t rows, size_t cols, float eps);
void orc_bitlinear(float* out, const float* x, const float* nw, const int8_t* wq, float scale_w,
                   size_t rows, size_t in_dim, size_t out_dim, float eps, float* norm_out,
                   int act_quant, int frac_bits, int32_t* acc_out);
void orc_hgrn_scan(float* out, const float* i, const float* f, size_t t, size_t d,
                   float* state_io);
void orc_rmsnorm_swishgate(float* out, const float* g, const float* o, const float* w,
                           size_t rows, size_t cols, float eps);

/* ---- model (cpp/src/model/hgrn_model.cpp) ---- */
typedef struct {
  const int8_t* wq;    /* [out, in] ternary */
  const float* normw;  /* [in] */
  float scale_w;
  size_t in_dim, out_dim;
} orc_proj;

enum { ORC_I = 0, ORC_F, ORC_G, ORC_O, ORC_GATE, ORC_DOWN, ORC_NPROJ };

typedef struct {
  const float* attn_norm;
  const float* mlp_norm;
  const float* g_norm;
  orc_proj proj[ORC_NPROJ];
} orc_layer;

typedef struct {
  size_t vocab, hidden, layers, inter;
  int use_lower_bound;
  float eps;
  const float* embeddings;   /* [V, H] */
  const float* final_norm;   /* [H] */
  const float* lower_bounds; /* [L, H] or NULL */
  orc_proj lm_head;
  const orc_layer* layer;    /* [L] */
} orc_model;

/* Full-prefix forward from zero state; logits [T, V]. */
int orc_model_forward(const orc_model* m, int act_quant, int frac_bits, const int64_t* ids,
                      size_t t, float* logits);
int orc_model_forward_trace(const orc_model* m, int act_quant, int frac_bits, const int64_t* ids,
                            size_t t, float* logits, float* trace);
/* Greedy generate (prefill + decode with carried state); out holds n + gen ids. */
int orc_model_generate(const orc_model* m, int act_quant, int frac_bits, const int64_t* ids,
                       size_t n, size_t gen, int64_t* out, float* last_logits);
/* Greedy lockstep serving; out is [B][stride]. */
int orc_model_generate_serve(const orc_model* m, int act_quant, int frac_bits, size_t b,
                             const int64_t* const* prompts, const size_t* lens, size_t gen,
                             int64_t* out, size_t stride, size_t* out_lens);

#ifdef __cplusplus
}
#endif
#endif
