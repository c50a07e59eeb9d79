/* mmfree_oracle.c -- TEST INFRASTRUCTURE ONLY (CPU checker for the CUDA path).
 *
 * Plain-C restatement of the reference engine's numerics. The reference's x86 build
 * (cpp/CMakeLists.txt:10,47: g++ -O2 -mavx2 -mfma, GCC default -ffp-contract=fast) fixes:
 *   - every AVX2 primitive's lane order (8 lanes, lane j owns elements 8i+j) and its
 *     horizontal-sum tree;
 *   - which mul+add pairs the compiler fused into one FMA.
 * This file is compiled with -ffp-contract=off, so every fused site is an explicit fmaf():
 *   1. hgrn_step state update      state = fma(f, state, in)   (simd.hpp:340, :354)
 *   2. forget-gate lower bound     f = fma(1-lb, f, lb)         (hgrn_model.cpp:121)
 *   3. the scalar tail (n % 8 != 0) of expf_poly, whose a*b+c forms GCC fuses
 *      (simd.hpp:215-224); the sumsq tail (simd.hpp:87) is NOT fused in that build
 * plus the FMAs the reference writes as intrinsics (sumsq, ternary_dot_f32, exp8_ps).
 * Parity of this file with the compiled reference is checked by tests/test_oracle.py.
 */
#include "mmfree_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- primitives */

/* _mm256 horizontal sum, simd.hpp:48-57: ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)). */
static float hsum8(const float v[8]) {
  float b0 = v[0] + v[4], b1 = v[1] + v[5], b2 = v[2] + v[6], b3 = v[3] + v[7];
  return (b0 + b1) + (b2 + b3);
}

/* simd.hpp:69-89. Lane j accumulates fma(x,x,acc) over elements 8i+j; then the tree. */
float orc_sumsq(const float* x, size_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t c = 0;
  for (; c + 8 <= n; c += 8)
    for (int j = 0; j < 8; ++j) acc[j] = fmaf(x[c + j], x[c + j], acc[j]);
  float s = hsum8(acc);
  for (; c < n; ++c) s += x[c] * x[c]; /* the compiled tail is not fused */
  return s;
}

/* _mm256_cvtps_epi32: round-half-even; NaN or out of int32 range gives INT32_MIN. */
static int32_t cvt_ps_epi32(float v) {
  if (isnan(v) || v >= 2147483648.0f || v < -2147483648.0f) return INT32_MIN;
  return (int32_t)nearbyintf(v);
}

/* simd.hpp:162-187: vector body (cvtps + int clamp) then scalar tail (float clamp). */
void orc_quant_q510(int32_t* yq, const float* y, float qs, size_t n) {
  size_t c = 0;
  for (; c + 8 <= n; c += 8)
    for (int j = 0; j < 8; ++j) {
      int32_t q = cvt_ps_epi32(y[c + j] * qs);
      yq[c + j] = q < -32768 ? -32768 : (q > 32767 ? 32767 : q);
    }
  for (; c < n; ++c) {
    float q = nearbyintf(y[c] * qs);
    if (q > 32767.0f) q = 32767.0f;
    else if (q < -32768.0f) q = -32768.0f;
    yq[c] = isnan(q) ? INT32_MIN : (int32_t)q; /* cvttss2si of NaN is INT32_MIN */
  }
}

/* Cephes single-precision exp constants (S. Moshier, Cephes Math Library, expf.c):
 * log2(e), ln2 split into C1 + C2, and the degree-6 minimax polynomial coefficients,
 * as the reference writes them (simd.hpp:208-249). */
#define EXP_HI 88.3762626647949f
#define EXP_LOG2E 1.44269504088896341f
#define EXP_C1 0.693359375f
#define EXP_C2 (-2.12194440e-4f)
#define EXP_P0 1.9875691500E-4f
#define EXP_P1 1.3981999507E-3f
#define EXP_P2 8.3334519073E-3f
#define EXP_P3 4.1665795894E-2f
#define EXP_P4 1.6666665459E-1f
#define EXP_P5 5.0000001201E-1f

static float pow2i(float fx) {
  uint32_t e = (uint32_t)((int32_t)fx + 127) << 23;
  float r;
  memcpy(&r, &e, sizeof r);
  return r;
}

/* One lane of exp8_ps, simd.hpp:232-249 (all FMAs are intrinsics there). */
float orc_exp8_lane(float x) {
  x = (x > -EXP_HI) ? x : -EXP_HI; /* vmaxps: NaN -> second operand */
  x = (x < EXP_HI) ? x : EXP_HI;   /* vminps */
  float fx = floorf(fmaf(x, EXP_LOG2E, 0.5f));
  float r = fmaf(-fx, EXP_C1, x);
  r = fmaf(-fx, EXP_C2, r);
  float p = EXP_P0;
  p = fmaf(p, r, EXP_P1);
  p = fmaf(p, r, EXP_P2);
  p = fmaf(p, r, EXP_P3);
  p = fmaf(p, r, EXP_P4);
  p = fmaf(p, r, EXP_P5);
  p = fmaf(p, r * r, r + 1.0f);
  return p * pow2i(fx);
}

/* expf_poly as the reference build compiles it (simd.hpp:212-229, GCC-fused). */
float orc_expf_tail(float x) {
  if (x > EXP_HI) x = EXP_HI;
  else if (x < -EXP_HI) x = -EXP_HI;
  float fx = floorf(fmaf(x, EXP_LOG2E, 0.5f));
  float r = fmaf(-fx, EXP_C1, x);
  r = fmaf(-fx, EXP_C2, r);
  float p = EXP_P0;
  p = fmaf(p, r, EXP_P1);
  p = fmaf(p, r, EXP_P2);
  p = fmaf(p, r, EXP_P3);
  p = fmaf(p, r, EXP_P4);
  p = fmaf(p, r, EXP_P5);
  p = fmaf(p, r * r, r) + 1.0f;
  return p * pow2i(fx);
}

static float neg(float x) { return -x; } /* sign flip, as the vector XOR with -0.0f */

/* simd.hpp:270-286 */
void orc_sigmoid(float* out, const float* x, size_t n) {
  size_t body = n / 8 * 8;
  for (size_t i = 0; i < body; ++i) out[i] = 1.0f / (1.0f + orc_exp8_lane(neg(x[i])));
  for (size_t i = body; i < n; ++i) out[i] = 1.0f / (1.0f + orc_expf_tail(-x[i]));
}

/* simd.hpp:289-307 */
void orc_silu(float* out, const float* x, size_t n) {
  size_t body = n / 8 * 8;
  for (size_t i = 0; i < body; ++i) out[i] = x[i] / (1.0f + orc_exp8_lane(neg(x[i])));
  for (size_t i = body; i < n; ++i) out[i] = x[i] / (1.0f + orc_expf_tail(-x[i]));
}

/* simd.hpp:310-330 */
void orc_swiglu(float* out, const float* a, const float* b, size_t n) {
  size_t body = n / 8 * 8;
  for (size_t i = 0; i < body; ++i) out[i] = (a[i] / (1.0f + orc_exp8_lane(neg(a[i])))) * b[i];
  for (size_t i = body; i < n; ++i) out[i] = (a[i] / (1.0f + orc_expf_tail(-a[i]))) * b[i];
}

/* simd.hpp:335-357, with the fused state update of the compiled reference. */
void orc_hgrn_step(float* state, float* out, const float* f, const float* in, size_t d) {
  for (size_t i = 0; i < d; ++i) {
    state[i] = fmaf(f[i], state[i], in[i]);
    out[i] = state[i];
  }
}

/* simd.hpp:92-122 */
float orc_ternary_dot_f32(const float* y, const int8_t* w, size_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t k = 0;
  for (; k + 8 <= n; k += 8)
    for (int j = 0; j < 8; ++j) acc[j] = fmaf(y[k + j], (float)w[k + j], acc[j]);
  float s = hsum8(acc);
  for (; k < n; ++k) {
    if (w[k] > 0) s += y[k];
    else if (w[k] < 0) s -= y[k];
  }
  return s;
}

/* simd.hpp:125-154: integer, wraps mod 2^32 like vpmulld/vpaddd. */
int32_t orc_ternary_dot_i32(const int32_t* yq, const int8_t* w, size_t n) {
  uint32_t s = 0;
  for (size_t k = 0; k < n; ++k) s += (uint32_t)yq[k] * (uint32_t)(int32_t)w[k];
  return (int32_t)s;
}

/* ---------------------------------------------------------------- kernels */

static float rms_rstd(const float* x, size_t cols, float eps) {
  float s = orc_sumsq(x, cols);
  return 1.0f / sqrtf(s / (float)cols + eps);
}

/* rmsnorm.cpp:11-22 */
void orc_rmsnorm(float* y, const float* x, const float* w, size_t rows, size_t cols, float eps) {
  for (size_t r = 0; r < rows; ++r) {
    const float* xr = x + r * cols;
    float rstd = rms_rstd(xr, cols, eps);
    for (size_t c = 0; c < cols; ++c) y[r * cols + c] = xr[c] * rstd * w[c];
  }
}

/* bitlinear.cpp:21-117 (FixedQ510 :39-94, Float :95-116). acc_out ([rows, out]) is filled
 * in FixedQ510 mode only. */
void orc_bitlinear(float* out, const float* x, const float* nw, const int8_t* wq, float scale_w,
                   size_t rows, size_t in_dim, size_t out_dim, float eps, float* norm_out,
                   int act_quant, int frac_bits, int32_t* acc_out) {
  const float qs = (float)(1u << frac_bits);
  const float inv_fixed = 1.0f / (qs * scale_w);
  const float inv_scale_w = 1.0f / scale_w;
  float* y = (float*)malloc(in_dim * sizeof(float));
  int32_t* yq = (int32_t*)malloc(in_dim * sizeof(int32_t));
  for (size_t r = 0; r < rows; ++r) {
    const float* xr = x + r * in_dim;
    float rstd = rms_rstd(xr, in_dim, eps);
    for (size_t c = 0; c < in_dim; ++c) y[c] = xr[c] * rstd * nw[c];
    if (norm_out) memcpy(norm_out + r * in_dim, y, in_dim * sizeof(float));
    float* orow = out + r * out_dim;
    if (act_quant == 1) {
      orc_quant_q510(yq, y, qs, in_dim);
#pragma omp parallel for schedule(static)
      for (size_t o = 0; o < out_dim; ++o) {
        int32_t a = orc_ternary_dot_i32(yq, wq + o * in_dim, in_dim);
        if (acc_out) acc_out[r * out_dim + o] = a;
        orow[o] = (float)a * inv_fixed;
      }
    } else {
#pragma omp parallel for schedule(static)
      for (size_t o = 0; o < out_dim; ++o)
        orow[o] = orc_ternary_dot_f32(y, wq + o * in_dim, in_dim) * inv_scale_w;
    }
  }
  free(y);
  free(yq);
}

/* hgrn_scan.cpp:11-19 */
void orc_hgrn_scan(float* out, const float* i, const float* f, size_t t, size_t d,
                   float* state_io) {
  float* local = NULL;
  float* state = state_io;
  if (!state) state = local = (float*)calloc(d, sizeof(float));
  for (size_t s = 0; s < t; ++s) orc_hgrn_step(state, out + s * d, f + s * d, i + s * d, d);
  free(local);
}

/* rmsnorm_swishgate.cpp:13-30 */
void orc_rmsnorm_swishgate(float* out, const float* g, const float* o, const float* w,
                           size_t rows, size_t cols, float eps) {
  float* so = (float*)malloc(cols * sizeof(float));
  for (size_t r = 0; r < rows; ++r) {
    const float* gr = g + r * cols;
    float rstd = rms_rstd(gr, cols, eps);
    orc_silu(so, o + r * cols, cols);
    for (size_t c = 0; c < cols; ++c) out[r * cols + c] = (gr[c] * rstd * w[c]) * so[c];
  }
  free(so);
}

/* ---------------------------------------------------------------- model */

typedef struct {
  size_t cap;
  float *hs, *i, *f, *g, *onemf, *scan, *recur, *oin, *oout, *resid, *y, *gate, *yh, *z;
} scratch;

static void scratch_init(scratch* s, size_t t, size_t h, size_t inter) {
  size_t th = t * h, ti = t * inter;
  s->cap = t;
  s->hs = malloc(th * 4); s->i = malloc(th * 4); s->f = malloc(th * 4); s->g = malloc(th * 4);
  s->onemf = malloc(th * 4); s->scan = malloc(th * 4); s->recur = malloc(th * 4);
  s->oin = malloc(th * 4); s->oout = malloc(th * 4); s->resid = malloc(th * 4);
  s->y = malloc(2 * ti * 4); s->gate = malloc(ti * 4); s->yh = malloc(ti * 4);
  s->z = malloc(ti * 4);
}

static void scratch_free(scratch* s) {
  free(s->hs); free(s->i); free(s->f); free(s->g); free(s->onemf); free(s->scan);
  free(s->recur); free(s->oin); free(s->oout); free(s->resid); free(s->y); free(s->gate);
  free(s->yh); free(s->z);
}

static void run_proj(const orc_proj* p, float* out, const float* x, size_t rows, float eps,
                     int aq, int frac) {
  orc_bitlinear(out, x, p->normw, p->wq, p->scale_w, rows, p->in_dim, p->out_dim, eps, NULL, aq,
                frac, NULL);
}

/* hgrn_model.cpp:80-195. stream_state: the T rows are T streams, each one step. */
/* optional per-layer trace: [recur, resid, h] x [t, H] per layer, after h0 = embeddings */
static float* g_trace = NULL;

static void block(const orc_model* m, scratch* s, float* h, size_t t, size_t l, float* rstate,
                  int stream_state, int aq, int frac) {
  const size_t H = m->hidden, I = m->inter, th = t * H;
  const orc_layer* L = &m->layer[l];
  const float eps = m->eps;
  memcpy(s->resid, h, th * 4);
  orc_rmsnorm(s->hs, h, L->attn_norm, t, H, eps);
  run_proj(&L->proj[ORC_I], s->i, s->hs, t, eps, aq, frac);
  run_proj(&L->proj[ORC_F], s->f, s->hs, t, eps, aq, frac);
  run_proj(&L->proj[ORC_G], s->g, s->hs, t, eps, aq, frac);
  orc_sigmoid(s->f, s->f, th);
  if (m->use_lower_bound && l > 0) {
    const float* lb = m->lower_bounds + l * H;
    for (size_t r = 0; r < t; ++r)
      for (size_t c = 0; c < H; ++c) s->f[r * H + c] = fmaf(1.0f - lb[c], s->f[r * H + c], lb[c]);
  }
  for (size_t n = 0; n < th; ++n) s->onemf[n] = 1.0f - s->f[n];
  orc_swiglu(s->scan, s->i, s->onemf, th);
  if (stream_state) {
    for (size_t b = 0; b < t; ++b)
      orc_hgrn_step(rstate + b * H, s->recur + b * H, s->f + b * H, s->scan + b * H, H);
  } else {
    orc_hgrn_scan(s->recur, s->scan, s->f, t, H, rstate);
  }
  orc_rmsnorm_swishgate(s->oin, s->g, s->recur, L->g_norm, t, H, eps);
  run_proj(&L->proj[ORC_O], s->oout, s->oin, t, eps, aq, frac);
  for (size_t n = 0; n < th; ++n) s->resid[n] += s->oout[n];
  orc_rmsnorm(s->hs, s->resid, L->mlp_norm, t, H, eps);
  run_proj(&L->proj[ORC_GATE], s->y, s->hs, t, eps, aq, frac);
  for (size_t r = 0; r < t; ++r) {
    memcpy(s->gate + r * I, s->y + r * 2 * I, I * 4);
    memcpy(s->yh + r * I, s->y + r * 2 * I + I, I * 4);
  }
  orc_swiglu(s->z, s->gate, s->yh, t * I);
  run_proj(&L->proj[ORC_DOWN], s->oout, s->z, t, eps, aq, frac);
  for (size_t n = 0; n < th; ++n) h[n] = s->resid[n] + s->oout[n];
  if (g_trace) {
    float* tr = g_trace + th + l * 3 * th;
    memcpy(tr, s->recur, th * 4);
    memcpy(tr + th, s->resid, th * 4);
    memcpy(tr + 2 * th, h, th * 4);
  }
}

static void embed(const orc_model* m, float* h, const int64_t* ids, size_t t) {
  for (size_t r = 0; r < t; ++r)
    memcpy(h + r * m->hidden, m->embeddings + (size_t)ids[r] * m->hidden, m->hidden * 4);
}

/* greedy pick, hgrn_model.cpp:271-273: strict '>' keeps the lowest index on ties. */
static int64_t argmax_first(const float* lg, size_t v) {
  size_t c = 0;
  for (size_t k = 1; k < v; ++k)
    if (lg[k] > lg[c]) c = k;
  return (int64_t)c;
}

static void head(const orc_model* m, const float* hrow, float* logits, size_t rows, int aq,
                 int frac) {
  float* fn = malloc(rows * m->hidden * 4);
  orc_rmsnorm(fn, hrow, m->final_norm, rows, m->hidden, m->eps);
  run_proj(&m->lm_head, logits, fn, rows, m->eps, aq, frac);
  free(fn);
}

static int check_ids(const orc_model* m, const int64_t* ids, size_t n) {
  for (size_t k = 0; k < n; ++k)
    if (ids[k] < 0 || (size_t)ids[k] >= m->vocab) return -1;
  return 0;
}

/* hgrn_model.cpp:220-247 */
int orc_model_forward(const orc_model* m, int aq, int frac, const int64_t* ids, size_t t,
                      float* logits) {
  if (t == 0 || check_ids(m, ids, t)) return -1;
  scratch s;
  scratch_init(&s, t, m->hidden, m->inter);
  float* h = malloc(t * m->hidden * 4);
  embed(m, h, ids, t);
  for (size_t l = 0; l < m->layers; ++l) block(m, &s, h, t, l, NULL, 0, aq, frac);
  head(m, h, logits, t, aq, frac);
  free(h);
  scratch_free(&s);
  return 0;
}

/* orc_model_forward plus trace (1 + 3L) x [t, H]: embeddings, then per layer the
 * recurrence output, the residual after o_proj and the layer output. */
int orc_model_forward_trace(const orc_model* m, int aq, int frac, const int64_t* ids, size_t t,
                            float* logits, float* trace) {
  if (t == 0 || check_ids(m, ids, t)) return -1;
  for (size_t r = 0; r < t; ++r)
    memcpy(trace + r * m->hidden, m->embeddings + (size_t)ids[r] * m->hidden, m->hidden * 4);
  g_trace = trace;
  int rc = orc_model_forward(m, aq, frac, ids, t, logits);
  g_trace = NULL;
  return rc;
}

/* hgrn_model.cpp:249-347 (greedy, no EOS). */
int orc_model_generate(const orc_model* m, int aq, int frac, const int64_t* ids, size_t n,
                       size_t gen, int64_t* out, float* last_logits) {
  if (n == 0 || check_ids(m, ids, n)) return -1;
  const size_t H = m->hidden, V = m->vocab, L = m->layers;
  scratch s;
  scratch_init(&s, n, H, m->inter);
  float* h = malloc(n * H * 4);
  float* state = calloc(L * H, 4);
  float* lg = malloc(V * 4);
  memcpy(out, ids, n * 8);
  size_t len = n;
  embed(m, h, ids, n);
  for (size_t l = 0; l < L; ++l) block(m, &s, h, n, l, state + l * H, 0, aq, frac);
  if (gen > 0) {
    head(m, h + (n - 1) * H, lg, 1, aq, frac);
    out[len++] = argmax_first(lg, V);
    for (size_t step = 1; step < gen; ++step) {
      embed(m, h, out + len - 1, 1);
      for (size_t l = 0; l < L; ++l) block(m, &s, h, 1, l, state + l * H, 0, aq, frac);
      head(m, h, lg, 1, aq, frac);
      out[len++] = argmax_first(lg, V);
    }
    if (last_logits) memcpy(last_logits, lg, V * 4);
  }
  free(h); free(state); free(lg);
  scratch_free(&s);
  return 0;
}

/* hgrn_model.cpp:349-454 (greedy, no EOS). Every stream gets at least one new token. */
int orc_model_generate_serve(const orc_model* m, int aq, int frac, size_t b,
                             const int64_t* const* prompts, const size_t* lens, size_t gen,
                             int64_t* out, size_t stride, size_t* out_lens) {
  const size_t H = m->hidden, V = m->vocab, L = m->layers;
  size_t maxt = b;
  for (size_t k = 0; k < b; ++k) {
    if (lens[k] == 0 || check_ids(m, prompts[k], lens[k])) return -1;
    if (lens[k] > maxt) maxt = lens[k];
    if (lens[k] + (gen > 0 ? gen : 1) > stride) return -1;
  }
  scratch s;
  scratch_init(&s, maxt, H, m->inter);
  float* h = malloc(maxt * H * 4);
  float* state = calloc(L * b * H, 4);
  float* lg = malloc(b * V * 4);
  for (size_t k = 0; k < b; ++k) {
    size_t t = lens[k];
    memcpy(out + k * stride, prompts[k], t * 8);
    out_lens[k] = t;
    embed(m, h, prompts[k], t);
    for (size_t l = 0; l < L; ++l) block(m, &s, h, t, l, state + (l * b + k) * H, 0, aq, frac);
    /* the first token is emitted even when gen == 0 (hgrn_model.cpp:422-427) */
    head(m, h + (t - 1) * H, lg, 1, aq, frac);
    out[k * stride + out_lens[k]++] = argmax_first(lg, V);
  }
  for (size_t step = 1; step < gen; ++step) {
    for (size_t k = 0; k < b; ++k) embed(m, h + k * H, out + k * stride + out_lens[k] - 1, 1);
    for (size_t l = 0; l < L; ++l) block(m, &s, h, b, l, state + l * b * H, 1, aq, frac);
    head(m, h, lg, b, aq, frac);
    for (size_t k = 0; k < b; ++k) out[k * stride + out_lens[k]++] = argmax_first(lg + k * V, V);
  }
  free(h); free(state); free(lg);
  scratch_free(&s);
  return 0;
}
