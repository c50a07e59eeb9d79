/* mmfree_cuda.h -- C ABI of the B200 (sm_100a) HGRN-Bit engine, libmmfree_cuda.so.
 *
 * Drop-in for the hot path of the matmulfreellmCPU C++ engine. Every entry point names the
 * reference interface it replaces (paths inside the reference project). Conventions:
 *   - every function returns MMFREE_OK (0) or a negative MMFREE_E_* code; the message of the
 *     last failure on the calling thread is mmfree_cuda_last_error();
 *   - kernel entry points take DEVICE pointers and a cudaStream_t passed as void* (NULL =
 *     the legacy default stream); they are asynchronous like any CUDA launch;
 *   - model entry points take HOST buffers and return when their results are in them;
 *   - act_quant is MMFREE_ACT_FLOAT (the reference's ActQuant::Float) or
 *     MMFREE_ACT_FIXED_Q510 (ActQuant::FixedQ510, static Q(15-f).f int16 activations with an
 *     int32 accumulator); frac_bits is the reference's --frac (10 = Q5.10).
 * FixedQ510 results are bit-identical to the reference's x86 AVX2 build; Float results agree
 * to fp32 reduction-order noise. There is no CPU fallback: without a CUDA device every call
 * fails with MMFREE_E_CUDA.
 * Like the reference kernels (bitlinear.cpp:49-53), the kernel entry points share one
 * library-owned scratch arena per device and are not re-entrant across host threads; the
 * arena grows with cudaMalloc on first use of a larger shape, so call once outside any
 * stream capture before capturing. A model handle must be used by one host thread at a time.
 */
#ifndef MMFREE_CUDA_H
#define MMFREE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MMFREE_CUDA_ABI_VERSION 2

enum {
  MMFREE_OK = 0,
  MMFREE_E_INVALID = -1, /* bad argument (null pointer, zero or oversize dimension, ...) */
  MMFREE_E_CUDA = -2,    /* CUDA runtime error (no device, launch failure, out of memory) */
  MMFREE_E_IO = -3,      /* blob file missing, unreadable or malformed */
  MMFREE_E_RANGE = -4,   /* token id outside [0, vocab_size) or code outside int16 */
  MMFREE_E_STATE = -5,   /* call out of order (e.g. serve_step without serve_begin) */
  MMFREE_E_INTERNAL = -6,
  MMFREE_E_TIMEOUT = -7  /* a bounded wait inside a kernel gave up (its outputs are undefined) */
};

enum { MMFREE_ACT_FLOAT = 0, MMFREE_ACT_FIXED_Q510 = 1 };

/* Largest in_dim accepted by the kernel entry points (one row is staged in shared memory). */
#define MMFREE_CUDA_MAX_IN_DIM 57344

const char* mmfree_cuda_last_error(void);
int mmfree_cuda_abi_version(void);

/* ---- packed ternary weights ---------------------------------------------------------
 * The reference keeps int8 {-1,0,+1} weights [out_dim, in_dim] (kernels.hpp:32-33,
 * weights.hpp:34). The CUDA engine streams them as 2 bits per weight in a tiled layout
 * (32-row groups x 64-column chunks, 512 bytes each); these calls produce it. */
size_t mmfree_cuda_packed_bytes(size_t out_dim, size_t in_dim);
/* device int8 [out_dim, in_dim] -> device packed (mmfree_cuda_packed_bytes bytes). */
int mmfree_cuda_repack_ternary(void* dst, const int8_t* wq, size_t out_dim, size_t in_dim,
                               void* stream);
/* Same format computed on the host (for offline caches and tests). */
int mmfree_cuda_pack_ternary_host(void* dst, const int8_t* wq, size_t out_dim, size_t in_dim);

/* ---- kernel entry points (device pointers) ------------------------------------------- */

/* Replaces mmfree::bitlinear (kernels.hpp:41-44, bitlinear.cpp:21-117): per row
 * RMSNorm(eps) * norm_weight, then Float or FixedQ510 activation handling, ternary
 * accumulate and dequant. out [rows, out_dim]; x [rows, in_dim]; norm_out (nullable)
 * [rows, in_dim]; acc_out (nullable, FixedQ510 only) [rows, out_dim] int32 accumulators,
 * the values a TernaryBackend would produce (ternary_backend.hpp:26-31). */
int mmfree_cuda_bitlinear(float* out, const float* x, const float* norm_weight,
                          const void* wpacked, float scale_w, size_t rows, size_t in_dim,
                          size_t out_dim, float eps, float* norm_out, int act_quant,
                          int frac_bits, int32_t* acc_out, void* stream);

/* Status of the asynchronous kernel entry points (mmfree_cuda_bitlinear,
 * mmfree_cuda_bitlinear_cluster, mmfree_cuda_bitlinear_noalloc). They return once their
 * kernels are queued; a failure inside a kernel (a bounded wait that gave up) is recorded in
 * a device error word instead. This call synchronizes `stream` (the stream those calls used),
 * reads and clears the calling device's words and returns MMFREE_OK, or MMFREE_E_TIMEOUT when
 * a call since the last check failed -- the outputs of those calls are then undefined. It
 * allocates nothing. No reference counterpart: the reference kernels are synchronous host
 * code that cannot time out. */
int mmfree_cuda_kernel_status(void* stream);

/* Diagnostic switch: the number of polls after which the BitLinear prologue's wait for its
 * staged input row gives up (raising the error mmfree_cuda_kernel_status reports) in kernels
 * launched from now on, by this process; a negative value restores the default (2^22).
 * 0 makes every staged wait give up at once: a way to test a caller's error handling without
 * faulting the GPU. Model handles capture the value in force when they build a decode graph. */
void mmfree_cuda_set_wait_limit(int64_t polls);

/* Size of the static device scratch used by mmfree_cuda_bitlinear_noalloc (4 MiB, of which
 * the first 256 bytes hold the calls' error word). */
#define MMFREE_CUDA_NOALLOC_SCRATCH_BYTES (4u << 20)

/* mmfree_cuda_bitlinear for callers that cannot allocate device memory. It has no
 * counterpart in the reference (whose CPU kernels keep their scratch in static host
 * buffers, bitlinear.cpp:49-53).
 *
 * Who needs it: code that runs where cudaMalloc is unavailable or forbidden -- a plugin
 * inside a host process whose allocator owns the whole device (a serving framework's
 * memory pool, a pre-partitioned GPU), a latency-critical decode loop that must never
 * block on an allocation, or work issued while a stream is being captured into a CUDA
 * graph, where cudaMalloc is not a legal call. mmfree_cuda_bitlinear grows a library-owned
 * scratch arena with cudaMalloc on first use of a larger shape; this variant instead uses
 * a fixed array compiled into the library (one per device that loads it, held until the
 * process exits) and calls no allocating routine on its success path.
 *
 * Same arguments, semantics, kernels and results as mmfree_cuda_bitlinear. Limits and rules:
 *   - scratch need: 256 bytes of error word, plus FixedQ510 2*rows*ceil64(in_dim) + 4*rows
 *     bytes or Float 4*rows*ceil64(in_dim) bytes (each rounded up to 256); a call needing
 *     more than MMFREE_CUDA_NOALLOC_SCRATCH_BYTES fails with MMFREE_E_INVALID and allocates
 *     nothing;
 *   - the first call on a device looks up that device's copy of the array
 *     (cudaGetSymbolAddress, which can load the module) and zeroes its error word: make it
 *     before any stream capture (a failed lookup is retried by the next call);
 *   - every call on a device shares the one array, which keeps the last call's contents;
 *     the planes need not start at zero (each call writes all it reads), but calls whose
 *     kernels overlap on the GPU (different streams, or different host threads) race on it;
 *   - a kernel that gives up a bounded wait sets the array's error word and leaves the
 *     call's outputs undefined; mmfree_cuda_kernel_status reports and clears it.
 */
int mmfree_cuda_bitlinear_noalloc(float* out, const float* x, const float* norm_weight,
                                  const void* wpacked, float scale_w, size_t rows,
                                  size_t in_dim, size_t out_dim, float eps, float* norm_out,
                                  int act_quant, int frac_bits, int32_t* acc_out, void* stream);

/* Replaces mmfree::bitlinear_cluster (kernels.hpp:50-53, bitlinear.cpp:119-159): k <= 3
 * FixedQ510 projections sharing x, each with its own norm weight, packed weight, scale and
 * output. outs / norm_weights / wpacked are HOST arrays of k device pointers, scale_w a
 * host array of k floats; acc_out (nullable) is [k, rows, out_dim]. */
int mmfree_cuda_bitlinear_cluster(float* const* outs, const float* x,
                                  const float* const* norm_weights,
                                  const void* const* wpacked, const float* scale_w, int k,
                                  size_t rows, size_t in_dim, size_t out_dim, float eps,
                                  int frac_bits, int32_t* acc_out, void* stream);

/* Replaces TernaryBackend::matmul_batch (ternary_backend.hpp:43-48): acc[i*M + m] =
 * sum_n x[i*N + n] * wq[m, n] for b rows of int32 activations in int16 range. */
int mmfree_cuda_ternary_matmul(int32_t* acc, const int32_t* x, const void* wpacked, size_t N,
                               size_t M, size_t b, void* stream);

/* The TernaryBackend seam on HOST buffers (ternary_backend.hpp:26-59), for callers that keep
 * the reference's own Model and offload only the integer accumulate, as an accelerator
 * backend does (include/mmfree_cuda_backend.hpp wraps it as a mmfree::TernaryBackend).
 * seam_matmul: acc[i*M + m] = sum_n x[i*N + n] * wq[m*N + n] for b rows (the arguments of
 * TernaryBackend::matmul_batch, ternary_backend.hpp:43-48); returns when acc is written.
 * wq is uploaded and repacked on the GPU the first time its (pointer, M, N) is seen and kept
 * until seam_close: the weights behind a pointer must not change meanwhile (the reference's
 * are an immutable mmap, weights.cpp:191-254). Codes outside int16 give MMFREE_E_RANGE.
 * A seam is used by one host thread at a time. */
typedef struct mmfree_cuda_seam mmfree_cuda_seam;
int mmfree_cuda_seam_open(int device, mmfree_cuda_seam** out);
int mmfree_cuda_seam_matmul(mmfree_cuda_seam* s, const int8_t* wq, size_t N, size_t M,
                            const int32_t* x, int32_t* acc, size_t b);
void mmfree_cuda_seam_close(mmfree_cuda_seam* s);

/* Replaces mmfree::rmsnorm (kernels.hpp:29-30, rmsnorm.cpp:11-22). */
int mmfree_cuda_rmsnorm(float* y, const float* x, const float* weight, size_t rows,
                        size_t cols, float eps, void* stream);
/* Replaces mmfree::swiglu (kernels.hpp:56, activations.cpp:9-15): out = silu(a) * b. */
int mmfree_cuda_swiglu(float* out, const float* a, const float* b, size_t n, void* stream);
/* Replaces mmfree::hgrn_scan (kernels.hpp:61-62, hgrn_scan.cpp:11-19); state_io nullable. */
int mmfree_cuda_hgrn_scan(float* out, const float* i, const float* f, size_t T, size_t D,
                          float* state_io, void* stream);
/* Replaces mmfree::rmsnorm_swishgate (kernels.hpp:65-66, rmsnorm_swishgate.cpp:13-30). */
int mmfree_cuda_rmsnorm_swishgate(float* out, const float* g, const float* o,
                                  const float* weight, size_t rows, size_t cols, float eps,
                                  void* stream);

/* ---- model (host buffers) ------------------------------------------------------------ */
typedef struct mmfree_cuda_model mmfree_cuda_model;

typedef struct {
  size_t vocab_size, hidden_size, num_hidden_layers, num_heads, expand_ratio,
      intermediate_size;
  int use_lower_bound, use_short_conv;
  float rms_norm_eps;
} mmfree_cuda_config; /* mirrors mmfree::Config (config.hpp:8-21) */

/* Parses only the header of a model.mmfree blob (mmfree::Weights(path).config(),
 * weights.cpp:191-235 + weights.hpp:44); needs no GPU. MMFREE_E_IO on a bad file. */
int mmfree_cuda_blob_config(const char* blob_path, mmfree_cuda_config* out);

/* Replaces mmfree::Weights(path) + mmfree::Model(w, aq, frac_bits) (weights.cpp:191-254,
 * model.hpp:33-34): parses model.mmfree, uploads it to `device` and repacks the ternary
 * weights. Errors: MMFREE_E_IO (file/format), MMFREE_E_CUDA, MMFREE_E_INVALID. */
int mmfree_cuda_model_open(const char* blob_path, int device, int act_quant, int frac_bits,
                           mmfree_cuda_model** out);
void mmfree_cuda_model_close(mmfree_cuda_model* m);

/* ---- tensor-parallel prefill (configuration 4: one process per GPU, NCCL over NVLink) ---
 * No reference counterpart: the reference is one CPU process. A TP handle is rank `rank` of
 * `world` and holds only its shards of the per-layer BitLinear weights; its prefill
 * (mmfree_cuda_forward, _forward_last, _serve_begin -- every rank calls it with the same
 * ids, and every rank gets the full result) splits each layer of hgrn_model.cpp:80-195:
 *   FixedQ510: every projection column-parallel, an NCCL all-gather of the column slices
 *              before each exact full-row norm; bit-identical to one GPU;
 *   Float:     i/f/g/gate column-parallel, o/down row-parallel; an NCCL all-reduce of
 *              per-row partial sums of squares before g_norm, o_proj and down_proj, and one
 *              of the row-parallel outputs; within the Float tolerance of one GPU.
 * Decode calls on a TP handle fail with MMFREE_E_STATE. hidden_size and intermediate_size
 * must be multiples of 32 * world; the blob must be the int8 model.mmfree. NCCL
 * (libnccl.so.2) is loaded when the first TP call needs it.
 * nccl_unique_id: 128 bytes that rank 0 creates and the caller sends to every rank (for
 * example with MPI_Bcast or torch.distributed.broadcast) before each calls model_open_tp;
 * model_open_tp is collective: it returns on a rank once every rank has called it. */
int mmfree_cuda_nccl_unique_id(unsigned char* out);
int mmfree_cuda_model_open_tp(const char* blob_path, int device, int act_quant, int frac_bits,
                              int rank, int world, const unsigned char* nccl_id,
                              mmfree_cuda_model** out);
int mmfree_cuda_model_config(const mmfree_cuda_model* m, mmfree_cuda_config* out);
size_t mmfree_cuda_model_weight_bytes(const mmfree_cuda_model* m); /* packed ternary bytes */

/* Replaces Model::generate (model.hpp:36-50): out_ids receives prompt + generated ids
 * (*out_len of them; out_cap >= n + new_tokens). temperature <= 0 is greedy. */
int mmfree_cuda_generate(mmfree_cuda_model* m, const int64_t* ids, size_t n,
                         size_t new_tokens, int64_t eos_id, float temperature, int top_k,
                         uint64_t seed, int64_t* out_ids, size_t out_cap, size_t* out_len);

/* Model::generate with its streaming hook (model.hpp:44-50, `on_token`): the same
 * arguments and results as mmfree_cuda_generate, and on_token(id, ctx) is called on the
 * calling thread with every generated id in order as soon as the host has it -- each step
 * when eos_id >= 0 (the step's id is read back to test it), otherwise once the device loop
 * is done. on_token may be NULL. */
typedef void (*mmfree_cuda_token_fn)(int64_t id, void* ctx);
int mmfree_cuda_generate_stream(mmfree_cuda_model* m, const int64_t* ids, size_t n,
                                size_t new_tokens, int64_t eos_id, float temperature, int top_k,
                                uint64_t seed, mmfree_cuda_token_fn on_token, void* ctx,
                                int64_t* out_ids, size_t out_cap, size_t* out_len);

/* Replaces Model::forward (model.hpp:34): logits [T, vocab_size]. */
int mmfree_cuda_forward(mmfree_cuda_model* m, const int64_t* ids, size_t T, float* logits);
/* The last row of Model::forward only (what mmfree-cli --logits-out writes, main.cpp:217-224). */
int mmfree_cuda_forward_last(mmfree_cuda_model* m, const int64_t* ids, size_t T,
                             float* logits);

/* Model::forward plus an intermediate trace for parity debugging (the counterpart of the
 * reference spec's capture hooks, tools/reference.py:108-117): logits [T, vocab_size] and
 * trace [(1 + 3 L), T, hidden_size] = embeddings, then per layer the recurrence output,
 * the residual after o_proj and the layer output. */
int mmfree_cuda_forward_trace(mmfree_cuda_model* m, const int64_t* ids, size_t T, float* logits,
                              float* trace);

/* Replaces Model::generate_serve (model.hpp:52-70): B prompts (host pointers + lengths);
 * out is [B, out_stride], stream b's full ids in out[b*out_stride ...], length out_lens[b]. */
int mmfree_cuda_generate_serve(mmfree_cuda_model* m, size_t B, const int64_t* const* prompts,
                               const size_t* lens, size_t new_tokens, int64_t eos_id,
                               float temperature, int top_k, uint64_t seed, int64_t* out,
                               size_t out_stride, size_t* out_lens);

/* Step-wise lockstep serving (the decode loop of hgrn_model.cpp:432-452 exposed one step per
 * call, greedy). begin prefills the B prompts and writes each stream's first token;
 * step feeds one token per stream and returns the next; run performs `steps` steps on the
 * device from the last tokens and writes [B, steps] ids; end releases the session. */
int mmfree_cuda_serve_begin(mmfree_cuda_model* m, size_t B, const int64_t* const* prompts,
                            const size_t* lens, int64_t* first_ids);
int mmfree_cuda_serve_step(mmfree_cuda_model* m, const int64_t* in_ids, int64_t* out_ids);
int mmfree_cuda_serve_run(mmfree_cuda_model* m, size_t steps, int64_t* out);
int mmfree_cuda_serve_end(mmfree_cuda_model* m);

/* ---- measurement (no reference counterpart: the reference times host code with its
 * Profiler, profile.hpp:20-73; device work is timed with CUDA events instead) ---------- */
/* The cudaStream_t (as void*) every kernel of the model is launched on, for event timing. */
void* mmfree_cuda_model_stream(mmfree_cuda_model* m);

typedef struct {
  const char* name;  /* kernel class: prep, bitlinear_matmul, lm_head_matmul, mixer, ... */
  double ms;         /* summed device time of its launches */
  int64_t launches;
  double bytes;      /* algorithmic bytes moved */
  double ops;        /* algorithmic ops (2*M*K*N per BitLinear matmul) */
} mmfree_cuda_kernel_stats;

/* Runs `steps` greedy decode steps of the active serving session (like serve_run, but not
 * graph-captured) with a CUDA event pair around every launch; fills up to max_classes
 * entries of out and sets *n_classes. */
int mmfree_cuda_serve_profile(mmfree_cuda_model* m, size_t steps, mmfree_cuda_kernel_stats* out,
                              int max_classes, int* n_classes);

#ifdef __cplusplus
}
#endif
#endif /* MMFREE_CUDA_H */
