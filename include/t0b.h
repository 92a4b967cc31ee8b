/*
 * t0b.h -- C ABI of the B200-native t0-alpha quantized forecast engine
 * (libt0b.so).  Plain pointers and sizes only; every entry point returns a
 * t0b_status and never aborts.  The message of the last failure on the
 * calling thread is available from t0b_last_error().
 *
 * Each entry point names the reference (idle-intelligence/t0-web) interface
 * it replaces.  The reference boundary is the Rust crate API of `t0-fast`
 * (crates/t0-fast/src/lib.rs) plus the GGUF codec of `t0-core`
 * (crates/t0-core/src/gguf.rs); a Rust engine crate binds these symbols
 * through an `extern "C"` block.
 *
 * Threading: an engine may be shared by several models; a model is not
 * thread-safe (mirrors `GpuModel`/`Pool` being !Sync, pool.rs:9-16).  All
 * device work of a model runs on the model's CUDA stream.
 */
#ifndef T0B_H
#define T0B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int t0b_status;
enum {
  T0B_OK = 0,
  T0B_ERR_INVALID = 1,     /* bad argument (shape, size, pointer) */
  T0B_ERR_FORMAT = 2,      /* malformed GGUF / metadata */
  T0B_ERR_UNSUPPORTED = 3, /* valid input outside what this engine runs */
  T0B_ERR_CUDA = 4,        /* CUDA runtime error */
  T0B_ERR_OOM = 5,         /* device allocation failed */
  T0B_ERR_DEVICE = 6       /* a kernel reported an error (e.g. a bounded wait ran out) */
};

/* ggml tensor type ids (gguf.rs:32-39) */
enum { T0B_F32 = 0, T0B_F16 = 1, T0B_Q4_0 = 2, T0B_Q8_0 = 8 };

typedef struct t0b_engine t0b_engine;
typedef struct t0b_model t0b_model;

typedef struct {
  int32_t embed_dim, num_layers, num_heads, mlp_hidden_dim, patch_size, group_every_n;
  float dropout;
  int32_t n_quantiles;
  float quantile_levels[32];
  int32_t scaler_use_arcsinh;
  float scaler_eps;
  int32_t variance_offset; /* 1 = "variance_offset", 0 = "std_clamp" */
  int32_t weight_type;     /* ggml type of the four big per-layer matmuls */
  uint64_t quantizable_gpu_bytes; /* GpuModel::quantizable_gpu_bytes, model.rs:194-199 */
  uint64_t total_weight_bytes;    /* GpuModel::total_weight_bytes, model.rs:208-225 */
} t0b_model_info;

/* Thread-local message of the last failure ("" if none). */
const char *t0b_last_error(void);

/* ---- engine: device context (replaces Engine::new, engine.rs:62-111) ---- */
t0b_status t0b_engine_create(int device, t0b_engine **out);
void t0b_engine_destroy(t0b_engine *e);

/* ---- model: GGUF-resident weights (replaces load_model_from_gguf,
 * lib.rs:42-44 -> GpuModel::load_from_gguf_bytes, model.rs:302-348).
 * The bytes are copied; Q8_0/Q4_0 blocks stay in llama.cpp's exact layout in
 * device memory, every other tensor is expanded from f16 to f32. */
t0b_status t0b_model_load_gguf(t0b_engine *e, const uint8_t *bytes, size_t len, t0b_model **out);
void t0b_model_destroy(t0b_model *m);
t0b_status t0b_model_info_get(const t0b_model *m, t0b_model_info *out);
/* Run the model's work on `stream` (a cudaStream_t; NULL = the model's own
 * stream). */
t0b_status t0b_model_set_stream(t0b_model *m, void *stream);
void *t0b_model_stream(const t0b_model *m);
/* Upper bound on tokens (rows x patches) per device pass; larger requests are
 * split into passes.  Default 393216 (about 8 GB of workspace for t0-alpha). */
t0b_status t0b_model_set_max_tokens(t0b_model *m, size_t max_tokens);
/* Replay each forecast pass from a CUDA graph (default on).  A pass's launch
 * sequence is captured the first time its shape, input/output pointers and
 * workspace are seen, and replayed afterwards, so per-kernel host launch
 * overhead is paid once per shape; graphs are not used while profiling is on.
 * No reference counterpart (t0-fast records one wgpu command buffer per
 * forward, model.rs:755-786). */
t0b_status t0b_model_use_graphs(t0b_model *m, int on);

/* ---- forecasts (host buffers; synchronous) ----
 * Output layout [rows, horizon, n_quantiles] row-major, quantile-minor.
 * NaN in a context marks a missing observation.  horizon rounded up to the
 * patch size must not exceed 1024 (lib.rs:58-62). */

/* One (possibly multivariate, joint) series of v rows sharing one group id:
 * t0_fast::forecast, lib.rs:102-109. */
t0b_status t0b_forecast(t0b_model *m, const float *ctx, size_t v, size_t t_ctx, size_t horizon, float *out);

/* n independent univariate series [n, t_ctx]: t0_fast::forecast_batch_chunked,
 * lib.rs:118-146.  `chunk` bounds series per device pass (0 = all). */
t0b_status t0b_forecast_batch(t0b_model *m, const float *ctx, size_t n, size_t t_ctx, size_t horizon,
                              size_t chunk, float *out);

/* n independent univariate series of different lengths, concatenated:
 * t0_fast::forecast_batch_rows_chunked, lib.rs:175-248. */
t0b_status t0b_forecast_batch_rows(t0b_model *m, const float *ctx, const size_t *lengths, size_t n,
                                   size_t horizon, size_t chunk, float *out);

/* n_series independent multivariate series; series i has n_variates[i] rows
 * (concatenated, [sum v_i, t_ctx]).  Each series is one joint forecast
 * (t0_fast::forecast semantics per series).  No reference counterpart: the
 * reference needs one `forecast` call per multivariate series. */
t0b_status t0b_forecast_multiseries(t0b_model *m, const float *ctx, const int32_t *n_variates,
                                    size_t n_series, size_t t_ctx, size_t horizon, float *out);

/* Same as t0b_forecast_multiseries with DEVICE pointers, asynchronous on the
 * model's stream (ctx_dev [sum v_i, t_ctx] f32, out_dev [sum v_i, horizon,
 * n_q] f32).  n_variates stays a host array. */
t0b_status t0b_forecast_multiseries_device(t0b_model *m, const float *ctx_dev, const int32_t *n_variates,
                                           size_t n_series, size_t t_ctx, size_t horizon, float *out_dev);

/* Autoregressive rollout for horizons beyond one forward pass (replaces
 * t0_fast::forecast_rollout, lib.rs:259-345, itself t0-core model.rs:582-665):
 * one univariate series; a first block of up to 1024 steps, then blocks in
 * which each query level's quantile path is fed back as observed context
 * (trailing window of round_up(t_ctx, patch) values), the paths forecast as
 * one batch, and each step re-reduced to the query levels (quantile.rs).
 * query: n_query levels ascending inside (0, 1).  Output
 * [prediction_length, n_query] row-major. */
t0b_status t0b_forecast_rollout(t0b_model *m, const float *ctx, size_t t_ctx, size_t prediction_length,
                                const float *query, size_t n_query, float *out);

/* Block until the model's stream is idle and report any kernel-side error. */
t0b_status t0b_model_sync(t0b_model *m);

/* ---- measurement (no reference counterpart: the reference times whole
 * forecasts with Instant, main.rs:719-740) ----
 * With profiling on, every kernel launch of the model is bracketed by CUDA
 * events on the model's stream; t0b_model_profile_read synchronizes and
 * returns, per kernel class, launches, total device time and algorithmic
 * work.  Classes: 0 gemm_tc, 1 gemm_small, 2 attn_time, 3 attn_group, 4 prep,
 * 5 sgemm, 6 other. */
typedef struct {
  char name[16];
  uint64_t launches;
  double total_ms;
  double flops; /* algorithmic (useful) FLOPs summed over launches */
  double bytes; /* algorithmic HBM bytes summed over launches */
} t0b_kernel_stats;
t0b_status t0b_model_profile_enable(t0b_model *m, int on); /* also resets the statistics */
t0b_status t0b_model_profile_read(t0b_model *m, t0b_kernel_stats *out, int max_classes, int *n_classes);
/* Kernel launches issued by this model since it was created. */
uint64_t t0b_model_launch_count(const t0b_model *m);

/* ---- standalone dequant-GEMMs (device pointers, model-independent) ----
 * y[M,N] = x[M,K] . deq(W)[N,K]^T (+ bias[N]); W is raw Q8_0/Q4_0 blocks in
 * llama.cpp layout, row n at n * (K/32) * block_bytes.  Replaces t0-fast's
 * internal linear() dispatcher (model.rs:406-504) for quantized weights.
 * Runs on `stream` (cudaStream_t, NULL = legacy default stream). */
t0b_status t0b_gemm_q(t0b_engine *e, int ggml_type, const void *w_dev, int N, int K, const float *x_dev, int M,
                      const float *bias_dev, float *y_dev, void *stream);

/* Fused SwiGLU MLP on quantized weights (ops.rs:49-62, silu_mul.wgsl):
 * w0 [2F, K] (gate rows [0,F), up rows [F,2F)), w2 [N2, F];
 * z = silu(x.gate^T + b0g) * (x.up^T + b0u) ([M, F], written to z_dev if
 * non-NULL), y = z . w2^T + b2 ([M, N2]).  Biases may be NULL. */
t0b_status t0b_swiglu_q(t0b_engine *e, int ggml_type, const void *w0_dev, const void *w2_dev, int F, int K,
                        int N2, const float *x_dev, int M, const float *b0_dev, const float *b2_dev,
                        float *z_dev, float *y_dev, void *stream);

/* ---- resident-weight dequant-GEMMs (asynchronous) ----
 * The same GEMMs as t0b_gemm_q / t0b_swiglu_q on a weight matrix that stays
 * resident, the way t0-fast's GpuModel keeps its quantized buffers
 * (model.rs:302-348) and runs linear() on them (model.rs:406-504).
 * t0b_qmatrix_create reads the matrix once (synchronously) for its
 * tensor-core prescale; the matrix must stay valid and unchanged while the
 * handle lives.  t0b_qmatrix_gemm and t0b_qmatrix_swiglu only queue work on
 * `stream` (no host synchronisation, so they can be captured in a CUDA graph)
 * except when the handle's activation scratch has to grow, which first waits
 * for `stream`.  Kernel-side errors are reported by t0b_qmatrix_sync.  The
 * handles of one engine share the engine's activation scratch (as
 * t0b_gemm_q does): their launches must not overlap on different streams,
 * and a handle is not thread-safe. */
typedef struct t0b_qmatrix t0b_qmatrix;
t0b_status t0b_qmatrix_create(t0b_engine *e, int ggml_type, const void *w_dev, int N, int K, t0b_qmatrix **out);
void t0b_qmatrix_destroy(t0b_qmatrix *q);
/* y[M, N] = x[M, K] . deq(W)^T (+ bias[N]) */
t0b_status t0b_qmatrix_gemm(t0b_qmatrix *q, const float *x_dev, int M, const float *bias_dev, float *y_dev,
                            void *stream);
/* q0 = w0 [2F, K] (gate rows, then up rows), q2 = w2 [N2, F]; same outputs as
 * t0b_swiglu_q.  Errors are reported by both handles. */
t0b_status t0b_qmatrix_swiglu(t0b_qmatrix *q0, t0b_qmatrix *q2, const float *x_dev, int M, const float *b0_dev,
                              const float *b2_dev, float *z_dev, float *y_dev, void *stream);
/* Wait for `stream` and report any kernel-side error of q's launches. */
t0b_status t0b_qmatrix_sync(t0b_qmatrix *q, void *stream);

/* ---- bounded-wait self-test (no reference counterpart; a diagnostic) ----
 * Every wait of a kernel on an mbarrier (TMA tiles, dequantized tiles,
 * accumulators) gives up after T0B_WAIT_CYCLES SM cycles (about 2 s), records
 * a device error code and returns, so a lost arrival becomes T0B_ERR_DEVICE
 * instead of a hung GPU.  This call exercises that path on the engine's
 * device: one warp waits with the same bounded wait on a barrier that nothing
 * arrives on.  Expected result: T0B_ERR_DEVICE after about 2 s, with
 * *device_code = 1 (the wait's code) and *outcome = 2 (the wait returned and
 * the kernel finished); the context stays usable.  It starts no TMA, tensor
 * memory or cluster work. */
t0b_status t0b_selftest_bounded_wait(t0b_engine *e, int *device_code, int *outcome);

/* ---- no-allocation dequant-GEMM (no reference counterpart) ----
 * The product of t0b_gemm_q, same arguments minus the engine, computed on
 * the calling thread's current device without allocating any device memory:
 * the split f16 copy of x, the weight-scale reduction word and the kernel
 * error word live in one fixed array compiled into the library
 * (T0B_NOALLOC_SCRATCH_BYTES per device, reserved when the library's device
 * code is loaded on that device).  Meant for hosts that cannot allocate at
 * call time: a process that has handed all of HBM to its own arena up front,
 * or a serving loop that must not pay cudaMalloc/cudaFree latency and their
 * implicit device-wide synchronisation in the middle of a request.
 *
 * Limits and rules:
 *  - M * K <= T0B_NOALLOC_MAX_X_ELEMENTS, else T0B_ERR_INVALID (nothing runs);
 *    K % 256 == 0 and N % 256 == 0 as for t0b_gemm_q.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress, with that device current) and caches it.
 *  - Every call synchronises `stream` (it reads the kernel error word back
 *    before returning), so it must not be called while `stream` is being
 *    captured into a CUDA graph.
 *  - All calls on one device share the array.  Each call clears the two
 *    control words it needs zeroed and overwrites the x copy before reading
 *    it, so no state carries over from one call to the next; but calls that
 *    overlap in time on one device (several host threads, or work enqueued
 *    on other streams before this call returns) race on it and must be
 *    serialised by the caller.  Each call synchronises `stream` before it
 *    returns. */
#define T0B_NOALLOC_MAX_X_ELEMENTS ((size_t)1 << 22)
#define T0B_NOALLOC_SCRATCH_BYTES ((size_t)256 + 4 * T0B_NOALLOC_MAX_X_ELEMENTS)
t0b_status t0b_gemm_q_noalloc(int ggml_type, const void *w_dev, int N, int K, const float *x_dev, int M,
                              const float *bias_dev, float *y_dev, void *stream);

/* ---- host codecs (gguf.rs) ---- */
/* Parse and validate a GGUF file without a device: gguf::read_gguf
 * (gguf.rs:347-405) + config_from_gguf_metadata (weights.rs:69-112) + the
 * tensor set and shapes this engine needs.  Fills *out (byte counts are the
 * GGUF-resident sizes). */
t0b_status t0b_gguf_validate(const uint8_t *bytes, size_t len, t0b_model_info *out);

/* quantize_q8_0 / quantize_q4_0, gguf.rs:100-157; n % 32 == 0 */
t0b_status t0b_quantize(int ggml_type, const float *x, size_t n, uint8_t *out);
/* dequantize_q8_0 / dequantize_q4_0 / f16 / f32, gguf.rs:116-174, 213-226 */
t0b_status t0b_dequantize(int ggml_type, const uint8_t *bytes, size_t n, float *out);
size_t t0b_row_bytes(int ggml_type, size_t n_elements);

/* Weights::export_gguf, weights.rs:187-227 (+ write_gguf, gguf.rs:299-345):
 * n named f32 tensors (ndims[i] in {1,2}; shapes[2i], shapes[2i+1]),
 * big_type in {T0B_F16, T0B_Q8_0, T0B_Q4_0} for the four big matmuls.
 * *out_len receives the size; call once with out == NULL to query it. */
t0b_status t0b_export_gguf(size_t n, const char *const *names, const int32_t *ndims, const int64_t *shapes,
                           const float *const *data, int big_type, const t0b_model_info *cfg, uint8_t *out,
                           size_t *out_len);

#ifdef __cplusplus
}
#endif
#endif
