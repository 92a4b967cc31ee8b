/*
 * t0_oracle.h -- CPU oracle for the t0-alpha quantized forecast path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * engine `t0-core` (idle-intelligence/t0-web, Rust, Burn on ndarray) used to
 * check the CUDA product.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * library never links or calls it.
 *
 * Parity pins (what ties this restatement to the reference):
 *   - gguf.rs:407-482 unit tests (Q8_0 / Q4_0 round-trip bounds, GGUF
 *     structure round trip), quant.rs:161-185 (exact unpack),
 *     ops_tests.rs:11-72 (rmsnorm known answers, RoPE seq-1 identity,
 *     halves-concat xpos scale) and the kernel recipe of
 *     t0-fast/src/model.rs:825-870 are re-run against this code by
 *     tests/test_oracle_pins.py.
 *   - Q8_0 / Q4_0 quantizers are checked bit-for-bit against gguf-py 0.19
 *     (llama.cpp's numpy port of quantize_row_q{8,4}_0_ref), the third-party
 *     algorithm the reference cites at gguf.rs:97-132.
 *   - End-to-end quantiles of the real t0-core cannot be reproduced here: the
 *     Rust toolchain and the t0-alpha checkpoint are both absent, so the
 *     whole-forward restatement is pinned only through the known answers
 *     above plus line-by-line restatement (every function cites the file:line
 *     it follows).  The forward pass is "parity partially pinned".
 */
#ifndef T0_ORACLE_H
#define T0_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, gguf.rs:32-39 */
enum { O_F32 = 0, O_F16 = 1, O_Q4_0 = 2, O_Q8_0 = 8 };

/* ---- f16 (IEEE binary16, round-to-nearest-even; `half 2.7.1`) ---- */
uint16_t o_f32_to_f16(float x);
float o_f16_to_f32(uint16_t h);

/* ---- block codecs, gguf.rs:100-174 ---- */
void o_quantize_q8_0(const float *x, size_t n, uint8_t *out);
void o_dequantize_q8_0(const uint8_t *bytes, size_t n, float *out);
void o_quantize_q4_0(const float *x, size_t n, uint8_t *out);
void o_dequantize_q4_0(const uint8_t *bytes, size_t n, float *out);
size_t o_row_bytes(int type, size_t n_elements);

/* ---- model config, config.rs:7-57 ---- */
typedef struct {
  int embed_dim, num_layers, num_heads, mlp_hidden_dim, patch_size;
  int group_every_n;
  float dropout;
  int n_quantiles;
  float quantile_levels[32];
  int scaler_use_arcsinh;
  float scaler_eps;
  int variance_offset; /* 1: "variance_offset", 0: "std_clamp" */
} o_config;

/* ---- GGUF export (weights.rs:187-227 + gguf.rs:299-345) ----
 * tensors: n named f32 tensors with 1..2 dims (row-major).  big_type is the
 * ggml type for the four big per-layer matmuls (O_F16 / O_Q8_0 / O_Q4_0).
 * Writes into a malloc'd buffer returned in *out (free with o_free). */
int o_export_gguf(int n, const char *const *names, const int *ndims,
                  const int64_t *shapes /* n x 2 */, const float *const *data,
                  int big_type, const o_config *cfg, uint8_t **out,
                  size_t *out_len);
void o_free(void *p);

/* ---- model (weights.rs:151-163 dequantizes everything to f32) ---- */
typedef struct o_model o_model;
int o_model_load_gguf(const uint8_t *bytes, size_t len, o_model **out);
void o_model_free(o_model *m);
int o_model_config(const o_model *m, o_config *out);
/* raw GGUF tensor lookup (type id, shape, byte pointer into the model's copy) */
int o_model_tensor(const o_model *m, const char *name, int *type, int64_t *rows,
                   int64_t *cols, const uint8_t **bytes, size_t *nbytes);

/* ---- forecast drivers ----
 * out layout [v, horizon, n_q] row-major.  Return 0 on success. */
int o_forecast(const o_model *m, const float *ctx, int v, int t_ctx,
               int horizon, float *out);                         /* model.rs:322-333 */
int o_forecast_batch(const o_model *m, const float *ctx, int n, int t_ctx,
                     int horizon, int chunk, float *out);        /* model.rs:385-407 */

/* ---- quantile utilities (t0-core quantile.rs) and autoregressive rollout
 * (t0-core model.rs:582-665).  Query levels sorted ascending, inside (0, 1).
 * o_forecast_rollout writes [prediction_length, nq] (query-level minor). */
void o_interpolate_quantiles(const float *query, int nq, const float *levels, const float *values, int n,
                             float *out);                                                  /* quantile.rs:17-43 */
void o_weighted_quantile(const float *query, int nq, const float *weights, const float *samples, int n,
                         float *out);                                                      /* quantile.rs:47-61 */
void o_prob_mass(const float *levels, int n, float *out);                                 /* quantile.rs:66-78 */
int o_forecast_rollout(const o_model *m, const float *ctx, int t_ctx, int prediction_length, const float *query,
                       int nq, float *out);
int o_forecast_batch_rows(const o_model *m, const float *ctx,
                          const int64_t *lengths, int n, int horizon,
                          int chunk, float *out);    /* t0-fast lib.rs:175-242 */
/* independent multivariate series, series i has n_variates[i] rows of t_ctx
 * values; each is a `forecast` call (a joint series sharing one group id).
 * Runs on n_threads host threads (one series per thread at a time). */
int o_forecast_multiseries(const o_model *m, const float *ctx,
                           const int32_t *n_variates, int n_series, int t_ctx,
                           int horizon, int n_threads, float *out);

/* Forward on an already scaled + padded window, with an optional trace of
 * the residual stream: trace (if non-NULL) receives [(L+1), v*p, E] floats:
 * index 0 = patch embedding (+type embedding), index l+1 = output of layer l.
 * `series` arrays are [v, t]; out = [v, p, patch, n_q].  model.rs:177-300 */
int o_forward(const o_model *m, int v, int t, const float *variates,
              const int8_t *mask, const int64_t *group_ids,
              const int64_t *variate_type, float *out, float *trace);

/* ---- primitives exposed for known-answer tests ---- */
void o_rmsnorm(const float *x, int rows, int dim, const float *g, float eps,
               float *out);                                   /* ops.rs:12-17 */
void o_rope_tables(int seq, int hd, float *cos_t, float *sin_t,
                   float *scale);                             /* ops.rs:78-115 */
/* Causal scaler of one padded TimeSeries (scaler.rs:44-118).  Writes loc,
 * scale and the scaled values, all [v, t]. */
void o_scale_input(const o_config *cfg, int v, int t, const float *variates,
                   const int8_t *mask, const int64_t *group_ids,
                   float *scaled, float *loc, float *scale);

/* ---- GEMM oracles (fp64 accumulation) for the standalone configs ----
 * y[M,N] = x[M,K] . deq(W)[N,K]^T (+ bias[N] if non-NULL). */
int o_gemm_q_f64(int type, const uint8_t *w, int N, int K, const float *x,
                 int M, const float *bias, double *y);
/* Fused SwiGLU on quantized weights: gate rows [0,F), up rows [F,2F) of w0
 * ([2F, K]); z = silu(x.gate^T) * (x.up^T) ([M,F]); y = z . w2^T ([M, N2]).
 * z_out (optional) receives z. */
int o_swiglu_q_f64(int type, const uint8_t *w0, int F, int K,
                   const uint8_t *w2, int N2, const float *x, int M,
                   double *z_out, double *y);

/* Precision study only: emulate tensor-core operand rounding inside the four
 * quantized matmuls (0 exact, 1 f16 x and w, 2 f16 x, 3 f16 w, 4 bf16 both). */
void o_set_gemm_emulation(int mode);

#ifdef __cplusplus
}
#endif
#endif
