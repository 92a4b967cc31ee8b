// t0b_internal.h -- kernel argument blocks and launcher prototypes shared by
// the host orchestration (t0b_model.cu) and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "epilogue.cuh"

// Raises the kernel's dynamic shared memory limit on the current device to at
// least `bytes`, never lowering it: a CUDA graph captured with a larger launch
// must stay launchable after smaller launches of the same kernel.
cudaError_t t0b_smem_limit(const void *kernel, size_t bytes);

struct PrepArgs {
  const float *ctx;      // raw context values (NaN = missing)
  const int64_t *row_off;  // start of row r's values in ctx
  const int *row_len;    // context steps of row r
  const int *row_lead;   // leading padding steps of row r (patch-aligns the context)
  int R, p, hp;          // rows, patches per row, horizon patches
  int use_arcsinh, variance_offset;
  float eps;
  float *feat;           // [R*p, 96]
  float *out_loc, *out_scale;  // [R*hp] stats at the last step of each output patch
  int *err;              // device error word (index checks of the checked build)
};

struct SgemmArgs {
  const float *A;
  int lda;
  const float *B;
  int ldb;
  const __half *B16;  // optional f16 copy of B, exact (B came from f16 on disk): tensor-core path
  float *C;
  int ldc;
  int M, N, K;
  const float *bias, *bias2, *bias3;
  int relu, accumulate;
};

struct AttnArgs {
  const float *qkv;  // [T, 3E]
  __half *oh, *ol;   // [T, E] split output
  float *o32;        // optional f32 output
  const int *row_first_valid;  // whole-padding patches at the start of each row
  const int *series_row0, *series_nrows;
  // per-head QK RMSNorm gains [hd] (eps 1e-8, ops.rs:175-177), applied to q
  // and k as they are read; on TIME layers (use_rope) then xpos RoPE with the
  // tables rope = [4][p][hd]: cos, sin, scale, 1/scale (k uses 1/scale).
  // hd = E / H is 64 or 128.
  const float *qn, *kn, *rope;
  // the same tables without duplicates, [p][2 hd]: cos[hd/2], sin[hd/2] per
  // rotated pair, scale[hd/2], 1/scale[hd/2] per dim mod hd/2
  const float *rope_c;
  int use_rope;
  int R, p, E, H, n_series;
  int max_nrows;  // largest series_nrows entry (host-side bound for the group kernel)
  int *err;       // device error word (a bounded wait that ran out)
  // time attention on f16 planes (t0b_launch_attn_time_planes): q | k | v as
  // (hi, lo) planes [R p][3E] written by the wQKV GEMM's EPI_QKV epilogue,
  // and the per-(token, head) sums of squares of q and k [R p][2H]
  const __half *qkv_h, *qkv_l;
  const float *ssq_qk;
};

// Tensor map of an f32 row-major [outer][inner] tensor with rows row_bytes
// apart and a [box_outer][box_inner] box, optionally 128-byte swizzled (a
// 32-float inner box); false if the driver entry point is unavailable or
// rejects the layout (k_gemm_tc.cu).
bool t0b_make_tmap_f32_2d(CUtensorMap *tm, const float *ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                          uint32_t box_inner, uint32_t box_outer, bool swizzle128);
bool t0b_make_tmap_f16_3d(CUtensorMap *tm, const void *ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                          uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2, bool swizzle128);

// Small-M dequant GEMM (k_gemm_small.cu): thread-block clusters along K,
// launched as a programmatic dependent of the previous kernel on `st`.  The
// activations are the f16 planes ah / al, or, when x32 is given, f32 rows
// that the kernel splits itself (ah / al unused).
cudaError_t t0b_launch_gemm_small(int qt, const __half *ah, const __half *al, int M, int K, const uint8_t *W,
                                  const Epi &epi, int *err, cudaStream_t st, const float *x32 = nullptr);
// Whether the small-M kernel runs this shape: K is split into at most 8
// slices of a multiple of 256 values (a divisor of K), which must fit in
// shared memory (x32: f32 input, K slices of 256 values only); otherwise
// callers use the tensor-core kernel (or, for x32, the planes of a split pass).
bool t0b_small_supports(int qt, int M, int K, const Epi &epi, bool x32 = false);
cudaError_t t0b_launch_gemm_tc(int qt, const __half *ah, const __half *al, int M, int K, const uint8_t *W, int wrows,
                               int wshift, const Epi &epi, int *err, cudaStream_t st);
cudaError_t t0b_launch_absmax_scale(const uint8_t *W, size_t nblocks, int bpb, unsigned int *out, cudaStream_t st);

// Exponent s of the power-of-two weight prescale for the split-f16 tensor-core
// path: the largest |d q| of the matrix (max_d * max|q|) times 2^s stays at
// or below 2^14, so W*2^s splits into two normal f16 terms without overflow.
inline int t0b_weight_shift(float max_d, int qt) {
  const float wmax = max_d * (qt == 8 ? 128.0f : 8.0f);
  if (!(wmax > 0.0f)) return 0;
  int s = 0;
  while (s < 24 && wmax * (float)(1 << (s + 1)) <= 16384.0f) ++s;
  return s;
}
cudaError_t t0b_launch_prep(const PrepArgs &a, cudaStream_t st);
cudaError_t t0b_launch_sgemm(const SgemmArgs &a, cudaStream_t st);
cudaError_t t0b_launch_rownorm_split(const float *x, const float *g, __half *xh, __half *xl, float *ssq, int M, int E,
                                     cudaStream_t st);
cudaError_t t0b_launch_attn_time(const AttnArgs &a, cudaStream_t st);
// Time attention for 64-dim heads on the planes of the EPI_QKV epilogue
// (qkv_h, qkv_l, ssq_qk), p <= 256.
cudaError_t t0b_launch_attn_time_planes(const AttnArgs &a, cudaStream_t st);
cudaError_t t0b_launch_attn_group(const AttnArgs &a, cudaStream_t st);
cudaError_t t0b_launch_dec_gather(const float *x, const float *g, float *xo, int R, int p, int hp, int E,
                                  cudaStream_t st);
cudaError_t t0b_launch_dec_head(const float *dec, const float *loc, const float *scale, float *out, const int *out_row,
                                int R, int hp, int horizon, int nq, int use_arcsinh, cudaStream_t st);
cudaError_t t0b_launch_split_f32(const float *x, __half *xh, __half *xl, size_t n, cudaStream_t st);
// Self-test of the bounded mbarrier wait (k_misc.cu): one warp waits on a
// barrier nobody arrives on; *outcome = 2 once the wait ran out and returned.
cudaError_t t0b_launch_bounded_wait_selftest(int *err, int *outcome, cudaStream_t st);
