// k_misc.cu -- the non-GEMM kernels of the forecast path:
//   * prep: padding + causal per-timestep scaler + patch features on device
//     (data.rs:52-155, scaler.rs:44-118, model.rs:185-199);
//   * sgemm_nt: f32 GEMM for the small f16-on-disk layers (patch encoder,
//     decoder), ops.rs:24-42;
//   * rownorm_split: x*g split into f16 hi/lo + sum of squares per row;
//   * time / group attention with implicit masks (mask.rs:49-82, ops.rs:153-190);
//   * decoder gather + out_norm, and the quantile head + inverse scaling +
//     forecast-region slice (ops.rs:195-210, scaler.rs:125-148,
//     model.rs:487-531).
#include "common.cuh"
#include <algorithm>
#include <cstring>

#include "t0b_internal.h"

// Launch as a programmatic dependent of the previous kernel on `st`: the
// kernel may start while that one finishes, and waits (griddepcontrol.wait)
// before it reads anything the previous kernel writes.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ============================================================== prep
// One warp per variate row.  The causal scaler is the reference's Welford
// recurrence in f32 (scaler.rs:44-118).  Per chunk of kPrepChunk steps each
// lane runs that recurrence over its own 1/32 of the chunk, starting from
// the state before its first step: the carried state of the previous chunks
// merged with the states of the lanes before it by the pairwise update of
// Chan, Golub and LeVeque (a warp scan over lanes' local Welford states);
// lane 0 continues the carried state exactly, so a row of at most
// kPrepChunk / 32 steps per lane reproduces the sequential recurrence bit for
// bit, and later lanes differ from it by the rounding of the merge.  The
// states after every step go to shared memory; then all 32 lanes turn them
// into the per-step loc / scale, the scaled value and the patch features
// (lane = step within the patch, so feature rows are written coalesced).
constexpr int kPrepChunk = 256;  // steps per chunk (a multiple of the patch size 32)
constexpr int kPrepWarps = 4;

// Welford state (ca, ma, qa) of earlier steps followed by (cb, mb, qb):
// count, mean and sum of squared deviations of both, into (cb, mb, qb).
T0B_DEV void welford_merge(float ca, float ma, float qa, float &cb, float &mb, float &qb) {
  if (ca == 0.0f) return;
  if (cb == 0.0f) {
    cb = ca;
    mb = ma;
    qb = qa;
    return;
  }
  const float n = ca + cb, d = mb - ma;
  mb = ma + d * (cb / n);
  qb = (qa + qb) + d * d * (ca * cb / n);
  cb = n;
}
// One Welford step (the reference's operation order; NaN = not observed).
T0B_DEV void welford_step(float x, float &count, float &mean, float &m2) {
  if (!isnan(x)) {
    count = __fadd_rn(count, 1.0f);
    const float delta = __fsub_rn(x, mean);
    mean = __fadd_rn(mean, __fdiv_rn(delta, count));
    const float delta2 = __fsub_rn(x, mean);
    m2 = __fadd_rn(m2, __fmul_rn(delta, delta2));
  }
}

__global__ void __launch_bounds__(32 * kPrepWarps) prep_kernel(PrepArgs a) {
  __shared__ __align__(16) float s_x[kPrepWarps][kPrepChunk];
  __shared__ __align__(16) float s_cnt[kPrepWarps][kPrepChunk];
  __shared__ __align__(16) float s_mean[kPrepWarps][kPrepChunk];
  __shared__ __align__(16) float s_m2[kPrepWarps][kPrepChunk];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kPrepWarps + w;
  if (r >= a.R) return;  // whole warp
  const int lead = a.row_lead[r];
  const int len = a.row_len[r];
  const float *src = a.ctx + a.row_off[r];
  const int steps = a.p * 32;
  const int hp0 = a.p - a.hp - 1;  // first output patch
  float count = 0.0f, mean = 0.0f, m2 = 0.0f;  // state after the previous chunks (same in every lane)
  // raw values of a chunk, coalesced (lane + 32 j); steps outside the context
  // read as NaN here (not observed), which only the recurrence looks at.
  // The next chunk's values are loaded while the current one is processed.
  constexpr int kPer = kPrepChunk / 32;
  float xr[kPer];
  auto load_chunk = [&](int c0) {
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int t = c0 + lane + 32 * j;
      xr[j] = (t < steps && t >= lead && t < lead + len) ? src[t - lead] : __int_as_float(0x7fc00000);
    }
  };
  load_chunk(0);
  for (int c0 = 0; c0 < steps; c0 += kPrepChunk) {
    const int n = min(kPrepChunk, steps - c0);
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (lane + 32 * j < n) s_x[w][lane + 32 * j] = xr[j];
    if (c0 + kPrepChunk < steps) load_chunk(c0 + kPrepChunk);
    __syncwarp();
    {
      // n is a multiple of 32: lane l takes steps [l seg, (l + 1) seg)
      const int seg = n >> 5, i0 = lane * seg;
      float lc = 0.0f, lm = 0.0f, lq = 0.0f;  // this lane's steps alone
      for (int i = 0; i < seg; ++i) welford_step(s_x[w][i0 + i], lc, lm, lq);
      // inclusive scan over lanes, then the state before this lane's steps
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float pc = __shfl_up_sync(0xffffffffu, lc, o), pm = __shfl_up_sync(0xffffffffu, lm, o),
                    pq = __shfl_up_sync(0xffffffffu, lq, o);
        if (lane >= o) welford_merge(pc, pm, pq, lc, lm, lq);
      }
      float c = __shfl_up_sync(0xffffffffu, lc, 1), m = __shfl_up_sync(0xffffffffu, lm, 1),
            q = __shfl_up_sync(0xffffffffu, lq, 1);
      if (lane == 0) c = m = q = 0.0f;
      welford_merge(count, mean, m2, c, m, q);
      for (int i = 0; i < seg; ++i) {
        welford_step(s_x[w][i0 + i], c, m, q);
        s_cnt[w][i0 + i] = c;
        s_mean[w][i0 + i] = m;
        s_m2[w][i0 + i] = q;
      }
      count = __shfl_sync(0xffffffffu, c, 31);
      mean = __shfl_sync(0xffffffffu, m, 31);
      m2 = __shfl_sync(0xffffffffu, q, 31);
    }
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const int t = c0 + i, patch = t >> 5, k = t & 31;
      int mask;  // 0 valid, 1 pad, 2 missing, 4 withheld
      float x = 0.0f;
      if (t < lead) {
        mask = 1;
      } else if (t < lead + len) {
        x = s_x[w][i];
        if (isnan(x)) {
          mask = 2;
          x = 0.0f;
        } else {
          mask = 0;
        }
      } else {
        mask = 4;
      }
      float lo = 0.0f, sc = 1.0f;
      if (mask != 1) {  // padding sentinel (group id < 0) keeps loc 0 / scale 1
        const float cnt = s_cnt[w][i];
        lo = s_mean[w][i];
        const float var = cnt > 1.0f ? fmaxf(__fdiv_rn(s_m2[w][i], __fsub_rn(cnt, 1.0f)), 0.0f) : 0.0f;
        sc = a.variance_offset ? __fsqrt_rn(__fadd_rn(var, a.eps)) : fmaxf(__fsqrt_rn(var), a.eps);
      }
      const float zv = __fdiv_rn(__fsub_rn(x, lo), sc);
      if (!T0B_CHECK(patch < a.p && k < 32, a.err)) continue;
      float *f = a.feat + ((size_t)r * a.p + patch) * 96;
      f[k] = a.use_arcsinh ? asinhf(zv) : zv;
      f[32 + k] = (float)k / 32.0f;
      f[64 + k] = mask == 0 ? 1.0f : 0.0f;
      if (k == 31 && patch >= hp0 && patch < hp0 + a.hp) {  // stats at the patch's last step
        const size_t o = (size_t)r * a.hp + (patch - hp0);
        a.out_loc[o] = lo;
        a.out_scale[o] = sc;
      }
    }
    __syncwarp();
  }
}

// ============================================================== sgemm
// C[M,N] (+)= A[M,K] . B[N,K]^T + bias (+ bias2) (relu), all f32 row-major.
// 64x64 tile, 256 threads, 4x4 outputs per thread, K tile 16.
__global__ void __launch_bounds__(256) sgemm_nt_kernel(SgemmArgs a) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < a.K; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      int row = i / 16, kk = i % 16;
      int m = m0 + row, n = n0 + row, k = k0 + kk;
      As[kk][row] = (m < a.M && k < a.K) ? a.A[(size_t)m * a.lda + k] : 0.0f;
      Bs[kk][row] = (n < a.N && k < a.K) ? a.B[(size_t)n * a.ldb + k] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int m = m0 + ty * 4 + i;
    if (m >= a.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int n = n0 + tx * 4 + j;
      if (n >= a.N) continue;
      float v = acc[i][j];
      if (a.bias) v = v + a.bias[n];
      if (a.bias2) v = v + a.bias2[n];
      if (a.bias3) v = v + a.bias3[n];
      if (a.relu) v = fmaxf(v, 0.0f);
      float *c = a.C + (size_t)m * a.ldc + n;
      *c = a.accumulate ? (*c + v) : v;
    }
  }
}

// Few rows (M <= 32 per CTA): a CTA owns 32 output columns and MT rows,
// stages its whole A [MT, K] and B [32, K] slices in shared memory with one
// round of 16-byte cp.async copies, and its 8 warps split K: lane n
// accumulates column n for every row (A values broadcast from shared
// memory), then the warps' partials are added in warp order.
constexpr int kSgemmSmallWarps = 8;

template <int MT>
__global__ void __launch_bounds__(32 * kSgemmSmallWarps) sgemm_small_kernel(SgemmArgs a) {
  extern __shared__ __align__(16) float sg_smem[];
  const int KP = a.K + 4;  // row pitch (floats): 16-byte pad keeps 128-bit row reads conflict-free
  float *As = sg_smem;                      // [MT][KP]
  float *Bs = As + (size_t)MT * KP;         // [32][KP]
  float *red = sg_smem;                     // [warps][MT][32], reuses A/B after the main loop
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MT, n0 = blockIdx.x * 32;
  const int g4 = a.K / 4;  // 16-byte granules per row
  // the weight rows first: they never change, so they are fetched while the
  // previous kernel (launched before this programmatic dependent) finishes
  for (int i = threadIdx.x; i < 32 * g4; i += blockDim.x) {
    const int row = i / g4, q = i - row * g4;
    const int n = min(n0 + row, a.N - 1);
    cp_async16(Bs + (size_t)row * KP + 4 * q, a.B + (size_t)n * a.ldb + 4 * q);
  }
  cp_async_commit();
  pdl_wait();
  for (int i = threadIdx.x; i < MT * g4; i += blockDim.x) {
    const int row = i / g4, q = i - row * g4;
    const int m = min(m0 + row, a.M - 1);  // rows past M duplicate a valid row; outputs dropped
    cp_async16(As + (size_t)row * KP + 4 * q, a.A + (size_t)m * a.lda + 4 * q);
  }
  cp_async_commit();
  pdl_launch_dependents();
  cp_async_wait<0>();
  __syncthreads();
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
  const int kw = a.K / kSgemmSmallWarps;  // a multiple of 4
  const float *brow = Bs + (size_t)lane * KP + w * kw;
  for (int k = 0; k < kw; k += 4) {
    const float4 b = *reinterpret_cast<const float4 *>(brow + k);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float4 x = *reinterpret_cast<const float4 *>(As + (size_t)m * KP + w * kw + k);
      acc[m] = fmaf(x.x, b.x, acc[m]);
      acc[m] = fmaf(x.y, b.y, acc[m]);
      acc[m] = fmaf(x.z, b.z, acc[m]);
      acc[m] = fmaf(x.w, b.w, acc[m]);
    }
  }
  __syncthreads();  // A/B no longer read: reuse as the partial tiles
#pragma unroll
  for (int m = 0; m < MT; ++m) red[((size_t)w * MT + m) * 32 + lane] = acc[m];
  __syncthreads();
  for (int i = threadIdx.x; i < MT * 32; i += blockDim.x) {
    const int m = m0 + i / 32, n = n0 + (i & 31);
    float v = red[i];
#pragma unroll
    for (int q = 1; q < kSgemmSmallWarps; ++q) v += red[(size_t)q * MT * 32 + i];
    if (m >= a.M || n >= a.N) continue;
    if (a.bias) v = v + a.bias[n];
    if (a.bias2) v = v + a.bias2[n];
    if (a.bias3) v = v + a.bias3[n];
    if (a.relu) v = fmaxf(v, 0.0f);
    float *c = a.C + (size_t)m * a.ldc + n;
    *c = a.accumulate ? (*c + v) : v;
  }
}

// Many rows, f16-exact weights (the patch encoder / decoder weights are f16
// on disk): C = A . B^T on the tensor cores as Ah.B + Al.B, A split into two
// f16 planes as it is read (products exact).  Each 32-wide K step is summed
// by the MMAs into a fresh partial that is then added to the f32 result
// (the tensor cores' own accumulation only ever spans 4 MMAs), i.e. the
// same f32-class arithmetic as the quantized GEMMs.  128 x 64 tile per CTA,
// 8 warps of 32 x 32, K steps double-buffered with cp.async.
constexpr int kSgH_BM = 128, kSgH_BN = 64, kSgH_BK = 32;
constexpr int kSgH_AP = kSgH_BK + 8;  // A row pitch (floats): conflict-free float2 fragment reads
constexpr int kSgH_BP = kSgH_BK + 8;  // B row pitch (halves): conflict-free ldmatrix rows
constexpr size_t kSgH_Stage = (size_t)kSgH_BM * kSgH_AP * 4 + (size_t)kSgH_BN * kSgH_BP * 2;

__global__ void __launch_bounds__(256, 2) sgemm_h_kernel(SgemmArgs a) {
  extern __shared__ __align__(16) uint8_t sgh_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wm = warp & 3, wn = warp >> 2;  // warp tile rows 32 wm.., cols 32 wn..
  const int m0 = blockIdx.y * kSgH_BM, n0 = blockIdx.x * kSgH_BN;
  auto As = [&](int st) { return reinterpret_cast<float *>(sgh_smem + st * kSgH_Stage); };
  auto Bs = [&](int st) { return reinterpret_cast<__half *>(sgh_smem + st * kSgH_Stage + (size_t)kSgH_BM * kSgH_AP * 4); };
  auto stage = [&](int st, int k0) {
    float *as = As(st);
    __half *bs = Bs(st);
    // A: 128 rows x 32 floats = 8 granules per row; B: 64 rows x 32 halves = 4 granules per row
    for (int i = threadIdx.x; i < kSgH_BM * 8; i += 256) {
      const int r = i >> 3, q = i & 7;
      const int m = min(m0 + r, a.M - 1);  // rows past M duplicate a valid row; outputs dropped
      cp_async16(as + r * kSgH_AP + 4 * q, a.A + (size_t)m * a.lda + k0 + 4 * q);
    }
    for (int i = threadIdx.x; i < kSgH_BN * 4; i += 256) {
      const int r = i >> 2, q = i & 3;
      const int n = min(n0 + r, a.N - 1);
      cp_async16(bs + r * kSgH_BP + 8 * q, a.B16 + (size_t)n * a.ldb + k0 + 8 * q);
    }
    cp_async_commit();
  };
  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0f;
  const int nk = a.K / kSgH_BK;
  stage(0, 0);
  for (int kt = 0; kt < nk; ++kt) {
    if (kt + 1 < nk) {
      stage((kt + 1) & 1, (kt + 1) * kSgH_BK);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float *as = As(kt & 1);
    const __half *bs = Bs(kt & 1);
    float pp[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) pp[i][j][0] = pp[i][j][1] = pp[i][j][2] = pp[i][j][3] = 0.0f;
#pragma unroll
    for (int kh = 0; kh < 2; ++kh) {  // two k16 steps per stage
      uint32_t ah[2][4], al[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const float *r0 = as + (32 * wm + 16 * mt + g) * kSgH_AP + 16 * kh + 2 * t;
        const float *r1 = r0 + 8 * kSgH_AP;
        const float2 x0 = *reinterpret_cast<const float2 *>(r0), x1 = *reinterpret_cast<const float2 *>(r1);
        const float2 x2 = *reinterpret_cast<const float2 *>(r0 + 8), x3 = *reinterpret_cast<const float2 *>(r1 + 8);
        split2(x0.x, x0.y, ah[mt][0], al[mt][0]);
        split2(x1.x, x1.y, ah[mt][1], al[mt][1]);
        split2(x2.x, x2.y, ah[mt][2], al[mt][2]);
        split2(x3.x, x3.y, ah[mt][3], al[mt][3]);
      }
#pragma unroll
      for (int n2 = 0; n2 < 2; ++n2) {  // n8 tiles 2 n2, 2 n2 + 1
        // ldmatrix: matrix mi = lane / 8 -> rows (n) (mi / 2) * 8 + lane % 8, k (mi % 2) * 8
        const __half *br = bs + (32 * wn + 16 * n2 + ((lane >> 4) << 3) + (lane & 7)) * kSgH_BP + 16 * kh +
                           ((lane >> 3) & 1) * 8;
        uint32_t b00, b01, b10, b11;
        ldsm_x4(br, b00, b01, b10, b11);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          float *c0 = pp[mt][2 * n2], *c1 = pp[mt][2 * n2 + 1];
          mma16816(c0[0], c0[1], c0[2], c0[3], ah[mt][0], ah[mt][1], ah[mt][2], ah[mt][3], b00, b01);
          mma16816(c0[0], c0[1], c0[2], c0[3], al[mt][0], al[mt][1], al[mt][2], al[mt][3], b00, b01);
          mma16816(c1[0], c1[1], c1[2], c1[3], ah[mt][0], ah[mt][1], ah[mt][2], ah[mt][3], b10, b11);
          mma16816(c1[0], c1[1], c1[2], c1[3], al[mt][0], al[mt][1], al[mt][2], al[mt][3], b10, b11);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][j][e] += pp[i][j][e];
    __syncthreads();  // this stage may be refilled next
  }
  // epilogue: rows g / g + 8 of each m16 tile, columns 2t, 2t + 1 of each n8 tile
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int m = m0 + 32 * wm + 16 * mt + g + 8 * hr;
      if (m >= a.M) continue;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int n = n0 + 32 * wn + 8 * nt + 2 * t;
        const float v[2] = {acc[mt][nt][2 * hr], acc[mt][nt][2 * hr + 1]};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (n + e >= a.N) continue;
          float x = v[e];
          if (a.bias) x = x + a.bias[n + e];
          if (a.bias2) x = x + a.bias2[n + e];
          if (a.bias3) x = x + a.bias3[n + e];
          if (a.relu) x = fmaxf(x, 0.0f);
          float *c = a.C + (size_t)m * a.ldc + n + e;
          *c = a.accumulate ? (*c + x) : x;
        }
      }
    }
}

// ============================================================== rownorm_split
// One warp per row: xh/xl = split(x * g), ssq[r] = sum x^2 (single slot).
__global__ void rownorm_split_kernel(const float *x, const float *g, __half *xh, __half *xl, float *ssq, int M,
                                     int E) {
  pdl_launch_dependents();  // the next small-M GEMM may prefetch its weights
  pdl_wait();               // x comes from the previous kernel
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  // 16-byte loads of x and g, 8-byte stores of each f16 plane (E % 4 == 0)
  const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)row * E);
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  uint2 *hr = reinterpret_cast<uint2 *>(xh + (size_t)row * E), *lr = reinterpret_cast<uint2 *>(xl + (size_t)row * E);
  float s = 0.0f;
  for (int c = lane; c < E / 4; c += 32) {
    const float4 v = xr[c], gg = g4[c];
    s += v.x * v.x;
    s += v.y * v.y;
    s += v.z * v.z;
    s += v.w * v.w;
    uint32_t h0, l0, h1, l1;
    split2(v.x * gg.x, v.y * gg.y, h0, l0);
    split2(v.z * gg.z, v.w * gg.w, h1, l1);
    hr[c] = make_uint2(h0, h1);
    lr[c] = make_uint2(l0, l1);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) ssq[row] = s;
}

// ============================================================== attention
T0B_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the 16 lanes of an aligned half-warp.
T0B_DEV float half_warp_sum(float v) {
#pragma unroll
  for (int o = 8; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Four consecutive head dims d..d+3 (d % 4 == 0) of one q or k vector whose
// sum of squares over the head is ss: RMSNorm with gains g (ops.rs:175-177),
// then, if tab != NULL, xpos RoPE at position pos on the adjacent pairs
// (d, d+1), (d+2, d+3): (x0, x1) -> (x0 c - x1 s, x1 c + x0 s) * scale
// (ops.rs:132-142); tab = cos table, sc = the scale table to use.
T0B_DEV float4 qk_norm_rope4(float4 v, float ss, const float *g, int d, const float *tab, const float *sc, int p,
                             int pos) {
  const float rdn = 1.0f / sqrtf(ss / 64.0f + 1e-8f);
  float x[4] = {v.x * rdn * g[d], v.y * rdn * g[d + 1], v.z * rdn * g[d + 2], v.w * rdn * g[d + 3]};
  if (tab) {
    const float *c = tab + pos * 64 + d, *sn = tab + (size_t)p * 64 + pos * 64 + d, *s = sc + pos * 64 + d;
#pragma unroll
    for (int k = 0; k < 4; k += 2) {
      const float x0 = x[k], x1 = x[k + 1];
      x[k] = x0 * c[k] * s[k] + (-x1) * sn[k] * s[k];
      x[k + 1] = x1 * c[k + 1] * s[k + 1] + x0 * sn[k + 1] * s[k + 1];
    }
  }
  return make_float4(x[0], x[1], x[2], x[3]);
}

// Time attention for one (variate row, head): causal over the row's p
// patches, keys restricted to non-padding patches (mask.rs:49-65).  A query
// in a whole-padding patch has every key blocked; the reference's softmax
// then averages V over all p patches (scores all equal -1e9), reproduced
// here.  q, k and v of the row's head are staged once in shared memory
// (16-byte loads), q and k normalised and rotated on the way in; K keeps a
// 65-float pitch so the lane-per-key score loop is bank-conflict free.
__global__ void __launch_bounds__(128) attn_time_kernel(AttnArgs a) {
  pdl_launch_dependents();  // the next small-M GEMM may prefetch its weights
  extern __shared__ float sm[];
  const int r = blockIdx.x, h = blockIdx.y;
  const int p = a.p, E = a.E;
  const int LD = 65;
  // Qs and Vs first: their rows take 16-byte accesses, so their offsets
  // stay multiples of 64 floats whatever p is; Ks (65-float pitch, scalar
  // accesses only) and Ps follow
  float *Qs = sm;                // [p][64]
  float *Vs = Qs + p * 64;       // [p][64]
  float *Ks = Vs + p * 64;       // [p][65]
  float *Ps = Ks + p * LD;       // [4 warps][p] probabilities
  const size_t tok0 = (size_t)r * p;
  const float *rope_c = a.use_rope ? a.rope : nullptr;
  const float *rsc = a.rope + (size_t)2 * p * 64, *rsc_inv = a.rope + (size_t)3 * p * 64;
  // 16 threads per token, 4 dims each; every thread runs every iteration so
  // the half-warp reductions see all 16 lanes
  for (int base = 0; base < p * 16; base += 128) {
    const int i = base + threadIdx.x;
    const bool ok = i < p * 16;
    const int j = ok ? i >> 4 : 0, d = (i & 15) * 4;
    const float *row = a.qkv + (tok0 + j) * 3 * E + h * 64 + d;
    float4 qv = ok ? *reinterpret_cast<const float4 *>(row) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 kv = ok ? *reinterpret_cast<const float4 *>(row + E) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float sq = half_warp_sum(qv.x * qv.x + qv.y * qv.y + qv.z * qv.z + qv.w * qv.w);
    const float sk = half_warp_sum(kv.x * kv.x + kv.y * kv.y + kv.z * kv.z + kv.w * kv.w);
    if (ok) {
      qv = qk_norm_rope4(qv, sq, a.qn, d, rope_c, rsc, p, j);
      kv = qk_norm_rope4(kv, sk, a.kn, d, rope_c, rsc_inv, p, j);
      *reinterpret_cast<float4 *>(Qs + j * 64 + d) = qv;
      float *kd = Ks + j * LD + d;
      kd[0] = kv.x;
      kd[1] = kv.y;
      kd[2] = kv.z;
      kd[3] = kv.w;
      *reinterpret_cast<float4 *>(Vs + j * 64 + d) = *reinterpret_cast<const float4 *>(row + 2 * E);
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lo = a.row_first_valid[r];
  float *pw = Ps + warp * p;
  for (int i = warp; i < p; i += 4) {
    const float *qi = Qs + i * 64;
    const bool masked = i < lo;
    const int j0 = masked ? 0 : lo, j1 = masked ? p - 1 : i;
    float mx = -INFINITY;
    for (int j = j0 + lane; j <= j1; j += 32) {
      const float *kj = Ks + j * LD;
      float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
#pragma unroll
      for (int d = 0; d < 64; d += 4) {
        s0 = fmaf(qi[d], kj[d], s0);
        s1 = fmaf(qi[d + 1], kj[d + 1], s1);
        s2 = fmaf(qi[d + 2], kj[d + 2], s2);
        s3 = fmaf(qi[d + 3], kj[d + 3], s3);
      }
      float s = (s0 + s1) + (s2 + s3);
      s = masked ? -1.0e9f : s * 0.125f;
      pw[j] = s;
      mx = fmaxf(mx, s);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int j = j0 + lane; j <= j1; j += 32) {
      float e = expf(pw[j] - mx);
      pw[j] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
    int j = j0;
    for (; j + 1 <= j1; j += 2) {
      const float p0 = pw[j], p1 = pw[j + 1];
      o0 = fmaf(p0, Vs[j * 64 + lane], o0);
      o1 = fmaf(p0, Vs[j * 64 + lane + 32], o1);
      o2 = fmaf(p1, Vs[(j + 1) * 64 + lane], o2);
      o3 = fmaf(p1, Vs[(j + 1) * 64 + lane + 32], o3);
    }
    if (j <= j1) {
      const float p0 = pw[j];
      o0 = fmaf(p0, Vs[j * 64 + lane], o0);
      o1 = fmaf(p0, Vs[j * 64 + lane + 32], o1);
    }
    const float inv = 1.0f / sum;
    o0 = (o0 + o2) * inv;
    o1 = (o1 + o3) * inv;
    __syncwarp();
    const size_t oo = (tok0 + i) * E + h * 64;
    __half hh, ll;
    split_f16(o0, hh, ll);
    a.oh[oo + lane] = hh;
    a.ol[oo + lane] = ll;
    split_f16(o1, hh, ll);
    a.oh[oo + lane + 32] = hh;
    a.ol[oo + lane + 32] = ll;
    if (a.o32) {
      a.o32[oo + lane] = o0;
      a.o32[oo + lane + 32] = o1;
    }
  }
}

// ---------------------------------------------------------- tensor-core time attention
// Time attention for one (variate row, head) on mma.sync tensor cores, for
// p <= 256 (same semantics as attn_time_kernel).  f32-class products from f16
// MMAs: every operand is split into hi + lo f16 terms and a product is
// hi.hi + hi.lo + lo.hi with f32 accumulation.
//   - staging: the row's q, k and v tiles arrive by TMA (128-byte swizzled
//     [p][32] f32 boxes); one thread per key token reads its k or v row,
//     applies QK-norm and RoPE to k, and stores k and v as f16 hi/lo planes
//     in shared memory;
//   - one warp per block of 16 queries keeps its q rows in registers (normed,
//     rotated, split into mma fragments), walks the key blocks up to the
//     diagonal with an online softmax on the score fragments, and accumulates
//     P.V with P re-split from the score registers (FlashAttention-2 style).
constexpr int kAttnMmaMaxP = 256;  // 16 warps, 147 KB of shared memory at p = 256

// RoPE of the adjacent pair (x0, x1) = dims (2i, 2i+1) from a compact table
// row (cos[32], sin[32] per pair, scale[32], 1/scale[32] per dim mod 32):
// (x0, x1) -> (x0 c - x1 s, x1 c + x0 s) * scale, k uses 1/scale.
T0B_DEV void rope_pair(float &x0, float &x1, const float *tab, int i, bool kside) {
  const float c = tab[i], sn = tab[32 + i];
  const float *sc = tab + (kside ? 96 : 64);
  const float s0 = sc[(2 * i) & 31], s1 = sc[(2 * i + 1) & 31];
  const float a0 = x0, a1 = x1;
  x0 = a0 * c * s0 + (-a1) * sn * s0;
  x1 = a1 * c * s1 + a0 * sn * s1;
}

T0B_DEV uint32_t pack_h2(__half lo_elem, __half hi_elem) {
  __half2 v = __halves2half2(lo_elem, hi_elem);
  return *reinterpret_cast<uint32_t *>(&v);
}


// Shared-memory layout of attn_time_mma_kernel past its 1024-byte aligned
// base: the four f16 planes [4][PK][72] (the k / v TMA tiles alias their
// start), the q tile [2][PK][32] f32 (1024-byte aligned), the mbarrier.
__host__ __device__ constexpr size_t attn_planes_bytes(int PK) { return (size_t)4 * PK * 72 * 2; }
__host__ __device__ constexpr size_t attn_q_off(int PK) { return (attn_planes_bytes(PK) + 1023) / 1024 * 1024; }
__host__ __device__ constexpr size_t attn_smem_bytes(int PK) { return attn_q_off(PK) + (size_t)PK * 256 + 16; }
T0B_DEV uint8_t *attn_qtile(__half *base, int PK) { return reinterpret_cast<uint8_t *>(base) + attn_q_off(PK); }
T0B_DEV uint64_t *attn_bar(__half *base, int PK) {
  return reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(base) + attn_q_off(PK) + (size_t)PK * 256);
}

// use_tma: bit 0 = q / k / v tiles by TMA loads (tm_qkv); bit 1 (with bit 0)
// = the output planes by TMA stores (tm_oh / tm_ol: [R][p][E] f16 maps,
// 64 x 16 x 1 boxes with the 128-byte swizzle), staged in this warp's rows of
// the q tile, which only this warp reads and only before the k / v barrier.
__global__ void __launch_bounds__(512, 1) attn_time_mma_kernel(AttnArgs a, const __grid_constant__ CUtensorMap tm_qkv,
                                                               const __grid_constant__ CUtensorMap tm_oh,
                                                               const __grid_constant__ CUtensorMap tm_ol,
                                                               int use_tma_flags) {
  const bool use_tma = (use_tma_flags & 1) != 0;
  const bool tma_out = use_tma && (use_tma_flags & 2) != 0;
  pdl_launch_dependents();  // the next small-M GEMM may prefetch its weights
  pdl_wait();               // q, k, v come from the previous kernel
  extern __shared__ __align__(128) uint4 smem_u4[];
  const int r = blockIdx.x, h = blockIdx.y;
  const int p = a.p, E = a.E;
  const int QB = (p + 15) >> 4;  // blocks of 16 queries (= keys)
  const int PK = QB * 16;
  // k and v row-major [PK][72] f16 (72-half pitch: conflict-free ldmatrix rows),
  // from a 1024-byte aligned base (the TMA swizzle atom)
  __half *Kh = reinterpret_cast<__half *>(smem_u4 + ((1024u - (smem_u32(smem_u4) & 1023u)) & 1023u) / 16);
  __half *Kl = Kh + PK * 72;
  __half *Vh = Kl + PK * 72;
  __half *Vl = Vh + PK * 72;
  const size_t tok0 = (size_t)r * p;
  const bool rope = a.use_rope != 0;
  const int lo = a.row_first_valid[r];

  // ---- staging (blockDim = 32 QB = 2 PK): threads [0, PK) take the v row of
  // token j, threads [PK, 2 PK) the k row.  With use_tma the row's k and v
  // tiles ([p][64] f32 each) arrive by TMA loads into the start of the (not
  // yet written) f16 planes and each thread reads its row from there;
  // otherwise every load of a row is issued from global memory before any
  // conversion.
  {
    const bool is_k = threadIdx.x >= PK;
    const int j = is_k ? threadIdx.x - PK : threadIdx.x;
    float xv[64];
    if (use_tma) {
      // four boxes of [p][32] f32 with the 128-byte swizzle (16-byte unit u
      // of row r at unit u ^ (r & 7)): k dims 0-31, k 32-63, v 0-31, v 32-63
      uint8_t *tb = reinterpret_cast<uint8_t *>(Kh);  // 1024-byte aligned
      uint64_t *bar = attn_bar(Kh, PK);
      if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(bar, (uint32_t)(6 * p * 32 * sizeof(float)));
#pragma unroll
        for (int bx = 0; bx < 4; ++bx) {
          const int x = (bx < 2 ? E : 2 * E) + h * 64 + 32 * (bx & 1);
          if (T0B_CHECK_TMA(x, 4, (int)tok0, a.err)) tma_load_2d(tb + (size_t)bx * PK * 128, &tm_qkv, bar, x, (int)tok0);
        }
        uint8_t *qt = attn_qtile(Kh, PK);  // q dims 0-31 and 32-63, kept past the staging
        if (T0B_CHECK_TMA(h * 64, 4, (int)tok0, a.err)) {
          tma_load_2d(qt, &tm_qkv, bar, h * 64, (int)tok0);
          tma_load_2d(qt + (size_t)PK * 128, &tm_qkv, bar, h * 64 + 32, (int)tok0);
        }
      }
      const bool ok = mbar_wait(bar, 0, a.err, T0B_DEVERR_WAIT_ATTN, nullptr) && j < p;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const uint8_t *rowp = tb + ((size_t)((is_k ? 0 : 2) + hf) * PK + j) * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 x4 = ok ? *reinterpret_cast<const float4 *>(rowp + ((u ^ (j & 7)) << 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
          xv[32 * hf + 4 * u] = x4.x, xv[32 * hf + 4 * u + 1] = x4.y;
          xv[32 * hf + 4 * u + 2] = x4.z, xv[32 * hf + 4 * u + 3] = x4.w;
        }
      }
      __syncthreads();  // every row is in registers before the planes overwrite the tiles
    } else {
      const float *src = a.qkv + (tok0 + (j < p ? j : 0)) * 3 * E + h * 64 + (is_k ? E : 2 * E);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float4 x4 = j < p ? *reinterpret_cast<const float4 *>(src + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
        xv[4 * c] = x4.x, xv[4 * c + 1] = x4.y, xv[4 * c + 2] = x4.z, xv[4 * c + 3] = x4.w;
      }
    }
    if (is_k && j < p) {  // QK-norm over the whole row, then RoPE
      float ss = 0.0f;
#pragma unroll
      for (int d = 0; d < 64; ++d) ss += xv[d] * xv[d];
      const float rdn = 1.0f / sqrtf(ss / 64.0f + 1e-8f);
      const float4 *g4 = reinterpret_cast<const float4 *>(a.kn);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float4 gg = g4[c];
        xv[4 * c] = xv[4 * c] * rdn * gg.x;
        xv[4 * c + 1] = xv[4 * c + 1] * rdn * gg.y;
        xv[4 * c + 2] = xv[4 * c + 2] * rdn * gg.z;
        xv[4 * c + 3] = xv[4 * c + 3] * rdn * gg.w;
      }
      if (rope) {
        const float *tab = a.rope_c + (size_t)j * 128;
#pragma unroll
        for (int cg = 0; cg < 4; ++cg) rope16(xv + 16 * cg, tab, cg, true);
      }
    }
    __half *dh = (is_k ? Kh : Vh) + j * 72, *dl = (is_k ? Kl : Vl) + j * 72;
#pragma unroll
    for (int u = 0; u < 8; ++u) {  // 8 dims per 16-byte unit
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) split2(xv[8 * u + 2 * e], xv[8 * u + 2 * e + 1], hw[e], lw[e]);
      *reinterpret_cast<uint4 *>(dh + 8 * u) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4 *>(dl + 8 * u) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }

  // ---- this warp's query rows
  const int qb = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int ia = qb * 16 + g, ib = ia + 8;  // this thread's two query rows
  float qa[16], qbv[16];                    // dims 16kc + {2t, 2t+1, 2t+8, 2t+9}
  if (use_tma) {  // from the swizzled q tile (16-byte unit u of row r at u ^ (r & 7))
    const uint8_t *qt = attn_qtile(Kh, PK);
    const int ra_ = min(ia, p - 1), rb_ = min(ib, p - 1);
#pragma unroll
    for (int kc = 0; kc < 4; ++kc)
#pragma unroll
      for (int u8 = 0; u8 < 2; ++u8) {
        const int d = 16 * kc + 2 * t + 8 * u8, hf = d >> 5, uu = (d & 31) >> 2, off = (d & 3) * 4;
        const float2 x = *reinterpret_cast<const float2 *>(qt + ((size_t)hf * PK + ra_) * 128 + ((uu ^ (ra_ & 7)) << 4) + off);
        const float2 y = *reinterpret_cast<const float2 *>(qt + ((size_t)hf * PK + rb_) * 128 + ((uu ^ (rb_ & 7)) << 4) + off);
        qa[4 * kc + 2 * u8] = x.x, qa[4 * kc + 2 * u8 + 1] = x.y;
        qbv[4 * kc + 2 * u8] = y.x, qbv[4 * kc + 2 * u8 + 1] = y.y;
      }
  } else {
    const float *ra = a.qkv + (tok0 + min(ia, p - 1)) * 3 * E + h * 64;
    const float *rb = a.qkv + (tok0 + min(ib, p - 1)) * 3 * E + h * 64;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const float2 u0 = *reinterpret_cast<const float2 *>(ra + 16 * kc + 2 * t);
      const float2 u1 = *reinterpret_cast<const float2 *>(ra + 16 * kc + 2 * t + 8);
      const float2 w0 = *reinterpret_cast<const float2 *>(rb + 16 * kc + 2 * t);
      const float2 w1 = *reinterpret_cast<const float2 *>(rb + 16 * kc + 2 * t + 8);
      qa[4 * kc] = u0.x, qa[4 * kc + 1] = u0.y, qa[4 * kc + 2] = u1.x, qa[4 * kc + 3] = u1.y;
      qbv[4 * kc] = w0.x, qbv[4 * kc + 1] = w0.y, qbv[4 * kc + 2] = w1.x, qbv[4 * kc + 3] = w1.y;
    }
  }

  // ---- q: QK-norm, RoPE, split into mma fragments (rows >= p are zero)
  uint32_t qh[4][4], ql[4][4];
  {
    if (ia >= p)
#pragma unroll
      for (int x = 0; x < 16; ++x) qa[x] = 0.0f;
    if (ib >= p)
#pragma unroll
      for (int x = 0; x < 16; ++x) qbv[x] = 0.0f;
    float sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int x = 0; x < 16; ++x) {
      sa += qa[x] * qa[x];
      sb += qbv[x] * qbv[x];
    }
    sa += __shfl_xor_sync(0xffffffffu, sa, 1);
    sa += __shfl_xor_sync(0xffffffffu, sa, 2);
    sb += __shfl_xor_sync(0xffffffffu, sb, 1);
    sb += __shfl_xor_sync(0xffffffffu, sb, 2);
    const float ra_n = 1.0f / sqrtf(sa / 64.0f + 1e-8f), rb_n = 1.0f / sqrtf(sb / 64.0f + 1e-8f);
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const float2 g0 = *reinterpret_cast<const float2 *>(a.qn + 16 * kc + 2 * t);
      const float2 g1 = *reinterpret_cast<const float2 *>(a.qn + 16 * kc + 2 * t + 8);
      const float gg[4] = {g0.x, g0.y, g1.x, g1.y};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qa[4 * kc + e] = qa[4 * kc + e] * ra_n * gg[e];
        qbv[4 * kc + e] = qbv[4 * kc + e] * rb_n * gg[e];
      }
    }
    if (rope) {
      const float *ta = a.rope_c + (size_t)min(ia, p - 1) * 128, *tb = a.rope_c + (size_t)min(ib, p - 1) * 128;
#pragma unroll
      for (int kc = 0; kc < 4; ++kc)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int pi = 8 * kc + t + (e >> 1) * 4;  // pair index of dims (2pi, 2pi+1)
          rope_pair(qa[4 * kc + e], qa[4 * kc + e + 1], ta, pi, false);
          rope_pair(qbv[4 * kc + e], qbv[4 * kc + e + 1], tb, pi, false);
        }
    }
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      split2(qa[4 * kc], qa[4 * kc + 1], qh[kc][0], ql[kc][0]);
      split2(qbv[4 * kc], qbv[4 * kc + 1], qh[kc][1], ql[kc][1]);
      split2(qa[4 * kc + 2], qa[4 * kc + 3], qh[kc][2], ql[kc][2]);
      split2(qbv[4 * kc + 2], qbv[4 * kc + 3], qh[kc][3], ql[kc][3]);
    }
  }
  __syncthreads();  // k and v staged

  const bool any_masked = qb * 16 < lo;  // a whole-padding query in this block
  const int kb0 = any_masked ? 0 : (lo >> 4), kb1 = any_masked ? QB - 1 : qb;
  float o[8][4];
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.0f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.0f, lb = 0.0f;
  for (int kb = kb0; kb <= kb1; ++kb) {
    float sc[2][4];
#pragma unroll
    for (int nh = 0; nh < 2; ++nh) sc[nh][0] = sc[nh][1] = sc[nh][2] = sc[nh][3] = 0.0f;
    // ldmatrix rows: matrix m = lane / 8 -> keys (m / 2) * 8 + (lane % 8), dims (m % 2) * 8
    const int koff = (kb * 16 + ((lane >> 4) << 3) + (lane & 7)) * 72 + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t h00, h01, h10, h11, l00, l01, l10, l11;  // [key half][dim half]
      ldsm_x4(Kh + koff + 16 * kc, h00, h01, h10, h11);
      ldsm_x4(Kl + koff + 16 * kc, l00, l01, l10, l11);
      mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], h00, h01);
      mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], h10, h11);
      mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], l00, l01);
      mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], l10, l11);
      mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], ql[kc][0], ql[kc][1], ql[kc][2], ql[kc][3], h00, h01);
      mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], ql[kc][0], ql[kc][1], ql[kc][2], ql[kc][3], h10, h11);
    }
    // scale + masks; e = 0,1: row ia, e = 2,3: row ib
    float bma = -INFINITY, bmb = -INFINITY;
#pragma unroll
    for (int nh = 0; nh < 2; ++nh)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = e < 2 ? ia : ib;
        const int key = kb * 16 + nh * 8 + 2 * t + (e & 1);
        float s = sc[nh][e] * 0.125f;
        if (row >= p || row < lo)  // padding row / whole-padding query: uniform over the p keys
          s = key < p ? -1.0e9f : -INFINITY;
        else if (key < lo || key > row)
          s = -INFINITY;
        sc[nh][e] = s;
        if (e < 2) bma = fmaxf(bma, s); else bmb = fmaxf(bmb, s);
      }
    bma = fmaxf(bma, __shfl_xor_sync(0xffffffffu, bma, 1));
    bma = fmaxf(bma, __shfl_xor_sync(0xffffffffu, bma, 2));
    bmb = fmaxf(bmb, __shfl_xor_sync(0xffffffffu, bmb, 1));
    bmb = fmaxf(bmb, __shfl_xor_sync(0xffffffffu, bmb, 2));
    const float na = fmaxf(ma, bma), nb = fmaxf(mb, bmb);
    const float ua = na == -INFINITY ? 0.0f : na, ub = nb == -INFINITY ? 0.0f : nb;
    const float ca = expf(ma - ua), cb = expf(mb - ub);  // rescale of what came before (0 at the start)
    ma = na;
    mb = nb;
    la *= ca;
    lb *= cb;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      o[nd][0] *= ca, o[nd][1] *= ca;
      o[nd][2] *= cb, o[nd][3] *= cb;
    }
#pragma unroll
    for (int nh = 0; nh < 2; ++nh)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = expf(sc[nh][e] - (e < 2 ? ua : ub));
        sc[nh][e] = pe;
        if (e < 2) la += pe; else lb += pe;
      }
    // P as the A operand (16 queries x 16 keys of this block), split hi/lo
    uint32_t ph[4], pl[4];
    split2(sc[0][0], sc[0][1], ph[0], pl[0]);
    split2(sc[0][2], sc[0][3], ph[1], pl[1]);
    split2(sc[1][0], sc[1][1], ph[2], pl[2]);
    split2(sc[1][2], sc[1][3], ph[3], pl[3]);
    // transposed ldmatrix rows: matrix m -> keys (m % 2) * 8 + (lane % 8), dims (m / 2) * 8
    const int voff = (kb * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * 72 + ((lane >> 4) << 3);
#pragma unroll
    for (int n2 = 0; n2 < 4; ++n2) {  // dims 16 n2 .. 16 n2 + 15 = n8 blocks 2 n2, 2 n2 + 1
      uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
      ldsm_x4_trans(Vh + voff + 16 * n2, h0, h1, h2, h3);
      ldsm_x4_trans(Vl + voff + 16 * n2, l0, l1, l2, l3);
      float *oa = o[2 * n2], *ob = o[2 * n2 + 1];
      mma16816(oa[0], oa[1], oa[2], oa[3], ph[0], ph[1], ph[2], ph[3], h0, h1);
      mma16816(ob[0], ob[1], ob[2], ob[3], ph[0], ph[1], ph[2], ph[3], h2, h3);
      mma16816(oa[0], oa[1], oa[2], oa[3], ph[0], ph[1], ph[2], ph[3], l0, l1);
      mma16816(ob[0], ob[1], ob[2], ob[3], ph[0], ph[1], ph[2], ph[3], l2, l3);
      mma16816(oa[0], oa[1], oa[2], oa[3], pl[0], pl[1], pl[2], pl[3], h0, h1);
      mma16816(ob[0], ob[1], ob[2], ob[3], pl[0], pl[1], pl[2], pl[3], h2, h3);
    }
  }
  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);
  const float inva = 1.0f / la, invb = 1.0f / lb;
  if (tma_out) {
    // this warp's 16 output rows: hi plane in its q-tile rows of dims 0-31,
    // lo plane in its rows of dims 32-63 (2 KB each, 128-byte swizzle:
    // 16-byte unit nd of row rr at unit nd ^ (rr & 7)); rows >= p are
    // clipped by the tensor maps
    uint8_t *qt = attn_qtile(Kh, PK);
    uint8_t *sh = qt + (size_t)(qb * 16) * 128, *sl = qt + (size_t)(PK + qb * 16) * 128;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      uint32_t hw, lw;
      const uint32_t ua = (uint32_t)g * 128 + (((uint32_t)nd ^ (uint32_t)g) << 4) + 4 * t;
      split2(o[nd][0] * inva, o[nd][1] * inva, hw, lw);
      *reinterpret_cast<uint32_t *>(sh + ua) = hw;
      *reinterpret_cast<uint32_t *>(sl + ua) = lw;
      split2(o[nd][2] * invb, o[nd][3] * invb, hw, lw);
      *reinterpret_cast<uint32_t *>(sh + ua + 8 * 128) = hw;
      *reinterpret_cast<uint32_t *>(sl + ua + 8 * 128) = lw;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (T0B_CHECK_TMA(h * 64, 2, qb * 16, a.err) && T0B_CHECK(r >= 0, a.err)) {
        tma_store_3d(&tm_oh, sh, h * 64, qb * 16, r);
        tma_store_3d(&tm_ol, sl, h * 64, qb * 16, r);
      }
      bulk_commit();
    }
  }
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) {
    const int d = nd * 8 + 2 * t;
    if (tma_out) {  // only the optional f32 copy
      if (a.o32 && ia < p)
        *reinterpret_cast<float2 *>(a.o32 + (tok0 + ia) * E + h * 64 + d) =
            make_float2(o[nd][0] * inva, o[nd][1] * inva);
      if (a.o32 && ib < p)
        *reinterpret_cast<float2 *>(a.o32 + (tok0 + ib) * E + h * 64 + d) =
            make_float2(o[nd][2] * invb, o[nd][3] * invb);
      continue;
    }
    if (ia < p) {
      const float x0 = o[nd][0] * inva, x1 = o[nd][1] * inva;
      const size_t oo = (tok0 + ia) * E + h * 64 + d;
      uint32_t hw, lw;
      split2(x0, x1, hw, lw);
      *reinterpret_cast<uint32_t *>(a.oh + oo) = hw;
      *reinterpret_cast<uint32_t *>(a.ol + oo) = lw;
      if (a.o32) *reinterpret_cast<float2 *>(a.o32 + oo) = make_float2(x0, x1);
    }
    if (ib < p) {
      const float x0 = o[nd][2] * invb, x1 = o[nd][3] * invb;
      const size_t oo = (tok0 + ib) * E + h * 64 + d;
      uint32_t hw, lw;
      split2(x0, x1, hw, lw);
      *reinterpret_cast<uint32_t *>(a.oh + oo) = hw;
      *reinterpret_cast<uint32_t *>(a.ol + oo) = lw;
      if (a.o32) *reinterpret_cast<float2 *>(a.o32 + oo) = make_float2(x0, x1);
    }
  }
  if (tma_out && lane == 0) bulk_wait_all();  // stores done before the CTA (and its shared memory) ends
}

// --------------------------------------- time attention on f16 planes
// Time attention for one (variate row, head) of 64 dims when the wQKV GEMM
// has written q, k and v as f16 (hi, lo) planes (its EPI_QKV epilogue): q
// and k arrive multiplied by their QK-norm gains and rotated by RoPE, and
// their QK-norm, 1/sqrt(mean(y^2) + 1e-8) per (token, head), enters here as
// a per-query and per-key scale of the scores (RoPE is linear, so this is
// the same product as norm-then-rotate, ops.rs:132-142, 175-190).  The six
// [PK][64] tiles (q, k, v; hi and lo) come in by one TMA load each with the
// 128-byte swizzle, straight into the layout the ldmatrix fragment loads
// read (16-byte unit u of row r at unit u ^ (r & 7)); rows p .. PK-1 lie
// outside the [R][p][3E] tensor map and arrive as zeros.  There is no
// per-row conversion: each warp takes one block of 16 queries through
// split-f16 QK^T and PV on mma.sync with an online softmax and the masks of
// attn_time_mma_kernel, and writes its 16 output rows as f16 planes by TMA
// stores staged in its own (already consumed) q rows.
__host__ __device__ constexpr size_t attn_pl_smem_bytes(int PK) {
  return (size_t)6 * PK * 128 + (size_t)2 * PK * 4 + 16 + 1024;  // tiles, norm factors, mbarrier, alignment
}
// Byte offset of 16-byte unit u of row r in a 128-byte-swizzled [rows][64] f16 tile.
T0B_DEV uint32_t sw128_unit(int r, int u) { return (uint32_t)r * 128u + ((uint32_t)(u ^ (r & 7)) << 4); }

__global__ void __launch_bounds__(512, 1) attn_time_pl_kernel(AttnArgs a, const __grid_constant__ CUtensorMap tm_h,
                                                              const __grid_constant__ CUtensorMap tm_l,
                                                              const __grid_constant__ CUtensorMap tm_oh,
                                                              const __grid_constant__ CUtensorMap tm_ol) {
  pdl_launch_dependents();  // the next small-M GEMM may prefetch its weights
  extern __shared__ __align__(128) uint4 smem_u4[];
  uint8_t *base = reinterpret_cast<uint8_t *>(smem_u4) + ((1024u - (smem_u32(smem_u4) & 1023u)) & 1023u);
  const int r = blockIdx.x, h = blockIdx.y;
  const int p = a.p, E = a.E, H = a.H;
  const int QB = (p + 15) >> 4;  // blocks of 16 queries (= keys), one per warp
  const int PK = QB * 16;
  const uint32_t tile = (uint32_t)PK * 128u;
  uint8_t *Qh = base, *Ql = base + tile, *Kh = base + 2 * tile, *Kl = base + 3 * tile;
  uint8_t *Vh = base + 4 * tile, *Vl = base + 5 * tile;
  float *rq = reinterpret_cast<float *>(base + 6 * tile);
  float *rk = rq + PK;
  uint64_t *bar = reinterpret_cast<uint64_t *>(rk + PK);
  const size_t tok0 = (size_t)r * p;
  const int lo = a.row_first_valid[r];

  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  for (int j = threadIdx.x; j < PK; j += blockDim.x) {  // QK-norm factors (rows >= p unused)
    float fq = 0.0f, fk = 0.0f;
    if (j < p) {
      const float *ss = a.ssq_qk + (tok0 + j) * 2 * H;
      fq = 1.0f / sqrtf(ss[h] / 64.0f + 1e-8f);
      fk = 1.0f / sqrtf(ss[H + h] / 64.0f + 1e-8f);
    }
    rq[j] = fq;
    rk[j] = fk;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(bar, 6 * tile);
#pragma unroll
    for (int sg = 0; sg < 3; ++sg) {  // q, k, v
      if (T0B_CHECK_TMA(sg * E + h * 64, 2, r, a.err)) {
        tma_load_3d(base + (2 * sg) * tile, &tm_h, bar, sg * E + h * 64, 0, r);
        tma_load_3d(base + (2 * sg + 1) * tile, &tm_l, bar, sg * E + h * 64, 0, r);
      }
    }
  }
  mbar_wait(bar, 0, a.err, T0B_DEVERR_WAIT_ATTN, nullptr);

  const int qb = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int ia = qb * 16 + g, ib = ia + 8;  // this thread's two query rows
  // q fragments of the block: ldmatrix matrix m = lane / 8 -> rows (m % 2) * 8 + lane % 8, dims (m / 2) * 8
  uint32_t qh[4][4], ql[4][4];
  {
    const int row = qb * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const uint32_t off = sw128_unit(row, 2 * kc + (lane >> 4));
      ldsm_x4(Qh + off, qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3]);
      ldsm_x4(Ql + off, ql[kc][0], ql[kc][1], ql[kc][2], ql[kc][3]);
    }
  }
  const float fa = rq[ia] * 0.125f, fb = rq[ib] * 0.125f;  // QK-norm of the two query rows x 1/sqrt(64)

  const bool any_masked = qb * 16 < lo;  // a whole-padding query in this block
  const int kb0 = any_masked ? 0 : (lo >> 4), kb1 = any_masked ? QB - 1 : qb;
  float o[8][4];
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.0f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.0f, lb = 0.0f;
  for (int kb = kb0; kb <= kb1; ++kb) {
    float sc[2][4];
#pragma unroll
    for (int nh = 0; nh < 2; ++nh) sc[nh][0] = sc[nh][1] = sc[nh][2] = sc[nh][3] = 0.0f;
    // ldmatrix rows: matrix m = lane / 8 -> keys (m / 2) * 8 + (lane % 8), dims (m % 2) * 8
    const int krow = kb * 16 + ((lane >> 4) << 3) + (lane & 7);
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t h00, h01, h10, h11, l00, l01, l10, l11;  // [key half][dim half]
      const uint32_t off = sw128_unit(krow, 2 * kc + ((lane >> 3) & 1));
      ldsm_x4(Kh + off, h00, h01, h10, h11);
      ldsm_x4(Kl + off, l00, l01, l10, l11);
      mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], h00, h01);
      mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], h10, h11);
      mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], l00, l01);
      mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], l10, l11);
      mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], ql[kc][0], ql[kc][1], ql[kc][2], ql[kc][3], h00, h01);
      mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], ql[kc][0], ql[kc][1], ql[kc][2], ql[kc][3], h10, h11);
    }
    // QK-norm scales + masks; e = 0,1: row ia, e = 2,3: row ib
    float bma = -INFINITY, bmb = -INFINITY;
#pragma unroll
    for (int nh = 0; nh < 2; ++nh) {
      const int k0 = kb * 16 + nh * 8 + 2 * t;
      const float2 fk = *reinterpret_cast<const float2 *>(rk + k0);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = e < 2 ? ia : ib;
        const int key = k0 + (e & 1);
        float s = sc[nh][e] * (e < 2 ? fa : fb) * ((e & 1) ? fk.y : fk.x);
        if (row >= p || row < lo)  // padding row / whole-padding query: uniform over the p keys
          s = key < p ? -1.0e9f : -INFINITY;
        else if (key < lo || key > row)
          s = -INFINITY;
        sc[nh][e] = s;
        if (e < 2) bma = fmaxf(bma, s); else bmb = fmaxf(bmb, s);
      }
    }
    bma = fmaxf(bma, __shfl_xor_sync(0xffffffffu, bma, 1));
    bma = fmaxf(bma, __shfl_xor_sync(0xffffffffu, bma, 2));
    bmb = fmaxf(bmb, __shfl_xor_sync(0xffffffffu, bmb, 1));
    bmb = fmaxf(bmb, __shfl_xor_sync(0xffffffffu, bmb, 2));
    const float na = fmaxf(ma, bma), nb = fmaxf(mb, bmb);
    const float ua = na == -INFINITY ? 0.0f : na, ub = nb == -INFINITY ? 0.0f : nb;
    const float ca = expf(ma - ua), cb = expf(mb - ub);  // rescale of what came before (0 at the start)
    ma = na;
    mb = nb;
    la *= ca;
    lb *= cb;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      o[nd][0] *= ca, o[nd][1] *= ca;
      o[nd][2] *= cb, o[nd][3] *= cb;
    }
#pragma unroll
    for (int nh = 0; nh < 2; ++nh)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = expf(sc[nh][e] - (e < 2 ? ua : ub));
        sc[nh][e] = pe;
        if (e < 2) la += pe; else lb += pe;
      }
    // P as the A operand (16 queries x 16 keys of this block), split hi/lo
    uint32_t ph[4], pl[4];
    split2(sc[0][0], sc[0][1], ph[0], pl[0]);
    split2(sc[0][2], sc[0][3], ph[1], pl[1]);
    split2(sc[1][0], sc[1][1], ph[2], pl[2]);
    split2(sc[1][2], sc[1][3], ph[3], pl[3]);
    // transposed ldmatrix rows: matrix m -> keys (m % 2) * 8 + (lane % 8), dims (m / 2) * 8
    const int vrow = kb * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int n2 = 0; n2 < 4; ++n2) {  // dims 16 n2 .. 16 n2 + 15 = n8 blocks 2 n2, 2 n2 + 1
      uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
      const uint32_t off = sw128_unit(vrow, 2 * n2 + (lane >> 4));
      ldsm_x4_trans(Vh + off, h0, h1, h2, h3);
      ldsm_x4_trans(Vl + off, l0, l1, l2, l3);
      float *oa = o[2 * n2], *ob = o[2 * n2 + 1];
      mma16816(oa[0], oa[1], oa[2], oa[3], ph[0], ph[1], ph[2], ph[3], h0, h1);
      mma16816(ob[0], ob[1], ob[2], ob[3], ph[0], ph[1], ph[2], ph[3], h2, h3);
      mma16816(oa[0], oa[1], oa[2], oa[3], ph[0], ph[1], ph[2], ph[3], l0, l1);
      mma16816(ob[0], ob[1], ob[2], ob[3], ph[0], ph[1], ph[2], ph[3], l2, l3);
      mma16816(oa[0], oa[1], oa[2], oa[3], pl[0], pl[1], pl[2], pl[3], h0, h1);
      mma16816(ob[0], ob[1], ob[2], ob[3], pl[0], pl[1], pl[2], pl[3], h2, h3);
    }
  }
  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);
  const float inva = 1.0f / la, invb = 1.0f / lb;
  // this warp's 16 output rows: hi plane in its q-tile rows of the hi tile, lo
  // plane in its rows of the lo tile (2 KB each, 128-byte swizzle); rows >= p
  // are clipped by the tensor maps
  uint8_t *sh = Qh + (size_t)(qb * 16) * 128, *sl = Ql + (size_t)(qb * 16) * 128;
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) {
    uint32_t hw, lw;
    const uint32_t ua = (uint32_t)g * 128 + (((uint32_t)nd ^ (uint32_t)g) << 4) + 4 * t;
    split2(o[nd][0] * inva, o[nd][1] * inva, hw, lw);
    *reinterpret_cast<uint32_t *>(sh + ua) = hw;
    *reinterpret_cast<uint32_t *>(sl + ua) = lw;
    split2(o[nd][2] * invb, o[nd][3] * invb, hw, lw);
    *reinterpret_cast<uint32_t *>(sh + ua + 8 * 128) = hw;
    *reinterpret_cast<uint32_t *>(sl + ua + 8 * 128) = lw;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (T0B_CHECK_TMA(h * 64, 2, qb * 16, a.err) && T0B_CHECK(r >= 0, a.err)) {
      tma_store_3d(&tm_oh, sh, h * 64, qb * 16, r);
      tma_store_3d(&tm_ol, sl, h * 64, qb * 16, r);
    }
    bulk_commit();
    bulk_wait_all();  // stores done before the CTA (and its shared memory) ends
  }
  if (a.o32) {  // optional f32 copy of the output
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      const int d = nd * 8 + 2 * t;
      if (ia < p)
        *reinterpret_cast<float2 *>(a.o32 + (tok0 + ia) * E + h * 64 + d) = make_float2(o[nd][0] * inva, o[nd][1] * inva);
      if (ib < p)
        *reinterpret_cast<float2 *>(a.o32 + (tok0 + ib) * E + h * 64 + d) = make_float2(o[nd][2] * invb, o[nd][3] * invb);
    }
  }
}

cudaError_t t0b_launch_attn_time_planes(const AttnArgs &a, cudaStream_t st) {
  if (a.E / a.H != 64 || a.E % 64 || a.p < 1 || a.p > 256 || !a.qkv_h || !a.qkv_l || !a.ssq_qk || !a.oh || !a.ol)
    return cudaErrorInvalidValue;
  const int QB = (a.p + 15) / 16, PK = 16 * QB;
  const size_t smem = attn_pl_smem_bytes(PK);
  cudaError_t e = t0b_smem_limit((const void *)attn_time_pl_kernel, smem);
  if (e != cudaSuccess) return e;
  // q | k | v planes as [R][p][3E] f16 with [1][PK][64] boxes (rows >= p zero);
  // output planes as [R][p][E] f16 with [1][16][64] boxes (rows >= p clipped)
  CUtensorMap th, tl, toh, tol;
  const uint64_t rs = (uint64_t)3 * a.E * 2, ss = rs * (uint64_t)a.p;
  const uint64_t ors = (uint64_t)a.E * 2, oss = ors * (uint64_t)a.p;
  if (!t0b_make_tmap_f16_3d(&th, a.qkv_h, (uint64_t)3 * a.E, (uint64_t)a.p, (uint64_t)a.R, rs, ss, 64, (uint32_t)PK, 1,
                            true) ||
      !t0b_make_tmap_f16_3d(&tl, a.qkv_l, (uint64_t)3 * a.E, (uint64_t)a.p, (uint64_t)a.R, rs, ss, 64, (uint32_t)PK, 1,
                            true) ||
      !t0b_make_tmap_f16_3d(&toh, a.oh, (uint64_t)a.E, (uint64_t)a.p, (uint64_t)a.R, ors, oss, 64, 16, 1, true) ||
      !t0b_make_tmap_f16_3d(&tol, a.ol, (uint64_t)a.E, (uint64_t)a.p, (uint64_t)a.R, ors, oss, 64, 16, 1, true))
    return cudaErrorInvalidValue;
  attn_time_pl_kernel<<<dim3(a.R, a.H), 32 * QB, smem, st>>>(a, th, tl, toh, tol);
  return cudaGetLastError();
}

// ------------------------------------------------- 128-dim heads (t0-beta)
// Time attention for heads of HD = 128 dims, p <= 256, with the arithmetic
// of attn_time_mma_kernel (split-f16 QK^T and PV on mma.sync, online
// softmax).  At most 8 warps, each taking query blocks warp, warp + 8, ...;
// k / v rows are staged in 64-dim halves after a sum-of-squares pass, so no
// thread holds a whole row.  VSPLIT = 1 stages all of V (p <= 192: 4 f16
// planes of [192][136], 209 KB of shared memory); VSPLIT = 2 stages K whole
// and V one 64-dim half at a time (p <= 256: 139 + 74 KB), running the
// queries once per half: the scores and softmax of the second run repeat
// the first bit for bit (same operations in the same order), and each run
// writes its half of the output dims.
constexpr int kAttnWideMaxP = 256;
constexpr int kAttnWideOnePassMaxP = 192;

// RoPE on dims 16cg .. 16cg + 15 from a compact table row [2 HD]
// (cos[HD/2], sin[HD/2] per pair, scale[HD/2], 1/scale[HD/2] per dim mod
// HD/2); same arithmetic as rope16.
template <int HD>
T0B_DEV void rope16_hd(float *x, const float *tab, int cg, bool kside) {
  constexpr int HALF = HD / 2;
  const float *cs = tab + 8 * cg, *sn = tab + HALF + 8 * cg;
  const float *sv = tab + (kside ? 3 * HALF : 2 * HALF) + ((16 * cg) % HALF);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a0 = x[2 * i], a1 = x[2 * i + 1];
    x[2 * i] = a0 * cs[i] * sv[2 * i] + (-a1) * sn[i] * sv[2 * i];
    x[2 * i + 1] = a1 * cs[i] * sv[2 * i + 1] + a0 * sn[i] * sv[2 * i + 1];
  }
}
template <int HD>
T0B_DEV void rope_pair_hd(float &x0, float &x1, const float *tab, int i, bool kside) {
  constexpr int HALF = HD / 2;
  const float c = tab[i], sn = tab[HALF + i];
  const float *sc = tab + (kside ? 3 * HALF : 2 * HALF);
  const float s0 = sc[(2 * i) % HALF], s1 = sc[(2 * i + 1) % HALF];
  const float a0 = x0, a1 = x1;
  x0 = a0 * c * s0 + (-a1) * sn * s0;
  x1 = a1 * c * s1 + a0 * sn * s1;
}

template <int HD, int VSPLIT>
__global__ void __launch_bounds__(256, 1) attn_time_wide_kernel(AttnArgs a) {
  pdl_launch_dependents();  // the next small-M GEMM may prefetch its weights
  constexpr int PITCH = HD + 8;  // halves: conflict-free ldmatrix rows
  constexpr int VD = HD / VSPLIT;  // V dims staged (and output dims written) per run
  constexpr int VPITCH = VD + 8;
  constexpr int NKC = HD / 16;   // 16-dim chunks of a head
  constexpr int NVC = VD / 16;   // 16-dim chunks of V per run
  constexpr int NDT = VD / 8;    // n8 tiles of the output per run
  static_assert(VD % 64 == 0, "V is staged in 64-dim halves");
  extern __shared__ uint4 smem_u4[];
  const int r = blockIdx.x, h = blockIdx.y;
  const int p = a.p, E = a.E;
  const int QB = (p + 15) >> 4;  // blocks of 16 queries (= keys)
  const int PK = QB * 16;
  __half *Kh = reinterpret_cast<__half *>(smem_u4);
  __half *Kl = Kh + PK * PITCH;
  __half *Vh = Kl + PK * PITCH;
  __half *Vl = Vh + PK * VPITCH;
  const size_t tok0 = (size_t)r * p;
  const bool rope = a.use_rope != 0;
  const int lo = a.row_first_valid[r];
  const float qk_scale = 1.0f / sqrtf((float)HD);

#pragma unroll 1
  for (int vp = 0; vp < VSPLIT; ++vp) {
  // ---- staging: rows [0, PK) are v rows (dims [vp VD, vp VD + VD)), [PK, 2 PK)
  // k rows (all dims, first run only); rows >= p are zero
  if (vp > 0) __syncthreads();  // the previous run has finished reading V
  for (int row = threadIdx.x; row < (vp == 0 ? 2 * PK : PK); row += blockDim.x) {
    const bool is_k = row >= PK;
    const int j = is_k ? row - PK : row;
    const float *src = a.qkv + (tok0 + (j < p ? j : 0)) * 3 * E + (is_k ? E : 2 * E) + h * HD;
    float rdn = 1.0f;
    if (is_k && j < p) {  // QK-norm over the whole head
      float ss = 0.0f;
#pragma unroll 4
      for (int c = 0; c < HD / 4; ++c) {
        const float4 x4 = reinterpret_cast<const float4 *>(src)[c];
        ss += x4.x * x4.x;
        ss += x4.y * x4.y;
        ss += x4.z * x4.z;
        ss += x4.w * x4.w;
      }
      rdn = 1.0f / sqrtf(ss / (float)HD + 1e-8f);
    }
    __half *dh = is_k ? Kh + j * PITCH : Vh + j * VPITCH, *dl = is_k ? Kl + j * PITCH : Vl + j * VPITCH;
    const int hf0 = is_k ? 0 : vp * (VD / 64), nhf = is_k ? HD / 64 : VD / 64;
#pragma unroll 1
    for (int hx = 0; hx < nhf; ++hx) {
      const int hf = hf0 + hx;  // 64-dim half of the head read here
      float xv[64];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float4 x4 = j < p ? reinterpret_cast<const float4 *>(src + 64 * hf)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        xv[4 * c] = x4.x, xv[4 * c + 1] = x4.y, xv[4 * c + 2] = x4.z, xv[4 * c + 3] = x4.w;
      }
      if (is_k && j < p) {
        const float *gk = a.kn + 64 * hf;
#pragma unroll
        for (int d = 0; d < 64; ++d) xv[d] = xv[d] * rdn * gk[d];
        if (rope) {
          const float *tab = a.rope_c + (size_t)j * 2 * HD;
#pragma unroll
          for (int cg = 0; cg < 4; ++cg) rope16_hd<HD>(xv + 16 * cg, tab, 4 * hf + cg, true);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) split2(xv[8 * u + 2 * e], xv[8 * u + 2 * e + 1], hw[e], lw[e]);
        *reinterpret_cast<uint4 *>(dh + 64 * hx + 8 * u) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(dl + 64 * hx + 8 * u) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  for (int qb = warp; qb < QB; qb += nw) {
    const int ia = qb * 16 + g, ib = ia + 8;  // this thread's two query rows
    uint32_t qh[NKC][4], ql[NKC][4];
    {
      // dims 16 kc + {2t, 2t+1, 2t+8, 2t+9} of rows ia, ib (rows >= p are zero)
      float qa[NKC][4], qv[NKC][4];
      const float *ra = a.qkv + (tok0 + min(ia, p - 1)) * 3 * E + h * HD;
      const float *rb = a.qkv + (tok0 + min(ib, p - 1)) * 3 * E + h * HD;
      float sa = 0.0f, sb = 0.0f;
#pragma unroll
      for (int kc = 0; kc < NKC; ++kc) {
        const float2 u0 = *reinterpret_cast<const float2 *>(ra + 16 * kc + 2 * t);
        const float2 u1 = *reinterpret_cast<const float2 *>(ra + 16 * kc + 2 * t + 8);
        const float2 w0 = *reinterpret_cast<const float2 *>(rb + 16 * kc + 2 * t);
        const float2 w1 = *reinterpret_cast<const float2 *>(rb + 16 * kc + 2 * t + 8);
        qa[kc][0] = ia < p ? u0.x : 0.0f, qa[kc][1] = ia < p ? u0.y : 0.0f;
        qa[kc][2] = ia < p ? u1.x : 0.0f, qa[kc][3] = ia < p ? u1.y : 0.0f;
        qv[kc][0] = ib < p ? w0.x : 0.0f, qv[kc][1] = ib < p ? w0.y : 0.0f;
        qv[kc][2] = ib < p ? w1.x : 0.0f, qv[kc][3] = ib < p ? w1.y : 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e) sa += qa[kc][e] * qa[kc][e], sb += qv[kc][e] * qv[kc][e];
      }
      sa += __shfl_xor_sync(0xffffffffu, sa, 1);
      sa += __shfl_xor_sync(0xffffffffu, sa, 2);
      sb += __shfl_xor_sync(0xffffffffu, sb, 1);
      sb += __shfl_xor_sync(0xffffffffu, sb, 2);
      const float ra_n = 1.0f / sqrtf(sa / (float)HD + 1e-8f), rb_n = 1.0f / sqrtf(sb / (float)HD + 1e-8f);
      const float *ta = a.rope_c + (size_t)min(ia, p - 1) * 2 * HD, *tb = a.rope_c + (size_t)min(ib, p - 1) * 2 * HD;
#pragma unroll
      for (int kc = 0; kc < NKC; ++kc) {
        const float2 g0 = *reinterpret_cast<const float2 *>(a.qn + 16 * kc + 2 * t);
        const float2 g1 = *reinterpret_cast<const float2 *>(a.qn + 16 * kc + 2 * t + 8);
        const float gg[4] = {g0.x, g0.y, g1.x, g1.y};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          qa[kc][e] = qa[kc][e] * ra_n * gg[e];
          qv[kc][e] = qv[kc][e] * rb_n * gg[e];
        }
        if (rope) {
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int pi = 8 * kc + t + (e >> 1) * 4;  // pair index of dims (2pi, 2pi+1)
            rope_pair_hd<HD>(qa[kc][e], qa[kc][e + 1], ta, pi, false);
            rope_pair_hd<HD>(qv[kc][e], qv[kc][e + 1], tb, pi, false);
          }
        }
        split2(qa[kc][0], qa[kc][1], qh[kc][0], ql[kc][0]);
        split2(qv[kc][0], qv[kc][1], qh[kc][1], ql[kc][1]);
        split2(qa[kc][2], qa[kc][3], qh[kc][2], ql[kc][2]);
        split2(qv[kc][2], qv[kc][3], qh[kc][3], ql[kc][3]);
      }
    }

    const bool any_masked = qb * 16 < lo;  // a whole-padding query in this block
    const int kb0 = any_masked ? 0 : (lo >> 4), kb1 = any_masked ? QB - 1 : qb;
    float o[NDT][4];
  #pragma unroll
    for (int nd = 0; nd < NDT; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.0f;
    float ma = -INFINITY, mb = -INFINITY, la = 0.0f, lb = 0.0f;
    for (int kb = kb0; kb <= kb1; ++kb) {
      float sc[2][4];
  #pragma unroll
      for (int nh = 0; nh < 2; ++nh) sc[nh][0] = sc[nh][1] = sc[nh][2] = sc[nh][3] = 0.0f;
      // ldmatrix rows: matrix m = lane / 8 -> keys (m / 2) * 8 + (lane % 8), dims (m % 2) * 8
      const int koff = (kb * 16 + ((lane >> 4) << 3) + (lane & 7)) * PITCH + ((lane >> 3) & 1) * 8;
  #pragma unroll
      for (int kc = 0; kc < NKC; ++kc) {
        uint32_t h00, h01, h10, h11, l00, l01, l10, l11;  // [key half][dim half]
        ldsm_x4(Kh + koff + 16 * kc, h00, h01, h10, h11);
        ldsm_x4(Kl + koff + 16 * kc, l00, l01, l10, l11);
        mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], h00, h01);
        mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], h10, h11);
        mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], l00, l01);
        mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], l10, l11);
        mma16816(sc[0][0], sc[0][1], sc[0][2], sc[0][3], ql[kc][0], ql[kc][1], ql[kc][2], ql[kc][3], h00, h01);
        mma16816(sc[1][0], sc[1][1], sc[1][2], sc[1][3], ql[kc][0], ql[kc][1], ql[kc][2], ql[kc][3], h10, h11);
      }
      // scale + masks; e = 0,1: row ia, e = 2,3: row ib
      float bma = -INFINITY, bmb = -INFINITY;
  #pragma unroll
      for (int nh = 0; nh < 2; ++nh)
  #pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = e < 2 ? ia : ib;
          const int key = kb * 16 + nh * 8 + 2 * t + (e & 1);
          float s = sc[nh][e] * qk_scale;
          if (row >= p || row < lo)  // padding row / whole-padding query: uniform over the p keys
            s = key < p ? -1.0e9f : -INFINITY;
          else if (key < lo || key > row)
            s = -INFINITY;
          sc[nh][e] = s;
          if (e < 2) bma = fmaxf(bma, s); else bmb = fmaxf(bmb, s);
        }
      bma = fmaxf(bma, __shfl_xor_sync(0xffffffffu, bma, 1));
      bma = fmaxf(bma, __shfl_xor_sync(0xffffffffu, bma, 2));
      bmb = fmaxf(bmb, __shfl_xor_sync(0xffffffffu, bmb, 1));
      bmb = fmaxf(bmb, __shfl_xor_sync(0xffffffffu, bmb, 2));
      const float na = fmaxf(ma, bma), nb = fmaxf(mb, bmb);
      const float ua = na == -INFINITY ? 0.0f : na, ub = nb == -INFINITY ? 0.0f : nb;
      const float ca = expf(ma - ua), cb = expf(mb - ub);  // rescale of what came before (0 at the start)
      ma = na;
      mb = nb;
      la *= ca;
      lb *= cb;
  #pragma unroll
      for (int nd = 0; nd < NDT; ++nd) {
        o[nd][0] *= ca, o[nd][1] *= ca;
        o[nd][2] *= cb, o[nd][3] *= cb;
      }
  #pragma unroll
      for (int nh = 0; nh < 2; ++nh)
  #pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float pe = expf(sc[nh][e] - (e < 2 ? ua : ub));
          sc[nh][e] = pe;
          if (e < 2) la += pe; else lb += pe;
        }
      // P as the A operand (16 queries x 16 keys of this block), split hi/lo
      uint32_t ph[4], pl[4];
      split2(sc[0][0], sc[0][1], ph[0], pl[0]);
      split2(sc[0][2], sc[0][3], ph[1], pl[1]);
      split2(sc[1][0], sc[1][1], ph[2], pl[2]);
      split2(sc[1][2], sc[1][3], ph[3], pl[3]);
      // transposed ldmatrix rows: matrix m -> keys (m % 2) * 8 + (lane % 8), dims (m / 2) * 8
      const int voff = (kb * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * VPITCH + ((lane >> 4) << 3);
  #pragma unroll
      for (int n2 = 0; n2 < NVC; ++n2) {  // dims 16 n2 .. 16 n2 + 15 = n8 blocks 2 n2, 2 n2 + 1
        uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
        ldsm_x4_trans(Vh + voff + 16 * n2, h0, h1, h2, h3);
        ldsm_x4_trans(Vl + voff + 16 * n2, l0, l1, l2, l3);
        float *oa = o[2 * n2], *ob = o[2 * n2 + 1];
        mma16816(oa[0], oa[1], oa[2], oa[3], ph[0], ph[1], ph[2], ph[3], h0, h1);
        mma16816(ob[0], ob[1], ob[2], ob[3], ph[0], ph[1], ph[2], ph[3], h2, h3);
        mma16816(oa[0], oa[1], oa[2], oa[3], ph[0], ph[1], ph[2], ph[3], l0, l1);
        mma16816(ob[0], ob[1], ob[2], ob[3], ph[0], ph[1], ph[2], ph[3], l2, l3);
        mma16816(oa[0], oa[1], oa[2], oa[3], pl[0], pl[1], pl[2], pl[3], h0, h1);
        mma16816(ob[0], ob[1], ob[2], ob[3], pl[0], pl[1], pl[2], pl[3], h2, h3);
      }
    }
    la += __shfl_xor_sync(0xffffffffu, la, 1);
    la += __shfl_xor_sync(0xffffffffu, la, 2);
    lb += __shfl_xor_sync(0xffffffffu, lb, 1);
    lb += __shfl_xor_sync(0xffffffffu, lb, 2);
    const float inva = 1.0f / la, invb = 1.0f / lb;
#pragma unroll
    for (int nd = 0; nd < NDT; ++nd) {
      const int d = vp * VD + nd * 8 + 2 * t;
      if (ia < p) {
        const float x0 = o[nd][0] * inva, x1 = o[nd][1] * inva;
        const size_t oo = (tok0 + ia) * E + h * HD + d;
        uint32_t hw, lw;
        split2(x0, x1, hw, lw);
        *reinterpret_cast<uint32_t *>(a.oh + oo) = hw;
        *reinterpret_cast<uint32_t *>(a.ol + oo) = lw;
        if (a.o32) *reinterpret_cast<float2 *>(a.o32 + oo) = make_float2(x0, x1);
      }
      if (ib < p) {
        const float x0 = o[nd][2] * invb, x1 = o[nd][3] * invb;
        const size_t oo = (tok0 + ib) * E + h * HD + d;
        uint32_t hw, lw;
        split2(x0, x1, hw, lw);
        *reinterpret_cast<uint32_t *>(a.oh + oo) = hw;
        *reinterpret_cast<uint32_t *>(a.ol + oo) = lw;
        if (a.o32) *reinterpret_cast<float2 *>(a.o32 + oo) = make_float2(x0, x1);
      }
    }
  }
  }  // vp
}

// Group attention for one (series, patch): every head (one warp each) over
// the series' variate rows at that patch (mask.rs:69-82).  Rows whose patch
// is whole padding are blocked keys; such a query averages V over the
// series' rows.  q and k get their per-head RMSNorm as they are read (no
// RoPE on GROUP layers).
template <int HD>
__global__ void __launch_bounds__(256) attn_group_kernel(AttnArgs a) {
  pdl_launch_dependents();  // the next small-M GEMM may prefetch its weights
  constexpr int DPL = HD / 32;  // dims per lane: lane + 32 c
  const int s = blockIdx.x, patch = blockIdx.y;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (h >= a.H) return;
  const int r0 = a.series_row0[s], nv = a.series_nrows[s];
  const int p = a.p, E = a.E;
  const float qk_scale = 1.0f / sqrtf((float)HD);
  float qg[DPL], kg[DPL];
#pragma unroll
  for (int c = 0; c < DPL; ++c) qg[c] = a.qn[lane + 32 * c], kg[c] = a.kn[lane + 32 * c];
  // the normalised key of row kb, this lane's dims
  auto key = [&](int kb, float *kv) {
    const float *krow = a.qkv + ((size_t)(r0 + kb) * p + patch) * 3 * E + E + h * HD;
    float sk = 0.0f;
#pragma unroll
    for (int c = 0; c < DPL; ++c) kv[c] = krow[lane + 32 * c], sk += kv[c] * kv[c];
    const float rdn = 1.0f / sqrtf(warp_sum(sk) / (float)HD + 1e-8f);
#pragma unroll
    for (int c = 0; c < DPL; ++c) kv[c] = kv[c] * rdn * kg[c];
  };
  for (int qa = 0; qa < nv; ++qa) {
    const size_t tq = (size_t)(r0 + qa) * p + patch;
    const float *qrow = a.qkv + tq * 3 * E + h * HD;
    float q[DPL], sq = 0.0f;
#pragma unroll
    for (int c = 0; c < DPL; ++c) q[c] = qrow[lane + 32 * c], sq += q[c] * q[c];
    const float rq = 1.0f / sqrtf(warp_sum(sq) / (float)HD + 1e-8f);
#pragma unroll
    for (int c = 0; c < DPL; ++c) q[c] = q[c] * rq * qg[c];
    const bool qmasked = patch < a.row_first_valid[r0 + qa];
    // two passes over keys: max, then exp-sum and output
    float mx = -INFINITY;
    for (int kb = 0; kb < nv; ++kb) {
      const bool kvalid = patch >= a.row_first_valid[r0 + kb];
      float kv[DPL], dp = 0.0f;
      key(kb, kv);
#pragma unroll
      for (int c = 0; c < DPL; ++c) dp += q[c] * kv[c];
      const float d = warp_sum(dp);
      mx = fmaxf(mx, qmasked ? -1.0e9f : (kvalid ? d * qk_scale : -INFINITY));
    }
    float sum = 0.0f, o[DPL];
#pragma unroll
    for (int c = 0; c < DPL; ++c) o[c] = 0.0f;
    for (int kb = 0; kb < nv; ++kb) {
      const bool kvalid = patch >= a.row_first_valid[r0 + kb];
      float kv[DPL], dp = 0.0f;
      key(kb, kv);
#pragma unroll
      for (int c = 0; c < DPL; ++c) dp += q[c] * kv[c];
      const float d = warp_sum(dp);
      const float e = expf((qmasked ? -1.0e9f : (kvalid ? d * qk_scale : -INFINITY)) - mx);
      sum += e;
      const float *vrow = a.qkv + ((size_t)(r0 + kb) * p + patch) * 3 * E + 2 * E + h * HD;
#pragma unroll
      for (int c = 0; c < DPL; ++c) o[c] = fmaf(e, vrow[lane + 32 * c], o[c]);
    }
    const size_t oo = tq * E + h * HD;
#pragma unroll
    for (int c = 0; c < DPL; ++c) {
      const float x = o[c] / sum;
      __half hh, ll;
      split_f16(x, hh, ll);
      a.oh[oo + lane + 32 * c] = hh;
      a.ol[oo + lane + 32 * c] = ll;
      if (a.o32) a.o32[oo + lane + 32 * c] = x;
    }
  }
}

// Group attention on the tensor cores, 64-dim heads, up to 16 variate rows
// per series: one warp per head of one (series, patch).  The rows are the 16
// MMA rows (queries) and the 16 keys of the tile, padded with zeros; scores
// Q.K^T and P.V use the split-f16 three-term products of the time attention
// (f32-class), the softmax runs on the score fragments.  Semantics as
// attn_group_kernel (mask.rs:69-82).
template <int NT>  // key / query tiles of 8 rows: 1 (up to 8 variates) or 2 (up to 16)
__global__ void __launch_bounds__(256, NT == 1 ? 4 : 2) attn_group_mma_kernel(AttnArgs a) {
  pdl_launch_dependents();  // the next small-M GEMM may prefetch its weights
  __shared__ __align__(16) __half vs[8][2][16 * 72];  // per warp: v rows as f16 hi / lo planes
  const int s = blockIdx.x, patch = blockIdx.y;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (h >= a.H) return;
  const int g = lane >> 2, t = lane & 3;
  const int r0 = a.series_row0[s], nv = a.series_nrows[s];
  const int p = a.p, E = a.E;
  // per row (g, then g + 8) and its dims 16 kc + {2t, 2t+1, 2t+8, 2t+9}:
  // QK-norm (the quad t = 0..3 holds the row's 64 dims), then the q / k
  // mma fragments and the v row into this warp's shared planes
  uint32_t qh[4][4], ql[4][4], kh[4][4], kl[4][4];
  bool valid[2] = {false, false};
#pragma unroll
  for (int kc = 0; kc < 4; ++kc)
#pragma unroll
    for (int x = 0; x < 4; ++x) qh[kc][x] = ql[kc][x] = kh[kc][x] = kl[kc][x] = 0u;  // rows >= 8 NT: zero
#pragma unroll
  for (int hr = 0; hr < NT; ++hr) {
    const int b = g + 8 * hr;
    const bool in = b < nv;
    valid[hr] = in && patch >= a.row_first_valid[r0 + min(b, nv - 1)];
    const float *row = a.qkv + ((size_t)(r0 + min(b, nv - 1)) * p + patch) * 3 * E + h * 64;
    float q[16], k[16];
    __half *vh = vs[h][0] + b * 72, *vl = vs[h][1] + b * 72;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int d = 16 * kc + 2 * t + 8 * u;
        const float2 qq = *reinterpret_cast<const float2 *>(row + d);
        const float2 kk = *reinterpret_cast<const float2 *>(row + E + d);
        const float2 vv = *reinterpret_cast<const float2 *>(row + 2 * E + d);
        q[4 * kc + 2 * u] = in ? qq.x : 0.0f, q[4 * kc + 2 * u + 1] = in ? qq.y : 0.0f;
        k[4 * kc + 2 * u] = in ? kk.x : 0.0f, k[4 * kc + 2 * u + 1] = in ? kk.y : 0.0f;
        uint32_t hw, lw;
        split2(in ? vv.x : 0.0f, in ? vv.y : 0.0f, hw, lw);
        *reinterpret_cast<uint32_t *>(vh + d) = hw;
        *reinterpret_cast<uint32_t *>(vl + d) = lw;
      }
    float sq = 0.0f, sk = 0.0f;
#pragma unroll
    for (int x = 0; x < 16; ++x) sq += q[x] * q[x], sk += k[x] * k[x];
    sq += __shfl_xor_sync(0xffffffffu, sq, 1);
    sq += __shfl_xor_sync(0xffffffffu, sq, 2);
    sk += __shfl_xor_sync(0xffffffffu, sk, 1);
    sk += __shfl_xor_sync(0xffffffffu, sk, 2);
    const float rq = 1.0f / sqrtf(sq / 64.0f + 1e-8f), rk = 1.0f / sqrtf(sk / 64.0f + 1e-8f);
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const float2 gq0 = *reinterpret_cast<const float2 *>(a.qn + 16 * kc + 2 * t);
      const float2 gq1 = *reinterpret_cast<const float2 *>(a.qn + 16 * kc + 2 * t + 8);
      const float2 gk0 = *reinterpret_cast<const float2 *>(a.kn + 16 * kc + 2 * t);
      const float2 gk1 = *reinterpret_cast<const float2 *>(a.kn + 16 * kc + 2 * t + 8);
      const float gq[4] = {gq0.x, gq0.y, gq1.x, gq1.y}, gk[4] = {gk0.x, gk0.y, gk1.x, gk1.y};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        q[4 * kc + e] = q[4 * kc + e] * rq * gq[e];
        k[4 * kc + e] = k[4 * kc + e] * rk * gk[e];
      }
      // A fragment (queries): regs 0/2 row g, 1/3 row g + 8; B fragment of key
      // tile hr (keys 8 hr + g): regs 2 hr (dims 2t..) and 2 hr + 1 (dims 2t+8..)
      split2(q[4 * kc], q[4 * kc + 1], qh[kc][hr], ql[kc][hr]);
      split2(q[4 * kc + 2], q[4 * kc + 3], qh[kc][2 + hr], ql[kc][2 + hr]);
      split2(k[4 * kc], k[4 * kc + 1], kh[kc][2 * hr], kl[kc][2 * hr]);
      split2(k[4 * kc + 2], k[4 * kc + 3], kh[kc][2 * hr + 1], kl[kc][2 * hr + 1]);
    }
  }
  if (NT == 1) {  // keys 8-15 enter P.V with P = 0: their v rows must be finite
    __half *vh = vs[h][0] + (g + 8) * 72, *vl = vs[h][1] + (g + 8) * 72;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        *reinterpret_cast<uint32_t *>(vh + 16 * kc + 2 * t + 8 * u) = 0u;
        *reinterpret_cast<uint32_t *>(vl + 16 * kc + 2 * t + 8 * u) = 0u;
      }
  }
  // scores S[query][key], key tiles 0 (keys 0-7) and 1 (keys 8-15)
  float sc[2][4];
#pragma unroll
  for (int nh = 0; nh < 2; ++nh) sc[nh][0] = sc[nh][1] = sc[nh][2] = sc[nh][3] = 0.0f;
#pragma unroll
  for (int kc = 0; kc < 4; ++kc)
#pragma unroll
    for (int nh = 0; nh < NT; ++nh) {
      mma16816(sc[nh][0], sc[nh][1], sc[nh][2], sc[nh][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], kh[kc][2 * nh],
               kh[kc][2 * nh + 1]);
      mma16816(sc[nh][0], sc[nh][1], sc[nh][2], sc[nh][3], qh[kc][0], qh[kc][1], qh[kc][2], qh[kc][3], kl[kc][2 * nh],
               kl[kc][2 * nh + 1]);
      mma16816(sc[nh][0], sc[nh][1], sc[nh][2], sc[nh][3], ql[kc][0], ql[kc][1], ql[kc][2], ql[kc][3], kh[kc][2 * nh],
               kh[kc][2 * nh + 1]);
    }
  // key validity of keys 2t, 2t+1 (+8 nh) comes from the lanes holding those rows
  uint32_t kvalid = 0;
#pragma unroll
  for (int hr = 0; hr < NT; ++hr) kvalid |= (valid[hr] ? 1u : 0u) << (g + 8 * hr);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) kvalid |= __shfl_xor_sync(0xffffffffu, kvalid, o);
  // e = 0,1: query row g, e = 2,3: query row g + 8
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nh = 0; nh < 2; ++nh)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int qrow = g + 8 * (e >> 1), key = 8 * nh + 2 * t + (e & 1);
      const bool qmasked = !((kvalid >> qrow) & 1u);
      float x = -INFINITY;
      if (key < nv) x = qmasked ? -1.0e9f : (((kvalid >> key) & 1u) ? sc[nh][e] * 0.125f : -INFINITY);
      sc[nh][e] = x;
      mx[e >> 1] = fmaxf(mx[e >> 1], x);
    }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
    mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
    if (mx[hr] == -INFINITY) mx[hr] = 0.0f;  // padding query rows (>= nv): all zero
  }
  float sum[2] = {0.0f, 0.0f};
#pragma unroll
  for (int nh = 0; nh < 2; ++nh)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float pe = expf(sc[nh][e] - mx[e >> 1]);
      sc[nh][e] = pe;
      sum[e >> 1] += pe;
    }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    sum[hr] += __shfl_xor_sync(0xffffffffu, sum[hr], 1);
    sum[hr] += __shfl_xor_sync(0xffffffffu, sum[hr], 2);
  }
  // P as the A operand (16 queries x 16 keys), split hi / lo
  uint32_t ph[4], pl[4];
  split2(sc[0][0], sc[0][1], ph[0], pl[0]);
  split2(sc[0][2], sc[0][3], ph[1], pl[1]);
  split2(sc[1][0], sc[1][1], ph[2], pl[2]);
  split2(sc[1][2], sc[1][3], ph[3], pl[3]);
  __syncwarp();  // this warp's v planes are written
  float o[8][4];
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.0f;
  // transposed ldmatrix rows: matrix m -> keys (m % 2) * 8 + (lane % 8), dims (m / 2) * 8
  const int voff = (((lane >> 3) & 1) * 8 + (lane & 7)) * 72 + ((lane >> 4) << 3);
#pragma unroll
  for (int n2 = 0; n2 < 4; ++n2) {
    uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
    ldsm_x4_trans(vs[h][0] + voff + 16 * n2, h0, h1, h2, h3);
    ldsm_x4_trans(vs[h][1] + voff + 16 * n2, l0, l1, l2, l3);
    float *oa = o[2 * n2], *ob = o[2 * n2 + 1];
    mma16816(oa[0], oa[1], oa[2], oa[3], ph[0], ph[1], ph[2], ph[3], h0, h1);
    mma16816(ob[0], ob[1], ob[2], ob[3], ph[0], ph[1], ph[2], ph[3], h2, h3);
    mma16816(oa[0], oa[1], oa[2], oa[3], ph[0], ph[1], ph[2], ph[3], l0, l1);
    mma16816(ob[0], ob[1], ob[2], ob[3], ph[0], ph[1], ph[2], ph[3], l2, l3);
    mma16816(oa[0], oa[1], oa[2], oa[3], pl[0], pl[1], pl[2], pl[3], h0, h1);
    mma16816(ob[0], ob[1], ob[2], ob[3], pl[0], pl[1], pl[2], pl[3], h2, h3);
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int qa = g + 8 * hr;
    if (qa >= nv) continue;
    const float inv = 1.0f / sum[hr];
    const size_t oo = ((size_t)(r0 + qa) * p + patch) * E + h * 64;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      const int d = nd * 8 + 2 * t;
      const float x0 = o[nd][2 * hr] * inv, x1 = o[nd][2 * hr + 1] * inv;
      uint32_t hw, lw;
      split2(x0, x1, hw, lw);
      *reinterpret_cast<uint32_t *>(a.oh + oo + d) = hw;
      *reinterpret_cast<uint32_t *>(a.ol + oo + d) = lw;
      if (a.o32) *reinterpret_cast<float2 *>(a.o32 + oo + d) = make_float2(x0, x1);
    }
  }
}

// Group attention with the series' keys and values held in registers: one
// warp per head loads k and v of all NV (>= the series' row count) variate
// rows at this patch with independent loads, normalises the keys once, then
// answers every query row (same semantics as attn_group_kernel).
template <int NV, int HD>
__global__ void __launch_bounds__(256) attn_group_reg_kernel(AttnArgs a) {
  pdl_launch_dependents();  // the next small-M GEMM may prefetch its weights
  constexpr int DPL = HD / 32;  // dims per lane: lane + 32 c
  const int s = blockIdx.x, patch = blockIdx.y;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (h >= a.H) return;
  const int r0 = a.series_row0[s], nv = a.series_nrows[s];
  const int p = a.p, E = a.E;
  const float qk_scale = 1.0f / sqrtf((float)HD);
  float q[NV][DPL], k[NV][DPL], v[NV][DPL];
  uint32_t kvalid = 0;
#pragma unroll
  for (int b = 0; b < NV; ++b) {
#pragma unroll
    for (int c = 0; c < DPL; ++c) q[b][c] = k[b][c] = v[b][c] = 0.0f;
    if (b < nv) {
      const float *row = a.qkv + ((size_t)(r0 + b) * p + patch) * 3 * E + h * HD;
#pragma unroll
      for (int c = 0; c < DPL; ++c) {
        q[b][c] = row[lane + 32 * c];
        k[b][c] = row[E + lane + 32 * c];
        v[b][c] = row[2 * E + lane + 32 * c];
      }
      if (patch >= a.row_first_valid[r0 + b]) kvalid |= 1u << b;
    }
  }
  float qg[DPL], kg[DPL];
#pragma unroll
  for (int c = 0; c < DPL; ++c) qg[c] = a.qn[lane + 32 * c], kg[c] = a.kn[lane + 32 * c];
#pragma unroll
  for (int b = 0; b < NV; ++b) {
    if (b < nv) {
      float sk = k[b][0] * k[b][0], sq = q[b][0] * q[b][0];
#pragma unroll
      for (int c = 1; c < DPL; ++c) sk += k[b][c] * k[b][c], sq += q[b][c] * q[b][c];
      const float rk = 1.0f / sqrtf(warp_sum(sk) / (float)HD + 1e-8f);
      const float rq = 1.0f / sqrtf(warp_sum(sq) / (float)HD + 1e-8f);
#pragma unroll
      for (int c = 0; c < DPL; ++c) {
        k[b][c] = k[b][c] * rk * kg[c];
        q[b][c] = q[b][c] * rq * qg[c];
      }
    }
  }
#pragma unroll
  for (int qa = 0; qa < NV; ++qa) {
    if (qa >= nv) break;
    const bool qmasked = !((kvalid >> qa) & 1u);  // a row's query and key share its first valid patch
    float sc[NV];
    float mx = -INFINITY;
#pragma unroll
    for (int b = 0; b < NV; ++b) {
      sc[b] = -INFINITY;
      if (b < nv) {
        float dp = q[qa][0] * k[b][0];
#pragma unroll
        for (int c = 1; c < DPL; ++c) dp += q[qa][c] * k[b][c];
        const float d = warp_sum(dp);
        sc[b] = qmasked ? -1.0e9f : (((kvalid >> b) & 1u) ? d * qk_scale : -INFINITY);
        mx = fmaxf(mx, sc[b]);
      }
    }
    float sum = 0.0f, o[DPL];
#pragma unroll
    for (int c = 0; c < DPL; ++c) o[c] = 0.0f;
#pragma unroll
    for (int b = 0; b < NV; ++b) {
      if (b < nv) {
        const float e = expf(sc[b] - mx);
        sum += e;
#pragma unroll
        for (int c = 0; c < DPL; ++c) o[c] = fmaf(e, v[b][c], o[c]);
      }
    }
    const size_t oo = ((size_t)(r0 + qa) * p + patch) * E + h * HD;
#pragma unroll
    for (int c = 0; c < DPL; ++c) {
      const float x = o[c] / sum;
      __half hh, ll;
      split_f16(x, hh, ll);
      a.oh[oo + lane + 32 * c] = hh;
      a.ol[oo + lane + 32 * c] = ll;
      if (a.o32) a.o32[oo + lane + 32 * c] = x;
    }
  }
}


// ============================================================== decoder
// Gather the output-patch tokens of every row and apply out_norm (one warp
// per output token): xo[r*hp + j] = rmsnorm(x[r*p + p-hp-1+j]) * g.
__global__ void dec_gather_kernel(const float *x, const float *g, float *xo, int R, int p, int hp, int E) {
  pdl_launch_dependents();
  pdl_wait();  // x comes from the previous kernel
  const int o = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (o >= R * hp) return;
  const int r = o / hp, j = o % hp;
  const float *xr = x + ((size_t)r * p + (p - hp - 1 + j)) * E;
  float s = 0.0f;
  for (int c = lane; c < E; c += 32) s += xr[c] * xr[c];
#pragma unroll
  for (int k = 16; k; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
  const float dn = sqrtf(s / (float)E + 1e-8f);
  for (int c = lane; c < E; c += 32) xo[(size_t)o * E + c] = xr[c] / dn * g[c];
}

// Quantile head (cumsum of softplus) + inverse scaling + forecast slice.
// dec [R*hp, 32*nq]; out [R, horizon, nq] (rows remapped by out_row).
__global__ void dec_head_kernel(const float *dec, const float *loc, const float *scale, float *out,
                                const int *out_row, int R, int hp, int horizon, int nq, int use_arcsinh) {
  pdl_launch_dependents();
  pdl_wait();  // dec comes from the previous kernel
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;  // (r, step)
  if (idx >= R * hp * 32) return;
  const int r = idx / (hp * 32), step = idx % (hp * 32);
  if (step >= horizon) return;
  const int j = step / 32, k = step % 32;
  const float *src = dec + ((size_t)r * hp + j) * 32 * nq + k * nq;
  const float lo = loc[(size_t)r * hp + j], sc = scale[(size_t)r * hp + j];
  const int orow = out_row ? out_row[r] : r;
  float *dst = out + ((size_t)orow * horizon + step) * nq;
  float running = src[0];
  dst[0] = (use_arcsinh ? sinhf(running) : running) * sc + lo;
  for (int i = 1; i < nq; ++i) {
    running = running + logf(1.0f + expf(src[i]));
    dst[i] = (use_arcsinh ? sinhf(running) : running) * sc + lo;
  }
}

// ============================================================== launchers
cudaError_t t0b_launch_prep(const PrepArgs &a, cudaStream_t st) {
  prep_kernel<<<(a.R + kPrepWarps - 1) / kPrepWarps, 32 * kPrepWarps, 0, st>>>(a);
  return cudaGetLastError();
}
template <int MT>
static cudaError_t launch_sgemm_small(const SgemmArgs &a, cudaStream_t st) {
  const size_t smem = std::max((size_t)(MT + 32) * (a.K + 4), (size_t)kSgemmSmallWarps * MT * 32) * sizeof(float);
  cudaError_t e = t0b_smem_limit((const void *)sgemm_small_kernel<MT>, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.N + 31) / 32, (a.M + MT - 1) / MT);
  return launch_pdl(sgemm_small_kernel<MT>, grid, dim3(32 * kSgemmSmallWarps), smem, st, a);
}

cudaError_t t0b_launch_sgemm(const SgemmArgs &a, cudaStream_t st) {
  // few rows: the staged small-M kernel (whole K in shared memory)
  const bool aligned = ((uintptr_t)a.A % 16 == 0) && ((uintptr_t)a.B % 16 == 0) && a.lda % 4 == 0 && a.ldb % 4 == 0;
  if (a.M > 0 && a.M <= 64 && a.K % 32 == 0 && (size_t)64 * (a.K + 4) * sizeof(float) <= 200 * 1024 && aligned) {
    if (a.M <= 8) return launch_sgemm_small<8>(a, st);
    if (a.M <= 16) return launch_sgemm_small<16>(a, st);
    return launch_sgemm_small<32>(a, st);
  }
  // many rows with f16-exact weights: tensor cores
  const bool h_ok = a.B16 && a.K % kSgH_BK == 0 && ((uintptr_t)a.B16 % 16 == 0) && a.ldb % 8 == 0;
  if (h_ok && aligned) {
    const size_t smem = 2 * kSgH_Stage;
    cudaError_t e = t0b_smem_limit((const void *)sgemm_h_kernel, smem);
    if (e != cudaSuccess) return e;
    sgemm_h_kernel<<<dim3((a.N + kSgH_BN - 1) / kSgH_BN, (a.M + kSgH_BM - 1) / kSgH_BM), 256, smem, st>>>(a);
    return cudaGetLastError();
  }
  dim3 grid((a.N + 63) / 64, (a.M + 63) / 64);
  sgemm_nt_kernel<<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t t0b_launch_rownorm_split(const float *x, const float *g, __half *xh, __half *xl, float *ssq, int M, int E,
                                     cudaStream_t st) {
  if (E % 4) return cudaErrorInvalidValue;
  return launch_pdl(rownorm_split_kernel, dim3((M + 7) / 8), dim3(256), 0, st, x, g, xh, xl, ssq, M, E);
}
cudaError_t t0b_launch_attn_time(const AttnArgs &a, cudaStream_t st) {
  if (a.E / a.H == 128) {
    if (a.p > kAttnWideMaxP) return cudaErrorInvalidValue;
    const int QB = (a.p + 15) / 16, PK = 16 * QB;
    const unsigned nthr = 32 * (QB < 8 ? QB : 8);
    if (a.p <= kAttnWideOnePassMaxP) {
      const size_t smem = (size_t)(4 * PK * (128 + 8)) * sizeof(__half);
      cudaError_t e = t0b_smem_limit((const void *)attn_time_wide_kernel<128, 1>, smem);
      if (e != cudaSuccess) return e;
      attn_time_wide_kernel<128, 1><<<dim3(a.R, a.H), nthr, smem, st>>>(a);
    } else {
      const size_t smem = (size_t)(2 * PK * (128 + 8) + 2 * PK * (64 + 8)) * sizeof(__half);
      cudaError_t e = t0b_smem_limit((const void *)attn_time_wide_kernel<128, 2>, smem);
      if (e != cudaSuccess) return e;
      attn_time_wide_kernel<128, 2><<<dim3(a.R, a.H), nthr, smem, st>>>(a);
    }
    return cudaGetLastError();
  }
  if (a.E / a.H != 64) return cudaErrorInvalidValue;
  if (a.p <= kAttnMmaMaxP) {
    const int QB = (a.p + 15) / 16, PK = 16 * QB;
    const size_t smem = attn_smem_bytes(PK) + 1024;  // planes, q tile, mbarrier, alignment slack
    cudaError_t e = t0b_smem_limit((const void *)attn_time_mma_kernel, smem);
    if (e != cudaSuccess) return e;
    // k / v tiles by TMA: a [p][64] f32 box of the [R p][3E] q|k|v tensor
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    CUtensorMap toh, tol;  // output planes as [R][p][E] f16, 64 x 16 x 1 boxes
    std::memset(&toh, 0, sizeof(toh));
    std::memset(&tol, 0, sizeof(tol));
    const uint64_t rs = (uint64_t)a.E * 2, ss = rs * (uint64_t)a.p;
    const bool out_ok =
        t0b_make_tmap_f16_3d(&toh, a.oh, (uint64_t)a.E, (uint64_t)a.p, (uint64_t)a.R, rs, ss, 64, 16, 1, true) &&
        t0b_make_tmap_f16_3d(&tol, a.ol, (uint64_t)a.E, (uint64_t)a.p, (uint64_t)a.R, rs, ss, 64, 16, 1, true);
    const int use_tma = t0b_make_tmap_f32_2d(&tm, a.qkv, (uint64_t)3 * a.E, (uint64_t)a.R * a.p,
                                             (uint64_t)3 * a.E * sizeof(float), 32, (uint32_t)a.p, true) ? 1 : 0;
    return launch_pdl(attn_time_mma_kernel, dim3(a.R, a.H), dim3(32 * QB), smem, st, a, tm, toh, tol,
                      use_tma | (use_tma && out_ok ? 2 : 0));
  }
  size_t smem = (size_t)(a.p * (65 + 64 + 64) + 4 * a.p) * sizeof(float);
  cudaError_t e = t0b_smem_limit((const void *)attn_time_kernel, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.R, a.H);
  attn_time_kernel<<<grid, 128, smem, st>>>(a);
  return cudaGetLastError();
}
template <int HD>
static cudaError_t launch_attn_group_hd(const AttnArgs &a, cudaStream_t st) {
  dim3 grid(a.n_series, a.p);
  if (HD == 64 && a.max_nrows <= 8 && a.H <= 8)
    attn_group_mma_kernel<1><<<grid, 32 * a.H, 0, st>>>(a);
  else if (HD == 64 && a.max_nrows <= 16 && a.H <= 8)
    attn_group_mma_kernel<2><<<grid, 32 * a.H, 0, st>>>(a);
  else if (a.max_nrows <= 8)
    attn_group_reg_kernel<8, HD><<<grid, 32 * a.H, 0, st>>>(a);
  else if (a.max_nrows <= 16)
    attn_group_reg_kernel<16, HD><<<grid, 32 * a.H, 0, st>>>(a);
  else
    attn_group_kernel<HD><<<grid, 32 * a.H, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t t0b_launch_attn_group(const AttnArgs &a, cudaStream_t st) {
  if (a.E / a.H == 128) return launch_attn_group_hd<128>(a, st);
  if (a.E / a.H == 64) return launch_attn_group_hd<64>(a, st);
  return cudaErrorInvalidValue;
}
cudaError_t t0b_launch_dec_gather(const float *x, const float *g, float *xo, int R, int p, int hp, int E,
                                  cudaStream_t st) {
  int n = R * hp;
  return launch_pdl(dec_gather_kernel, dim3((n + 7) / 8), dim3(256), 0, st, x, g, xo, R, p, hp, E);
}
cudaError_t t0b_launch_dec_head(const float *dec, const float *loc, const float *scale, float *out, const int *out_row,
                                int R, int hp, int horizon, int nq, int use_arcsinh, cudaStream_t st) {
  int n = R * hp * 32;
  return launch_pdl(dec_head_kernel, dim3((n + 255) / 256), dim3(256), 0, st, dec, loc, scale, out, out_row, R, hp,
                    horizon, nq, use_arcsinh);
}

// ============================================================== split
// x -> (hi, lo) f16 planes.  Launched as a programmatic dependent: it lets
// the next kernel (a small-M GEMM prefetching its weights) start at once,
// and touches memory only after the previous kernel has completed.
__global__ void split_f32_kernel(const float *x, __half *h, __half *l, size_t n) {
  pdl_launch_dependents();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    __half a, b;
    split_f16(x[i], a, b);
    h[i] = a;
    l[i] = b;
  }
}
cudaError_t t0b_launch_split_f32(const float *x, __half *xh, __half *xl, size_t n, cudaStream_t st) {
  size_t blocks = std::min<size_t>((n + 255) / 256, 148 * 16);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)std::max<size_t>(blocks, 1));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, split_f32_kernel, x, xh, xl, n);
}

// ============================================================== bounded-wait self-test
// One warp initialises an mbarrier with an expected count of one and waits
// on its first phase with the same bounded wait every pipeline kernel uses
// (mbar_wait).  Nothing ever arrives, so the wait runs out after
// T0B_WAIT_CYCLES, records T0B_DEVERR_WAIT_X in the error word and returns
// false; the kernel then exits normally.  No TMA, tensor memory, cluster or
// other asynchronous work is started, so nothing is left in flight.
__global__ void bounded_wait_selftest_kernel(int *err, int *outcome) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  bool got = true;
  if (threadIdx.x == 0) got = mbar_wait(&bar, 0, err, T0B_DEVERR_WAIT_X, nullptr);
  got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
  if (threadIdx.x == 0) *outcome = got ? 1 : 2;  // 2: the wait ran out and returned
}
cudaError_t t0b_launch_bounded_wait_selftest(int *err, int *outcome, cudaStream_t st) {
  bounded_wait_selftest_kernel<<<1, 32, 0, st>>>(err, outcome);
  return cudaGetLastError();
}
