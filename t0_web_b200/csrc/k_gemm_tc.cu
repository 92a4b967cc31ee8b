// k_gemm_tc.cu -- large-token-count dequant GEMM on the 5th-generation tensor
// cores (tcgen05), raw Q8_0 / Q4_0 weight blocks resident in HBM.
//
// Y[M, N] = A[M, K] . deq(W)[N, K]^T with f32-class accuracy from f16 MMAs:
//   A = Ah + Al (two f16 terms, written by the producing kernel) and
//   W = Wh + Wl (two f16 terms from the exact product d * q, made here);
//   D = Ah.Wh + Ah.Wl + Al.Wh accumulated in f32 in tensor memory (the
//   dropped Al.Wl term is ~2^-22 relative).  Single-term f16 or bf16 MMAs
//   miss the 1e-3 quantile tolerance on t0-alpha-shaped models.
//
// CTA tile 128 tokens x 256 weight rows, 64 K-values per pipeline stage,
// two stages.  Warp roles (192 threads):
//   warp 0      TMA producer: Ah/Al tiles (128x64 f16, 128-byte swizzle) and
//               the raw blocks of the 256 weight rows (one 32-value block
//               column per load, 16-byte aligned superset of the 34/18-byte
//               block), both with mbarrier completion.
//   warp 1      allocates 256 TMEM columns; lane 0 issues tcgen05.mma and
//               tcgen05.commit.
//   warps 2-5   dequantize raw blocks -> Wh/Wl tiles in the canonical K-major
//               SW128 layout (generic stores + proxy fence), then run the
//               fused epilogue from TMEM (tcgen05.ld, one token row per
//               thread).
#include <cuda.h>

#include "common.cuh"
#include "epilogue.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 2;
constexpr uint32_t X_TILE = BM * BK * 2;  // 16 KB
constexpr uint32_t W_TILE = BN * BK * 2;  // 32 KB
constexpr uint32_t OFF_XH = 0;
constexpr uint32_t OFF_XL = OFF_XH + STAGES * X_TILE;
constexpr uint32_t OFF_WH = OFF_XL + STAGES * X_TILE;
constexpr uint32_t OFF_WL = OFF_WH + STAGES * W_TILE;
constexpr uint32_t OFF_RAW = OFF_WL + STAGES * W_TILE;  // 192 KB

template <int QT>
struct TQ;
template <>
struct TQ<8> {
  static constexpr int bpb = 34, rawb = 48;  // 34-byte block inside a 48-byte aligned window
};
template <>
struct TQ<4> {
  static constexpr int bpb = 18, rawb = 32;
};

template <int QT>
__host__ __device__ constexpr uint32_t raw_slot_bytes() {
  return (uint32_t)TQ<QT>::rawb * BN;
}
template <int QT>
__host__ __device__ constexpr uint32_t smem_bytes() {
  return OFF_RAW + 2 * raw_slot_bytes<QT>() + 256 /* barriers */ + 1024 /* alignment slack */;
}

struct TcParams {
  int M, N, K;
  // power-of-two weight prescale: W is split as (2^s d q) = Wh + Wl so that Wl
  // stays a normal f16; the accumulator is multiplied by 2^-s (both exact)
  float wscale, acc_scale;
  int swiglu_F;  // >0: SWIGLU tile = 128 gate rows + 128 up rows
  Epi epi;
  int *err;
};

// 32 columns of (main + correction) accumulator for this thread's row.
T0B_DEV void tmem_ld_pair(uint32_t taddr, float *v) {
  float c[32];
  tmem_ld32(taddr, v);
  tmem_ld32(taddr + BN, c);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] += c[i];
}

template <int QT>
__global__ void __launch_bounds__(192, 1)
    gemm_q_tc_kernel(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
                     const __grid_constant__ CUtensorMap tm_w, TcParams prm) {
  constexpr int BPB = TQ<QT>::bpb, RAWB = TQ<QT>::rawb;
  constexpr uint32_t RAW_SLOT = raw_slot_bytes<QT>();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base_u32 - smem_u32(smem_raw));

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_RAW + 2 * RAW_SLOT);
  uint64_t *x_full = bars + 0;     // [2]
  uint64_t *raw_full = bars + 2;   // [2]
  uint64_t *raw_empty = bars + 4;  // [2]
  uint64_t *w_full = bars + 6;     // [2]
  uint64_t *empty = bars + 8;      // [2] MMA released stage
  uint64_t *acc_full = bars + 10;  // [1]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 11);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = prm.M, K = prm.K;
  const int S = K / BK;
  const int m0 = blockIdx.y * BM;
  // weight rows of the two 128-row halves of this tile
  int wr0, wr1;
  if (prm.swiglu_F > 0) {
    wr0 = blockIdx.x * 128;
    wr1 = prm.swiglu_F + blockIdx.x * 128;
  } else {
    wr0 = blockIdx.x * BN;
    wr1 = wr0 + 128;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 128);
      mbar_init(&w_full[i], 128);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_xh);
    prefetch_tmap(&tm_xl);
    prefetch_tmap(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);  // main accumulator + correction accumulator
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int s = 0; s < S && !*abort_flag; ++s) {
        // raw weight blocks of this stage: block columns 2s, 2s+1 -> slots 0, 1
        for (int h = 0; h < 2; ++h) {
          if (s >= 1 && !mbar_wait(&raw_empty[h], (s - 1) & 1, prm.err, T0B_DEVERR_WAIT_EMPTY, abort_flag)) break;
          int j = 2 * s + h;
          int x = (j * BPB) & ~15;
          mbar_arrive_expect_tx(&raw_full[h], RAW_SLOT);
          uint8_t *dst = smem + OFF_RAW + h * RAW_SLOT;
          tma_load_2d(dst, &tm_w, &raw_full[h], x, wr0);
          tma_load_2d(dst + RAWB * 128, &tm_w, &raw_full[h], x, wr1);
        }
        const int xs = s & 1;
        if (s >= 2 && !mbar_wait(&empty[xs], ((s >> 1) - 1) & 1, prm.err, T0B_DEVERR_WAIT_EMPTY, abort_flag))
          break;
        mbar_arrive_expect_tx(&x_full[xs], 2 * X_TILE);
        tma_load_2d(smem + OFF_XH + xs * X_TILE, &tm_xh, &x_full[xs], s * BK, m0);
        tma_load_2d(smem + OFF_XL + xs * X_TILE, &tm_xl, &x_full[xs], s * BK, m0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
      bool ok = true;
      for (int s = 0; s < S; ++s) {
        const int xs = s & 1;
        if (!mbar_wait(&x_full[xs], (s >> 1) & 1, prm.err, T0B_DEVERR_WAIT_X, abort_flag) ||
            !mbar_wait(&w_full[xs], (s >> 1) & 1, prm.err, T0B_DEVERR_WAIT_DEQ, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t xh = base_u32 + OFF_XH + xs * X_TILE, xl = base_u32 + OFF_XL + xs * X_TILE;
        const uint32_t wh = base_u32 + OFF_WH + xs * W_TILE, wl = base_u32 + OFF_WL + xs * W_TILE;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint32_t ko = kk * 32;  // 16 f16 along K inside the 128-byte swizzled row
          const uint32_t acc = (s > 0 || kk > 0) ? 1u : 0u;
          // main term and the two ~2^-11 correction terms go to separate
          // accumulators: the tensor core's f32 accumulation error grows with
          // the number of MMAs chained into one accumulator
          umma_f16(tmem, sw128_desc(xh + ko), sw128_desc(wh + ko), idesc, acc);
          umma_f16(tmem + BN, sw128_desc(xh + ko), sw128_desc(wl + ko), idesc, acc);
          umma_f16(tmem + BN, sw128_desc(xl + ko), sw128_desc(wh + ko), idesc, 1u);
        }
        umma_commit(&empty[xs]);
      }
      umma_commit(acc_full);  // also fires after an abort, once issued MMAs drain
      (void)ok;
    }
  } else {
    // ------------------------------------------------------------ dequant
    const int t = threadIdx.x - 64;  // 0..127
    for (int s = 0; s < S && !*abort_flag; ++s) {
      const int ws = s & 1;
      if (s >= 2 && !mbar_wait(&empty[ws], ((s >> 1) - 1) & 1, prm.err, T0B_DEVERR_WAIT_EMPTY, abort_flag)) break;
      uint8_t *whs = smem + OFF_WH + ws * W_TILE;
      uint8_t *wls = smem + OFF_WL + ws * W_TILE;
      bool ok = true;
      for (int h = 0; h < 2; ++h) {
        if (!mbar_wait(&raw_full[h], s & 1, prm.err, T0B_DEVERR_WAIT_W, abort_flag)) {
          ok = false;
          break;
        }
        const int j = 2 * s + h;
        const int off = (j * BPB) & 15;  // block start inside the aligned window
        const uint8_t *slot = smem + OFF_RAW + h * RAW_SLOT;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int r = t + 128 * rr;  // tile row 0..255
          const uint32_t *src = reinterpret_cast<const uint32_t *>(slot + r * RAWB);
          uint32_t wv[RAWB / 4 + 1];
#pragma unroll
          for (int i = 0; i < RAWB / 16; ++i) {
            uint4 q4 = reinterpret_cast<const uint4 *>(src)[i];
            wv[4 * i] = q4.x;
            wv[4 * i + 1] = q4.y;
            wv[4 * i + 2] = q4.z;
            wv[4 * i + 3] = q4.w;
          }
          wv[RAWB / 4] = 0u;
          auto word_at = [&](int byte) -> uint32_t {  // 4 bytes starting at `byte`
            int w = byte >> 2, sh = (byte & 3) * 8;
            return sh ? __funnelshift_r(wv[w], wv[w + 1], sh) : wv[w];
          };
          const uint32_t dbits = word_at(off) & 0xFFFFu;
          const __half dh =
              __float2half_rn(__half2float(__ushort_as_half((unsigned short)dbits)) * prm.wscale);  // exact
          const __half2 d2 = __halves2half2(dh, dh);
          // 32 values of this block -> 4 chunks of 8 f16 at k = 32h + 8c
          uint32_t hv[16], lv[16];
          if (QT == 8) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              uint32_t q = word_at(off + 2 + 4 * i);  // 4 int8 values
              uint32_t qa = i8x2_to_h2(q & 0xFFFFu), qb = i8x2_to_h2(q >> 16);
              __half2 ha = __hmul2(d2, *reinterpret_cast<__half2 *>(&qa));
              __half2 hb = __hmul2(d2, *reinterpret_cast<__half2 *>(&qb));
              __half2 la = __hfma2(d2, *reinterpret_cast<__half2 *>(&qa), __hneg2(ha));
              __half2 lb = __hfma2(d2, *reinterpret_cast<__half2 *>(&qb), __hneg2(hb));
              hv[2 * i] = *reinterpret_cast<uint32_t *>(&ha);
              hv[2 * i + 1] = *reinterpret_cast<uint32_t *>(&hb);
              lv[2 * i] = *reinterpret_cast<uint32_t *>(&la);
              lv[2 * i + 1] = *reinterpret_cast<uint32_t *>(&lb);
            }
          } else {
            // bytes b0..b15: low nibble = value b, high nibble = value b+16
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t q = word_at(off + 2 + 4 * i);  // bytes 4i..4i+3
#pragma unroll
              for (int hi = 0; hi < 2; ++hi) {
                uint32_t qa = nib2_to_h2(q & 0xFFFFu, hi), qb = nib2_to_h2(q >> 16, hi);
                __half2 ha = __hmul2(d2, *reinterpret_cast<__half2 *>(&qa));
                __half2 hb = __hmul2(d2, *reinterpret_cast<__half2 *>(&qb));
                __half2 la = __hfma2(d2, *reinterpret_cast<__half2 *>(&qa), __hneg2(ha));
                __half2 lb = __hfma2(d2, *reinterpret_cast<__half2 *>(&qb), __hneg2(hb));
                const int v0 = 16 * hi + 4 * i;  // value index of qa.x
                hv[v0 / 2] = *reinterpret_cast<uint32_t *>(&ha);
                hv[v0 / 2 + 1] = *reinterpret_cast<uint32_t *>(&hb);
                lv[v0 / 2] = *reinterpret_cast<uint32_t *>(&la);
                lv[v0 / 2 + 1] = *reinterpret_cast<uint32_t *>(&lb);
              }
            }
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t o = sw128_offset(r, 32 * h + 8 * c);
            *reinterpret_cast<uint4 *>(whs + o) = make_uint4(hv[4 * c], hv[4 * c + 1], hv[4 * c + 2], hv[4 * c + 3]);
            *reinterpret_cast<uint4 *>(wls + o) = make_uint4(lv[4 * c], lv[4 * c + 1], lv[4 * c + 2], lv[4 * c + 3]);
          }
        }
        mbar_arrive(&raw_empty[h]);
      }
      if (!ok) break;
      fence_proxy_async_smem();
      mbar_arrive(&w_full[ws]);
    }

    // ------------------------------------------------------------ epilogue
    const bool have = mbar_wait(acc_full, 0, prm.err, T0B_DEVERR_WAIT_ACC, abort_flag) && !*abort_flag;
    tc_fence_after();
    if (have) {
      const int q = warp & 3;  // TMEM lane quadrant this warp may access
      const int m = m0 + 32 * q + lane;
      const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
      const Epi &e = prm.epi;
      const bool live = m < M;
      const float denom = live ? epi_row_denom(e, m) : 1.0f;
      if (e.kind == EPI_QKV) {
        for (int hh = 0; hh < 4; ++hh) {
          float v[64];
          tmem_ld_pair(trow + 64 * hh, v);
          tmem_ld_pair(trow + 64 * hh + 32, v + 32);
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] *= prm.acc_scale;
          if (live) epi_qkv64(e, m, blockIdx.x * BN + 64 * hh, v, denom);
        }
      } else if (e.kind == EPI_SWIGLU) {
        for (int c = 0; c < 4; ++c) {
          float gv[32], uv[32];
          tmem_ld_pair(trow + 32 * c, gv);
          tmem_ld_pair(trow + 128 + 32 * c, uv);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            gv[i] *= prm.acc_scale;
            uv[i] *= prm.acc_scale;
          }
          if (live) epi_swiglu32(e, m, blockIdx.x * 128 + 32 * c, gv, uv, denom);
        }
      } else {
        float ss = 0.0f;
        for (int c = 0; c < 8; ++c) {
          float v[32];
          tmem_ld_pair(trow + 32 * c, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= prm.acc_scale;
          if (live) ss += epi_cols32(e, m, blockIdx.x * BN + 32 * c, v, denom);
        }
        if (live && e.kind == EPI_RESID) e.ssq_out[(size_t)m * e.ssq_out_nt + blockIdx.x] = ss;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, int esize, const void *ptr, uint64_t inner,
                  uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  (void)esize;
  CUresult r = fn(tm, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int QT>
cudaError_t launch_tc_t(const __half *ah, const __half *al, int M, int K, const uint8_t *W, int wrows, int wshift,
                        const Epi &epi, int *err, cudaStream_t st) {
  CUtensorMap txh, txl, tw;
  const uint64_t rb = (uint64_t)(K / 32) * TQ<QT>::bpb;
  if (!make_tmap_2d(&txh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ah, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&txl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, al, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W, rb, (uint64_t)wrows, rb, TQ<QT>::rawb, 128,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  TcParams prm;
  prm.M = M;
  prm.N = epi.N;
  prm.K = K;
  prm.swiglu_F = epi.kind == EPI_SWIGLU ? epi.F : 0;
  prm.wscale = ldexpf(1.0f, wshift);
  prm.acc_scale = ldexpf(1.0f, -wshift);
  prm.epi = epi;
  prm.err = err;
  constexpr uint32_t smem = smem_bytes<QT>();
  auto kfn = gemm_q_tc_kernel<QT>;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(epi.kind == EPI_SWIGLU ? epi.F / 128 : epi.N / BN, (M + BM - 1) / BM);
  kfn<<<grid, 192, smem, st>>>(txh, txl, tw, prm);
  return cudaGetLastError();
}

}  // namespace

// Host entry.  qt: 8 = Q8_0, 4 = Q4_0.  Requires K % 256 == 0, N % 256 == 0
// (SWIGLU: F % 128 == 0), M >= 1, 16-byte aligned A rows.  `wrows` is the
// number of rows of W (N, or 2F for SWIGLU); `wshift` the weight prescale
// exponent from t0b_weight_shift.
cudaError_t t0b_launch_gemm_tc(int qt, const __half *ah, const __half *al, int M, int K, const uint8_t *W, int wrows,
                               int wshift, const Epi &epi, int *err, cudaStream_t st) {
  if (qt == 8) return launch_tc_t<8>(ah, al, M, K, W, wrows, wshift, epi, err, st);
  return launch_tc_t<4>(ah, al, M, K, W, wrows, wshift, epi, err, st);
}

// Largest |scale| of a Q8_0 / Q4_0 matrix (device), as the f32 bit pattern of
// a non-negative float (so an integer max is a float max).
__global__ void absmax_scale_kernel(const uint8_t *W, size_t nblocks, int bpb, unsigned int *out) {
  unsigned int mx = 0;
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
    const uint16_t bits = (uint16_t)(W[b * bpb] | (W[b * bpb + 1] << 8));
    mx = max(mx, __float_as_uint(fabsf(__half2float(__ushort_as_half(bits)))));
  }
  for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, mx);
}

cudaError_t t0b_launch_absmax_scale(const uint8_t *W, size_t nblocks, int bpb, unsigned int *out, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return e;
  absmax_scale_kernel<<<148, 256, 0, st>>>(W, nblocks, bpb, out);
  return cudaGetLastError();
}
