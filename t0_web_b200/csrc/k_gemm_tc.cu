// k_gemm_tc.cu -- large-token-count dequant GEMM on the 5th-generation tensor
// cores (tcgen05), raw Q8_0 / Q4_0 weight blocks resident in HBM.
//
// Y[M, N] = A[M, K] . deq(W)[N, K]^T with f32-class accuracy from f16 MMAs:
//   A = Ah + Al (two f16 terms, written by the producing kernel) and
//   W = Wh + Wl (two f16 terms from the exact product 2^s d q, made here);
//   D = Ah.Wh (main accumulator) + [Ah.Wl + Al.Wh] (correction accumulator),
//   both f32 in tensor memory.  The dropped Al.Wl term is ~2^-22 relative.
//   Single-term f16 or bf16 MMAs miss the 1e-3 quantile tolerance on
//   t0-alpha-shaped models, and chaining all three terms into one
//   accumulator triples the tensor core's accumulation error.
//
// Persistent kernel on CTA pairs (cta_group::2): each 2-CTA cluster (the
// two SMs of a TPC) walks a queue of 256-token x 256-column output tiles
// (weight-row tiles fastest so the pairs in flight share their activation
// tiles in L2).  CTA r of a pair holds tokens 128 r .. 128 r + 127 of the
// tile and half of its weight rows; one M = 256 MMA issued by CTA 0 reads
// both CTAs' operand tiles and leaves each CTA's 128 rows x 256 columns in
// its own TMEM.  One 32-value block column of K per pipeline stage, with
// rings for the activation tiles (TMA, 64-byte swizzle), the raw weight
// blocks (TMA) and the dequantized weight tiles.  The main and correction
// accumulators fill all 512 TMEM columns; the epilogue reads them chunk by
// chunk and releases TMEM to the next tile's MMAs after its last load
// (PLAIN: two 16-column chunks are loaded before the first is stored;
// SWIGLU: both chunks are computed before either is stored).  Its
// only global load is the row's RMSNorm sum of squares, fetched before the
// accumulator is ready (the bias is staged in shared memory); its global
// writes are asynchronous TMA stores (or TMA reduce-adds into the residual
// stream) of swizzled 32-row chunks.  QK-norm and RoPE run in the attention
// kernels.
//
// Why pairs: a single CTA per 128 x 256 tile moves ~144 KB through shared
// memory per K stage (72 KB of it the three MMA terms' operand reads)
// against 768 MMA cycles and measured exactly shared-memory bound; with the
// weight half-tiles split across the pair it is ~92 KB per CTA.
//
// Warp roles (896 threads per CTA, both CTAs unless noted):
//   warp 0      TMA producer of the Ah/Al tiles (byte counts of both CTAs
//               land on CTA 0's barrier).
//   warp 1      allocates the pair's 512 TMEM columns; in CTA 0 lane 0
//               issues tcgen05.mma and the commits.
//   warp 2      TMA producer of the raw blocks of this CTA's weight rows
//               (16-byte aligned superset window of the 34/18-byte block).
//   warps 4-11  dequantize raw blocks (one weight row per thread per stage,
//               two groups of four warps taking alternate stages) -> Wh/Wl
//               tiles in the canonical K-major SW64 layout (generic stores +
//               proxy fence).
//   warps 12-27 epilogue, four warps per TMEM lane quadrant (64 columns
//               each): bias + RMSNorm row scale (PLAIN) or SwiGLU, staged
//               in shared memory and written by TMA.
#include <cuda.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "epilogue.cuh"
#include "t0b_internal.h"

namespace {

constexpr int BM = 128, BN = 256, BK = 32;  // per CTA: 128 tokens; per pair: 256 columns; BK: one block column
constexpr int NTHREADS = 896;
constexpr int EPI_WARPS = 16;  // warps 12-27, four per TMEM lane quadrant
constexpr uint32_t X_TILE = BM * BK * 2;  // 8 KB, one of hi / lo
constexpr uint32_t STG_BYTES = 2048;      // per epilogue warp and buffer: one 32-row output chunk

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

struct TcParams {
  int M, N, K;
  int swiglu_F;  // > 0: a tile is 128 gate rows + the matching 128 up rows
  int n_tiles_n, n_tiles;
  // split-K (PLAIN only): each (m, n) tile is k_split work items over
  // consecutive K ranges whose partial tiles the epilogue reduce-adds into a
  // zeroed y; only the first split adds the bias
  int k_split;
  // power-of-two weight prescale: W is split as (2^s d q) = Wh + Wl so that Wl
  // stays a normal f16; the accumulator is multiplied by 2^-s (both exact)
  float wscale, acc_scale;
  Epi epi;
  int *err;
};

T0B_DEV void store_f32x16(float *dst, const float *v) {
  float4 *d = reinterpret_cast<float4 *>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// Dequantize one 32-value block of one weight row (raw window `src`, block
// starting OFF bytes in) into tile row r of the Wh / Wl tiles:
// hi = f16(2^s d q), lo = f16(2^s d q - hi), in the canonical K-major SW64
// layout (16-byte unit c of row r at sw64_offset(r, 8c)).  OFF is a
// compile-time constant (the block start inside the 16-byte aligned window
// is 34 s mod 16 or 18 s mod 16, always even), so every word index and shift
// is static and the window stays in registers; each 16-byte unit is stored
// as soon as its 8 values are made, which keeps the dequant warps within
// their register share.
template <int QT, int OFF>
T0B_DEV void dequant_row(const uint8_t *src, float wscale, uint8_t *whs, uint8_t *wls, int r) {
  constexpr int RAWB = TQ<QT>::rawb;
  constexpr int NW = QT == 8 ? 8 : 4;  // 32-bit words of quants in a block
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
  const uint32_t dbits = (wv[OFF >> 2] >> ((OFF & 3) * 8)) & 0xFFFFu;
  constexpr int QB = OFF + 2, W0 = QB >> 2, SH = (QB & 3) * 8;
  static_assert(W0 + NW < RAWB / 4 + 1, "block overruns the raw window");
  auto word_q = [&](int i) -> uint32_t {  // quant bytes 4i..4i+3
    return SH ? __funnelshift_r(wv[W0 + i], wv[W0 + i + 1], SH) : wv[W0 + i];
  };
  const __half dh = __float2half_rn(__half2float(__ushort_as_half((unsigned short)dbits)) * wscale);  // exact
  const __half2 d2 = __halves2half2(dh, dh);
  auto emit = [&](uint32_t qv, uint32_t &hv, uint32_t &lv) {
    __half2 h = __hmul2(d2, *reinterpret_cast<__half2 *>(&qv));
    __half2 l = __hfma2(d2, *reinterpret_cast<__half2 *>(&qv), __hneg2(h));  // exact residual, rounded once
    hv = *reinterpret_cast<uint32_t *>(&h);
    lv = *reinterpret_cast<uint32_t *>(&l);
  };
  auto put = [&](int c, const uint32_t *hv, const uint32_t *lv) {  // 16-byte unit c = values 8c .. 8c + 7
    const uint32_t o = sw64_offset(r, 8 * c);
    *reinterpret_cast<uint4 *>(whs + o) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    *reinterpret_cast<uint4 *>(wls + o) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
  };
  if (QT == 8) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t hv[4], lv[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t a, b;
        i8x4_to_h2x2(word_q(2 * c + j), a, b);  // int8 values 8c + 4j .. 8c + 4j + 3
        emit(a, hv[2 * j], lv[2 * j]);
        emit(b, hv[2 * j + 1], lv[2 * j + 1]);
      }
      put(c, hv, lv);
    }
  } else {
    // byte b holds value b (low nibble) and value b+16 (high nibble): words
    // 2 hf and 2 hf + 1 make units hf (values 8 hf ..) and 2 + hf (16 + 8 hf ..)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      uint32_t h0[4], l0[4], h1[4], l1[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t rr[4];
        nib8_to_h2x4(word_q(2 * hf + j), rr);
        emit(rr[0], h0[2 * j], l0[2 * j]);          // values 8hf + 4j, +1
        emit(rr[1], h0[2 * j + 1], l0[2 * j + 1]);  // values 8hf + 4j + 2, +3
        emit(rr[2], h1[2 * j], l1[2 * j]);          // values 16 + 8hf + 4j, +1
        emit(rr[3], h1[2 * j + 1], l1[2 * j + 1]);  // values 16 + 8hf + 4j + 2, +3
      }
      put(hf, h0, l0);
      put(2 + hf, h1, l1);
    }
  }
}

template <int QT>
T0B_DEV void dequant_row_at(int off, const uint8_t *src, float wscale, uint8_t *whs, uint8_t *wls, int r) {
  switch (off) {  // uniform across the CTA: the stage's block offset
    case 0: dequant_row<QT, 0>(src, wscale, whs, wls, r); break;
    case 2: dequant_row<QT, 2>(src, wscale, whs, wls, r); break;
    case 4: dequant_row<QT, 4>(src, wscale, whs, wls, r); break;
    case 6: dequant_row<QT, 6>(src, wscale, whs, wls, r); break;
    case 8: dequant_row<QT, 8>(src, wscale, whs, wls, r); break;
    case 10: dequant_row<QT, 10>(src, wscale, whs, wls, r); break;
    case 12: dequant_row<QT, 12>(src, wscale, whs, wls, r); break;
    default: dequant_row<QT, 14>(src, wscale, whs, wls, r); break;
  }
}

T0B_DEV void epi_bar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }  // the 16 epilogue warps only

// ---------------------------------------------------------------- the kernel
// Barriers that the peer CTA feeds live in CTA 0: the activation-full
// barrier (TMA byte counts of both CTAs), the dequantized-full barrier and
// the accumulator-empty barrier.  CTA 0's MMA thread signals the
// stage-empty and accumulator-full barriers of both CTAs with one commit
// each.  Ring depths and staging buffers per epilogue warp can be set at
// compile time (defaults measured best; deeper rings did not help).
#ifndef T0B_PXS
#define T0B_PXS 4
#endif
#ifndef T0B_PWS
#define T0B_PWS 4
#endif
#ifndef T0B_PRS
#define T0B_PRS 4
#endif
#ifndef T0B_STG_N
#define T0B_STG_N 2
#endif
constexpr int PXS = T0B_PXS, PWS = T0B_PWS, PRS = T0B_PRS;  // ring depths per CTA
constexpr int STG_N = T0B_STG_N;                             // staging buffers per epilogue warp
// The activation and dequantized-weight slots of a stage are freed together
// by one commit per stage on the stage-empty barrier of the activation slot
// (a second commit per stage measured 3.4 % slower): the activation ring is
// at least as deep as the weight ring, and the weight slot of stage g waits
// on the barrier of stage g - PWS.
static_assert(PXS >= PWS, "one stage-empty barrier per activation slot frees both rings");
static_assert(STG_N >= 1, "at least one staging buffer per epilogue warp");
// Register split between the warpgroups (setmaxnreg), out of the 72 per
// thread the kernel is launched with (896 x 72 = 64,512 of the SM's 65,536):
// producers / MMA 32, dequant 40, epilogue 96, so that an epilogue warp
// holds its whole 64-column slice of the accumulator in registers and
// releases tensor memory before any staging or store.  The host checks the
// kernel's launch register count before every launch (a split above the
// launch pool would wait forever).
constexpr int REG_LAUNCH = 72, REG_WG0 = 32, REG_DEQ = 40, REG_EPI = 96;
static_assert(REG_WG0 * 128 + REG_DEQ * 256 + REG_EPI * 512 <= REG_LAUNCH * NTHREADS, "register split over the pool");
constexpr uint32_t PW_TILE = 128 * BK * 2;    // 8 KB: one of hi / lo for this CTA's 128 weight rows
constexpr uint32_t P_OFF_XH = 0;
constexpr uint32_t P_OFF_XL = P_OFF_XH + PXS * X_TILE;
constexpr uint32_t P_OFF_WH = P_OFF_XL + PXS * X_TILE;
constexpr uint32_t P_OFF_WL = P_OFF_WH + PWS * PW_TILE;
constexpr uint32_t P_OFF_RAW = P_OFF_WL + PWS * PW_TILE;  // 128 KB

template <int QT>
struct PCfg {
  static constexpr uint32_t RAW_SLOT = (uint32_t)TQ<QT>::rawb * 128;
  static constexpr uint32_t OFF_EPI = P_OFF_RAW + PRS * RAW_SLOT;
  static constexpr uint32_t OFF_STG = (OFF_EPI + 2 * BN * 4 + 1023u) & ~1023u;  // bias [BN] + QKV gains [BN]
  static constexpr uint32_t OFF_BAR = OFF_STG + STG_N * EPI_WARPS * STG_BYTES;
  static constexpr uint32_t SMEM = OFF_BAR + 256 + 1024;
  static_assert(SMEM <= 232448, "shared memory over the 227 KB per-block limit");
};

// 16 columns of (main + correction) accumulator for this thread's row.
T0B_DEV void tmem_ld_pair16(uint32_t taddr, float *v, float scale) {
  float c[16];
  tmem_ld16x2(taddr, taddr + BN, v, c);
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = (v[i] + c[i]) * scale;
}
// The same for two 16-column chunks at once (one wait for four loads).
T0B_DEV void tmem_ld_pair16x2(uint32_t ta, uint32_t tb, float *va, float *vb, float scale) {
  float ca[16], cb[16];
  tmem_ld16x4(ta, ta + BN, tb, tb + BN, va, ca, vb, cb);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    va[i] = (va[i] + ca[i]) * scale;
    vb[i] = (vb[i] + cb[i]) * scale;
  }
}

template <int N>
T0B_DEV void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int QT, int EK>  // EK: the epilogue kind (EPI_PLAIN, EPI_SWIGLU, EPI_QKV or EPI_RESID)
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_q_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
                          const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_y,
                          const __grid_constant__ CUtensorMap tm_zh, const __grid_constant__ CUtensorMap tm_zl,
                          TcParams prm) {
  using C = PCfg<QT>;
  constexpr int BPB = TQ<QT>::bpb, RAWB = TQ<QT>::rawb;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base_u32 - smem_u32(smem_raw));
  if (cluster_size() != 2) {  // launched without the 2-CTA cluster: nothing is touched
    if (threadIdx.x == 0) record_error(prm.err, T0B_DEVERR_SHAPE);
    return;
  }
  const uint32_t rank = cluster_rank();

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
  uint64_t *x_full = bars;               // [PXS] TMA bytes of both CTAs -> MMA (CTA 0's)
  uint64_t *x_empty = x_full + PXS;      // [PXS] MMA -> TMA and dequant: the stage's slots are free (each CTA's)
  uint64_t *raw_full = x_empty + PXS;    // [PRS] TMA -> dequant
  uint64_t *raw_empty = raw_full + PRS;  // [PRS] dequant -> TMA
  uint64_t *w_full = raw_empty + PRS;    // [PWS] dequant warps of both CTAs -> MMA (CTA 0's)
  uint64_t *acc_full = w_full + PWS;     // MMA -> epilogue (each CTA's)
  uint64_t *acc_empty = acc_full + 1;    // epilogue warps of both CTAs -> MMA (CTA 0's)
  uint64_t *mma_done = acc_empty + 1;    // every issued MMA has completed (CTA 0)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(mma_done + 2);
  float *epi_s = reinterpret_cast<float *>(smem + C::OFF_EPI);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = prm.M, K = prm.K;
  const int S = K / BK;
  const int SK = S / prm.k_split;  // K stages per work item
  constexpr bool swiglu = EK == EPI_SWIGLU;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PXS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < PRS; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 128);
    }
    for (int i = 0; i < PWS; ++i) {
      mbar_init(&w_full[i], 8);  // lane 0 of the 4 dequant warps of a stage, in both CTAs
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * EPI_WARPS);  // lane 0 of every epilogue warp, both CTAs
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_xh);
    prefetch_tmap(&tm_xl);
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_y);  // the unused kinds' maps repeat a valid one
    prefetch_tmap(&tm_zh);
    prefetch_tmap(&tm_zl);
  }
  if (warp == 1) {  // the same warp in both CTAs allocates the pair's columns
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // work item -> its first K stage (items of one tile are adjacent K splits)
  auto tile_s0 = [&](int tile) { return ((tile / prm.n_tiles_n) % prm.k_split) * SK; };
  // pair tile -> (this CTA's first token, this CTA's first weight row, n tile)
  auto tile_rows = [&](int tile, int &m0, int &wrow, int &nt) {
    nt = tile % prm.n_tiles_n;
    m0 = (tile / prm.n_tiles_n / prm.k_split) * (2 * BM) + BM * (int)rank;
    if (swiglu)
      wrow = (rank == 0 ? 0 : prm.swiglu_F) + nt * 128;
    else
      wrow = nt * BN + 128 * (int)rank;
  };
  auto lead = [](const uint64_t *b) { return mapa_shared(smem_u32(b), 0); };

  if (warp < 4) {
    setmaxnreg_dec<REG_WG0>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- activation producer (both CTAs)
      uint32_t g = 0;
      for (int tile = pair; tile < prm.n_tiles && !*abort_flag; tile += npairs) {
        int m0, wrow, nt;
        tile_rows(tile, m0, wrow, nt);
        const int s0 = tile_s0(tile);
        for (int s = s0; s < s0 + SK && !*abort_flag; ++s, ++g) {
          const uint32_t xs = g % PXS;
          if (g >= PXS && !mbar_wait(&x_empty[xs], ((g / PXS) - 1) & 1, prm.err, T0B_DEVERR_WAIT_EMPTY, abort_flag))
            break;
          if (rank == 0) mbar_arrive_expect_tx(&x_full[xs], 4 * X_TILE);  // hi + lo of both CTAs
          const uint32_t fb = lead(&x_full[xs]);
          if (T0B_CHECK_TMA(s * BK, 2, m0, prm.err) && T0B_CHECK(s * BK < prm.K, prm.err)) {
            tma_load_2d_pair(smem + P_OFF_XH + xs * X_TILE, &tm_xh, fb, s * BK, m0);
            tma_load_2d_pair(smem + P_OFF_XL + xs * X_TILE, &tm_xl, fb, s * BK, m0);
          }
        }
      }
    } else if (warp == 2 && lane == 0) {
      // ---------------------------------------------------------- raw weight producer (both CTAs)
      // separate from the activation producer so that raw blocks run ahead
      // as far as the dequant warps allow, whatever the MMAs are waiting for
      uint32_t g = 0;
      for (int tile = pair; tile < prm.n_tiles && !*abort_flag; tile += npairs) {
        int m0, wrow, nt;
        tile_rows(tile, m0, wrow, nt);
        const int s0 = tile_s0(tile);
        for (int s = s0; s < s0 + SK && !*abort_flag; ++s, ++g) {
          const uint32_t rs = g % PRS;
          if (g >= PRS && !mbar_wait(&raw_empty[rs], ((g / PRS) - 1) & 1, prm.err, T0B_DEVERR_WAIT_EMPTY, abort_flag))
            break;
          const int x = (s * BPB) & ~15;  // aligned window holding block column s
          mbar_arrive_expect_tx(&raw_full[rs], C::RAW_SLOT);
          if (T0B_CHECK_TMA(x, 1, wrow, prm.err))
            tma_load_2d(smem + P_OFF_RAW + rs * C::RAW_SLOT, &tm_w, &raw_full[rs], x, wrow);
        }
      }
    } else if (warp == 1 && lane == 0 && rank == 0) {
      // ---------------------------------------------------------- MMA issuer (CTA 0)
      constexpr uint32_t idesc = idesc_f16_f32(2 * BM, BN);
      uint32_t g = 0, it = 0;
      for (int tile = pair; tile < prm.n_tiles && !*abort_flag; tile += npairs, ++it) {
        if (it >= 1 && !mbar_wait(acc_empty, (it - 1) & 1, prm.err, T0B_DEVERR_WAIT_ACC, abort_flag)) break;
        tc_fence_after();
        const int s0 = tile_s0(tile);
        for (int s = s0; s < s0 + SK; ++s, ++g) {
          const uint32_t xs = g % PXS, ws = g % PWS;
          if (!mbar_wait(&x_full[xs], (g / PXS) & 1, prm.err, T0B_DEVERR_WAIT_X, abort_flag) ||
              !mbar_wait(&w_full[ws], (g / PWS) & 1, prm.err, T0B_DEVERR_WAIT_DEQ, abort_flag))
            break;
          tc_fence_after();
          const uint32_t xh = base_u32 + P_OFF_XH + xs * X_TILE, xl = base_u32 + P_OFF_XL + xs * X_TILE;
          const uint32_t wh = base_u32 + P_OFF_WH + ws * PW_TILE, wl = base_u32 + P_OFF_WL + ws * PW_TILE;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t ko = kk * 32;  // 16 f16 along K inside the 64-byte swizzled row
            const uint32_t acc = (s > s0 || kk > 0) ? 1u : 0u;
            umma_f16_pair(tmem, sw64_desc(xh + ko), sw64_desc(wh + ko), idesc, acc);
            umma_f16_pair(tmem + BN, sw64_desc(xh + ko), sw64_desc(wl + ko), idesc, acc);
            umma_f16_pair(tmem + BN, sw64_desc(xl + ko), sw64_desc(wh + ko), idesc, 1u);
          }
          umma_commit_pair_both(&x_empty[xs]);  // frees the stage's activation and weight slots
        }
        if (*abort_flag) break;
        umma_commit_pair_both(acc_full);
      }
      // every issued MMA completes before the pair reaches the TMEM release
      umma_commit_pair(smem_u32(mma_done));
      mbar_wait(mma_done, 0, prm.err, T0B_DEVERR_WAIT_ACC, nullptr);
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------ dequant (both CTAs)
    setmaxnreg_dec<REG_DEQ>();
    const int grp = (warp - 4) >> 2;            // stages g with g % 2 == grp
    const int r = (threadIdx.x - 128) & 127;    // tile row 0..127 of this CTA's weight rows
    uint32_t g = 0;
    bool ok = true;
    for (int tile = pair; tile < prm.n_tiles && ok && !*abort_flag; tile += npairs) {
      const int s0 = tile_s0(tile);
      for (int s = s0; s < s0 + SK; ++s, ++g) {
        if ((int)(g & 1) != grp) continue;
        const uint32_t ws = g % PWS, rs = g % PRS;
        bool got = true;
        if (lane == 0)
          got = (g < PWS ||
                 mbar_wait(&x_empty[(g - PWS) % PXS], ((g - PWS) / PXS) & 1, prm.err, T0B_DEVERR_WAIT_EMPTY,
                           abort_flag)) &&
                mbar_wait(&raw_full[rs], (g / PRS) & 1, prm.err, T0B_DEVERR_WAIT_W, abort_flag);
        got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
        __syncwarp();
        if (!got) {
          ok = false;
          break;
        }
        uint8_t *whs = smem + P_OFF_WH + ws * PW_TILE;
        uint8_t *wls = smem + P_OFF_WL + ws * PW_TILE;
        const int off = (s * BPB) & 15;  // block start inside the aligned window
        const uint8_t *slot = smem + P_OFF_RAW + rs * C::RAW_SLOT;
        dequant_row_at<QT>(off, slot + r * RAWB, prm.wscale, whs, wls, r);
        mbar_arrive(&raw_empty[rs]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead(&w_full[ws]));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    setmaxnreg_inc<REG_EPI>();
    const int q = warp & 3;
    const int quarter = (warp - 12) >> 2;
    const int et = threadIdx.x - 384;
    const Epi &e = prm.epi;
    float *sb = epi_s;
    uint8_t *stg0 = smem + C::OFF_STG + (warp - 12) * STG_N * STG_BYTES;
    uint32_t ck = 0;  // chunks written by this warp (staging buffer = ck % STG_N)
    uint32_t it = 0;
    for (int tile = pair; tile < prm.n_tiles; tile += npairs, ++it) {
      int m0, wrow, nt;
      tile_rows(tile, m0, wrow, nt);
      epi_bar();
      if (et < BN) {
        const int c = et;
        const int f = swiglu ? (c < 128 ? nt * 128 + c : e.F + nt * 128 + (c - 128)) : nt * BN + c;
        sb[c] = (e.bias && tile_s0(tile) == 0) ? e.bias[f] : 0.0f;
        if constexpr (EK == EPI_RESID) sb[BN + c] = e.gnext[f];  // the next RMSNorm's gains
        if constexpr (EK == EPI_QKV) {  // QK-norm gains of the tile's columns (1 for v)
          const int seg = f / e.E;
          sb[BN + c] = seg == 0 ? e.qn[c & 63] : (seg == 1 ? e.kn[c & 63] : 1.0f);
        }
      }
      epi_bar();
      const int row0 = m0 + 32 * q;
      const int m = row0 + lane;
      const bool live = m < M;
      const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
      const float sc = prm.acc_scale * (live ? 1.0f / epi_row_denom(e, m) : 1.0f);
      bool have = mbar_wait(acc_full, it & 1, prm.err, T0B_DEVERR_WAIT_ACC, abort_flag) && !*abort_flag;
      have = __all_sync(0xffffffffu, have);
      tc_fence_after();
      bool released = false;
      auto release = [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead(acc_empty));
        released = true;
      };
      auto next_stage_buf = [&]() -> uint8_t * {
        uint8_t *b = stg0 + (ck % STG_N) * STG_BYTES;
        ++ck;
        if (lane == 0) bulk_wait_read<STG_N - 1>();  // the store that last used this buffer has read it
        __syncwarp();
        return b;
      };
      if (have) {
        // every epilogue kind loads its whole slice of the accumulator (64
        // values per thread: main + correction summed, scaled) and releases
        // tensor memory before it computes, stages or stores anything
        float v[4][16];
        // three load round trips: two chunks, then one, then one
        if constexpr (swiglu) {
          // gate columns 32 quarter .. + 31 and the matching up columns
          tmem_ld_pair16x2(trow + 32 * quarter, trow + 128 + 32 * quarter, v[0], v[2], sc);
          tmem_ld_pair16(trow + 32 * quarter + 16, v[1], sc);
          tmem_ld_pair16(trow + 128 + 32 * quarter + 16, v[3], sc);
        } else {
          tmem_ld_pair16x2(trow + 64 * quarter, trow + 64 * quarter + 16, v[0], v[1], sc);
          tmem_ld_pair16(trow + 64 * quarter + 32, v[2], sc);
          tmem_ld_pair16(trow + 64 * quarter + 48, v[3], sc);
        }
        release();
        // one 16-column chunk split in place (word 2i: f16x2 hi of values
        // 2i, 2i+1; word 2i+1: their lo) -> staged -> two TMA stores
        auto store_hl = [&](const uint32_t *w, int x) {
          uint8_t *stg = next_stage_buf();
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint32_t o = lane * 32 + ((j ^ ((lane >> 2) & 1)) << 4);
            *reinterpret_cast<uint4 *>(stg + o) = make_uint4(w[8 * j], w[8 * j + 2], w[8 * j + 4], w[8 * j + 6]);
            *reinterpret_cast<uint4 *>(stg + 1024 + o) =
                make_uint4(w[8 * j + 1], w[8 * j + 3], w[8 * j + 5], w[8 * j + 7]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (T0B_CHECK_TMA(x, 2, row0, prm.err)) {
              tma_store_2d(&tm_zh, stg, x, row0);
              tma_store_2d(&tm_zl, stg + 1024, x, row0);
            }
            bulk_commit();
          }
        };
        if constexpr (swiglu) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int g0 = 32 * quarter + 16 * c;
            float *gv = v[c], *uv = v[2 + c];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float gg = gv[i] + sb[g0 + i];
              const float uu = uv[i] + sb[128 + g0 + i];
              gv[i] = gg * __frcp_rn(1.0f + __expf(-gg)) * uu;
            }
            if (e.z32 && live) store_f32x16(e.z32 + (size_t)m * e.F + (size_t)nt * 128 + g0, gv);
            uint32_t *w = reinterpret_cast<uint32_t *>(gv);
#pragma unroll
            for (int i = 0; i < 8; ++i) split2(gv[2 * i], gv[2 * i + 1], w[2 * i], w[2 * i + 1]);
            store_hl(w, nt * 128 + g0);
          }
        } else if constexpr (EK == EPI_QKV) {
          // this warp's 64 columns are one head of q, k or v: bias, then for
          // q and k the sum of squares of y (their QK-norm, applied to the
          // attention scores), the norm gain and the RoPE of the token's
          // patch position; each 16-column chunk is split into f16 hi / lo
          // and written by TMA stores like the SwiGLU output
          const int col0 = nt * BN + 64 * quarter;  // first column of the head
          const int seg = col0 / e.E;               // 0: q, 1: k, 2: v
          const int pos = live ? m % e.p : 0;       // patch position of this thread's token
          float ss = 0.0f;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const int c0 = 64 * quarter + 16 * ch;
            float *x = v[ch];
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] += sb[c0 + i];
            if (seg < 2) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                ss += x[i] * x[i];
                x[i] *= sb[BN + c0 + i];
              }
              rope16_t(x, e.rope_t, e.p, pos, ch, seg == 1);
            }
            uint32_t *w = reinterpret_cast<uint32_t *>(x);
#pragma unroll
            for (int i = 0; i < 8; ++i) split2(x[2 * i], x[2 * i + 1], w[2 * i], w[2 * i + 1]);
            store_hl(w, col0 + 16 * ch);
          }
          if (seg < 2 && live) e.ssq_qk[(size_t)m * 2 * e.H + seg * e.H + ((col0 - seg * e.E) >> 6)] = ss;
        } else if constexpr (EK == EPI_RESID) {
          // residual branch output (wO, mlp.2): x[m, n] += y + bias; the new
          // x is stored back (each element belongs to one tile), x * gnext is
          // split into the f16 planes of the next RMSNorm-fused GEMM, and the
          // sum of x^2 over this warp's 64 columns goes to its slot of the
          // row's partial sums (the next GEMM's row scale adds the N / 64 slots)
          const int col0 = nt * BN + 64 * quarter;
          float ss = 0.0f;
          const float4 *xo = reinterpret_cast<const float4 *>(e.x + (size_t)(live ? m : 0) * e.N + col0);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int c0 = 64 * quarter + 16 * c;
            float *xv = v[c];
#pragma unroll
            for (int i = 0; i < 4; ++i) {  // x + (branch + bias), the order of the reduce-add path
              const float4 o = live ? xo[4 * c + i] : make_float4(0.f, 0.f, 0.f, 0.f);
              xv[4 * i] = o.x + (xv[4 * i] + sb[c0 + 4 * i]);
              xv[4 * i + 1] = o.y + (xv[4 * i + 1] + sb[c0 + 4 * i + 1]);
              xv[4 * i + 2] = o.z + (xv[4 * i + 2] + sb[c0 + 4 * i + 2]);
              xv[4 * i + 3] = o.w + (xv[4 * i + 3] + sb[c0 + 4 * i + 3]);
            }
            uint8_t *stg = next_stage_buf();
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<float4 *>(stg + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                  make_float4(xv[4 * j], xv[4 * j + 1], xv[4 * j + 2], xv[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (T0B_CHECK_TMA(col0 + 16 * c, 4, row0, prm.err)) tma_store_2d(&tm_y, stg, col0 + 16 * c, row0);
              bulk_commit();
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              ss += xv[i] * xv[i];
              xv[i] *= sb[BN + c0 + i];
            }
            uint32_t *w = reinterpret_cast<uint32_t *>(xv);
#pragma unroll
            for (int i = 0; i < 8; ++i) split2(xv[2 * i], xv[2 * i + 1], w[2 * i], w[2 * i + 1]);
            store_hl(w, col0 + 16 * c);
          }
          if (live && T0B_CHECK((col0 >> 6) < e.ssq_out_nt, prm.err)) e.ssq_out[(size_t)m * e.ssq_out_nt + (col0 >> 6)] = ss;
        } else {  // EPI_PLAIN: bias, then f32 chunks stored (or reduce-added) by TMA
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int c0 = 64 * quarter + 16 * c;
#pragma unroll
            for (int i = 0; i < 16; ++i) v[c][i] += sb[c0 + i];
            uint8_t *stg = next_stage_buf();
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<float4 *>(stg + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                  make_float4(v[c][4 * j], v[c][4 * j + 1], v[c][4 * j + 2], v[c][4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (!T0B_CHECK_TMA(nt * BN + c0, 4, row0, prm.err)) {
              } else if (e.reduce_add) {
                tma_reduce_add_2d(&tm_y, stg, nt * BN + c0, row0);
              } else {
                tma_store_2d(&tm_y, stg, nt * BN + c0, row0);
              }
              bulk_commit();
            }
          }
        }
      }
      if (!released) release();
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA frees the pair's TMEM while the other may still use it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
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

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *ptr, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// SM count of device `dev` (callers hold max_pairs' lock or accept a
// repeated query; nothing is cached here).
int sm_count(int dev) {
  int n_sm = 0;
  if (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n_sm <= 0) {
    cudaGetLastError();
    n_sm = 148;
  }
  return n_sm;
}

// Number of 2-CTA clusters of `kfn` (launched as `cfg`) that fit on the
// device at once, cached per kernel and device.
int max_pairs(const void *kfn, const cudaLaunchConfig_t &cfg) {
  static std::mutex mu;
  static std::map<std::pair<const void *, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find({kfn, dev});
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t c = cfg;
  c.gridDim = dim3(2 * sm_count(dev));
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kfn, &c) != cudaSuccess || n < 1) {
    cudaGetLastError();
    return 0;
  }
  cache[{kfn, dev}] = n;
  return n;
}

template <int QT, int EK>
cudaError_t launch_tc_k(const CUtensorMap &txh, const CUtensorMap &txl, const CUtensorMap &tw, const CUtensorMap &ty,
                        const CUtensorMap &tzh, const CUtensorMap &tzl, const TcParams &prm, cudaStream_t st) {
  using P = PCfg<QT>;
  auto kfn = gemm_q_tc_pair_kernel<QT, EK>;
  // the warpgroups' register split (setmaxnreg) is sized for a launch with
  // REG_LAUNCH registers per thread; any other count is refused, never run
  static const int launch_regs = [&] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, (const void *)kfn) == cudaSuccess ? fa.numRegs : -1;
  }();
  if (launch_regs != REG_LAUNCH) return cudaErrorInvalidConfiguration;
  cudaError_t e = t0b_smem_limit((const void *)kfn, P::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = P::SMEM;
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const int pairs = max_pairs((const void *)kfn, cfg);
  if (pairs < 1) return cudaErrorInvalidConfiguration;
  const int np = prm.n_tiles < pairs ? prm.n_tiles : pairs;  // persistent: one CTA pair per SM pair
  cfg.gridDim = dim3(2 * np);
  return cudaLaunchKernelEx(&cfg, kfn, txh, txl, tw, ty, tzh, tzl, prm);
}

template <int QT>
cudaError_t launch_tc_t(const __half *ah, const __half *al, int M, int K, const uint8_t *W, int wrows, int wshift,
                        const Epi &epi, int *err, cudaStream_t st) {
  CUtensorMap txh, txl, tw;
  const uint64_t rb = (uint64_t)(K / 32) * TQ<QT>::bpb;
  if (!make_tmap_2d(&txh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ah, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, BM,
                    CU_TENSOR_MAP_SWIZZLE_64B) ||
      !make_tmap_2d(&txl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, al, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, BM,
                    CU_TENSOR_MAP_SWIZZLE_64B) ||
      !make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, W, rb, (uint64_t)wrows, rb, TQ<QT>::rawb, 128,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (epi.kind != EPI_PLAIN && epi.kind != EPI_SWIGLU && epi.kind != EPI_QKV && epi.kind != EPI_RESID)
    return cudaErrorInvalidValue;
  if (epi.kind == EPI_RESID &&
      (!epi.x || !epi.gnext || !epi.ssq_out || epi.ssq_out_nt != epi.N / 64 || epi.F != epi.N || epi.zh != epi.xh ||
       epi.zl != epi.xl || epi.y != epi.x || epi.ldy != epi.N))
    return cudaErrorInvalidValue;
  if (epi.kind == EPI_QKV &&
      (epi.F != 3 * epi.E || epi.N != epi.F || epi.E % 64 || epi.E / 64 != epi.H || !epi.qn || !epi.kn ||
       !epi.rope_t || !epi.ssq_qk || epi.p < 1))
    return cudaErrorInvalidValue;
  // output maps for the epilogue's TMA stores (the unused kind's maps repeat
  // a valid one; the kernel never touches them)
  CUtensorMap ty, tzh, tzl;
  if (epi.kind == EPI_RESID) {  // x (f32) and the split planes of x * gnext
    if (!make_tmap_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, epi.y, (uint64_t)epi.N, (uint64_t)M,
                      (uint64_t)epi.ldy * 4, 16, 32, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_tmap_2d(&tzh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, epi.zh, (uint64_t)epi.F, (uint64_t)M,
                      (uint64_t)epi.F * 2, 16, 32, CU_TENSOR_MAP_SWIZZLE_32B) ||
        !make_tmap_2d(&tzl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, epi.zl, (uint64_t)epi.F, (uint64_t)M,
                      (uint64_t)epi.F * 2, 16, 32, CU_TENSOR_MAP_SWIZZLE_32B))
      return cudaErrorInvalidValue;
  } else if (epi.kind == EPI_PLAIN) {
    if (!epi.y || epi.ldy < epi.N || epi.ldy % 4 ||
        !make_tmap_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, epi.y, (uint64_t)epi.N, (uint64_t)M,
                      (uint64_t)epi.ldy * 4, 16, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return cudaErrorInvalidValue;
    tzh = tzl = ty;
  } else {  // SWIGLU and QKV: f16 (hi, lo) planes of F columns
    if (!epi.zh || !epi.zl ||
        !make_tmap_2d(&tzh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, epi.zh, (uint64_t)epi.F, (uint64_t)M,
                      (uint64_t)epi.F * 2, 16, 32, CU_TENSOR_MAP_SWIZZLE_32B) ||
        !make_tmap_2d(&tzl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, epi.zl, (uint64_t)epi.F, (uint64_t)M,
                      (uint64_t)epi.F * 2, 16, 32, CU_TENSOR_MAP_SWIZZLE_32B))
      return cudaErrorInvalidValue;
    ty = tzh;
  }
  TcParams prm;
  prm.M = M;
  prm.N = epi.N;
  prm.K = K;
  prm.swiglu_F = epi.kind == EPI_SWIGLU ? epi.F : 0;
  prm.n_tiles_n = epi.kind == EPI_SWIGLU ? epi.F / 128 : epi.N / BN;
  prm.k_split = 1;
  prm.wscale = ldexpf(1.0f, wshift);
  prm.acc_scale = ldexpf(1.0f, -wshift);
  prm.epi = epi;
  prm.err = err;
  prm.n_tiles = prm.n_tiles_n * ((M + 2 * BM - 1) / (2 * BM));
  {
    // few tiles for the SMs (the standalone shapes at a few hundred tokens):
    // split K in two, the partial tiles reduce-added into a zeroed y.  Two
    // addends into zero give the same sum in either order, so the result
    // stays deterministic.
    int dev = 0;
    cudaGetDevice(&dev);
    const int pairs_est = sm_count(dev) / 2, S = K / BK;
    if (epi.kind == EPI_PLAIN && !epi.reduce_add && 2 * prm.n_tiles <= pairs_est && S % 2 == 0 && S / 2 >= 8) {
      cudaError_t ze = epi.ldy == epi.N ? cudaMemsetAsync(epi.y, 0, (size_t)M * epi.N * 4, st)
                                        : cudaMemset2DAsync(epi.y, (size_t)epi.ldy * 4, 0, (size_t)epi.N * 4, M, st);
      if (ze != cudaSuccess) return ze;
      prm.k_split = 2;
      prm.n_tiles *= 2;
      prm.epi.reduce_add = 1;
    }
  }
  if (epi.kind == EPI_SWIGLU) return launch_tc_k<QT, EPI_SWIGLU>(txh, txl, tw, ty, tzh, tzl, prm, st);
  if (epi.kind == EPI_QKV) return launch_tc_k<QT, EPI_QKV>(txh, txl, tw, ty, tzh, tzl, prm, st);
  if (epi.kind == EPI_RESID) return launch_tc_k<QT, EPI_RESID>(txh, txl, tw, ty, tzh, tzl, prm, st);
  return launch_tc_k<QT, EPI_PLAIN>(txh, txl, tw, ty, tzh, tzl, prm, st);
}

}  // namespace

// f32 row-major [outer][inner] tensor (rows row_bytes apart), box
// [box_outer][box_inner], optionally with the 128-byte swizzle: for other
// kernels' TMA loads.
bool t0b_make_tmap_f32_2d(CUtensorMap *tm, const float *ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                          uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  return make_tmap_2d(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ptr, inner, outer, row_bytes, box_inner, box_outer,
                      swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

// f16 tensor of dims {d0, d1, d2} (innermost first; d1 rows s1 bytes apart,
// d2 slabs s2 bytes apart), box {b0, b1, b2}, optionally with the 128-byte
// swizzle: for the attention kernels' TMA stores.
bool t0b_make_tmap_f16_3d(CUtensorMap *tm, const void *ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                          uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Host entry.  qt: 8 = Q8_0, 4 = Q4_0.  Requires K % 256 == 0, N % 256 == 0
// (SWIGLU: F % 128 == 0), M >= 1, 16-byte aligned A rows.  `wrows` is the
// number of rows of W (N, or 2F for SWIGLU); `wshift` the weight prescale
// exponent from t0b_weight_shift.  Epilogue kinds: PLAIN (bias + optional
// RMSNorm row scale; with reduce_add the tile is added into y by TMA
// reduce-adds), SWIGLU and QKV (N = F = 3E, 64-dim heads); others are
// rejected (cudaErrorInvalidValue).
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
