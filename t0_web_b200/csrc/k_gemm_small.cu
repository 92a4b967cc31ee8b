// k_gemm_small.cu -- small-token-count dequant GEMM on raw Q8_0 / Q4_0 blocks.
//
// Y[M, N] = A[M, K] . deq(W)[N, K]^T for M up to a few dozen tokens (a single
// forecast: M = v * p = 19 at context 512 / horizon 96).  Work is bounded by
// the weight bytes, so the kernel streams each weight row once:
//   * each warp owns 16 weight rows and walks K in 256-value chunks, staging
//     the raw 34-byte (Q8_0) / 18-byte (Q4_0) blocks of its rows into shared
//     memory with 16-byte cp.async copies (rows are 16-byte aligned because
//     K % 256 == 0);
//   * the int8 values / nibbles are unpacked in registers to f16 *exactly*
//     (q is an integer of at most 8 bits) and multiplied on the tensor cores
//     (mma.sync m16n8k16) against the activations split as A = Ah + Al
//     (two f16 terms), so every product is exact to about 2^-22;
//   * the block's f16 scale d is applied in f32 to the 32-value block sum
//     ("promotion"), i.e. y = sum_b d_b * sum_{k in b} a_k q_k, which is the
//     reference's f32 dot product up to summation order
//     (linear_q8.wgsl / linear_q4.wgsl, gguf.rs:116-174).
// Parallelism: a CTA owns 32 weight rows (two warps); when that gives too few
// CTAs to keep the memory system busy, K is split across CTAs too.  Each
// split CTA writes its partial 32 x M tile to a workspace and the last CTA to
// finish a tile (an arrival counter, reset to zero by that CTA) adds the
// partials in split order -- deterministic -- and runs the epilogue.
// The 32 x M output tile goes through shared memory into the fused epilogue.
#include "common.cuh"
#include "epilogue.cuh"

namespace {

constexpr int kWarps = 2;
constexpr int kRows = kWarps * 16;  // weight rows (output columns) per CTA
constexpr int kRowsPerWarp = 16;
constexpr int kChunkK = 256;  // values per staged chunk (8 blocks)

template <int QT>
struct QInfo;
template <>
struct QInfo<8> {
  static constexpr int bpb = 34;
};
template <>
struct QInfo<4> {
  static constexpr int bpb = 18;
};

template <int QT, int NT8>
__global__ void __launch_bounds__(64) gemm_q_small_kernel(const __half *__restrict__ ah,
                                                          const __half *__restrict__ al, int M, int K,
                                                          const uint8_t *__restrict__ W, Epi epi, int *err,
                                                          float *part, int *cnt) {
  constexpr int BPB = QInfo<QT>::bpb;
  constexpr int CB = 8 * BPB;  // bytes per row per chunk: 272 / 144, multiple of 16
  constexpr int MT = 8 * NT8;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t *stage = smem;  // [warps][2][16][CB]
  float *tile = reinterpret_cast<float *>(smem + kWarps * 2 * kRowsPerWarp * CB);  // [kRows][MT+1]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int m0 = blockIdx.y * MT;
  const size_t RB = (size_t)(K / 32) * BPB;

  // weight rows of this warp (SWIGLU: warp 0 gate rows, warp 1 the matching up rows)
  int wrow0;
  if (epi.kind == EPI_SWIGLU) {
    const int f0 = blockIdx.x * 16;
    wrow0 = warp == 0 ? f0 : epi.F + f0;
  } else {
    wrow0 = blockIdx.x * kRows + 16 * warp;
  }
  const uint8_t *wbase = W + (size_t)wrow0 * RB;
  uint8_t *my = stage + warp * 2 * kRowsPerWarp * CB;

  float acc[NT8][4];
#pragma unroll
  for (int j = 0; j < NT8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

  // this CTA's share of the K chunks (split-K along gridDim.z)
  const int nchunks_all = K / kChunkK, ksplit = gridDim.z;
  const int per = (nchunks_all + ksplit - 1) / ksplit;
  const int c_begin = blockIdx.z * per, c_end = min(nchunks_all, c_begin + per);
  const int nchunks = c_end > c_begin ? c_end - c_begin : 0;
  auto stage_chunk = [&](int c, int buf) {
    uint8_t *dst = my + buf * kRowsPerWarp * CB;
    for (int i = lane; i < kRowsPerWarp * (CB / 16); i += 32) {
      int r = i / (CB / 16), q = i % (CB / 16);
      cp_async16(dst + r * CB + q * 16, wbase + (size_t)r * RB + (size_t)(c_begin + c) * CB + q * 16);
    }
    cp_async_commit();
  };
  if (nchunks > 0) stage_chunk(0, 0);
  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) {
      stage_chunk(c + 1, (c + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    const uint8_t *sb = my + (c & 1) * kRowsPerWarp * CB;
#pragma unroll 2
    for (int b = 0; b < 8; ++b) {
      const uint8_t *r0 = sb + g * CB + b * BPB;
      const uint8_t *r1 = sb + (g + 8) * CB + b * BPB;
      float d0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(r0));
      float d1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(r1));
      uint32_t a[2][4];
      if (QT == 8) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          a[h][0] = i8x2_to_h2(*reinterpret_cast<const uint16_t *>(r0 + 2 + 16 * h + 2 * tig));
          a[h][1] = i8x2_to_h2(*reinterpret_cast<const uint16_t *>(r1 + 2 + 16 * h + 2 * tig));
          a[h][2] = i8x2_to_h2(*reinterpret_cast<const uint16_t *>(r0 + 2 + 16 * h + 8 + 2 * tig));
          a[h][3] = i8x2_to_h2(*reinterpret_cast<const uint16_t *>(r1 + 2 + 16 * h + 8 + 2 * tig));
        }
      } else {
        uint32_t w00 = *reinterpret_cast<const uint16_t *>(r0 + 2 + 2 * tig);
        uint32_t w10 = *reinterpret_cast<const uint16_t *>(r1 + 2 + 2 * tig);
        uint32_t w01 = *reinterpret_cast<const uint16_t *>(r0 + 2 + 8 + 2 * tig);
        uint32_t w11 = *reinterpret_cast<const uint16_t *>(r1 + 2 + 8 + 2 * tig);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          a[h][0] = nib2_to_h2(w00, h);
          a[h][1] = nib2_to_h2(w10, h);
          a[h][2] = nib2_to_h2(w01, h);
          a[h][3] = nib2_to_h2(w11, h);
        }
      }
      const int kb = (c_begin + c) * kChunkK + b * 32;
#pragma unroll
      for (int j = 0; j < NT8; ++j) {
        int m = m0 + 8 * j + g;
        float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
        // tokens past M load zeros; the mma itself is warp-wide and unconditional
        uint32_t bh[2][2] = {{0u, 0u}, {0u, 0u}}, bl[2][2] = {{0u, 0u}, {0u, 0u}};
        if (m < M) {
          const __half *xh = ah + (size_t)m * K + kb + 2 * tig;
          const __half *xl = al + (size_t)m * K + kb + 2 * tig;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            bh[h][0] = *reinterpret_cast<const uint32_t *>(xh + 16 * h);
            bh[h][1] = *reinterpret_cast<const uint32_t *>(xh + 16 * h + 8);
            bl[h][0] = *reinterpret_cast<const uint32_t *>(xl + 16 * h);
            bl[h][1] = *reinterpret_cast<const uint32_t *>(xl + 16 * h + 8);
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          mma16816(p0, p1, p2, p3, a[h][0], a[h][1], a[h][2], a[h][3], bh[h][0], bh[h][1]);
          mma16816(p0, p1, p2, p3, a[h][0], a[h][1], a[h][2], a[h][3], bl[h][0], bl[h][1]);
        }
        acc[j][0] += d0 * p0;
        acc[j][1] += d0 * p1;
        acc[j][2] += d1 * p2;
        acc[j][3] += d1 * p3;
      }
    }
    __syncwarp();
  }

  // accumulators -> tile[weight row 0..63][token 0..MT)
  constexpr int LD = MT + 1;
#pragma unroll
  for (int j = 0; j < NT8; ++j) {
    int r = 16 * warp + g;
    int t = 8 * j + 2 * tig;
    tile[r * LD + t] = acc[j][0];
    tile[r * LD + t + 1] = acc[j][1];
    tile[(r + 8) * LD + t] = acc[j][2];
    tile[(r + 8) * LD + t + 1] = acc[j][3];
  }
  __syncthreads();

  if (ksplit > 1) {
    // publish this CTA's partial tile; the last CTA of the tile reduces
    const int tile_id = blockIdx.y * gridDim.x + blockIdx.x;
    float *mine = part + ((size_t)tile_id * ksplit + blockIdx.z) * kRows * LD;
    for (int i = threadIdx.x; i < kRows * LD; i += blockDim.x) mine[i] = tile[i];
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) last = atomicAdd(&cnt[tile_id], 1) == ksplit - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float *all = part + (size_t)tile_id * ksplit * kRows * LD;
    for (int i = threadIdx.x; i < kRows * LD; i += blockDim.x) {
      float v = 0.0f;
      for (int z = 0; z < ksplit; ++z) v += __ldcg(all + (size_t)z * kRows * LD + i);
      tile[i] = v;
    }
    if (threadIdx.x == 0) cnt[tile_id] = 0;  // ready for the next launch
    __syncthreads();
  }

  // epilogue: one thread per token, its 32 (SWIGLU: 16 gate + 16 up) columns
  for (int t = threadIdx.x; t < MT; t += blockDim.x) {
    if (m0 + t >= M) continue;
    const int m = m0 + t;
    float denom = epi_row_denom(epi, m);
    float v[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) v[r] = tile[r * LD + t];
    if (epi.kind == EPI_SWIGLU) {
      epi_swiglu<16>(epi, m, blockIdx.x * 16, v, v + 16, denom);
    } else {
      float ss = epi_cols32(epi, m, blockIdx.x * kRows, v, denom);
      if (epi.kind == EPI_RESID) epi.ssq_out[(size_t)m * epi.ssq_out_nt + blockIdx.x] = ss;
    }
  }
}

// Split-K factor for a launch: enough CTAs for ~2 per SM, at most one split
// per 256-value chunk of K.
int small_ksplit(int M, int K, const Epi &epi, int nt8) {
  const int mt = 8 * (nt8 <= 4 ? nt8 : 8);
  const int cols = epi.kind == EPI_SWIGLU ? epi.F / 16 : epi.N / kRows;
  const int tiles = cols * ((M + mt - 1) / mt);
  const int target = 296;
  if (tiles >= target) return 1;
  const int ks = (target + tiles - 1) / tiles;
  return ks < K / kChunkK ? ks : K / kChunkK;
}

template <int QT, int NT8>
cudaError_t launch_small_t(const __half *ah, const __half *al, int M, int K, const uint8_t *W, const Epi &epi,
                           int *err, cudaStream_t st, float *part, int *cnt, int ksplit) {
  constexpr int CB = 8 * QInfo<QT>::bpb;
  constexpr int MT = 8 * NT8;
  size_t smem = (size_t)kWarps * 2 * kRowsPerWarp * CB + (size_t)kRows * (MT + 1) * sizeof(float);
  auto kfn = gemm_q_small_kernel<QT, NT8>;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int gx = epi.kind == EPI_SWIGLU ? epi.F / 16 : epi.N / kRows;
  dim3 grid(gx, (M + MT - 1) / MT, ksplit);
  kfn<<<grid, 32 * kWarps, smem, st>>>(ah, al, M, K, W, epi, err, part, cnt);
  return cudaGetLastError();
}

}  // namespace

// Workspace the split-K form of a small-M launch needs (0, 0 when it runs
// unsplit): part_floats for the partial tiles, cnt_ints for the per-tile
// arrival counters, which must be zero before the first launch and are left
// at zero by every launch.
void t0b_small_workspace(int M, int K, const Epi &epi, size_t *part_floats, size_t *cnt_ints) {
  const int nt8 = (M + 7) / 8;
  const int ks = small_ksplit(M, K, epi, nt8);
  const int mt = 8 * (nt8 <= 4 ? nt8 : 8);
  const size_t tiles = (size_t)(epi.kind == EPI_SWIGLU ? epi.F / 16 : epi.N / kRows) * ((M + mt - 1) / mt);
  *part_floats = ks > 1 ? tiles * ks * kRows * (mt + 1) : 0;
  *cnt_ints = ks > 1 ? tiles : 0;
}

// Host entry.  qt: 8 = Q8_0, 4 = Q4_0.  Requires K % 256 == 0 and the output
// column count (N, or F for SWIGLU) a multiple of 32 (16 for SWIGLU).  With
// part/cnt = NULL the launch is not split along K; otherwise they must be
// sized by t0b_small_workspace.
cudaError_t t0b_launch_gemm_small(int qt, const __half *ah, const __half *al, int M, int K, const uint8_t *W,
                                  const Epi &epi, int *err, cudaStream_t st, float *part, int *cnt) {
  const int nt8 = (M + 7) / 8;
  const int ks = (part && cnt) ? small_ksplit(M, K, epi, nt8) : 1;
  if (qt == 8) {
    if (nt8 <= 1) return launch_small_t<8, 1>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
    if (nt8 <= 2) return launch_small_t<8, 2>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
    if (nt8 <= 3) return launch_small_t<8, 3>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
    if (nt8 <= 4) return launch_small_t<8, 4>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
    return launch_small_t<8, 8>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
  } else {
    if (nt8 <= 1) return launch_small_t<4, 1>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
    if (nt8 <= 2) return launch_small_t<4, 2>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
    if (nt8 <= 3) return launch_small_t<4, 3>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
    if (nt8 <= 4) return launch_small_t<4, 4>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
    return launch_small_t<4, 8>(ah, al, M, K, W, epi, err, st, part, cnt, ks);
  }
}
