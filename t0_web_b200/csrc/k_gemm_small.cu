// k_gemm_small.cu -- small-token-count dequant GEMM on raw Q8_0 / Q4_0 blocks.
//
// Y[M, N] = A[M, K] . deq(W)[N, K]^T for M up to a few dozen tokens (a single
// forecast: M = v * p = 19 at context 512 / horizon 96).  One such GEMM moves
// well under a megabyte or two of weights, less than HBM's bandwidth-delay
// product, so its time is set by how many dependent memory round trips it
// makes, not by bytes.  The kernel is built for one round trip:
//   * a CTA owns 32 weight rows (output columns; SWIGLU: 16 gate rows and the
//     matching 16 up rows) and one K slice of KS values; the K slices of a
//     row group form a thread-block cluster (up to 8 CTAs along K);
//   * every load is issued up front with 16-byte cp.async: the CTA's raw
//     34-byte (Q8_0) / 18-byte (Q4_0) blocks -- before waiting on the
//     previous kernel (programmatic dependent launch), since weights never
//     change -- then its tokens' activations (split A = Ah + Al, two f16
//     planes) for the slice;
//   * the int8 values / nibbles are unpacked in registers to f16 *exactly*
//     (q is an integer of at most 8 bits) and multiplied on the tensor cores
//     (mma.sync m16n8k16, activation fragments by ldmatrix), so every product
//     is exact to about 2^-22; each block's f16 scale d is applied in f32 to
//     the 32-value block sum, i.e. y = sum_b d_b * sum_{k in b} a_k q_k, the
//     reference's f32 dot product up to summation order (linear_q8.wgsl /
//     linear_q4.wgsl, gguf.rs:116-174);
//   * the epilogue's operands ride in the same cp.async groups (bias and the
//     next norm's gain with the weights; the residual rows and the RMSNorm
//     partial sums with the activations), so the epilogue reads only shared
//     memory;
//   * 16 warps: 8 groups split the slice's blocks, each with one warp per
//     16-row tile; the groups' partial tiles are added through shared memory; every CTA of a cluster then pushes its tile into
//     a slot of the first CTA's shared memory (distributed shared memory),
//     which adds the slots in slice order (deterministic) and runs the fused
//     epilogue, one warp per token row and one lane per output column.
#include <cooperative_groups.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "t0b_internal.h"

namespace cg = cooperative_groups;

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kKGroups = 8;  // warps split a slice's blocks 8 ways and its 32 rows into 2 tiles of 16
constexpr int kRows = 32;        // weight rows (output columns) per CTA
constexpr int kMaxCluster = 8;   // K slices per row group (portable cluster size)
// the partial-tile region holds the f32 activation rows of a 256-wide K slice
static_assert(kKGroups * kRows == 256, "f32 staging of x32 calls relies on an [8][32] partial-tile region");
constexpr size_t kSmemCap = 200 * 1024;

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

struct SmallLayout {
  size_t wpitch, apitch, w_off, a_off, red_off, slot_off, eb_off, eg_off, ex_off, es_off, xs_off, bytes;
};

// Shared memory of one CTA: raw weights [32][KS/32 blocks], activations
// [2 planes][MT tokens][KS (+8 pad) halves], per-K-group partial tiles
// [8][32][MT] f32, cluster slots [cs][32][MT+1] f32 (slot z: the tile of K
// slice z; only the first CTA's slots are used), then the epilogue operands:
// bias [32], next-norm gain [32], residual rows [MT][32], RMSNorm partial
// sums [MT][nt].  With f32 input (x32, K slices of 256 only) the f32
// activation rows [MT][256] that the planes are split from sit in the
// per-K-group partial-tile region, which is the same size and unused until
// the MMAs are done.
__host__ __device__ inline SmallLayout small_layout(int qt, int KS, int MT, int cs, int nt, bool x32 = false) {
  SmallLayout L;
  L.wpitch = (size_t)(KS / 32) * (qt == 8 ? 34 : 18);  // multiple of 16: KS % 256 == 0
  L.apitch = (size_t)KS * 2 + 16;                       // 16-byte pad: conflict-free ldmatrix rows
  L.w_off = 0;
  L.a_off = L.w_off + kRows * L.wpitch;
  L.red_off = L.a_off + 2 * (size_t)MT * L.apitch;
  L.slot_off = L.red_off + (size_t)kKGroups * kRows * MT * 4;
  L.eb_off = L.slot_off + (size_t)cs * kRows * (MT + 1) * 4;
  L.eg_off = L.eb_off + kRows * 4;
  L.ex_off = L.eg_off + kRows * 4;
  L.es_off = L.ex_off + (size_t)MT * kRows * 4;
  L.bytes = L.es_off + (size_t)MT * nt * 4;
  L.xs_off = L.red_off;  // (x32) MT * KS * 4 == kKGroups * kRows * MT * 4 bytes at KS == 256
  (void)x32;
  return L;
}

T0B_DEV void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
T0B_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
T0B_DEV void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
T0B_DEV void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Activations: the f16 planes ah / al [M][K], or, when x32 is given, the
// f32 rows x32 [M][K], which each CTA splits into the planes of its K slice
// in shared memory (standalone calls: no separate split kernel).
template <int QT, int NT8>
__global__ void __launch_bounds__(kThreads) gemm_q_small_kernel(const __half *__restrict__ ah,
                                                                const __half *__restrict__ al,
                                                                const float *__restrict__ x32, int M, int K,
                                                                int KS, const uint8_t *__restrict__ W, Epi epi,
                                                                int *err) {
  constexpr int BPB = QInfo<QT>::bpb;
  constexpr int MT = 8 * NT8;
  constexpr int LD = MT + 1;
  extern __shared__ __align__(16) uint8_t smem[];
  const int cs = gridDim.z, z = blockIdx.z;  // cluster = the cs K slices of one row group
  const int nt = epi.ssq_in ? epi.ssq_in_nt : 0;
  const SmallLayout L = small_layout(QT, KS, MT, cs, nt, x32 != nullptr);
  uint8_t *wst = smem + L.w_off;
  uint8_t *act = smem + L.a_off;
  float *red = reinterpret_cast<float *>(smem + L.red_off);
  float *slots = reinterpret_cast<float *>(smem + L.slot_off);
  float *e_bias = reinterpret_cast<float *>(smem + L.eb_off);
  float *e_gain = reinterpret_cast<float *>(smem + L.eg_off);
  float *e_x = reinterpret_cast<float *>(smem + L.ex_off);
  float *e_ssq = reinterpret_cast<float *>(smem + L.es_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int m0 = blockIdx.y * MT;
  const size_t RB = (size_t)(K / 32) * BPB;
  const int KB = KS / 32;  // blocks in this CTA's slice
  const bool swiglu = epi.kind == EPI_SWIGLU, resid = epi.kind == EPI_RESID;
  const int n0 = blockIdx.x * kRows;  // first output column (PLAIN / RESID)
  const int f0 = blockIdx.x * 16;     // first hidden column (SWIGLU)
  if (cs > 1) cluster_arrive_relaxed();  // matched by the wait before the slot push

  // 1. constant operands (may be fetched while the previous kernel is still
  //    running): the raw weight blocks of the 32 rows for this K slice, the
  //    bias and the next norm's gain
  {
    // warp w stages rows w, w + 4, ...; lane q its 16-byte granules q, q + 32, ...
    const int gpr = (int)(L.wpitch / 16);  // granules per row: 17 (Q8_0) / 9 (Q4_0) per 256 values
    for (int r = warp; r < kRows; r += kWarps) {
      const int wrow = swiglu ? (r < 16 ? 0 : epi.F) + f0 + (r & 15) : n0 + r;
      const uint8_t *src = W + (size_t)wrow * RB + (size_t)z * L.wpitch;
      if (!T0B_CHECK(wrow < (swiglu ? 2 * epi.F : epi.N), err)) continue;
      for (int q = lane; q < gpr; q += 32) cp_async16(wst + r * L.wpitch + q * 16, src + q * 16);
    }
    if (threadIdx.x < kRows) {
      const int c = threadIdx.x;
      if (epi.bias)
        cp_async4(e_bias + c, epi.bias + (swiglu ? (c < 16 ? 0 : epi.F) + f0 + (c & 15) : n0 + c));
      else
        e_bias[c] = 0.0f;
      if (resid) cp_async4(e_gain + c, epi.gnext + n0 + c);
    }
    cp_async_commit();
  }
  // 2. operands written by earlier kernels: activations, residual rows and
  //    RMSNorm partial sums
  pdl_wait();
  {
    if (x32) {
      // f32 activation rows (token) by warp, 16-byte granules by lane
      float *xs = reinterpret_cast<float *>(smem + L.xs_off);
      for (int t = warp; t < MT; t += kWarps) {
        const int m = min(m0 + t, M - 1);  // rows past M duplicate a valid row; their outputs are dropped
        const float *src = x32 + (size_t)m * K + (size_t)z * KS;
        for (int q = lane; q < KS / 4; q += 32) cp_async16(xs + (size_t)t * KS + 4 * q, src + 4 * q);
      }
    } else {
      // activation rows (plane * MT + token) by warp, granules by lane
      const int gpt = KS / 8;  // 16-byte granules per token row per plane: a multiple of 32
      for (int row = warp; row < 2 * MT; row += kWarps) {
        const int pl = row >= MT, t = row - pl * MT;
        const int m = min(m0 + t, M - 1);  // rows past M duplicate a valid row; their outputs are dropped
        const __half *src = (pl ? al : ah) + (size_t)m * K + (size_t)z * KS;
        uint8_t *dst = act + (size_t)row * L.apitch;
        for (int q = lane; q < gpt; q += 32) cp_async16(dst + q * 16, src + q * 8);
      }
    }
    if (z == 0) {
      if (resid) {
        for (int i = threadIdx.x; i < MT * (kRows / 4); i += kThreads) {
          const int t = i / (kRows / 4), q = i % (kRows / 4);
          const int m = min(m0 + t, M - 1);
          cp_async16(e_x + t * kRows + 4 * q, epi.x + (size_t)m * epi.N + n0 + 4 * q);
        }
      }
      for (int i = threadIdx.x; i < MT * nt; i += kThreads) {
        const int t = i / nt, s = i - t * nt;
        const int m = min(m0 + t, M - 1);
        cp_async4(e_ssq + i, epi.ssq_in + (size_t)m * nt + s);
      }
    }
    cp_async_commit();
  }
  pdl_launch_dependents();
  cp_async_wait<0>();
  __syncthreads();
  if (x32) {  // split the f32 rows into the two planes, two values per thread and step
    const float *xs = reinterpret_cast<const float *>(smem + L.xs_off);
    for (int i = threadIdx.x; i < MT * KS / 2; i += kThreads) {
      const int t = i / (KS / 2), k2 = i - t * (KS / 2);
      const float2 v = *reinterpret_cast<const float2 *>(xs + (size_t)t * KS + 2 * k2);
      uint32_t hw, lw;
      split2(v.x, v.y, hw, lw);
      *reinterpret_cast<uint32_t *>(act + (size_t)t * L.apitch + 4 * k2) = hw;
      *reinterpret_cast<uint32_t *>(act + (size_t)(MT + t) * L.apitch + 4 * k2) = lw;
    }
    __syncthreads();
  }
  // RMSNorm row denominators, one thread per token (slot order); read by the
  // epilogue after the barriers below
  if (z == 0 && nt && threadIdx.x < MT) {
    float s = 0.0f;
    for (int i = 0; i < nt; ++i) s += e_ssq[threadIdx.x * nt + i];
    e_ssq[threadIdx.x * nt] = sqrtf(s / (float)epi.ssq_dim + 1e-8f);
  }

  // 3. warp (kg, rt): row tile rt (16 rows) over K group kg's blocks of the slice
  const int kg = warp % kKGroups, rt = warp / kKGroups;
  float acc[NT8][4];
#pragma unroll
  for (int j = 0; j < NT8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  const int bpw = KB / kKGroups;  // KB is a multiple of 8
  for (int bi = 0; bi < bpw; ++bi) {
    const int b = kg * bpw + bi;
    uint32_t a[2][4];
    const uint8_t *r0 = wst + (size_t)(rt * 16 + g) * L.wpitch + b * BPB;
    const uint8_t *r1 = r0 + 8 * L.wpitch;
    const float d0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(r0));
    const float d1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(r1));
    if (QT == 8) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        a[h][0] = i8x2_to_h2(*reinterpret_cast<const uint16_t *>(r0 + 2 + 16 * h + 2 * tig));
        a[h][1] = i8x2_to_h2(*reinterpret_cast<const uint16_t *>(r1 + 2 + 16 * h + 2 * tig));
        a[h][2] = i8x2_to_h2(*reinterpret_cast<const uint16_t *>(r0 + 2 + 16 * h + 8 + 2 * tig));
        a[h][3] = i8x2_to_h2(*reinterpret_cast<const uint16_t *>(r1 + 2 + 16 * h + 8 + 2 * tig));
      }
    } else {
      // byte j of a Q4_0 block holds value j (low nibble) and j + 16 (high)
      const uint32_t w00 = *reinterpret_cast<const uint16_t *>(r0 + 2 + 2 * tig);
      const uint32_t w10 = *reinterpret_cast<const uint16_t *>(r1 + 2 + 2 * tig);
      const uint32_t w01 = *reinterpret_cast<const uint16_t *>(r0 + 2 + 8 + 2 * tig);
      const uint32_t w11 = *reinterpret_cast<const uint16_t *>(r1 + 2 + 8 + 2 * tig);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        a[h][0] = nib2_to_h2(w00, h);
        a[h][1] = nib2_to_h2(w10, h);
        a[h][2] = nib2_to_h2(w01, h);
        a[h][3] = nib2_to_h2(w11, h);
      }
    }
#pragma unroll
    for (int j = 0; j < NT8; ++j) {
      // B fragments: matrix mi = lane / 8 covers k16 half mi / 2, k sub-block mi % 2
      const int mi = lane >> 3;
      const size_t roff = (size_t)(8 * j + (lane & 7)) * L.apitch + (size_t)(b * 32 + (mi >> 1) * 16 + (mi & 1) * 8) * 2;
      uint32_t bh[4], bl[4];
      ldsm_x4(act + roff, bh[0], bh[1], bh[2], bh[3]);
      ldsm_x4(act + (size_t)MT * L.apitch + roff, bl[0], bl[1], bl[2], bl[3]);
      float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mma16816(p0, p1, p2, p3, a[h][0], a[h][1], a[h][2], a[h][3], bh[2 * h], bh[2 * h + 1]);
        mma16816(p0, p1, p2, p3, a[h][0], a[h][1], a[h][2], a[h][3], bl[2 * h], bl[2 * h + 1]);
      }
      acc[j][0] += d0 * p0;
      acc[j][1] += d0 * p1;
      acc[j][2] += d1 * p2;
      acc[j][3] += d1 * p3;
    }
  }

  // 4. K groups' partial tiles (group order: deterministic) -> slot z of the
  //    first CTA of the cluster
  {
    float *mine = red + (size_t)kg * kRows * MT;
#pragma unroll
    for (int j = 0; j < NT8; ++j) {
      const int r = rt * 16 + g, t = 8 * j + 2 * tig;
      mine[r * MT + t] = acc[j][0];
      mine[r * MT + t + 1] = acc[j][1];
      mine[(r + 8) * MT + t] = acc[j][2];
      mine[(r + 8) * MT + t + 1] = acc[j][3];
    }
  }
  __syncthreads();
  float *slot = slots + (size_t)z * kRows * LD;
  if (cs > 1) {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA of the cluster has started
    slot = cg::this_cluster().map_shared_rank(slot, 0);
  }
  for (int i = threadIdx.x; i < kRows * MT; i += kThreads) {
    float v = red[i];
#pragma unroll
    for (int w = 1; w < kKGroups; ++w) v += red[(size_t)w * kRows * MT + i];
    slot[(i / MT) * LD + i % MT] = v;
  }
  if (cs > 1) {
    cluster_arrive_release();
    cluster_wait_acquire();
    if (z != 0) return;
    for (int i = threadIdx.x; i < kRows * MT; i += kThreads) {
      const int off = (i / MT) * LD + i % MT;
      float v = slots[off];
      for (int q = 1; q < cs; ++q) v += slots[(size_t)q * kRows * LD + off];
      slots[off] = v;
    }
  }
  __syncthreads();

  // 5. epilogue (first CTA of the cluster): warp w takes tokens w, w + 4, ...;
  //    lane c output column c (SWIGLU: lanes 0-15, gate row c and up row 16+c)
  const float *tile = slots;
  for (int t = warp; t < MT; t += kWarps) {
    const int m = m0 + t;
    if (m >= M) break;
    const float denom = nt ? e_ssq[t * nt] : 1.0f;
    const int c = lane;
    if (!T0B_CHECK(swiglu ? f0 + 16 <= epi.F : n0 + kRows <= epi.N, err)) break;
    if (swiglu) {
      if (c < 16) {
        const float gt = tile[c * LD + t] / denom + e_bias[c];
        const float up = tile[(16 + c) * LD + t] / denom + e_bias[16 + c];
        const float zv = gt / (1.0f + expf(-gt)) * up;
        const size_t o = (size_t)m * epi.F + f0 + c;
        if (epi.zh) {
          __half h, l;
          split_f16(zv, h, l);
          epi.zh[o] = h;
          epi.zl[o] = l;
        }
        if (epi.z32) epi.z32[o] = zv;
      }
    } else if (!resid) {
      const float yv = tile[c * LD + t] / denom + e_bias[c];
      const size_t o = (size_t)m * epi.ldy + n0 + c;
      if (epi.zh) {  // the split straight into f16 planes (the next GEMM's operand)
        __half h, l;
        split_f16(yv, h, l);
        epi.zh[o] = h;
        epi.zl[o] = l;
      } else {
        epi.y[o] = yv;
      }
    } else {
      const float xn = e_x[t * kRows + c] + (tile[c * LD + t] / denom + e_bias[c]);
      const size_t o = (size_t)m * epi.N + n0 + c;
      epi.x[o] = xn;
      __half h, l;
      split_f16(xn * e_gain[c], h, l);
      epi.xh[o] = h;
      epi.xl[o] = l;
      float ss = xn * xn;
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sh);
      if (c == 0 && T0B_CHECK((int)blockIdx.x < epi.ssq_out_nt, err)) epi.ssq_out[(size_t)m * epi.ssq_out_nt + blockIdx.x] = ss;
    }
  }
}

// K slice per CTA: K itself up to 1024 (one CTA per row group: a cluster's
// reduction through distributed shared memory cost more than the extra MMA
// work per CTA, 0.704 -> 0.655 ms per single forecast at K = 512; at
// K = 1024, M = 16 a GEMM 8.1 -> 6.0 us with the split pass, a SwiGLU MLP
// 24.1 -> 13.6 us), else the smallest multiple of 256 dividing K that leaves
// at most kMaxCluster slices.
int small_slice(int K) {
  if (K <= 1024) return K;
  const int c = K / 256;
  for (int d = (c + kMaxCluster - 1) / kMaxCluster; d <= c; ++d)
    if (c % d == 0) return 256 * d;
  return K;
}

template <int QT, int NT8>
cudaError_t launch_small_t(const __half *ah, const __half *al, const float *x32, int M, int K, int KS,
                           const uint8_t *W, const Epi &epi, int *err, cudaStream_t st) {
  constexpr int MT = 8 * NT8;
  const int cs = K / KS;
  const SmallLayout L = small_layout(QT, KS, MT, cs, epi.ssq_in ? epi.ssq_in_nt : 0, x32 != nullptr);
  auto kfn = gemm_q_small_kernel<QT, NT8>;
  cudaError_t e = t0b_smem_limit((const void *)kfn, L.bytes);
  if (e != cudaSuccess) return e;
  const int gx = epi.kind == EPI_SWIGLU ? epi.F / 16 : epi.N / kRows;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(gx, (M + MT - 1) / MT, cs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.bytes;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = cs;
  // may start while the previous kernel on the stream finishes; the kernel
  // waits (griddepcontrol.wait) before touching anything that kernel writes
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kfn, ah, al, x32, M, K, KS, W, epi, err);
}

// Tokens per CTA (8 * nt8) that fit in shared memory for this K; 0 if none.
template <int QT>
int small_nt8(int M, int K, const Epi &epi, bool x32 = false) {
  const int KS = small_slice(K);
  int nt8 = (M + 7) / 8 < 4 ? (M + 7) / 8 : 4;
  const int cs = K / KS, nt = epi.ssq_in ? epi.ssq_in_nt : 0;
  while (nt8 > 1 && small_layout(QT, KS, 8 * nt8, cs, nt, x32).bytes > kSmemCap) --nt8;
  return small_layout(QT, KS, 8 * nt8, cs, nt, x32).bytes > kSmemCap ? 0 : nt8;
}

template <int QT>
cudaError_t launch_small_q(const __half *ah, const __half *al, const float *x32, int M, int K, const uint8_t *W,
                           const Epi &epi, int *err, cudaStream_t st) {
  const int KS = small_slice(K);
  // tokens per CTA: up to 32, fewer when a wide slice would not fit in
  // shared memory
  const int nt8 = small_nt8<QT>(M, K, epi, x32 != nullptr);
  if (!nt8) return cudaErrorInvalidValue;
  switch (nt8) {
    case 1: return launch_small_t<QT, 1>(ah, al, x32, M, K, KS, W, epi, err, st);
    case 2: return launch_small_t<QT, 2>(ah, al, x32, M, K, KS, W, epi, err, st);
    case 3: return launch_small_t<QT, 3>(ah, al, x32, M, K, KS, W, epi, err, st);
    default: return launch_small_t<QT, 4>(ah, al, x32, M, K, KS, W, epi, err, st);
  }
}

}  // namespace

bool t0b_small_supports(int qt, int M, int K, const Epi &epi, bool x32) {
  if (M <= 0 || K <= 0 || K % 256) return false;
  if (x32 && small_slice(K) != 256) return false;  // the f32 rows are staged in the 256-wide partial-tile region
  return (qt == 8 ? small_nt8<8>(M, K, epi, x32) : small_nt8<4>(M, K, epi, x32)) > 0;
}

// Host entry.  qt: 8 = Q8_0, 4 = Q4_0.  Requires K % 256 == 0 and the output
// column count (N, or F for SWIGLU) a multiple of 32 (16 for SWIGLU).
cudaError_t t0b_launch_gemm_small(int qt, const __half *ah, const __half *al, int M, int K, const uint8_t *W,
                                  const Epi &epi, int *err, cudaStream_t st, const float *x32) {
  if (M <= 0 || K <= 0 || K % 256) return cudaErrorInvalidValue;
  if (x32 && small_slice(K) != 256) return cudaErrorInvalidValue;
  return qt == 8 ? launch_small_q<8>(ah, al, x32, M, K, W, epi, err, st)
                 : launch_small_q<4>(ah, al, x32, M, K, W, epi, err, st);
}
