// epilogue.cuh -- fused GEMM epilogues shared by the small-M (mma.sync) and
// large-M (tcgen05) dequant-GEMM paths.
//
// A thread owns one output row m and a run of consecutive columns.  The
// accumulator it receives is sum_k A'[m,k] * W[n,k] where A' is the A
// operand as stored (for the RMSNorm-fused GEMMs A' = x * g, the row's
// 1/sqrt(mean(x^2)+eps) factor is applied here: rmsnorm(x)*g . W^T ==
// (x*g . W^T) / sqrt(mean(x^2)+eps), ops.rs:12-17).
#pragma once

#include "common.cuh"

enum : int { EPI_PLAIN = 0, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_QKV = 4 };

struct Epi {
  int kind;
  int M, N;
  const float *bias;  // [N] (SWIGLU: [2F], gate then up)
  // optional fused RMSNorm row scale: partial sums of squares of the
  // un-normalised row, ssq_in[m * ssq_in_nt + slot], over ssq_dim columns
  const float *ssq_in;
  int ssq_in_nt, ssq_dim;
  // EPI_PLAIN: y [M, ldy] = acc / row denominator + bias (reduce_add: y +=
  // that instead; tensor-core kernel only).  Small-M kernel with zh set: that
  // value split into f16 planes zh / zl [M, ldy] instead of y.
  float *y;
  int ldy;
  int reduce_add;
  // EPI_RESID: x[m, n] += acc + bias (f32 residual stream, in place); then
  // x*gnext split into f16 (xh, xl) for the next RMSNorm-fused GEMM and the
  // sum of x^2 over this thread's columns written to ssq_out[m*nt + slot].
  float *x;
  const float *gnext;
  __half *xh, *xl;
  float *ssq_out;
  int ssq_out_nt;
  // EPI_SWIGLU: z = silu(gate) * up over F columns (ops.rs:49-62), split to
  // (zh, zl) f16 and optionally written as f32 (z32).
  int F;
  __half *zh, *zl;
  float *z32;
  // EPI_QKV (tensor-core kernel, head_dim 64, TIME layers): the wQKV output
  // y (q | k | v, E columns each) leaves as f16 (hi, lo) planes in zh / zl
  // [M][F = 3E] with q and k already multiplied by their QK-norm gains
  // (qn / kn) and rotated by the xpos RoPE of the token's patch position
  // (m mod p, transposed compact table rope_t [128][p]); v is only split.  The QK-norm
  // itself, 1/sqrt(mean(y^2) + 1e-8) of each (token, head) of q and k, is a
  // per-row scale of the attention scores: the sums of squares of y go to
  // ssq_qk[m * 2H + h] (q) and ssq_qk[m * 2H + H + h] (k).  RoPE is linear,
  // so rope(g * y * s) == s * rope(g * y) (ops.rs:132-142, 175-177).
  const float *qn, *kn, *rope_t;
  float *ssq_qk;
  int p, E, H;
};

// RoPE on 16 consecutive dims 16cg..16cg+15 (8 pairs) of a 64-dim head with
// 16-byte loads from the compact table row `tab` [128]: cos[32], sin[32] per
// rotated pair, scale[32] (q side), 1/scale[32] (k side) per dim mod 32
// (ops.rs:132-142: x0' = (x0 c - x1 s) scale, x1' = (x1 c + x0 s) scale).
T0B_DEV void rope16(float *x, const float *tab, int cg, bool kside) {
  const float4 *t4 = reinterpret_cast<const float4 *>(tab);
  const float4 c0 = t4[2 * cg], c1 = t4[2 * cg + 1], n0 = t4[8 + 2 * cg], n1 = t4[8 + 2 * cg + 1];
  const float4 *sp = t4 + (kside ? 24 : 16) + ((16 * cg) & 31) / 4;
  const float4 s0 = sp[0], s1 = sp[1], s2 = sp[2], s3 = sp[3];
  const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float sn[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
  const float sv[16] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w,
                        s2.x, s2.y, s2.z, s2.w, s3.x, s3.y, s3.z, s3.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a0 = x[2 * i], a1 = x[2 * i + 1];
    x[2 * i] = a0 * cs[i] * sv[2 * i] + (-a1) * sn[i] * sv[2 * i];
    x[2 * i + 1] = a1 * cs[i] * sv[2 * i + 1] + a0 * sn[i] * sv[2 * i + 1];
  }
}

// The same rotation with the table transposed, rope_t [128][p] (entry j of
// position pos at j * p + pos): the lanes of a warp hold consecutive tokens,
// so each entry is one coalesced load across the warp.
T0B_DEV void rope16_t(float *x, const float *tabt, int p, int pos, int cg, bool kside) {
  const float *ct = tabt + (size_t)(8 * cg) * p + pos, *st = ct + (size_t)32 * p;
  const float *sv = tabt + (size_t)((kside ? 96 : 64) + ((16 * cg) & 31)) * p + pos;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float c = ct[(size_t)i * p], sn = st[(size_t)i * p];
    const float s0 = sv[(size_t)(2 * i) * p], s1 = sv[(size_t)(2 * i + 1) * p];
    const float a0 = x[2 * i], a1 = x[2 * i + 1];
    x[2 * i] = a0 * c * s0 + (-a1) * sn * s0;
    x[2 * i + 1] = a1 * c * s1 + a0 * sn * s1;
  }
}

T0B_DEV float epi_row_denom(const Epi &e, int m) {
  if (!e.ssq_in) return 1.0f;
  float s = 0.0f;
  for (int i = 0; i < e.ssq_in_nt; ++i) s += e.ssq_in[(size_t)m * e.ssq_in_nt + i];
  return sqrtf(s / (float)e.ssq_dim + 1e-8f);
}

T0B_DEV void store_split(__half *hi, __half *lo, size_t off, const float *v, int n) {
  for (int i = 0; i < n; i += 2) {
    __half h0, l0, h1, l1;
    split_f16(v[i], h0, l0);
    split_f16(v[i + 1], h1, l1);
    *reinterpret_cast<__half2 *>(hi + off + i) = __halves2half2(h0, h1);
    *reinterpret_cast<__half2 *>(lo + off + i) = __halves2half2(l0, l1);
  }
}

// 32 columns n0..n0+31 of row m, kinds PLAIN and RESID.  Returns the sum of
// squares of the new residual row values (RESID) or 0.
T0B_DEV float epi_cols32(const Epi &e, int m, int n0, float *v, float denom) {
  if (e.kind == EPI_PLAIN) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = v[i] / denom + (e.bias ? e.bias[n0 + i] : 0.0f);
    float4 *dst = reinterpret_cast<float4 *>(e.y + (size_t)m * e.ldy + n0);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    return 0.0f;
  }
  // EPI_RESID
  float *xr = e.x + (size_t)m * e.N + n0;
  float ss = 0.0f;
  float g[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 xo = reinterpret_cast<const float4 *>(xr)[i];
    float xs[4] = {xo.x, xo.y, xo.z, xo.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int c = 4 * i + j;
      float a = v[c] / denom + e.bias[n0 + c];
      float xn = xs[j] + a;
      v[c] = xn;
      ss += xn * xn;
      g[c] = xn * e.gnext[n0 + c];
    }
    reinterpret_cast<float4 *>(xr)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
  store_split(e.xh, e.xl, (size_t)m * e.N + n0, g, 32);
  return ss;
}

// SwiGLU on NF features: gate columns f0..f0+NF-1 and the matching up
// columns (ops.rs:49-62).
template <int NF>
T0B_DEV void epi_swiglu(const Epi &e, int m, int f0, const float *gacc, const float *uacc, float denom) {
  float z[NF];
#pragma unroll
  for (int i = 0; i < NF; ++i) {
    float g = gacc[i] / denom + (e.bias ? e.bias[f0 + i] : 0.0f);
    float u = uacc[i] / denom + (e.bias ? e.bias[e.F + f0 + i] : 0.0f);
    z[i] = g / (1.0f + expf(-g)) * u;
  }
  if (e.zh) store_split(e.zh, e.zl, (size_t)m * e.F + f0, z, NF);
  if (e.z32) {
    float4 *dst = reinterpret_cast<float4 *>(e.z32 + (size_t)m * e.F + f0);
#pragma unroll
    for (int i = 0; i < NF / 4; ++i) dst[i] = make_float4(z[4 * i], z[4 * i + 1], z[4 * i + 2], z[4 * i + 3]);
  }
}
