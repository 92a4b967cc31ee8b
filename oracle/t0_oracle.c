/*
 * t0_oracle.c -- TEST INFRASTRUCTURE: plain-C CPU restatement of the
 * reference engine `t0-core` (idle-intelligence/t0-web, crates/t0-core) for
 * the quantized t0-alpha forecast path.  It exists to check the CUDA product
 * and to time the reference algorithm on host cores; nothing in the product
 * links it.  See t0_oracle.h for what pins it to the reference.
 *
 * Arithmetic follows the reference in f32 (weights dequantized to f32 at
 * load, weights.rs:151-163).  Compile with -ffp-contract=off and without
 * fast-math: the quantizers depend on exact f32 products and roundings.
 * GEMM dot products use 16 fixed partial sums (matrixmultiply's summation
 * order is not pinned by any reference test; only ulps differ).
 */
#define _GNU_SOURCE
#include "t0_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define QK 32
#define MAX_HORIZON 1024 /* model.rs:26 */
#define BLOCK_MASK (-1.0e9f) /* mask.rs:8 */

enum { MASK_VALID = 0, MASK_PAD = 1, MASK_MISSING = 2, MASK_WITHHELD = 4 }; /* data.rs:7-13 */
enum { VT_TARGET = 0, VT_FUTURE = 2 };                                    /* data.rs:15-20 */

/* ------------------------------------------------------------------------ */
/* f16 <-> f32.  IEEE binary16 with round-to-nearest-even on the way down,   */
/* subnormals kept, overflow to infinity, NaN kept quiet.  This is the       */
/* conversion `half 2.7.1` (Cargo.lock) performs for f16::from_f32/to_f32.   */
/* ------------------------------------------------------------------------ */
uint16_t o_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp8 = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp8 == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x0200u | (man >> 13) : 0));
  int e = (int)exp8 - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    int shift = 14 - e; /* drop this many bits of the 24-bit significand */
    if (shift > 24) return (uint16_t)sign;
    uint32_t m = man | 0x800000u;
    uint32_t h = m >> shift;
    uint32_t rb = 1u << (shift - 1);
    /* round half to even: round bit set and (sticky bits or odd result) */
    if ((m & rb) && (m & (3u * rb - 1u))) h += 1;
    return (uint16_t)(sign | h);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  uint32_t rb = 0x1000u;
  if ((man & rb) && (man & (3u * rb - 1u))) h += 1; /* carry may bump exponent: correct */
  return (uint16_t)h;
}

float o_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t x;
  if (e == 0x1f) {
    x = sign | 0x7f800000u | (m << 13);
  } else if (e == 0) {
    if (m == 0) {
      x = sign;
    } else { /* subnormal: value = m * 2^-24 */
      float v = (float)m * (1.0f / 16777216.0f);
      memcpy(&x, &v, 4);
      x |= sign;
    }
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/* ------------------------------------------------------------------------ */
/* Q8_0 / Q4_0 block codecs, gguf.rs:100-174                                  */
/* ------------------------------------------------------------------------ */
/* gguf.rs:100-114: d = amax/127, id = 1/d (0 if d == 0),
 * q = clamp(round(x*id), -128, 127) with round = half away from zero. */
void o_quantize_q8_0(const float *x, size_t n, uint8_t *out) {
  for (size_t b = 0; b < n / QK; ++b) {
    const float *blk = x + b * QK;
    float amax = 0.0f;
    for (int i = 0; i < QK; ++i) amax = fmaxf(amax, fabsf(blk[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = o_f32_to_f16(d);
    uint8_t *o = out + b * (2 + QK);
    o[0] = (uint8_t)(dh & 0xff);
    o[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < QK; ++i) {
      float q = roundf(blk[i] * id);
      if (q < -128.0f) q = -128.0f;
      if (q > 127.0f) q = 127.0f;
      o[2 + i] = (uint8_t)(int8_t)q;
    }
  }
}

/* gguf.rs:116-126 */
void o_dequantize_q8_0(const uint8_t *bytes, size_t n, float *out) {
  for (size_t b = 0; b < n / QK; ++b) {
    const uint8_t *blk = bytes + b * (2 + QK);
    float d = o_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    for (int i = 0; i < QK; ++i) out[b * QK + i] = d * (float)(int8_t)blk[2 + i];
  }
}

/* gguf.rs:133-157: max = signed value of largest |x| (first wins, strict >),
 * d = max/-8, id = 1/d, nibble = clamp(floor(x*id + 8.5), 0, 15);
 * byte j = nib(x_j) | nib(x_{j+16}) << 4. */
void o_quantize_q4_0(const float *x, size_t n, uint8_t *out) {
  for (size_t b = 0; b < n / QK; ++b) {
    const float *blk = x + b * QK;
    float amax = 0.0f, mx = 0.0f;
    for (int i = 0; i < QK; ++i) {
      if (fabsf(blk[i]) > amax) {
        amax = fabsf(blk[i]);
        mx = blk[i];
      }
    }
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = o_f32_to_f16(d);
    uint8_t *o = out + b * (2 + QK / 2);
    o[0] = (uint8_t)(dh & 0xff);
    o[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < QK / 2; ++j) {
      float x0 = blk[j] * id;
      float x1 = blk[j + QK / 2] * id;
      int i0 = (int)floorf(x0 + 8.5f);
      int i1 = (int)floorf(x1 + 8.5f);
      i0 = i0 < 0 ? 0 : (i0 > 15 ? 15 : i0);
      i1 = i1 < 0 ? 0 : (i1 > 15 ? 15 : i1);
      o[2 + j] = (uint8_t)(i0 | (i1 << 4));
    }
  }
}

/* gguf.rs:159-174 */
void o_dequantize_q4_0(const uint8_t *bytes, size_t n, float *out) {
  for (size_t b = 0; b < n / QK; ++b) {
    const uint8_t *blk = bytes + b * (2 + QK / 2);
    float d = o_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    for (int j = 0; j < QK / 2; ++j) {
      uint8_t byte = blk[2 + j];
      out[b * QK + j] = d * ((float)(byte & 0x0f) - 8.0f);
      out[b * QK + j + QK / 2] = d * ((float)(byte >> 4) - 8.0f);
    }
  }
}

/* gguf.rs:61-70 */
size_t o_row_bytes(int type, size_t n) {
  switch (type) {
    case O_F32: return n * 4;
    case O_F16: return n * 2;
    case O_Q4_0: return (n / QK) * (2 + QK / 2);
    case O_Q8_0: return (n / QK) * (2 + QK);
    default: return 0;
  }
}

static void dequantize_for(int type, const uint8_t *bytes, size_t n, float *out) {
  switch (type) { /* gguf.rs:213-226 */
    case O_F32:
      memcpy(out, bytes, n * 4);
      break;
    case O_F16:
      for (size_t i = 0; i < n; ++i) out[i] = o_f16_to_f32((uint16_t)(bytes[2 * i] | (bytes[2 * i + 1] << 8)));
      break;
    case O_Q8_0: o_dequantize_q8_0(bytes, n, out); break;
    case O_Q4_0: o_dequantize_q4_0(bytes, n, out); break;
  }
}

static void quantize_for(int type, const float *x, size_t n, uint8_t *out) {
  switch (type) { /* gguf.rs:192-211 */
    case O_F32: memcpy(out, x, n * 4); break;
    case O_F16:
      for (size_t i = 0; i < n; ++i) {
        uint16_t h = o_f32_to_f16(x[i]);
        out[2 * i] = (uint8_t)(h & 0xff);
        out[2 * i + 1] = (uint8_t)(h >> 8);
      }
      break;
    case O_Q8_0: o_quantize_q8_0(x, n, out); break;
    case O_Q4_0: o_quantize_q4_0(x, n, out); break;
  }
}

void o_free(void *p) { free(p); }

/* ------------------------------------------------------------------------ */
/* GGUF v3 subset writer / reader, gguf.rs:228-405                            */
/* ------------------------------------------------------------------------ */
typedef struct {
  uint8_t *p;
  size_t len, cap;
} buf_t;

static void buf_put(buf_t *b, const void *src, size_t n) {
  if (b->len + n > b->cap) {
    size_t c = b->cap ? b->cap : 4096;
    while (c < b->len + n) c *= 2;
    b->p = (uint8_t *)realloc(b->p, c);
    b->cap = c;
  }
  memcpy(b->p + b->len, src, n);
  b->len += n;
}
static void put_u8(buf_t *b, uint8_t v) { buf_put(b, &v, 1); }
static void put_u32(buf_t *b, uint32_t v) {
  uint8_t t[4] = {(uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24)};
  buf_put(b, t, 4);
}
static void put_u64(buf_t *b, uint64_t v) {
  put_u32(b, (uint32_t)v);
  put_u32(b, (uint32_t)(v >> 32));
}
static void put_f32(buf_t *b, float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  put_u32(b, u);
}
static void put_str(buf_t *b, const char *s) { /* gguf.rs:228-232 */
  put_u64(b, (uint64_t)strlen(s));
  buf_put(b, s, strlen(s));
}

/* weights.rs:32-37 */
static int is_quantizable(const char *name) {
  return strstr(name, ".attention.wQKV.weight") || strstr(name, ".attention.wO.weight") ||
         strstr(name, ".mlp.0.weight") || strstr(name, ".mlp.2.weight");
}

static int cmp_idx_names(const void *a, const void *b, void *ctx) {
  const char *const *names = (const char *const *)ctx;
  return strcmp(names[*(const int *)a], names[*(const int *)b]);
}

/* weights.rs:187-227 (names sorted, 2-D && quantizable -> big type, else
 * F16; metadata keys 208-220) + gguf.rs:299-345 (offsets 32-aligned relative
 * to a data blob that starts right after the tensor infos, no pad before). */
int o_export_gguf(int n, const char *const *names, const int *ndims, const int64_t *shapes,
                  const float *const *data, int big_type, const o_config *cfg, uint8_t **out,
                  size_t *out_len) {
  int *order = (int *)malloc(sizeof(int) * (size_t)n);
  for (int i = 0; i < n; ++i) order[i] = i;
  qsort_r(order, (size_t)n, sizeof(int), cmp_idx_names, (void *)names);

  buf_t b = {0};
  buf_put(&b, "GGUF", 4);
  put_u32(&b, 3);
  put_u64(&b, (uint64_t)n);
  put_u64(&b, 11);
#define KEY_U32(k, v) (put_str(&b, k), put_u32(&b, 4), put_u32(&b, (uint32_t)(v)))
  KEY_U32("t0.embed_dim", cfg->embed_dim);
  KEY_U32("t0.num_layers", cfg->num_layers);
  KEY_U32("t0.num_heads", cfg->num_heads);
  KEY_U32("t0.mlp_hidden_dim", cfg->mlp_hidden_dim);
  KEY_U32("t0.patch_size", cfg->patch_size);
  KEY_U32("t0.group_every_n", cfg->group_every_n);
#undef KEY_U32
  put_str(&b, "t0.dropout");
  put_u32(&b, 6);
  put_f32(&b, cfg->dropout);
  put_str(&b, "t0.quantile_levels");
  put_u32(&b, 9);
  put_u32(&b, 6);
  put_u64(&b, (uint64_t)cfg->n_quantiles);
  for (int i = 0; i < cfg->n_quantiles; ++i) put_f32(&b, cfg->quantile_levels[i]);
  put_str(&b, "t0.scaler_use_arcsinh");
  put_u32(&b, 7);
  put_u8(&b, cfg->scaler_use_arcsinh ? 1 : 0);
  put_str(&b, "t0.scaler_eps");
  put_u32(&b, 6);
  put_f32(&b, cfg->scaler_eps);
  put_str(&b, "t0.scaler_eps_mode");
  put_u32(&b, 8);
  put_str(&b, cfg->variance_offset ? "variance_offset" : "std_clamp");

  int *types = (int *)malloc(sizeof(int) * (size_t)n);
  uint64_t *offs = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)n);
  size_t *nbytes = (size_t *)malloc(sizeof(size_t) * (size_t)n);
  uint64_t cursor = 0;
  for (int oi = 0; oi < n; ++oi) {
    int i = order[oi];
    size_t ne = (size_t)shapes[2 * i] * (size_t)(ndims[i] == 2 ? shapes[2 * i + 1] : 1);
    types[i] = (ndims[i] == 2 && is_quantizable(names[i])) ? big_type : O_F16;
    nbytes[i] = o_row_bytes(types[i], ne);
    offs[i] = cursor;
    cursor += nbytes[i];
    if (cursor % 32) cursor += 32 - cursor % 32;
  }
  for (int oi = 0; oi < n; ++oi) {
    int i = order[oi];
    put_str(&b, names[i]);
    put_u32(&b, (uint32_t)ndims[i]);
    for (int d = ndims[i] - 1; d >= 0; --d) put_u64(&b, (uint64_t)shapes[2 * i + d]);
    put_u32(&b, (uint32_t)types[i]);
    put_u64(&b, offs[i]);
  }
  uint64_t pos = 0;
  for (int oi = 0; oi < n; ++oi) {
    int i = order[oi];
    while (pos < offs[i]) {
      put_u8(&b, 0);
      ++pos;
    }
    size_t ne = (size_t)shapes[2 * i] * (size_t)(ndims[i] == 2 ? shapes[2 * i + 1] : 1);
    uint8_t *tmp = (uint8_t *)malloc(nbytes[i] ? nbytes[i] : 1);
    quantize_for(types[i], data[i], ne, tmp);
    buf_put(&b, tmp, nbytes[i]);
    free(tmp);
    pos = offs[i] + nbytes[i];
  }
  free(order);
  free(types);
  free(offs);
  free(nbytes);
  *out = b.p;
  *out_len = b.len;
  return 0;
}

typedef struct {
  const uint8_t *p;
  size_t len, pos;
  int err;
} rd_t;

static int rd(rd_t *r, void *dst, size_t n) {
  if (r->err || r->pos + n > r->len) {
    r->err = 1;
    memset(dst, 0, n);
    return -1;
  }
  memcpy(dst, r->p + r->pos, n);
  r->pos += n;
  return 0;
}
static uint32_t rd_u32(rd_t *r) {
  uint8_t t[4];
  rd(r, t, 4);
  return (uint32_t)t[0] | ((uint32_t)t[1] << 8) | ((uint32_t)t[2] << 16) | ((uint32_t)t[3] << 24);
}
static uint64_t rd_u64(rd_t *r) {
  uint64_t lo = rd_u32(r);
  return lo | ((uint64_t)rd_u32(r) << 32);
}
static float rd_f32(rd_t *r) {
  uint32_t u = rd_u32(r);
  float f;
  memcpy(&f, &u, 4);
  return f;
}

typedef struct {
  char name[128];
  int ndim;
  int64_t shape[4]; /* row-major */
  int type;
  uint64_t offset;
  const uint8_t *bytes;
  size_t nbytes;
  float *f32; /* dequantized (weights.rs:151-163) */
} o_tensor;

struct o_model {
  o_config cfg;
  int n_tensors;
  o_tensor *tensors;
  uint8_t *file; /* private copy of the GGUF bytes */
  size_t file_len;
};

static const o_tensor *find_tensor(const o_model *m, const char *name) {
  for (int i = 0; i < m->n_tensors; ++i)
    if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
  return NULL;
}

/* gguf.rs:347-405 + weights.rs:69-112 */
int o_model_load_gguf(const uint8_t *bytes, size_t len, o_model **out) {
  *out = NULL;
  o_model *m = (o_model *)calloc(1, sizeof(o_model));
  m->file = (uint8_t *)malloc(len ? len : 1);
  memcpy(m->file, bytes, len);
  m->file_len = len;
  rd_t r = {m->file, len, 0, 0};
  char magic[4];
  rd(&r, magic, 4);
  if (r.err || memcmp(magic, "GGUF", 4) != 0) goto fail; /* gguf.rs:350-352 */
  if (rd_u32(&r) != 3) goto fail;                      /* gguf.rs:353-356 */
  uint64_t n_t = rd_u64(&r), n_kv = rd_u64(&r);
  if (r.err || n_t > 100000 || n_kv > 100000) goto fail;
  /* defaults of config_from_gguf_metadata for optional keys */
  o_config *c = &m->cfg;
  int have[6] = {0}, have_q = 0;
  c->dropout = 0.0f;
  c->scaler_use_arcsinh = 1;
  c->scaler_eps = 0.1f;
  c->variance_offset = 1;
  for (uint64_t i = 0; i < n_kv && !r.err; ++i) {
    uint64_t kl = rd_u64(&r);
    if (kl > 4096) goto fail;
    char key[4097];
    rd(&r, key, kl);
    key[kl] = 0;
    uint32_t ty = rd_u32(&r);
    if (ty == 4) {
      uint32_t v = rd_u32(&r);
      static const char *ks[6] = {"t0.embed_dim", "t0.num_layers", "t0.num_heads", "t0.mlp_hidden_dim",
                                  "t0.patch_size", "t0.group_every_n"};
      int *dst[6] = {&c->embed_dim, &c->num_layers, &c->num_heads, &c->mlp_hidden_dim, &c->patch_size,
                     &c->group_every_n};
      for (int k = 0; k < 6; ++k)
        if (!strcmp(key, ks[k])) {
          *dst[k] = (int)v;
          have[k] = 1;
        }
    } else if (ty == 6) {
      float v = rd_f32(&r);
      if (!strcmp(key, "t0.dropout")) c->dropout = v;
      if (!strcmp(key, "t0.scaler_eps")) c->scaler_eps = v;
    } else if (ty == 7) {
      uint8_t v;
      rd(&r, &v, 1);
      if (!strcmp(key, "t0.scaler_use_arcsinh")) c->scaler_use_arcsinh = v != 0;
    } else if (ty == 8) {
      uint64_t sl = rd_u64(&r);
      if (sl > (1u << 20) || r.pos + sl > len) goto fail;
      char *s = (char *)malloc(sl + 1);
      rd(&r, s, sl);
      s[sl] = 0;
      if (!strcmp(key, "t0.scaler_eps_mode")) c->variance_offset = strcmp(s, "std_clamp") != 0;
      free(s);
    } else if (ty == 9) {
      uint32_t et = rd_u32(&r);
      uint64_t al = rd_u64(&r);
      if (et != 6 || al > (1u << 24)) goto fail; /* gguf.rs:281-283 */
      for (uint64_t k = 0; k < al; ++k) {
        float v = rd_f32(&r);
        if (!strcmp(key, "t0.quantile_levels") && k < 32) c->quantile_levels[k] = v;
      }
      if (!strcmp(key, "t0.quantile_levels")) {
        if (al > 32) goto fail;
        c->n_quantiles = (int)al;
        have_q = 1;
      }
    } else {
      goto fail; /* gguf.rs:290 */
    }
  }
  for (int k = 0; k < 6; ++k)
    if (!have[k]) goto fail; /* weights.rs:70-75 */
  if (!have_q) goto fail;    /* weights.rs:94-97 */

  m->n_tensors = (int)n_t;
  m->tensors = (o_tensor *)calloc(n_t ? n_t : 1, sizeof(o_tensor));
  for (uint64_t i = 0; i < n_t; ++i) {
    o_tensor *t = &m->tensors[i];
    uint64_t nl = rd_u64(&r);
    if (nl >= sizeof(t->name)) goto fail;
    rd(&r, t->name, nl);
    t->name[nl] = 0;
    uint32_t nd = rd_u32(&r);
    if (nd < 1 || nd > 4) goto fail;
    t->ndim = (int)nd;
    for (uint32_t d = 0; d < nd; ++d) t->shape[nd - 1 - d] = (int64_t)rd_u64(&r); /* reversed */
    uint32_t ty = rd_u32(&r);
    if (ty != O_F32 && ty != O_F16 && ty != O_Q4_0 && ty != O_Q8_0) goto fail; /* gguf.rs:41-49 */
    t->type = (int)ty;
    t->offset = rd_u64(&r);
  }
  if (r.err) goto fail;
  size_t blob = r.pos; /* gguf.rs:387-389: blob starts right after the infos */
  for (uint64_t i = 0; i < n_t; ++i) {
    o_tensor *t = &m->tensors[i];
    size_t ne = 1;
    for (int d = 0; d < t->ndim; ++d) ne *= (size_t)t->shape[d];
    if ((t->type == O_Q4_0 || t->type == O_Q8_0) && ne % QK) goto fail;
    t->nbytes = o_row_bytes(t->type, ne);
    if (t->offset > len - blob || t->nbytes > len - blob - t->offset) goto fail; /* gguf.rs:397-399 */
    t->bytes = m->file + blob + t->offset;
    t->f32 = (float *)malloc(ne * sizeof(float));
    dequantize_for(t->type, t->bytes, ne, t->f32);
  }
  *out = m;
  return 0;
fail:
  o_model_free(m);
  return -1;
}

void o_model_free(o_model *m) {
  if (!m) return;
  for (int i = 0; i < m->n_tensors; ++i) free(m->tensors[i].f32);
  free(m->tensors);
  free(m->file);
  free(m);
}

int o_model_config(const o_model *m, o_config *out) {
  *out = m->cfg;
  return 0;
}

int o_model_tensor(const o_model *m, const char *name, int *type, int64_t *rows, int64_t *cols,
                   const uint8_t **bytes, size_t *nbytes) {
  const o_tensor *t = find_tensor(m, name);
  if (!t) return -1;
  *type = t->type;
  *rows = t->shape[0];
  *cols = t->ndim > 1 ? t->shape[1] : 1;
  *bytes = t->bytes;
  *nbytes = t->nbytes;
  return 0;
}

/* ------------------------------------------------------------------------ */
/* ops.rs primitives (f32)                                                    */
/* ------------------------------------------------------------------------ */
static float dot_f32(const float *a, const float *b, int K) {
  float acc[16] = {0};
  int k = 0;
  for (; k + 16 <= K; k += 16)
    for (int j = 0; j < 16; ++j) acc[j] += a[k + j] * b[k + j];
  float tail = 0.0f;
  for (; k < K; ++k) tail += a[k] * b[k];
  for (int s = 8; s >= 1; s >>= 1)
    for (int j = 0; j < s; ++j) acc[j] += acc[j + s];
  return acc[0] + tail;
}

/* Operand-rounding emulation for precision studies of a tensor-core GEMM:
 * 0 = exact f32 (the reference), 1 = x and w rounded to f16, 2 = x only,
 * 3 = w only, 4 = x and w rounded to bf16.  Applies to the four quantized
 * matmuls only.  Default 0; set by o_set_gemm_emulation. */
static int g_emul = 0;
void o_set_gemm_emulation(int mode) { g_emul = mode; }
static float round_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  memcpy(&f, &u, 4);
  return f;
}
static float emul(float v, int is_w) {
  int m = g_emul;
  if (m == 1 || (m == 2 && !is_w) || (m == 3 && is_w)) return o_f16_to_f32(o_f32_to_f16(v));
  if (m == 4) return round_bf16(v);
  return v;
}

/* ops.rs:40-42: y = x . w^T + b.  w is [N, K]. */
static void linear(const float *x, int M, int K, const float *w, const float *b, int N, float *y);
static void linear_q(const float *x, int M, int K, const float *w, const float *b, int N, float *y) {
  if (!g_emul) {
    linear(x, M, K, w, b, N, y);
    return;
  }
  if (g_emul >= 5) { /* split-f16: x = xh + xl, w = wh + wl; y = xh.wh + xh.wl + xl.wh */
    float sx = g_emul == 6 ? 256.0f : 1.0f, sw = g_emul == 6 ? 1024.0f : 1.0f;
    float *xh = (float *)malloc(sizeof(float) * (size_t)M * K), *xl = (float *)malloc(sizeof(float) * (size_t)M * K);
    float *wh = (float *)malloc(sizeof(float) * (size_t)N * K), *wl = (float *)malloc(sizeof(float) * (size_t)N * K);
    for (size_t i = 0; i < (size_t)M * K; ++i) {
      float v = x[i] * sx;
      xh[i] = o_f16_to_f32(o_f32_to_f16(v));
      xl[i] = o_f16_to_f32(o_f32_to_f16(v - xh[i]));
    }
    for (size_t i = 0; i < (size_t)N * K; ++i) {
      float v = w[i] * sw;
      wh[i] = o_f16_to_f32(o_f32_to_f16(v));
      wl[i] = o_f16_to_f32(o_f32_to_f16(v - wh[i]));
    }
    for (int n = 0; n < N; ++n)
      for (int m = 0; m < M; ++m) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) {
          acc += xh[(size_t)m * K + k] * wh[(size_t)n * K + k];
          acc += xh[(size_t)m * K + k] * wl[(size_t)n * K + k];
          acc += xl[(size_t)m * K + k] * wh[(size_t)n * K + k];
        }
        y[(size_t)m * N + n] = acc / (sx * sw) + b[n];
      }
    free(xh); free(xl); free(wh); free(wl);
    return;
  }
  float *xe = (float *)malloc(sizeof(float) * (size_t)M * K);
  float *we = (float *)malloc(sizeof(float) * (size_t)N * K);
  for (size_t i = 0; i < (size_t)M * K; ++i) xe[i] = emul(x[i], 0);
  for (size_t i = 0; i < (size_t)N * K; ++i) we[i] = emul(w[i], 1);
  linear(xe, M, K, we, b, N, y);
  free(xe);
  free(we);
}
static void linear(const float *x, int M, int K, const float *w, const float *b, int N, float *y) {
  for (int n = 0; n < N; ++n) {
    const float *wr = w + (size_t)n * K;
    for (int m = 0; m < M; ++m) y[(size_t)m * N + n] = dot_f32(x + (size_t)m * K, wr, K) + b[n];
  }
}

/* ops.rs:12-17: x / sqrt(mean(x^2) + eps) * g */
void o_rmsnorm(const float *x, int rows, int dim, const float *g, float eps, float *out) {
  for (int r = 0; r < rows; ++r) {
    const float *xr = x + (size_t)r * dim;
    float s = 0.0f;
    for (int i = 0; i < dim; ++i) s += xr[i] * xr[i];
    float denom = sqrtf(s / (float)dim + eps);
    for (int i = 0; i < dim; ++i) out[(size_t)r * dim + i] = xr[i] / denom * g[i];
  }
}

/* ops.rs:78-115: theta 10000, xpos scale base 512; cos/sin duplicated as
 * interleaved pairs, xpos scale duplicated as concatenated halves. */
void o_rope_tables(int seq, int hd, float *cos_t, float *sin_t, float *scale) {
  int half = hd / 2;
  double theta = 10000.0, scale_base = 512.0;
  double max_half = floor((double)(seq - 1) / 2.0);
  for (int p = 0; p < seq; ++p) {
    double power = ((double)p - max_half) / scale_base;
    for (int j = 0; j < half; ++j) {
      double inv_freq = 1.0 / pow(theta, (double)(2 * j) / (double)hd);
      double angle = (double)p * inv_freq;
      double base = (2.0 * j + 0.4 * hd) / (1.4 * hd);
      float s = (float)pow(base, power);
      for (int k = 0; k < 2; ++k) {
        cos_t[p * hd + 2 * j + k] = (float)cos(angle);
        sin_t[p * hd + 2 * j + k] = (float)sin(angle);
      }
      scale[p * hd + j] = s;
      scale[p * hd + half + j] = s;
    }
  }
}

/* Rust std f32::asinh: (|x| + |x|/(hypot(1, 1/|x|) + 1/|x|)).ln_1p() with
 * the sign of x. */
static float rust_asinh(float x) {
  float ax = fabsf(x);
  float ix = 1.0f / ax;
  return copysignf(log1pf(ax + ax / (hypotf(1.0f, ix) + ix)), x);
}

/* scaler.rs:44-118 */
void o_scale_input(const o_config *cfg, int v, int t, const float *variates, const int8_t *mask,
                   const int64_t *group_ids, float *scaled, float *loc, float *scale) {
  for (int row = 0; row < v; ++row) {
    size_t base = (size_t)row * t;
    float count = 0.0f, mean = 0.0f, m2 = 0.0f;
    for (int col = 0; col < t; ++col) {
      if (mask[base + col] == MASK_VALID) {
        count += 1.0f;
        float delta = variates[base + col] - mean;
        mean += delta / count;
        float delta2 = variates[base + col] - mean;
        m2 += delta * delta2;
      }
      loc[base + col] = mean;
      float var = count > 1.0f ? fmaxf(m2 / (count - 1.0f), 0.0f) : 0.0f;
      scale[base + col] = cfg->variance_offset ? sqrtf(var + cfg->scaler_eps) : fmaxf(sqrtf(var), cfg->scaler_eps);
    }
    for (int col = 0; col < t; ++col)
      if (group_ids[base + col] < 0) {
        loc[base + col] = 0.0f;
        scale[base + col] = 1.0f;
      }
  }
  for (size_t i = 0; i < (size_t)v * t; ++i) {
    float x = (variates[i] - loc[i]) / scale[i];
    scaled[i] = cfg->scaler_use_arcsinh ? rust_asinh(x) : x;
  }
}

/* ops.rs:132-142 on one head vector: x*cos*s + rotate_half(x)*sin*s, with
 * rotate_half((x0, x1)) = (-x1, x0) per adjacent pair; k uses 1/s. */
static void apply_rope_vec(float *x, int hd, const float *cos_r, const float *sin_r, const float *sc_r,
                           int invert) {
  float tmp[256];
  for (int d = 0; d < hd; ++d) {
    float s = invert ? 1.0f / sc_r[d] : sc_r[d];
    float rot = (d & 1) ? x[d - 1] : -x[d + 1];
    tmp[d] = x[d] * cos_r[d] * s + rot * sin_r[d] * s;
  }
  memcpy(x, tmp, sizeof(float) * (size_t)hd);
}

/* ------------------------------------------------------------------------ */
/* model.rs forward                                                           */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float *hw, *hb, *ow, *ob, *rw, *rb;
  int in_dim, hidden, out_dim;
} resblock_t;

static int get_rb(const o_model *m, const char *prefix, resblock_t *rb) {
  char nm[256];
  const o_tensor *t;
#define G(field, suffix)                                  \
  snprintf(nm, sizeof nm, "%s.%s", prefix, suffix);       \
  if (!(t = find_tensor(m, nm))) return -1;               \
  rb->field = t->f32;
  G(hw, "mlp.hidden_layer.weight");
  rb->in_dim = (int)t->shape[1];
  rb->hidden = (int)t->shape[0];
  G(hb, "mlp.hidden_layer.bias");
  G(ow, "mlp.output_layer.weight");
  rb->out_dim = (int)t->shape[0];
  G(ob, "mlp.output_layer.bias");
  G(rw, "residual_layer.weight");
  G(rb, "residual_layer.bias");
#undef G
  return 0;
}

/* ops.rs:24-37 */
static void residual_block(const float *x, int M, const resblock_t *w, float *y) {
  float *h = (float *)malloc(sizeof(float) * (size_t)M * w->hidden);
  float *r = (float *)malloc(sizeof(float) * (size_t)M * w->out_dim);
  linear(x, M, w->in_dim, w->hw, w->hb, w->hidden, h);
  for (size_t i = 0; i < (size_t)M * w->hidden; ++i) h[i] = h[i] > 0.0f ? h[i] : 0.0f;
  linear(h, M, w->hidden, w->ow, w->ob, w->out_dim, y);
  linear(x, M, w->in_dim, w->rw, w->rb, w->out_dim, r);
  for (size_t i = 0; i < (size_t)M * w->out_dim; ++i) y[i] = y[i] + r[i];
  free(h);
  free(r);
}

static const float *tf(const o_model *m, const char *fmt, int layer) {
  char nm[256];
  snprintf(nm, sizeof nm, fmt, layer);
  const o_tensor *t = find_tensor(m, nm);
  return t ? t->f32 : NULL;
}

/* ops.rs:153-190.  xin: normed activations laid out [outer, seq, E];
 * mask [outer, seq, seq] (additive); rope tables [seq, hd] or NULL.
 * Returns the wO projection (+bias) in out [outer, seq, E]. */
static void mhsa(const float *xin, int outer, int seq, int E, int H, const float *wqkv, const float *bqkv,
                 const float *wo, const float *bo, const float *qn, const float *kn, const float *mask,
                 const float *rcos, const float *rsin, const float *rsc, float *out) {
  int hd = E / H;
  int M = outer * seq;
  float *qkv = (float *)malloc(sizeof(float) * (size_t)M * 3 * E);
  linear_q(xin, M, E, wqkv, bqkv, 3 * E, qkv);
  /* QK-norm (eps 1e-8) then RoPE, in place on the fused buffer */
  for (int r = 0; r < M; ++r) {
    int pos = r % seq;
    for (int h = 0; h < H; ++h) {
      float *q = qkv + (size_t)r * 3 * E + h * hd;
      float *k = qkv + (size_t)r * 3 * E + E + h * hd;
      o_rmsnorm(q, 1, hd, qn, 1e-8f, q);
      o_rmsnorm(k, 1, hd, kn, 1e-8f, k);
      if (rcos) {
        apply_rope_vec(q, hd, rcos + pos * hd, rsin + pos * hd, rsc + pos * hd, 0);
        apply_rope_vec(k, hd, rcos + pos * hd, rsin + pos * hd, rsc + pos * hd, 1);
      }
    }
  }
  float *att = (float *)malloc(sizeof(float) * (size_t)M * E);
  float *sc = (float *)malloc(sizeof(float) * (size_t)seq);
  float scl = 1.0f / sqrtf((float)hd);
  for (int o = 0; o < outer; ++o)
    for (int h = 0; h < H; ++h)
      for (int i = 0; i < seq; ++i) {
        const float *q = qkv + (size_t)(o * seq + i) * 3 * E + h * hd;
        float mx = -INFINITY;
        for (int j = 0; j < seq; ++j) {
          const float *k = qkv + (size_t)(o * seq + j) * 3 * E + E + h * hd;
          float s = 0.0f;
          for (int d = 0; d < hd; ++d) s += q[d] * k[d];
          sc[j] = s * scl + mask[((size_t)o * seq + i) * seq + j];
          mx = fmaxf(mx, sc[j]);
        }
        float sum = 0.0f;
        for (int j = 0; j < seq; ++j) {
          sc[j] = expf(sc[j] - mx);
          sum += sc[j];
        }
        for (int j = 0; j < seq; ++j) sc[j] = sc[j] / sum;
        float *dst = att + (size_t)(o * seq + i) * E + h * hd;
        for (int d = 0; d < hd; ++d) {
          float a = 0.0f;
          for (int j = 0; j < seq; ++j) a += sc[j] * qkv[(size_t)(o * seq + j) * 3 * E + 2 * E + h * hd + d];
          dst[d] = a;
        }
      }
  linear_q(att, M, E, wo, bo, E, out);
  free(sc);
  free(att);
  free(qkv);
}

/* mask.rs:12-28 */
static void reduce_patch_metadata(const int64_t *meta, const int8_t *mask, int v, int t, int P, int64_t *out) {
  int p = t / P;
  for (int row = 0; row < v; ++row)
    for (int patch = 0; patch < p; ++patch) {
      out[row * p + patch] = -1;
      for (int k = 0; k < P; ++k) {
        size_t idx = (size_t)row * t + patch * P + k;
        if (mask[idx] != MASK_PAD) {
          out[row * p + patch] = meta[idx];
          break;
        }
      }
    }
}

int o_forward(const o_model *m, int v, int t, const float *variates, const int8_t *mask,
              const int64_t *group_ids, const int64_t *variate_type, float *out, float *trace) {
  const o_config *c = &m->cfg;
  int P = c->patch_size, E = c->embed_dim, H = c->num_heads, hd = E / H, F = c->mlp_hidden_dim;
  if (t % P) return -1;
  int p = t / P, M = v * p, nq = c->n_quantiles;
  resblock_t enc, dec;
  if (get_rb(m, "patch_encoder.projection", &enc) || get_rb(m, "decoder", &dec)) return -2;
  const float *type_emb = tf(m, "patch_encoder.type_embeddings.weight", 0);
  const float *out_norm = tf(m, "transformer.out_norm.scale", 0);
  if (!type_emb || !out_norm) return -2;

  /* model.rs:185-199 patch concat [values(P) | k/P (P) | valid (P)] */
  float *cat = (float *)malloc(sizeof(float) * (size_t)M * 3 * P);
  for (int row = 0; row < v; ++row)
    for (int patch = 0; patch < p; ++patch)
      for (int k = 0; k < P; ++k) {
        size_t src = (size_t)row * t + patch * P + k;
        size_t base = ((size_t)row * p + patch) * 3 * P;
        cat[base + k] = variates[src];
        cat[base + P + k] = (float)k / (float)P;
        cat[base + 2 * P + k] = mask[src] == MASK_VALID ? 1.0f : 0.0f;
      }
  float *x = (float *)malloc(sizeof(float) * (size_t)M * E);
  residual_block(cat, M, &enc, x);
  free(cat);

  int64_t *pvt = (int64_t *)malloc(sizeof(int64_t) * (size_t)M);
  int64_t *pgid = (int64_t *)malloc(sizeof(int64_t) * (size_t)M);
  int8_t *attendable = (int8_t *)malloc((size_t)M);
  reduce_patch_metadata(variate_type, mask, v, t, P, pvt);
  reduce_patch_metadata(group_ids, mask, v, t, P, pgid);
  for (int row = 0; row < v; ++row) /* mask.rs:32-43 */
    for (int patch = 0; patch < p; ++patch) {
      attendable[row * p + patch] = 0;
      for (int k = 0; k < P; ++k)
        if (mask[(size_t)row * t + patch * P + k] != MASK_PAD) attendable[row * p + patch] = 1;
    }
  /* model.rs:205-207: + type_emb[max(type, 0)] (one-hot matmul == gather) */
  for (int r = 0; r < M; ++r) {
    int64_t ti = pvt[r] > 0 ? pvt[r] : 0;
    for (int e = 0; e < E; ++e) x[(size_t)r * E + e] = x[(size_t)r * E + e] + type_emb[ti * E + e];
  }
  if (trace) memcpy(trace, x, sizeof(float) * (size_t)M * E);

  /* mask.rs:49-82 */
  float *tmask = (float *)malloc(sizeof(float) * (size_t)v * p * p);
  for (int row = 0; row < v; ++row) {
    int is_future = pvt[row * p] == VT_FUTURE;
    for (int i = 0; i < p; ++i)
      for (int j = 0; j < p; ++j) {
        int64_t gi = pgid[row * p + i], gj = pgid[row * p + j];
        int att = gi >= 0 && gi == gj && (is_future || j <= i) && attendable[row * p + j];
        tmask[((size_t)row * p + i) * p + j] = att ? 0.0f : BLOCK_MASK;
      }
  }
  float *gmask = (float *)malloc(sizeof(float) * (size_t)p * v * v);
  for (int patch = 0; patch < p; ++patch)
    for (int i = 0; i < v; ++i)
      for (int j = 0; j < v; ++j) {
        int64_t gi = pgid[i * p + patch], gj = pgid[j * p + patch];
        gmask[((size_t)patch * v + i) * v + j] = (gi >= 0 && gi == gj) ? 0.0f : BLOCK_MASK;
      }
  float *rcos = (float *)malloc(sizeof(float) * (size_t)p * hd);
  float *rsin = (float *)malloc(sizeof(float) * (size_t)p * hd);
  float *rsc = (float *)malloc(sizeof(float) * (size_t)p * hd);
  o_rope_tables(p, hd, rcos, rsin, rsc);

  float *xn = (float *)malloc(sizeof(float) * (size_t)M * E);
  float *xt = (float *)malloc(sizeof(float) * (size_t)M * E);
  float *ao = (float *)malloc(sizeof(float) * (size_t)M * E);
  float *hid = (float *)malloc(sizeof(float) * (size_t)M * 2 * F);
  float *gated = (float *)malloc(sizeof(float) * (size_t)M * F);
  /* config.rs:45-56: TIME x (n-1), GROUP repeated; only whole blocks run */
  int n_layers = c->group_every_n > 0 ? (c->num_layers / c->group_every_n) * c->group_every_n : c->num_layers;
  for (int l = 0; l < n_layers; ++l) { /* model.rs:246-300 */
    int is_group = c->group_every_n > 0 && (l % c->group_every_n) == c->group_every_n - 1;
    const float *an = tf(m, "transformer.layers.%d.attention_block.norm.scale", l);
    const float *wqkv = tf(m, "transformer.layers.%d.attention_block.attention.wQKV.weight", l);
    const float *bqkv = tf(m, "transformer.layers.%d.attention_block.attention.wQKV.bias", l);
    const float *wo = tf(m, "transformer.layers.%d.attention_block.attention.wO.weight", l);
    const float *bo = tf(m, "transformer.layers.%d.attention_block.attention.wO.bias", l);
    const float *qn = tf(m, "transformer.layers.%d.attention_block.attention.q_norm.scale", l);
    const float *kn = tf(m, "transformer.layers.%d.attention_block.attention.k_norm.scale", l);
    const float *mn = tf(m, "transformer.layers.%d.norm.scale", l);
    const float *w0 = tf(m, "transformer.layers.%d.mlp.0.weight", l);
    const float *b0 = tf(m, "transformer.layers.%d.mlp.0.bias", l);
    const float *w2 = tf(m, "transformer.layers.%d.mlp.2.weight", l);
    const float *b2 = tf(m, "transformer.layers.%d.mlp.2.bias", l);
    if (!an || !wqkv || !bqkv || !wo || !bo || !qn || !kn || !mn || !w0 || !b0 || !w2 || !b2) return -2;
    o_rmsnorm(x, M, E, an, 1e-8f, xn);
    if (!is_group) {
      mhsa(xn, v, p, E, H, wqkv, bqkv, wo, bo, qn, kn, tmask, rcos, rsin, rsc, ao);
    } else { /* [v,p,E] -> [p,v,E], attention over variates, no RoPE */
      for (int r = 0; r < v; ++r)
        for (int q = 0; q < p; ++q)
          memcpy(xt + ((size_t)q * v + r) * E, xn + ((size_t)r * p + q) * E, sizeof(float) * (size_t)E);
      mhsa(xt, p, v, E, H, wqkv, bqkv, wo, bo, qn, kn, gmask, NULL, NULL, NULL, xn);
      for (int r = 0; r < v; ++r)
        for (int q = 0; q < p; ++q)
          memcpy(ao + ((size_t)r * p + q) * E, xn + ((size_t)q * v + r) * E, sizeof(float) * (size_t)E);
    }
    for (size_t i = 0; i < (size_t)M * E; ++i) x[i] = x[i] + ao[i];
    o_rmsnorm(x, M, E, mn, 1e-8f, xn); /* ops.rs:49-62 swiglu, gate first */
    linear_q(xn, M, E, w0, b0, 2 * F, hid);
    for (int r = 0; r < M; ++r)
      for (int f = 0; f < F; ++f) {
        float g = hid[(size_t)r * 2 * F + f];
        float u = hid[(size_t)r * 2 * F + F + f];
        gated[(size_t)r * F + f] = (g / (1.0f + expf(-g))) * u;
      }
    linear_q(gated, M, F, w2, b2, E, ao);
    for (size_t i = 0; i < (size_t)M * E; ++i) x[i] = x[i] + ao[i];
    if (trace) memcpy(trace + (size_t)(l + 1) * M * E, x, sizeof(float) * (size_t)M * E);
  }
  /* model.rs:230-237 */
  o_rmsnorm(x, M, E, out_norm, 1e-8f, xn);
  float *dd = (float *)malloc(sizeof(float) * (size_t)M * dec.out_dim);
  residual_block(xn, M, &dec, dd);
  /* ops.rs:195-210 quantile head: q0 = r0, qi = q0 + sum softplus(rj) */
  size_t rows = (size_t)M * P;
  for (size_t r = 0; r < rows; ++r) {
    const float *src = dd + r * nq;
    float *dst = out + r * nq;
    float running = src[0];
    dst[0] = running;
    for (int i = 1; i < nq; ++i) {
      running = running + logf(1.0f + expf(src[i]));
      dst[i] = running;
    }
  }
  free(dd);
  free(xn);
  free(xt);
  free(ao);
  free(hid);
  free(gated);
  free(rcos);
  free(rsin);
  free(rsc);
  free(tmask);
  free(gmask);
  free(pvt);
  free(pgid);
  free(attendable);
  free(x);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* forecast drivers: data.rs + model.rs:448-531 (+ t0-fast lib.rs:175-242)   */
/* ------------------------------------------------------------------------ */
typedef struct {
  int v, t;
  float *variates;
  int8_t *mask;
  int64_t *gid, *vt;
} series_t;

static void series_alloc(series_t *s, int v, int t) {
  s->v = v;
  s->t = t;
  s->variates = (float *)calloc((size_t)v * t, sizeof(float));
  s->mask = (int8_t *)calloc((size_t)v * t, 1);
  s->gid = (int64_t *)calloc((size_t)v * t, sizeof(int64_t));
  s->vt = (int64_t *)calloc((size_t)v * t, sizeof(int64_t));
}
static void series_free(series_t *s) {
  free(s->variates);
  free(s->mask);
  free(s->gid);
  free(s->vt);
}

/* data.rs:52-86: NaN -> Missing (value 0); horizon -> Withheld; group 0 */
static void from_context(const float *ctx, int v, int t_ctx, int horizon, series_t *s) {
  series_alloc(s, v, t_ctx + horizon);
  for (int row = 0; row < v; ++row) {
    for (int col = 0; col < t_ctx; ++col) {
      float xv = ctx[(size_t)row * t_ctx + col];
      size_t idx = (size_t)row * s->t + col;
      if (isnan(xv)) {
        s->variates[idx] = 0.0f;
        s->mask[idx] = MASK_MISSING;
      } else {
        s->variates[idx] = xv;
        s->mask[idx] = MASK_VALID;
      }
    }
    for (int col = t_ctx; col < s->t; ++col) s->mask[(size_t)row * s->t + col] = MASK_WITHHELD;
  }
}

/* data.rs:110-155 */
static void pad_series(const series_t *in, int P, int context_end, series_t *out) {
  int horizon = in->t - context_end;
  int pad_left = (P - context_end % P) % P;
  int pad_right = ((horizon + P - 1) / P) * P - horizon;
  int nt = pad_left + in->t + pad_right;
  series_alloc(out, in->v, nt);
  for (int row = 0; row < in->v; ++row) {
    int64_t rg = in->gid[(size_t)row * in->t + in->t - 1];
    int64_t rt = in->vt[(size_t)row * in->t + in->t - 1];
    for (int col = 0; col < nt; ++col) {
      size_t d = (size_t)row * nt + col;
      out->mask[d] = MASK_PAD;
      out->gid[d] = -1;
      out->vt[d] = -1;
    }
    for (int col = 0; col < in->t; ++col) {
      size_t src = (size_t)row * in->t + col, dst = (size_t)row * nt + pad_left + col;
      out->variates[dst] = in->variates[src];
      out->mask[dst] = in->mask[src];
      out->gid[dst] = in->gid[src];
      out->vt[dst] = in->vt[src];
    }
    for (int col = 0; col < pad_right; ++col) {
      size_t dst = (size_t)row * nt + pad_left + in->t + col;
      out->gid[dst] = rg;
      out->vt[dst] = rt;
      out->mask[dst] = rt == VT_TARGET ? MASK_WITHHELD : MASK_PAD;
    }
  }
}

/* model.rs:448-531: pad, scale, forward, rescale, slice */
static int forecast_series(const o_model *m, const series_t *raw, int t_ctx, int horizon, float *out) {
  const o_config *c = &m->cfg;
  int P = c->patch_size, nq = c->n_quantiles, v = raw->v;
  int pad_left = (P - t_ctx % P) % P;
  int padded_h = ((horizon + P - 1) / P) * P;
  int padded_ctx = t_ctx + pad_left;
  if (padded_h > MAX_HORIZON) return -3; /* model.rs:468-471 */
  for (size_t i = 0; i < (size_t)raw->v * raw->t; ++i)
    if (raw->vt[i] == VT_FUTURE) return -4; /* scaler.rs:57-61 */
  series_t w;
  pad_series(raw, P, t_ctx, &w);
  size_t vt = (size_t)w.v * w.t;
  float *scaled = (float *)malloc(sizeof(float) * vt);
  float *loc = (float *)malloc(sizeof(float) * vt);
  float *scl = (float *)malloc(sizeof(float) * vt);
  o_scale_input(c, w.v, w.t, w.variates, w.mask, w.gid, scaled, loc, scl);
  int np = w.t / P;
  float *pred = (float *)malloc(sizeof(float) * (size_t)v * np * P * nq);
  int rc = o_forward(m, w.v, w.t, scaled, w.mask, w.gid, w.vt, pred, NULL);
  if (rc == 0) {
    /* scaler.rs:125-148: stats at the last step of each patch */
    for (int row = 0; row < v; ++row)
      for (int q = 0; q < np; ++q) {
        size_t ti = (size_t)row * w.t + (size_t)q * P + (P - 1);
        float lo = loc[ti], sc = scl[ti];
        size_t base = ((size_t)row * np + q) * P * nq;
        for (int i = 0; i < P * nq; ++i) {
          float r = pred[base + i];
          float un = c->scaler_use_arcsinh ? sinhf(r) : r;
          pred[base + i] = un * sc + lo;
        }
      }
    int cp = padded_ctx / P;
    for (int row = 0; row < v; ++row)
      for (int h = 0; h < horizon; ++h) {
        int hp = h / P, k = h % P;
        size_t src = (((size_t)row * np + cp - 1 + hp) * P + k) * nq;
        memcpy(out + ((size_t)row * horizon + h) * nq, pred + src, sizeof(float) * (size_t)nq);
      }
  }
  free(pred);
  free(scaled);
  free(loc);
  free(scl);
  series_free(&w);
  return rc;
}

int o_forecast(const o_model *m, const float *ctx, int v, int t_ctx, int horizon, float *out) {
  series_t s;
  from_context(ctx, v, t_ctx, horizon, &s);
  int rc = forecast_series(m, &s, t_ctx, horizon, out);
  series_free(&s);
  return rc;
}

/* model.rs:385-407 + data.rs:96-105 (group id = row within the chunk) */
int o_forecast_batch(const o_model *m, const float *ctx, int n, int t_ctx, int horizon, int chunk, float *out) {
  int cs = (chunk == 0 || chunk > n) ? n : chunk;
  int nq = m->cfg.n_quantiles;
  for (int start = 0; start < n; start += cs) {
    int k = (n - start) < cs ? (n - start) : cs;
    series_t s;
    from_context(ctx + (size_t)start * t_ctx, k, t_ctx, horizon, &s);
    for (int row = 0; row < k; ++row)
      for (int col = 0; col < s.t; ++col) s.gid[(size_t)row * s.t + col] = row;
    int rc = forecast_series(m, &s, t_ctx, horizon, out + (size_t)start * horizon * nq);
    series_free(&s);
    if (rc) return rc;
  }
  return 0;
}

/* t0-fast lib.rs:175-242: ragged rows left-padded to a common patch-aligned
 * width with whole Pad patches. */
int o_forecast_batch_rows(const o_model *m, const float *ctx, const int64_t *lengths, int n, int horizon,
                          int chunk, float *out) {
  int P = m->cfg.patch_size, nq = m->cfg.n_quantiles;
  int cs = (chunk == 0 || chunk > n) ? n : chunk;
  size_t off = 0;
  for (int start = 0; start < n; start += cs) {
    int k = (n - start) < cs ? (n - start) : cs;
    int common = 0;
    for (int r = 0; r < k; ++r) {
      int al = (int)((lengths[start + r] + P - 1) / P) * P;
      if (al > common) common = al;
    }
    series_t s;
    series_alloc(&s, k, common + horizon);
    for (size_t i = 0; i < (size_t)k * s.t; ++i) {
      s.mask[i] = MASK_PAD;
      s.gid[i] = -1;
      s.vt[i] = -1;
    }
    for (int r = 0; r < k; ++r) {
      int len = (int)lengths[start + r];
      int lead = common - len;
      for (int col = 0; col < len; ++col) {
        size_t idx = (size_t)r * s.t + lead + col;
        float xv = ctx[off + col];
        if (isnan(xv)) {
          s.variates[idx] = 0.0f;
          s.mask[idx] = MASK_MISSING;
        } else {
          s.variates[idx] = xv;
          s.mask[idx] = MASK_VALID;
        }
        s.gid[idx] = r;
        s.vt[idx] = VT_TARGET;
      }
      for (int col = common; col < s.t; ++col) {
        size_t idx = (size_t)r * s.t + col;
        s.gid[idx] = r;
        s.vt[idx] = VT_TARGET;
        s.mask[idx] = MASK_WITHHELD;
      }
      off += (size_t)len;
    }
    int rc = forecast_series(m, &s, common, horizon, out + (size_t)start * horizon * nq);
    series_free(&s);
    if (rc) return rc;
  }
  return 0;
}

typedef struct {
  const o_model *m;
  const float *ctx;
  const int32_t *nv;
  const size_t *row_off;
  int n_series, t_ctx, horizon, rc;
  float *out;
  atomic_int next;
} ms_job_t;

static void *ms_worker(void *arg) {
  ms_job_t *j = (ms_job_t *)arg;
  int nq = j->m->cfg.n_quantiles;
  for (;;) {
    int s = atomic_fetch_add(&j->next, 1);
    if (s >= j->n_series) break;
    size_t r0 = j->row_off[s];
    int rc = o_forecast(j->m, j->ctx + r0 * j->t_ctx, j->nv[s], j->t_ctx, j->horizon,
                        j->out + r0 * (size_t)j->horizon * nq);
    if (rc) j->rc = rc;
  }
  return NULL;
}

int o_forecast_multiseries(const o_model *m, const float *ctx, const int32_t *n_variates, int n_series, int t_ctx,
                           int horizon, int n_threads, float *out) {
  size_t *row_off = (size_t *)malloc(sizeof(size_t) * ((size_t)n_series + 1));
  row_off[0] = 0;
  for (int s = 0; s < n_series; ++s) row_off[s + 1] = row_off[s] + (size_t)n_variates[s];
  ms_job_t job = {m, ctx, n_variates, row_off, n_series, t_ctx, horizon, 0, out, 0};
  if (n_threads < 1) n_threads = 1;
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n_threads);
  for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, ms_worker, &job);
  for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
  free(th);
  free(row_off);
  return job.rc;
}

/* ------------------------------------------------------------------------ */
/* fp64 GEMM oracles for the standalone dequant-GEMM configurations          */
/* ------------------------------------------------------------------------ */
static float *deq_rows(int type, const uint8_t *w, int N, int K) {
  float *d = (float *)malloc(sizeof(float) * (size_t)N * K);
  size_t rb = o_row_bytes(type, (size_t)K);
  for (int n = 0; n < N; ++n) dequantize_for(type, w + (size_t)n * rb, (size_t)K, d + (size_t)n * K);
  return d;
}

int o_gemm_q_f64(int type, const uint8_t *w, int N, int K, const float *x, int M, const float *bias, double *y) {
  if (K % QK) return -1;
  float *d = deq_rows(type, w, N, K);
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      double acc = 0.0;
      const float *xr = x + (size_t)m * K, *wr = d + (size_t)n * K;
      for (int k = 0; k < K; ++k) acc += (double)xr[k] * (double)wr[k];
      y[(size_t)m * N + n] = acc + (bias ? (double)bias[n] : 0.0);
    }
  free(d);
  return 0;
}

int o_swiglu_q_f64(int type, const uint8_t *w0, int F, int K, const uint8_t *w2, int N2, const float *x, int M,
                   double *z_out, double *y) {
  if (K % QK || F % QK) return -1;
  float *d0 = deq_rows(type, w0, 2 * F, K);
  float *d2 = deq_rows(type, w2, N2, F);
  double *z = (double *)malloc(sizeof(double) * (size_t)F);
  for (int m = 0; m < M; ++m) {
    const float *xr = x + (size_t)m * K;
    for (int f = 0; f < F; ++f) {
      double g = 0.0, u = 0.0;
      const float *wg = d0 + (size_t)f * K, *wu = d0 + (size_t)(F + f) * K;
      for (int k = 0; k < K; ++k) {
        g += (double)xr[k] * (double)wg[k];
        u += (double)xr[k] * (double)wu[k];
      }
      z[f] = g / (1.0 + exp(-g)) * u;
      if (z_out) z_out[(size_t)m * F + f] = z[f];
    }
    for (int n = 0; n < N2; ++n) {
      double acc = 0.0;
      const float *wr = d2 + (size_t)n * F;
      for (int f = 0; f < F; ++f) acc += z[f] * (double)wr[f];
      y[(size_t)m * N2 + n] = acc;
    }
  }
  free(z);
  free(d0);
  free(d2);
  return 0;
}

/* ===================================================== quantile utilities
 * quantile.rs restated in f32 with the same operation order.  Sorting is
 * stable (Rust's sort_by), done by insertion on index arrays. */
static void stable_order(const float *key, int n, int *idx) {
  for (int i = 0; i < n; ++i) {
    int j = i;
    while (j > 0 && key[idx[j - 1]] > key[i]) {
      idx[j] = idx[j - 1];
      --j;
    }
    idx[j] = i;
  }
}

/* quantile.rs:17-43 */
void o_interpolate_quantiles(const float *query, int nq, const float *levels, const float *values, int n,
                             float *out) {
  if (n < 1) return;
  int *idx = (int *)malloc(sizeof(int) * (size_t)n);
  float *lv = (float *)malloc(sizeof(float) * (size_t)(n + 2));
  float *vv = (float *)malloc(sizeof(float) * (size_t)(n + 2));
  stable_order(levels, n, idx);
  int len = 0;
  if (levels[idx[0]] > 0.0f) {  /* insert (0, first value) */
    lv[len] = 0.0f;
    vv[len] = values[idx[0]];
    ++len;
  }
  for (int i = 0; i < n; ++i, ++len) {
    lv[len] = levels[idx[i]];
    vv[len] = values[idx[i]];
  }
  if (lv[len - 1] < 1.0f) {  /* push (1, last value) */
    lv[len] = 1.0f;
    vv[len] = vv[len - 1];
    ++len;
  }
  for (int k = 0; k < nq; ++k) {
    const float q = query[k];
    int upper = 0;  /* partition_point(l <= q) */
    while (upper < len && lv[upper] <= q) ++upper;
    if (upper > len - 1) upper = len - 1;
    const int lower = upper > 0 ? upper - 1 : 0;
    const float ll = lv[lower], ul = lv[upper], lo = vv[lower], uo = vv[upper];
    const float diff = ul - ll;
    const float w = diff == 0.0f ? 0.0f : (q - ll) / diff;
    out[k] = lo + w * (uo - lo);
  }
  free(idx);
  free(lv);
  free(vv);
}

/* quantile.rs:47-61 */
void o_weighted_quantile(const float *query, int nq, const float *weights, const float *samples, int n,
                         float *out) {
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) sum += weights[i];
  int *idx = (int *)malloc(sizeof(int) * (size_t)n);
  float *ss = (float *)malloc(sizeof(float) * (size_t)n);
  float *cw = (float *)malloc(sizeof(float) * (size_t)n);
  stable_order(samples, n, idx);
  float cum = 0.0f;
  for (int i = 0; i < n; ++i) {
    ss[i] = samples[idx[i]];
    cum += weights[idx[i]] / sum;
    cw[i] = cum < 0.0f ? 0.0f : (cum > 1.0f ? 1.0f : cum);
  }
  o_interpolate_quantiles(query, nq, cw, ss, n, out);
  free(idx);
  free(ss);
  free(cw);
}

/* quantile.rs:66-78 */
void o_prob_mass(const float *levels, int n, float *out) {
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float lo = i == 0 ? 0.0f : levels[i - 1];
    const float hi = i == n - 1 ? 1.0f : levels[i + 1];
    out[i] = (hi - lo) / 2.0f;
  }
  for (int i = 0; i < n; ++i) sum += out[i];
  for (int i = 0; i < n; ++i) out[i] /= sum;
}

/* ================================================ autoregressive rollout
 * t0-core model.rs:582-665: a first single-window block of up to
 * MAX_HORIZON steps, then blocks in which each query-level path feeds its
 * own previous block back as observed context (trailing context_width
 * window), the paths are forecast as one batch, and every step's
 * path x trained-level outputs are reduced back to the query levels by
 * weighted_quantile over the trained-mass x query-mass grid. */
int o_forecast_rollout(const o_model *m, const float *ctx, int t_ctx, int prediction_length, const float *query,
                       int nq, float *out) {
  const int P = m->cfg.patch_size, ntr = m->cfg.n_quantiles, MAXH = 1024;
  const float *trained = m->cfg.quantile_levels;
  if (t_ctx < 1 || prediction_length < 1 || nq < 1) return -1;
  float trained_mass[32], *query_mass = (float *)malloc(sizeof(float) * (size_t)nq);
  o_prob_mass(trained, ntr, trained_mass);
  o_prob_mass(query, nq, query_mass);
  const int context_width = (t_ctx + P - 1) / P * P;
  int horizon0 = (prediction_length + P - 1) / P * P;
  if (horizon0 > MAXH) horizon0 = MAXH;
  const int total = prediction_length + MAXH + P;  /* output buffer incl. the last block's overshoot */
  float *res = (float *)malloc(sizeof(float) * (size_t)total * nq);
  float *block0 = (float *)malloc(sizeof(float) * (size_t)horizon0 * ntr);
  int rc = o_forecast(m, ctx, 1, t_ctx, horizon0, block0);
  if (rc) goto done;
  for (int h = 0; h < horizon0; ++h) o_interpolate_quantiles(query, nq, trained, block0 + (size_t)h * ntr, ntr,
                                                             res + (size_t)h * nq);
  if (prediction_length > horizon0) {
    const int npath = nq;
    /* each path's buffer: the context followed by everything fed back */
    const int cap = t_ctx + prediction_length + MAXH + P;
    float *paths = (float *)malloc(sizeof(float) * (size_t)npath * cap);
    int plen = t_ctx;
    for (int j = 0; j < npath; ++j) memcpy(paths + (size_t)j * cap, ctx, sizeof(float) * (size_t)t_ctx);
    int remaining = prediction_length - horizon0, prev_off = 0, prev_width = horizon0, done_steps = horizon0;
    float *batch = (float *)malloc(sizeof(float) * (size_t)npath * context_width);
    float *blocks = (float *)malloc(sizeof(float) * (size_t)npath * MAXH * ntr);
    float *samples = (float *)malloc(sizeof(float) * (size_t)npath * ntr);
    float *weights = (float *)malloc(sizeof(float) * (size_t)npath * ntr);
    for (int j = 0; j < npath; ++j)
      for (int pq = 0; pq < ntr; ++pq) weights[j * ntr + pq] = trained_mass[pq] * query_mass[j];
    while (remaining > 0 && rc == 0) {
      for (int j = 0; j < npath; ++j)
        for (int h = 0; h < prev_width; ++h) paths[(size_t)j * cap + plen + h] = res[(size_t)(prev_off + h) * nq + j];
      plen += prev_width;
      int horizon = (remaining + P - 1) / P * P;
      if (horizon > MAXH) horizon = MAXH;
      for (int j = 0; j < npath; ++j) {
        const int w = plen < context_width ? plen : context_width;
        float *dst = batch + (size_t)j * context_width;
        memset(dst, 0, sizeof(float) * (size_t)context_width);
        memcpy(dst + (context_width - w), paths + (size_t)j * cap + (plen - w), sizeof(float) * (size_t)w);
      }
      rc = o_forecast_batch(m, batch, npath, context_width, horizon, npath, blocks);
      if (rc) break;
      for (int h = 0; h < horizon; ++h) {
        for (int j = 0; j < npath; ++j)
          for (int pq = 0; pq < ntr; ++pq)
            samples[j * ntr + pq] = blocks[((size_t)j * horizon + h) * ntr + pq];
        o_weighted_quantile(query, nq, weights, samples, npath * ntr, res + (size_t)(done_steps + h) * nq);
      }
      prev_off = done_steps;
      prev_width = horizon;
      done_steps += horizon;
      remaining = remaining > horizon ? remaining - horizon : 0;
    }
    free(paths);
    free(batch);
    free(blocks);
    free(samples);
    free(weights);
  }
  if (rc == 0) memcpy(out, res, sizeof(float) * (size_t)prediction_length * nq);
done:
  free(res);
  free(block0);
  free(query_mass);
  return rc;
}
