// t0b_model.cu -- engine / model / forecast drivers behind the C ABI (t0b.h).
//
// Host side of the forecast path (t0-fast lib.rs:50-248 + model.rs:302-808):
// GGUF parse, weight residency (Q8_0 / Q4_0 blocks copied byte-for-byte to
// device memory, every other tensor expanded from f16 to f32), the per-pass
// launch sequence, and the batching drivers.  Independent series are packed
// as variate rows of p patches each (p = context patches + horizon patches);
// group attention is scoped per series, so no cross-series mask exists.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../../include/t0b.h"
#include "gguf_host.h"
#include "t0b_internal.h"

namespace {

// An NVTX range over the object's lifetime (host-side annotation for
// profilers; a no-op when no tool is attached).  Ranges: every forecast
// call, every pass, every layer of a pass that is launched rather than
// replayed from its CUDA graph (graphs off, or profiling on).
struct NvtxRange {
  explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange &) = delete;
  NvtxRange &operator=(const NvtxRange &) = delete;
};

thread_local std::string g_last_error;

t0b_status fail(t0b_status s, const std::string &msg) {
  g_last_error = msg;
  return s;
}

#define CUDA_TRY(expr)                                                                           \
  do {                                                                                           \
    cudaError_t e_ = (expr);                                                                     \
    if (e_ != cudaSuccess) return fail(T0B_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

constexpr int kMaxHorizon = 1024;  // model.rs:26

// grow-only device buffer
struct DBuf {
  void *p = nullptr;
  size_t bytes = 0;
  ~DBuf() {
    if (p) cudaFree(p);
  }
  cudaError_t reserve(size_t n) {
    if (n <= bytes) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    cudaError_t e = cudaMalloc(&p, n);
    if (e == cudaSuccess) bytes = n;
    return e;
  }
  template <class T>
  T *as() const {
    return reinterpret_cast<T *>(p);
  }
};

// grow-only pinned host buffer
struct HBuf {
  void *p = nullptr;
  size_t bytes = 0;
  ~HBuf() {
    if (p) cudaFreeHost(p);
  }
  cudaError_t reserve(size_t n) {
    if (n <= bytes) return cudaSuccess;
    if (p) cudaFreeHost(p);
    p = nullptr;
    bytes = 0;
    cudaError_t e = cudaMallocHost(&p, n);
    if (e == cudaSuccess) bytes = n;
    return e;
  }
};

struct LayerW {
  const uint8_t *wqkv, *wo, *w0, *w2;
  int sh_qkv, sh_o, sh_0, sh_2;  // weight prescale exponents (t0b_weight_shift)
  const float *bqkv, *bo, *b0, *b2, *g_attn, *g_mlp, *qn, *kn;
  bool group;
};

}  // namespace

struct t0b_engine {
  int device = 0;
  int *d_err = nullptr;
  DBuf scratch_xh, scratch_xl, scratch_zh, scratch_zl, scratch_red;
};

struct t0b_model {
  t0b_engine *eng = nullptr;
  t0b_model_info info{};
  int E = 0, H = 0, F = 0, L = 0, P = 0, nq = 0, qt = 8;
  std::vector<LayerW> layers;
  std::vector<void *> allocs;  // every device allocation of the weights
  const float *enc_hw, *enc_hb, *enc_ow, *enc_ob, *enc_rw, *enc_rb, *temb, *out_g;
  const float *dec_hw, *dec_hb, *dec_ow, *dec_ob, *dec_rw, *dec_rb;
  // f16 copies of the encoder / decoder matrices when the file stores them as
  // f16 (exact), for the tensor-core path; NULL otherwise
  const __half *enc_hw16 = nullptr, *enc_ow16 = nullptr, *enc_rw16 = nullptr;
  const __half *dec_hw16 = nullptr, *dec_ow16 = nullptr, *dec_rw16 = nullptr;
  int dec_out = 0, enc_in = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int *d_err = nullptr;
  size_t max_tokens = 393216;
  int tc_min_tokens = 128;
  std::map<int, float *> rope;  // p -> [4][p][hd] device tables: cos, sin, scale, 1/scale
  // workspace
  DBuf x, qkv, feat, ssq, xo, dhid, dout, loc, scl;
  DBuf ssqk;  // per-(token, head) sums of squares of q and k (TIME layers on the tensor-core path)
  DBuf xh, xl, ah, al, hh, hl;
  DBuf meta;  // row/series metadata
  HBuf hmeta;
  DBuf ctx_stage, out_stage;
  // host-buffer forecasts: a copy stream and events that overlap each pass's
  // context upload and the previous pass's quantile download with compute
  cudaStream_t io_stream = nullptr;
  cudaEvent_t io_in[2] = {nullptr, nullptr}, io_done[2] = {nullptr, nullptr};
  // measurement
  uint64_t launches = 0;
  bool prof = false;
  struct Rec {
    int cls;
    cudaEvent_t a, b;
    double flops, bytes;
  };
  std::vector<Rec> recs;
  std::vector<cudaEvent_t> ev_pool;
  t0b_kernel_stats stats[7];
  // CUDA graphs of whole passes, keyed by everything the captured launch
  // sequence depends on (shape, input/output and workspace pointers)
  bool use_graphs = true;
  struct GraphEntry {
    cudaGraphExec_t exec;
    uint64_t launches, last_use;
  };
  std::map<std::vector<uint64_t>, GraphEntry> graphs;
  uint64_t graph_clock = 0;
  std::vector<uint64_t> graph_sig;  // workspace allocations the cached graphs were captured against
  void drop_graphs() {
    for (auto &kv : graphs) cudaGraphExecDestroy(kv.second.exec);
    graphs.clear();
  }
  ~t0b_model() {
    drop_graphs();
    for (auto &r : recs) {
      cudaEventDestroy(r.a);
      cudaEventDestroy(r.b);
    }
    for (auto e : ev_pool) cudaEventDestroy(e);
    for (auto &kv : rope) cudaFree(kv.second);
    for (void *p : allocs) cudaFree(p);
    if (own_stream && stream) cudaStreamDestroy(stream);
    if (io_stream) cudaStreamDestroy(io_stream);
    for (int i = 0; i < 2; ++i) {
      if (io_in[i]) cudaEventDestroy(io_in[i]);
      if (io_done[i]) cudaEventDestroy(io_done[i]);
    }
    if (d_err) cudaFree(d_err);
  }
};

extern "C" const char *t0b_last_error(void) { return g_last_error.c_str(); }

// =================================================================== engine
extern "C" t0b_status t0b_engine_create(int device, t0b_engine **out) {
  if (!out) return fail(T0B_ERR_INVALID, "t0b_engine_create: out is NULL");
  *out = nullptr;
  int n = 0;
  CUDA_TRY(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return fail(T0B_ERR_INVALID, "t0b_engine_create: no such device");
  CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(T0B_ERR_UNSUPPORTED, "t0b: this engine is built for sm_100a (B200); device is sm_" +
                                         std::to_string(prop.major) + std::to_string(prop.minor));
  auto *e = new t0b_engine();
  e->device = device;
  if (cudaMalloc(&e->d_err, sizeof(int)) != cudaSuccess || cudaMemset(e->d_err, 0, sizeof(int)) != cudaSuccess) {
    delete e;
    return fail(T0B_ERR_OOM, "t0b_engine_create: device allocation failed");
  }
  *out = e;
  return T0B_OK;
}

extern "C" void t0b_engine_destroy(t0b_engine *e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->d_err) cudaFree(e->d_err);
  delete e;
}

// ==================================================================== model
namespace {

t0b_status upload_f32(t0b_model *m, const t0b::GgufFile &f, const std::string &name, const float **dst,
                      size_t expect) {
  auto it = f.tensors.find(name);
  if (it == f.tensors.end()) return fail(T0B_ERR_FORMAT, "gguf: missing tensor " + name);
  const auto &t = it->second;
  if (expect && t.n_elements != expect)
    return fail(T0B_ERR_FORMAT, "gguf: tensor " + name + " has " + std::to_string(t.n_elements) +
                                    " elements, expected " + std::to_string(expect));
  std::vector<float> h(t.n_elements);
  t0b::dequantize(t.type, t.data, t.n_elements, h.data());
  void *d = nullptr;
  if (cudaMalloc(&d, h.size() * 4) != cudaSuccess) return fail(T0B_ERR_OOM, "t0b: out of device memory");
  m->allocs.push_back(d);
  CUDA_TRY(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
  m->info.total_weight_bytes += h.size() * 4;
  *dst = (const float *)d;
  return T0B_OK;
}

// The f16 bytes of a tensor stored as F16 (exact), or NULL for other types.
t0b_status upload_f16_copy(t0b_model *m, const t0b::GgufFile &f, const std::string &name, const __half **dst) {
  *dst = nullptr;
  auto it = f.tensors.find(name);
  if (it == f.tensors.end()) return fail(T0B_ERR_FORMAT, "gguf: missing tensor " + name);
  const auto &t = it->second;
  if (t.type != t0b::GG_F16) return T0B_OK;
  void *d = nullptr;
  if (cudaMalloc(&d, t.n_elements * 2) != cudaSuccess) return fail(T0B_ERR_OOM, "t0b: out of device memory");
  m->allocs.push_back(d);
  CUDA_TRY(cudaMemcpy(d, t.data, t.n_elements * 2, cudaMemcpyHostToDevice));
  *dst = (const __half *)d;
  return T0B_OK;
}

t0b_status upload_q(t0b_model *m, const t0b::GgufFile &f, const std::string &name, int64_t rows, int64_t cols,
                    const uint8_t **dst, int *shift) {
  auto it = f.tensors.find(name);
  if (it == f.tensors.end()) return fail(T0B_ERR_FORMAT, "gguf: missing tensor " + name);
  const auto &t = it->second;
  if (t.shape.size() != 2 || t.shape[0] != rows || t.shape[1] != cols)
    return fail(T0B_ERR_FORMAT, "gguf: tensor " + name + " has an unexpected shape");
  if (t.type != t0b::GG_Q8_0 && t.type != t0b::GG_Q4_0)
    return fail(T0B_ERR_UNSUPPORTED, "t0b: tensor " + name +
                                         " is not Q8_0/Q4_0; this engine keeps only quantized big matmuls resident");
  void *d = nullptr;
  // 16 extra bytes: vectorised tail reads past the last block stay in bounds
  if (cudaMalloc(&d, t.nbytes + 16) != cudaSuccess) return fail(T0B_ERR_OOM, "t0b: out of device memory");
  m->allocs.push_back(d);
  CUDA_TRY(cudaMemcpy(d, t.data, t.nbytes, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemset((uint8_t *)d + t.nbytes, 0, 16));
  m->info.quantizable_gpu_bytes += t.nbytes;
  m->info.total_weight_bytes += t.nbytes;
  *dst = (const uint8_t *)d;
  // largest block scale of the matrix -> prescale exponent of the TC path
  const int bpb = t.type == t0b::GG_Q8_0 ? 34 : 18;
  float maxd = 0.0f;
  for (size_t b = 0; b < t.n_elements / 32; ++b) {
    uint16_t bits;
    std::memcpy(&bits, t.data + b * bpb, 2);
    maxd = std::max(maxd, std::fabs(t0b::f16_to_f32(bits)));
  }
  *shift = t0b_weight_shift(maxd, bpb == 34 ? 8 : 4);
  return T0B_OK;
}

bool meta_u32(const t0b::GgufFile &f, const char *k, int32_t *v) {
  auto it = f.meta.find(k);
  if (it == f.meta.end() || it->second.type != 4) return false;
  *v = (int32_t)it->second.u;
  return true;
}

t0b_status parse_config(const t0b::GgufFile &f, t0b_model *m);
t0b_status upload_all(t0b_model *m, const t0b::GgufFile &f);

t0b_status load_model(t0b_model *m, const uint8_t *bytes, size_t len) {
  t0b::GgufFile f;
  std::string err;
  if (!t0b::parse_gguf(bytes, len, f, err)) return fail(T0B_ERR_FORMAT, err);
  t0b_status s = parse_config(f, m);
  if (s != T0B_OK) return s;
  return upload_all(m, f);
}

t0b_status parse_config(const t0b::GgufFile &f, t0b_model *m) {
  // weights.rs:69-112 config_from_gguf_metadata
  auto &I = m->info;
  static const char *req[6] = {"t0.embed_dim", "t0.num_layers", "t0.num_heads", "t0.mlp_hidden_dim",
                               "t0.patch_size", "t0.group_every_n"};
  int32_t *dst[6] = {&I.embed_dim, &I.num_layers, &I.num_heads, &I.mlp_hidden_dim, &I.patch_size, &I.group_every_n};
  for (int i = 0; i < 6; ++i)
    if (!meta_u32(f, req[i], dst[i]))
      return fail(T0B_ERR_FORMAT, std::string("gguf: missing or wrong-typed metadata key ") + req[i]);
  auto q = f.meta.find("t0.quantile_levels");
  if (q == f.meta.end() || q->second.type != 9) return fail(T0B_ERR_FORMAT, "gguf: missing t0.quantile_levels metadata");
  if (q->second.arr.empty() || q->second.arr.size() > 32)
    return fail(T0B_ERR_UNSUPPORTED, "t0b: 1..32 quantile levels supported");
  I.n_quantiles = (int32_t)q->second.arr.size();
  for (size_t i = 0; i < q->second.arr.size(); ++i) I.quantile_levels[i] = q->second.arr[i];
  auto getf = [&](const char *k, float d) {
    auto it = f.meta.find(k);
    return (it != f.meta.end() && it->second.type == 6) ? it->second.f : d;
  };
  I.dropout = getf("t0.dropout", 0.0f);
  I.scaler_eps = getf("t0.scaler_eps", 0.1f);
  auto ab = f.meta.find("t0.scaler_use_arcsinh");
  I.scaler_use_arcsinh = (ab != f.meta.end() && ab->second.type == 7) ? ab->second.b : 1;
  auto em = f.meta.find("t0.scaler_eps_mode");
  I.variance_offset = (em != f.meta.end() && em->second.type == 8) ? (em->second.s != "std_clamp") : 1;
  I.weight_type = -1;

  m->E = I.embed_dim;
  m->H = I.num_heads;
  m->F = I.mlp_hidden_dim;
  m->P = I.patch_size;
  m->nq = I.n_quantiles;
  // config.rs:45-56: TIME x (n-1), GROUP; only whole blocks of n layers run
  const int gen = I.group_every_n;
  m->L = gen > 0 ? (I.num_layers / gen) * gen : I.num_layers;
  if (m->P != 32) return fail(T0B_ERR_UNSUPPORTED, "t0b: patch_size must be 32");
  if (m->H <= 0 || m->E % m->H || (m->E / m->H != 64 && m->E / m->H != 128))
    return fail(T0B_ERR_UNSUPPORTED, "t0b: head_dim (embed_dim / num_heads) must be 64 or 128");
  if (m->E % 256 || m->F % 256)
    return fail(T0B_ERR_UNSUPPORTED, "t0b: embed_dim and mlp_hidden_dim must be multiples of 256");
  if (m->H > 8) return fail(T0B_ERR_UNSUPPORTED, "t0b: at most 8 heads");
  // every tensor the forward pass needs, with its shape and type
  const int E = m->E, F = m->F, P = m->P, nq = m->nq;
  auto need = [&](const std::string &name, int64_t r, int64_t c, bool quant) -> t0b_status {
    auto it = f.tensors.find(name);
    if (it == f.tensors.end()) return fail(T0B_ERR_FORMAT, "gguf: missing tensor " + name);
    const auto &t = it->second;
    const size_t ne = (size_t)r * (size_t)(c ? c : 1);
    if (t.n_elements != ne || (c && (t.shape.size() != 2 || t.shape[0] != r || t.shape[1] != c)))
      return fail(T0B_ERR_FORMAT, "gguf: tensor " + name + " has an unexpected shape");
    if (quant) {
      if (t.type != t0b::GG_Q8_0 && t.type != t0b::GG_Q4_0)
        return fail(T0B_ERR_UNSUPPORTED, "t0b: tensor " + name +
                                             " is not Q8_0/Q4_0; this engine keeps only quantized big matmuls resident");
      if (m->info.weight_type == -1) m->info.weight_type = t.type;
      if (t.type != m->info.weight_type) return fail(T0B_ERR_UNSUPPORTED, "t0b: mixed Q8_0/Q4_0 big matmuls");
      m->info.quantizable_gpu_bytes += t.nbytes;
    }
    return T0B_OK;
  };
  t0b_status s;
#define NEED(name, r, c, q) \
  if ((s = need(name, r, c, q)) != T0B_OK) return s
  NEED("patch_encoder.projection.mlp.hidden_layer.weight", E, 3 * P, false);
  NEED("patch_encoder.projection.mlp.output_layer.weight", E, E, false);
  NEED("patch_encoder.projection.residual_layer.weight", E, 3 * P, false);
  NEED("patch_encoder.type_embeddings.weight", 3, E, false);
  NEED("decoder.mlp.hidden_layer.weight", E, E, false);
  NEED("decoder.mlp.output_layer.weight", P * nq, E, false);
  NEED("decoder.residual_layer.weight", P * nq, E, false);
  // 1-D tensors (c == 0: element count only)
  NEED("patch_encoder.projection.mlp.hidden_layer.bias", E, 0, false);
  NEED("patch_encoder.projection.mlp.output_layer.bias", E, 0, false);
  NEED("patch_encoder.projection.residual_layer.bias", E, 0, false);
  NEED("transformer.out_norm.scale", E, 0, false);
  NEED("decoder.mlp.hidden_layer.bias", E, 0, false);
  NEED("decoder.mlp.output_layer.bias", P * nq, 0, false);
  NEED("decoder.residual_layer.bias", P * nq, 0, false);
  for (int l = 0; l < m->L; ++l) {
    const std::string p = "transformer.layers." + std::to_string(l);
    NEED(p + ".attention_block.attention.wQKV.weight", 3 * E, E, true);
    NEED(p + ".attention_block.attention.wO.weight", E, E, true);
    NEED(p + ".mlp.0.weight", 2 * F, E, true);
    NEED(p + ".mlp.2.weight", E, F, true);
    NEED(p + ".attention_block.norm.scale", E, 0, false);
    NEED(p + ".attention_block.attention.wQKV.bias", 3 * E, 0, false);
    NEED(p + ".attention_block.attention.wO.bias", E, 0, false);
    NEED(p + ".attention_block.attention.q_norm.scale", E / m->H, 0, false);
    NEED(p + ".attention_block.attention.k_norm.scale", E / m->H, 0, false);
    NEED(p + ".norm.scale", E, 0, false);
    NEED(p + ".mlp.0.bias", 2 * F, 0, false);
    NEED(p + ".mlp.2.bias", E, 0, false);
  }
#undef NEED
  if (m->info.weight_type == -1) return fail(T0B_ERR_FORMAT, "gguf: model has no layers");
  m->qt = m->info.weight_type == t0b::GG_Q8_0 ? 8 : 4;
  return T0B_OK;
}

t0b_status upload_all(t0b_model *m, const t0b::GgufFile &f) {
  const int E = m->E, F = m->F, P = m->P, nq = m->nq, gen = m->info.group_every_n;
  m->info.quantizable_gpu_bytes = 0;
  m->info.total_weight_bytes = 0;
  t0b_status s;
#define UP(name, ptr, n) \
  if ((s = upload_f32(m, f, name, &(ptr), (n))) != T0B_OK) return s
  UP("patch_encoder.projection.mlp.hidden_layer.weight", m->enc_hw, (size_t)E * 3 * P);
  UP("patch_encoder.projection.mlp.hidden_layer.bias", m->enc_hb, (size_t)E);
  UP("patch_encoder.projection.mlp.output_layer.weight", m->enc_ow, (size_t)E * E);
  UP("patch_encoder.projection.mlp.output_layer.bias", m->enc_ob, (size_t)E);
  UP("patch_encoder.projection.residual_layer.weight", m->enc_rw, (size_t)E * 3 * P);
  UP("patch_encoder.projection.residual_layer.bias", m->enc_rb, (size_t)E);
  UP("patch_encoder.type_embeddings.weight", m->temb, (size_t)3 * E);
  UP("transformer.out_norm.scale", m->out_g, (size_t)E);
  UP("decoder.mlp.hidden_layer.weight", m->dec_hw, (size_t)E * E);
  UP("decoder.mlp.hidden_layer.bias", m->dec_hb, (size_t)E);
  UP("decoder.mlp.output_layer.weight", m->dec_ow, (size_t)P * nq * E);
  UP("decoder.mlp.output_layer.bias", m->dec_ob, (size_t)P * nq);
  UP("decoder.residual_layer.weight", m->dec_rw, (size_t)P * nq * E);
  UP("decoder.residual_layer.bias", m->dec_rb, (size_t)P * nq);
  m->dec_out = P * nq;
  m->enc_in = 3 * P;
#define UP16(name, ptr) \
  if ((s = upload_f16_copy(m, f, name, &(ptr))) != T0B_OK) return s
  UP16("patch_encoder.projection.mlp.hidden_layer.weight", m->enc_hw16);
  UP16("patch_encoder.projection.mlp.output_layer.weight", m->enc_ow16);
  UP16("patch_encoder.projection.residual_layer.weight", m->enc_rw16);
  UP16("decoder.mlp.hidden_layer.weight", m->dec_hw16);
  UP16("decoder.mlp.output_layer.weight", m->dec_ow16);
  UP16("decoder.residual_layer.weight", m->dec_rw16);
#undef UP16
  for (int l = 0; l < m->L; ++l) {
    LayerW w{};
    const std::string p = "transformer.layers." + std::to_string(l);
    w.group = gen > 0 && (l % gen) == gen - 1;
    if ((s = upload_q(m, f, p + ".attention_block.attention.wQKV.weight", 3 * E, E, &w.wqkv, &w.sh_qkv)) != T0B_OK) return s;
    if ((s = upload_q(m, f, p + ".attention_block.attention.wO.weight", E, E, &w.wo, &w.sh_o)) != T0B_OK) return s;
    if ((s = upload_q(m, f, p + ".mlp.0.weight", 2 * F, E, &w.w0, &w.sh_0)) != T0B_OK) return s;
    if ((s = upload_q(m, f, p + ".mlp.2.weight", E, F, &w.w2, &w.sh_2)) != T0B_OK) return s;
    UP(p + ".attention_block.attention.wQKV.bias", w.bqkv, (size_t)3 * E);
    UP(p + ".attention_block.attention.wO.bias", w.bo, (size_t)E);
    UP(p + ".mlp.0.bias", w.b0, (size_t)2 * F);
    UP(p + ".mlp.2.bias", w.b2, (size_t)E);
    UP(p + ".attention_block.norm.scale", w.g_attn, (size_t)E);
    UP(p + ".norm.scale", w.g_mlp, (size_t)E);
    UP(p + ".attention_block.attention.q_norm.scale", w.qn, (size_t)(E / m->H));
    UP(p + ".attention_block.attention.k_norm.scale", w.kn, (size_t)(E / m->H));
    m->layers.push_back(w);
  }
#undef UP
  return T0B_OK;
}

// RoPE tables for p patches, ops.rs:78-115 (f64 math, cast to f32).
t0b_status rope_tables(t0b_model *m, int p, const float **out) {
  auto it = m->rope.find(p);
  if (it != m->rope.end()) {
    *out = it->second;
    return T0B_OK;
  }
  const int hd = m->E / m->H, half = hd / 2;
  // [4][p][hd] full tables, then the [p][2 hd] compact copy, then the same
  // compact table transposed, [2 hd][p] (entry-major: a warp of consecutive
  // tokens reads one entry of consecutive positions in one coalesced access)
  std::vector<float> h((size_t)4 * p * hd + (size_t)2 * p * 2 * hd);
  float *cs = h.data(), *sn = cs + (size_t)p * hd, *sc = sn + (size_t)p * hd, *si = sc + (size_t)p * hd;
  const double theta = 10000.0, base512 = 512.0;
  const double max_half = std::floor((double)(p - 1) / 2.0);
  for (int pos = 0; pos < p; ++pos) {
    const double power = ((double)pos - max_half) / base512;
    for (int j = 0; j < half; ++j) {
      const double inv_freq = 1.0 / std::pow(theta, (double)(2 * j) / (double)hd);
      const double ang = (double)pos * inv_freq;
      const double b = (2.0 * j + 0.4 * hd) / (1.4 * hd);
      const float s = (float)std::pow(b, power);
      cs[pos * hd + 2 * j] = cs[pos * hd + 2 * j + 1] = (float)std::cos(ang);  // interleaved pairs
      sn[pos * hd + 2 * j] = sn[pos * hd + 2 * j + 1] = (float)std::sin(ang);
      sc[pos * hd + j] = sc[pos * hd + half + j] = s;  // concatenated halves
      si[pos * hd + j] = si[pos * hd + half + j] = 1.0f / s;  // k side (ops.rs:135-136 recip)
    }
  }
  float *cc = si + (size_t)p * hd;
  for (int pos = 0; pos < p; ++pos)
    for (int j = 0; j < half; ++j) {
      cc[pos * 2 * hd + j] = cs[pos * hd + 2 * j];
      cc[pos * 2 * hd + half + j] = sn[pos * hd + 2 * j];
      cc[pos * 2 * hd + 2 * half + j] = sc[pos * hd + j];
      cc[pos * 2 * hd + 3 * half + j] = si[pos * hd + j];
    }
  float *ct = cc + (size_t)p * 2 * hd;
  for (int pos = 0; pos < p; ++pos)
    for (int j = 0; j < 2 * hd; ++j) ct[(size_t)j * p + pos] = cc[pos * 2 * hd + j];
  float *d = nullptr;
  if (cudaMalloc(&d, h.size() * 4) != cudaSuccess) return fail(T0B_ERR_OOM, "t0b: out of device memory");
  CUDA_TRY(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
  m->rope[p] = d;
  *out = d;
  return T0B_OK;
}

// ------------------------------------------------------------------ passes
struct Pass {
  int R = 0, p = 0, hp = 0, horizon = 0;
  std::vector<int64_t> row_off;
  std::vector<int> row_len, row_lead, row_fv, s_row0, s_nrows;
  const float *ctx = nullptr;  // device
  float *out = nullptr;        // device [R, horizon, nq]
};

bool use_tc(const t0b_model *m, int M) { return M >= m->tc_min_tokens; }
// the tensor-core kernel also takes the small shapes the small-M kernel cannot
bool use_tc(const t0b_model *m, int M, int K, const Epi &epi) {
  return use_tc(m, M) || !t0b_small_supports(m->qt, M, K, epi);
}

enum { KC_GEMM_TC = 0, KC_GEMM_SMALL, KC_ATTN_TIME, KC_ATTN_GROUP, KC_PREP, KC_SGEMM, KC_OTHER, KC_N };
const char *kKcNames[KC_N] = {"gemm_tc", "gemm_small", "attn_time", "attn_group", "prep", "sgemm", "other"};

cudaEvent_t take_event(t0b_model *m) {
  if (!m->ev_pool.empty()) {
    cudaEvent_t e = m->ev_pool.back();
    m->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Every kernel launch of a pass goes through here: counts it and, when
// profiling is on, brackets it with events on the model's stream.
template <class F>
cudaError_t launch(t0b_model *m, int cls, double flops, double bytes, F &&fn) {
  ++m->launches;
  if (!m->prof) return fn();
  t0b_model::Rec r{cls, take_event(m), take_event(m), flops, bytes};
  cudaEventRecord(r.a, m->stream);
  cudaError_t e = fn();
  cudaEventRecord(r.b, m->stream);
  m->recs.push_back(r);
  return e;
}

void fold_records(t0b_model *m) {
  for (auto &r : m->recs) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      auto &st = m->stats[r.cls];
      st.launches += 1;
      st.total_ms += ms;
      st.flops += r.flops;
      st.bytes += r.bytes;
    }
    m->ev_pool.push_back(r.a);
    m->ev_pool.push_back(r.b);
  }
  m->recs.clear();
}

cudaError_t qgemm(t0b_model *m, const __half *ah, const __half *al, int M, int K, const uint8_t *W, int wrows,
                  int wshift, Epi &epi) {
  // algorithmic work: 2 M N K flops; bytes = raw weight blocks + A (as f32) +
  // the f32 output (SWIGLU writes F columns; RESID also reads the residual)
  const double wbytes = (double)wrows * K / 32.0 * (m->qt == 8 ? 34.0 : 18.0);
  const double outc = epi.kind == EPI_SWIGLU ? (double)epi.F : (double)epi.N;
  const double flops = 2.0 * M * (double)wrows * K;
  const double bytes = wbytes + 4.0 * M * K + 4.0 * M * outc * (epi.kind == EPI_RESID ? 2.0 : 1.0);
  if (use_tc(m, M, K, epi)) {
    return launch(m, KC_GEMM_TC, flops, bytes, [&] {
      return t0b_launch_gemm_tc(m->qt, ah, al, M, K, W, wrows, wshift, epi, m->d_err, m->stream);
    });
  }
  if (epi.kind == EPI_RESID) epi.ssq_out_nt = epi.N / 32;
  return launch(m, KC_GEMM_SMALL, flops, bytes, [&] {
    return t0b_launch_gemm_small(m->qt, ah, al, M, K, W, epi, m->d_err, m->stream);
  });
}

// Residual branch output GEMM (wO or mlp.2): x += A . W^T + bias, then the
// split of x * gnext and its sums of squares for the next RMSNorm-fused GEMM,
// all in the GEMM's epilogue (EPI_RESID) on both paths: the tensor-core
// epilogue reads its x tile, stores the new x and the split planes by TMA and
// writes one partial sum of squares per 64 columns (N / 64 per row); the
// small-M epilogue one per 32 columns.  Sets *ssq_nt to the number of partial
// sums per row.
cudaError_t resid_gemm(t0b_model *m, const __half *ah, const __half *al, int M, int K, const uint8_t *W,
                       int wshift, const float *bias, float *x, const float *gnext, int *ssq_nt) {
  const int E = m->E;
  Epi r{};
  r.M = M;
  r.N = E;
  r.bias = bias;
  r.kind = EPI_RESID;
  r.x = x;
  r.gnext = gnext;
  r.xh = m->xh.as<__half>();
  r.xl = m->xl.as<__half>();
  r.ssq_out = m->ssq.as<float>();
  if (use_tc(m, M, K, r)) {
    r.y = x;
    r.ldy = E;
    r.F = E;
    r.zh = r.xh;
    r.zl = r.xl;
    r.ssq_out_nt = E / 64;
    *ssq_nt = E / 64;
    return qgemm(m, ah, al, M, K, W, E, wshift, r);
  }
  *ssq_nt = E / 32;
  return qgemm(m, ah, al, M, K, W, E, wshift, r);
}

t0b_status ensure_ws(t0b_model *m, size_t T, size_t R, size_t nout) {
  const size_t E = m->E, F = m->F;
  CUDA_TRY(m->x.reserve(T * E * 4));
  CUDA_TRY(m->qkv.reserve(T * 3 * E * 4));
  CUDA_TRY(m->feat.reserve(T * 96 * 4));
  CUDA_TRY(m->ssq.reserve(T * std::max<size_t>(16, E / 32) * 4));
  CUDA_TRY(m->ssqk.reserve(T * 2 * (size_t)m->H * 4));
  CUDA_TRY(m->xh.reserve(T * E * 2));
  CUDA_TRY(m->xl.reserve(T * E * 2));
  CUDA_TRY(m->ah.reserve(T * E * 2));
  CUDA_TRY(m->al.reserve(T * E * 2));
  CUDA_TRY(m->hh.reserve(T * F * 2));
  CUDA_TRY(m->hl.reserve(T * F * 2));
  CUDA_TRY(m->xo.reserve(nout * E * 4));
  CUDA_TRY(m->dhid.reserve(nout * E * 4));
  CUDA_TRY(m->dout.reserve(nout * m->dec_out * 4));
  CUDA_TRY(m->loc.reserve(nout * 4));
  CUDA_TRY(m->scl.reserve(nout * 4));
  (void)R;
  return T0B_OK;
}

#define LAUNCH(expr)                                                                                    \
  do {                                                                                                  \
    cudaError_t e_ = (expr);                                                                            \
    if (e_ != cudaSuccess) return fail(T0B_ERR_CUDA, std::string("launch failed: ") + cudaGetErrorString(e_)); \
  } while (0)

t0b_status run_pass(t0b_model *m, const Pass &ps) {
  const int R = ps.R, p = ps.p, hp = ps.hp, E = m->E, F = m->F;
  const size_t T = (size_t)R * p;
  char pass_name[64];
  std::snprintf(pass_name, sizeof(pass_name), "t0b pass rows=%d patches=%d", R, p);
  const NvtxRange pass_range(pass_name);
  const int ns = (int)ps.s_row0.size();
  if (T == 0) return T0B_OK;
  // the previous pass must be done before buffers are grown or the pinned
  // metadata staging buffer is rewritten
  CUDA_TRY(cudaStreamSynchronize(m->stream));
  t0b_status st = ensure_ws(m, T, R, (size_t)R * hp);
  if (st != T0B_OK) return st;
  // metadata: row_off (i64) | row_len | row_lead | row_fv | s_row0 | s_nrows,
  // each section padded to 16 bytes
  const size_t mbytes = (size_t)R * 20 + (size_t)ns * 8 + 256;
  CUDA_TRY(m->meta.reserve(mbytes));
  CUDA_TRY(m->hmeta.reserve(mbytes));
  uint8_t *hb = (uint8_t *)m->hmeta.p;
  size_t o = 0;
  auto put = [&](const void *src, size_t n) {
    std::memcpy(hb + o, src, n);
    size_t at = o;
    o += (n + 15) / 16 * 16;
    return at;
  };
  const size_t o_off = put(ps.row_off.data(), (size_t)R * 8);
  const size_t o_len = put(ps.row_len.data(), (size_t)R * 4);
  const size_t o_lead = put(ps.row_lead.data(), (size_t)R * 4);
  const size_t o_fv = put(ps.row_fv.data(), (size_t)R * 4);
  const size_t o_s0 = put(ps.s_row0.data(), (size_t)ns * 4);
  const size_t o_sn = put(ps.s_nrows.data(), (size_t)ns * 4);
  uint8_t *db = (uint8_t *)m->meta.p;
  const float *rope = nullptr;
  if ((st = rope_tables(m, p, &rope)) != T0B_OK) return st;

  // Everything from here on is stream work only (the metadata copy from the
  // pinned staging buffer and the kernels), so without profiling it is
  // captured once per pass shape into a CUDA graph and replayed.
  const bool graph = m->use_graphs && !m->prof && m->stream != nullptr;
  std::vector<uint64_t> key;
  if (graph) {
    // a workspace buffer that was reallocated invalidates every cached graph
    // (a graph may hold its old allocation, even at an address reused since)
    std::vector<uint64_t> sig{(uint64_t)(uintptr_t)m->hmeta.p, (uint64_t)m->hmeta.bytes};
    for (const DBuf *b : {&m->x, &m->qkv, &m->feat, &m->ssq, &m->ssqk, &m->xo, &m->dhid, &m->dout, &m->loc, &m->scl,
                          &m->xh, &m->xl, &m->ah, &m->al, &m->hh, &m->hl, &m->meta, &m->ctx_stage, &m->out_stage}) {
      sig.push_back((uint64_t)(uintptr_t)b->p);
      sig.push_back((uint64_t)b->bytes);
    }
    if (sig != m->graph_sig) {
      m->drop_graphs();
      m->graph_sig = std::move(sig);
    }
    key = {(uint64_t)R, (uint64_t)p, (uint64_t)hp, (uint64_t)ns, (uint64_t)ps.horizon, (uint64_t)o,
           (uint64_t)(uintptr_t)ps.ctx, (uint64_t)(uintptr_t)ps.out, (uint64_t)(uintptr_t)hb,
           (uint64_t)(uintptr_t)rope, (uint64_t)m->tc_min_tokens,
           // the group-attention kernel variant depends on the largest series
           (uint64_t)(ps.s_nrows.empty() ? 0 : *std::max_element(ps.s_nrows.begin(), ps.s_nrows.end()))};
    for (const DBuf *b : {&m->x, &m->qkv, &m->feat, &m->ssq, &m->ssqk, &m->xo, &m->dhid, &m->dout, &m->loc, &m->scl,
                          &m->xh, &m->xl, &m->ah, &m->al, &m->hh, &m->hl, &m->meta})
      key.push_back((uint64_t)(uintptr_t)b->p);
    auto it = m->graphs.find(key);
    if (it != m->graphs.end()) {
      it->second.last_use = ++m->graph_clock;
      m->launches += it->second.launches;
      CUDA_TRY(cudaGraphLaunch(it->second.exec, m->stream));
      return T0B_OK;
    }
  }
  auto body = [&]() -> t0b_status {
  CUDA_TRY(cudaMemcpyAsync(m->meta.p, hb, o, cudaMemcpyHostToDevice, m->stream));

  // 1. pad + causal scaler + patch features
  PrepArgs pa{};
  pa.ctx = ps.ctx;
  pa.row_off = (const int64_t *)(db + o_off);
  pa.row_len = (const int *)(db + o_len);
  pa.row_lead = (const int *)(db + o_lead);
  pa.R = R;
  pa.p = p;
  pa.hp = hp;
  pa.use_arcsinh = m->info.scaler_use_arcsinh;
  pa.variance_offset = m->info.variance_offset;
  pa.eps = m->info.scaler_eps;
  pa.feat = m->feat.as<float>();
  pa.out_loc = m->loc.as<float>();
  pa.out_scale = m->scl.as<float>();
  pa.err = m->d_err;
  LAUNCH(launch(m, KC_PREP, 0.0, (double)R * p * 32 * 4 + T * 96.0 * 4, [&] { return t0b_launch_prep(pa, m->stream); }));

  // 2. patch encoder: x = relu(f.hw^T+hb).ow^T + ob + f.rw^T + rb + type_emb[0]
  float *x = m->x.as<float>();
  float *hid = m->qkv.as<float>();  // scratch [T, E]
  SgemmArgs g{};
  g.A = m->feat.as<float>();
  g.lda = 96;
  g.B = m->enc_hw;
  g.B16 = m->enc_hw16;
  g.ldb = 96;
  g.C = hid;
  g.ldc = E;
  g.M = (int)T;
  g.N = E;
  g.K = 96;
  g.bias = m->enc_hb;
  g.relu = 1;
  LAUNCH(launch(m, KC_SGEMM, 2.0 * g.M * g.N * g.K, 0.0, [&] { return t0b_launch_sgemm(g, m->stream); }));
  g.B = m->enc_rw;
  g.B16 = m->enc_rw16;
  g.C = x;
  g.bias = m->enc_rb;
  g.bias2 = m->enc_ob;
  g.bias3 = m->temb;  // row 0: TARGET type embedding (every patch of a target row)
  g.relu = 0;
  LAUNCH(launch(m, KC_SGEMM, 2.0 * g.M * g.N * g.K, 0.0, [&] { return t0b_launch_sgemm(g, m->stream); }));
  g.A = hid;
  g.lda = E;
  g.B = m->enc_ow;
  g.B16 = m->enc_ow16;
  g.ldb = E;
  g.K = E;
  g.bias = g.bias2 = g.bias3 = nullptr;
  g.accumulate = 1;
  LAUNCH(launch(m, KC_SGEMM, 2.0 * g.M * g.N * g.K, 0.0, [&] { return t0b_launch_sgemm(g, m->stream); }));
  LAUNCH(launch(m, KC_OTHER, 0.0, T * E * 8.0, [&] {
    return t0b_launch_rownorm_split(x, m->layers[0].g_attn, m->xh.as<__half>(), m->xl.as<__half>(),
                                    m->ssq.as<float>(), (int)T, E, m->stream);
  }));
  int ssq_nt = 1;

  AttnArgs aa{};
  aa.qkv = m->qkv.as<float>();
  aa.oh = m->ah.as<__half>();
  aa.ol = m->al.as<__half>();
  aa.row_first_valid = (const int *)(db + o_fv);
  aa.series_row0 = (const int *)(db + o_s0);
  aa.series_nrows = (const int *)(db + o_sn);
  aa.R = R;
  aa.p = p;
  aa.E = E;
  aa.H = m->H;
  aa.n_series = ns;
  aa.max_nrows = ps.s_nrows.empty() ? 0 : *std::max_element(ps.s_nrows.begin(), ps.s_nrows.end());
  aa.err = m->d_err;
  const int M = (int)T;
  aa.rope = rope;
  aa.rope_c = rope + (size_t)4 * p * (E / m->H);  // after the [4][p][hd] full tables
  // TIME layers on the tensor-core path with 64-dim heads: the wQKV epilogue
  // writes gain-scaled, rotated q / k and v as f16 planes (the qkv buffer's
  // bytes) plus the QK-norm sums of squares, and the time attention reads the
  // planes by TMA without a conversion pass
  const bool qkv_planes = E / m->H == 64 && p <= 256 && use_tc(m, M);
  const bool univariate = ns == R;  // one variate row per series
  aa.qkv_h = m->qkv.as<__half>();
  aa.qkv_l = aa.qkv_h + T * 3 * E;
  aa.ssq_qk = m->ssqk.as<float>();

  for (int l = 0; l < m->L; ++l) {
    const LayerW &w = m->layers[l];
    char layer_name[32];
    std::snprintf(layer_name, sizeof(layer_name), "layer %d %s", l, w.group ? "GROUP" : "TIME");
    const NvtxRange layer_range(layer_name);
    // q | k | v = rmsnorm(x) . wQKV^T + b; QK-norm and RoPE happen in the
    // attention kernels as q and k are read, or in the epilogue (planes)
    const bool planes = qkv_planes && !w.group;
    Epi e{};
    e.kind = planes ? EPI_QKV : EPI_PLAIN;
    e.M = M;
    e.N = 3 * E;
    e.bias = w.bqkv;
    e.ssq_in = m->ssq.as<float>();
    e.ssq_in_nt = ssq_nt;
    e.ssq_dim = E;
    e.y = m->qkv.as<float>();
    e.ldy = 3 * E;
    if (planes) {
      e.F = 3 * E;
      e.zh = m->qkv.as<__half>();
      e.zl = e.zh + T * 3 * E;
      e.qn = w.qn;
      e.kn = w.kn;
      e.rope_t = aa.rope_c + (size_t)p * 2 * (E / m->H);  // the transposed compact table
      e.ssq_qk = m->ssqk.as<float>();
      e.p = p;
      e.E = E;
      e.H = m->H;
    }
    if (w.group && univariate) {
      // every series has one variate: the group attention of a token is a
      // softmax over its own key alone, exactly 1, so its output is exactly
      // v (mask.rs:69-82 makes a lone whole-padding query average the same
      // single v).  Only the v third of wQKV is computed, as the wO GEMM's
      // f16 planes: split in the small-M epilogue, by a split pass after
      // the tensor-core GEMM.
      const size_t rb = (size_t)(E / 32) * (m->qt == 8 ? 34 : 18);  // bytes per weight row
      Epi ev = e;
      ev.kind = EPI_PLAIN;
      ev.N = E;
      ev.bias = w.bqkv + 2 * E;
      ev.ldy = E;
      const bool tc_v = use_tc(m, M, E, ev);
      if (!tc_v) {
        ev.zh = m->ah.as<__half>();
        ev.zl = m->al.as<__half>();
      }
      LAUNCH(qgemm(m, m->xh.as<__half>(), m->xl.as<__half>(), M, E, w.wqkv + 2 * (size_t)E * rb, E, w.sh_qkv, ev));
      if (tc_v)
        LAUNCH(launch(m, KC_OTHER, 0.0, T * E * 8.0, [&] {
          return t0b_launch_split_f32(m->qkv.as<float>(), m->ah.as<__half>(), m->al.as<__half>(), T * (size_t)E,
                                      m->stream);
        }));
      LAUNCH(resid_gemm(m, m->ah.as<__half>(), m->al.as<__half>(), M, E, w.wo, w.sh_o, w.bo, x, w.g_mlp, &ssq_nt));
    } else {
    LAUNCH(qgemm(m, m->xh.as<__half>(), m->xl.as<__half>(), M, E, w.wqkv, 3 * E, w.sh_qkv, e));
    aa.qn = w.qn;
    aa.kn = w.kn;
    aa.use_rope = w.group ? 0 : 1;
    if (w.group) {
      LAUNCH(launch(m, KC_ATTN_GROUP, 0.0, T * (3.0 * E * 4 + E * 4.0), [&] { return t0b_launch_attn_group(aa, m->stream); }));
    } else {
      // causal pairs per row: p(p+1)/2, each 2*hd flops for q.k and 2*hd for p.v, per head
      const double fl = (double)R * m->H * (p * (p + 1) / 2.0) * 4.0 * (E / m->H);
      LAUNCH(launch(m, KC_ATTN_TIME, fl, T * (3.0 * E * 4 + E * 4.0), [&] {
        return planes ? t0b_launch_attn_time_planes(aa, m->stream) : t0b_launch_attn_time(aa, m->stream);
      }));
    }
    LAUNCH(resid_gemm(m, m->ah.as<__half>(), m->al.as<__half>(), M, E, w.wo, w.sh_o, w.bo, x, w.g_mlp, &ssq_nt));
    }

    Epi sg{};
    sg.kind = EPI_SWIGLU;
    sg.M = M;
    sg.N = 2 * F;
    sg.F = F;
    sg.bias = w.b0;
    sg.ssq_in = m->ssq.as<float>();
    sg.ssq_in_nt = ssq_nt;
    sg.ssq_dim = E;
    sg.zh = m->hh.as<__half>();
    sg.zl = m->hl.as<__half>();
    LAUNCH(qgemm(m, m->xh.as<__half>(), m->xl.as<__half>(), M, E, w.w0, 2 * F, w.sh_0, sg));

    const float *gnext = (l + 1 < m->L) ? m->layers[l + 1].g_attn : m->out_g;
    LAUNCH(resid_gemm(m, m->hh.as<__half>(), m->hl.as<__half>(), M, F, w.w2, w.sh_2, w.b2, x, gnext, &ssq_nt));
  }

  // decoder on the output patches only: rmsnorm(out_norm) -> residual block
  const int nout = R * hp;
  LAUNCH(launch(m, KC_OTHER, 0.0, nout * E * 8.0,
                [&] { return t0b_launch_dec_gather(x, m->out_g, m->xo.as<float>(), R, p, hp, E, m->stream); }));
  SgemmArgs d{};
  d.A = m->xo.as<float>();
  d.lda = E;
  d.B = m->dec_hw;
  d.B16 = m->dec_hw16;
  d.ldb = E;
  d.C = m->dhid.as<float>();
  d.ldc = E;
  d.M = nout;
  d.N = E;
  d.K = E;
  d.bias = m->dec_hb;
  d.relu = 1;
  LAUNCH(launch(m, KC_SGEMM, 2.0 * d.M * d.N * d.K, 0.0, [&] { return t0b_launch_sgemm(d, m->stream); }));
  d.B = m->dec_rw;
  d.B16 = m->dec_rw16;
  d.C = m->dout.as<float>();
  d.ldc = m->dec_out;
  d.N = m->dec_out;
  d.bias = m->dec_rb;
  d.bias2 = m->dec_ob;
  d.relu = 0;
  LAUNCH(launch(m, KC_SGEMM, 2.0 * d.M * d.N * d.K, 0.0, [&] { return t0b_launch_sgemm(d, m->stream); }));
  d.A = m->dhid.as<float>();
  d.B = m->dec_ow;
  d.B16 = m->dec_ow16;
  d.bias = d.bias2 = nullptr;
  d.accumulate = 1;
  LAUNCH(launch(m, KC_SGEMM, 2.0 * d.M * d.N * d.K, 0.0, [&] { return t0b_launch_sgemm(d, m->stream); }));
  LAUNCH(launch(m, KC_OTHER, 0.0, (double)nout * m->dec_out * 8.0, [&] {
    return t0b_launch_dec_head(m->dout.as<float>(), m->loc.as<float>(), m->scl.as<float>(), ps.out, nullptr, R, hp,
                               ps.horizon, m->nq, m->info.scaler_use_arcsinh, m->stream);
  }));
  return T0B_OK;
  };
  if (!graph) return body();
  const uint64_t launches0 = m->launches;
  CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeRelaxed));
  const t0b_status bs = body();
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(m->stream, &g);
  if (bs != T0B_OK) {
    if (g) cudaGraphDestroy(g);
    return bs;
  }
  if (ce != cudaSuccess) return fail(T0B_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
  cudaGraphExec_t ex = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return fail(T0B_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ie));
  if (m->graphs.size() >= 32) {  // keep the 32 most recently used pass shapes
    auto lru = m->graphs.begin();
    for (auto it = m->graphs.begin(); it != m->graphs.end(); ++it)
      if (it->second.last_use < lru->second.last_use) lru = it;
    cudaGraphExecDestroy(lru->second.exec);
    m->graphs.erase(lru);
  }
  m->graphs[key] = {ex, m->launches - launches0, ++m->graph_clock};
  CUDA_TRY(cudaGraphLaunch(ex, m->stream));
  return T0B_OK;
}

t0b_status check_horizon(size_t horizon) {
  if (horizon == 0) return fail(T0B_ERR_INVALID, "t0b: horizon must be >= 1");
  if ((horizon + 31) / 32 * 32 > (size_t)kMaxHorizon)
    return fail(T0B_ERR_INVALID,
                "single-window forecast can't exceed max_horizon (1024) in one pass -- use forecast_rollout");
  return T0B_OK;
}

t0b_status sync_model(t0b_model *m) {
  CUDA_TRY(cudaStreamSynchronize(m->stream));
  int herr = 0;
  CUDA_TRY(cudaMemcpy(&herr, m->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (herr) {
    cudaMemset(m->d_err, 0, sizeof(int));
    return fail(T0B_ERR_DEVICE, "t0b: a kernel reported device error code " + std::to_string(herr));
  }
  return T0B_OK;
}

// One group of whole series into one or more passes.  rows: (ctx offset,
// length) per variate row; series: consecutive row counts.  All rows of one
// call share the padded context width `ctx_w` (a multiple of 32).
struct RowSpec {
  int64_t off;
  int len;
};

// Host buffers behind a device forecast: the contexts at the same offsets as
// ctx_dev, the quantiles at the same offsets as out_dev.
struct HostIO {
  const float *ctx;
  float *out;
};

t0b_status run_series(t0b_model *m, const float *ctx_dev, const std::vector<RowSpec> &rows,
                      const std::vector<int> &series_nrows, int ctx_w, int horizon, float *out_dev,
                      size_t max_rows_hint, const HostIO *hio = nullptr) {
  const NvtxRange range("t0b forecast");
  const int hpad = (horizon + 31) / 32 * 32;
  const int p = (ctx_w + hpad) / 32, hp = hpad / 32;
  if (m->E / m->H == 128 && p > 256)
    return fail(T0B_ERR_UNSUPPORTED, "t0b: 128-dim heads run at most 256 patches per row (context + horizon)");
  size_t max_rows = std::max<size_t>(1, m->max_tokens / (size_t)p);
  if (max_rows_hint) max_rows = std::min(max_rows, max_rows_hint);
  {
    // balanced passes: as many as the token budget needs, of near-equal size
    // (whole series per pass), instead of full passes and a small remainder
    const size_t total = rows.size();
    const size_t npass = (total + max_rows - 1) / max_rows;
    const int maxnv = series_nrows.empty() ? 1 : *std::max_element(series_nrows.begin(), series_nrows.end());
    if (npass > 1) max_rows = std::min(max_rows, (total + npass - 1) / npass + (size_t)maxnv - 1);
  }
  size_t s = 0, row = 0;
  std::vector<Pass> passes;
  std::vector<std::pair<size_t, size_t>> pass_rows;  // [row0, row1) of each pass
  while (s < series_nrows.size()) {
    Pass ps;
    ps.p = p;
    ps.hp = hp;
    ps.horizon = horizon;
    ps.ctx = ctx_dev;
    size_t row0 = row;
    while (s < series_nrows.size()) {
      const int nv = series_nrows[s];
      if (ps.R > 0 && (size_t)(ps.R + nv) > max_rows) break;
      ps.s_row0.push_back(ps.R);
      ps.s_nrows.push_back(nv);
      for (int v = 0; v < nv; ++v, ++row) {
        const RowSpec &rs = rows[row];
        ps.row_off.push_back(rs.off);
        ps.row_len.push_back(rs.len);
        const int lead = ctx_w - rs.len;
        ps.row_lead.push_back(lead);
        ps.row_fv.push_back(lead / 32);
      }
      ps.R += nv;
      ++s;
    }
    ps.out = out_dev + row0 * (size_t)horizon * m->nq;
    pass_rows.push_back({row0, row});
    passes.push_back(std::move(ps));
  }
  if (!hio) {
    for (const Pass &ps : passes) {
      t0b_status st = run_pass(m, ps);
      if (st != T0B_OK) return st;
    }
    return T0B_OK;
  }
  // host buffers: pass i's contexts go up on the copy stream while pass i-1
  // computes, and pass i-1's quantiles come down while pass i computes
  if (!m->io_stream) CUDA_TRY(cudaStreamCreateWithFlags(&m->io_stream, cudaStreamNonBlocking));
  for (int i = 0; i < 2; ++i) {
    if (!m->io_in[i]) CUDA_TRY(cudaEventCreateWithFlags(&m->io_in[i], cudaEventDisableTiming));
    if (!m->io_done[i]) CUDA_TRY(cudaEventCreateWithFlags(&m->io_done[i], cudaEventDisableTiming));
  }
  const size_t per_row_out = (size_t)horizon * m->nq;
  auto h2d = [&](size_t i) -> t0b_status {
    const RowSpec &a = rows[pass_rows[i].first], &b = rows[pass_rows[i].second - 1];
    const size_t n = (size_t)(b.off + b.len - a.off);
    CUDA_TRY(cudaMemcpyAsync(const_cast<float *>(ctx_dev) + a.off, hio->ctx + a.off, n * 4, cudaMemcpyHostToDevice,
                             m->io_stream));
    CUDA_TRY(cudaEventRecord(m->io_in[i & 1], m->io_stream));
    return T0B_OK;
  };
  auto d2h = [&](size_t i) -> t0b_status {
    const size_t r0 = pass_rows[i].first, r1 = pass_rows[i].second;
    CUDA_TRY(cudaStreamWaitEvent(m->io_stream, m->io_done[i & 1], 0));
    CUDA_TRY(cudaMemcpyAsync(hio->out + r0 * per_row_out, out_dev + r0 * per_row_out, (r1 - r0) * per_row_out * 4,
                             cudaMemcpyDeviceToHost, m->io_stream));
    return T0B_OK;
  };
  t0b_status st = passes.empty() ? T0B_OK : h2d(0);
  for (size_t i = 0; i < passes.size() && st == T0B_OK; ++i) {
    CUDA_TRY(cudaStreamWaitEvent(m->stream, m->io_in[i & 1], 0));
    if ((st = run_pass(m, passes[i])) != T0B_OK) break;
    CUDA_TRY(cudaEventRecord(m->io_done[i & 1], m->stream));
    if (i + 1 < passes.size() && (st = h2d(i + 1)) != T0B_OK) break;
    if (i >= 1) st = d2h(i - 1);
  }
  if (st == T0B_OK && !passes.empty()) st = d2h(passes.size() - 1);
  CUDA_TRY(cudaStreamSynchronize(m->io_stream));
  return st;
}

struct Staged {
  float *ctx;
  float *out;
};

t0b_status stage_io(t0b_model *m, const float *ctx, size_t n_ctx, size_t n_out, Staged *sg) {
  CUDA_TRY(m->ctx_stage.reserve(std::max<size_t>(n_ctx, 1) * 4));
  CUDA_TRY(m->out_stage.reserve(std::max<size_t>(n_out, 1) * 4));
  CUDA_TRY(cudaMemcpyAsync(m->ctx_stage.p, ctx, n_ctx * 4, cudaMemcpyHostToDevice, m->stream));
  sg->ctx = m->ctx_stage.as<float>();
  sg->out = m->out_stage.as<float>();
  return T0B_OK;
}

t0b_status finish_io(t0b_model *m, const Staged &sg, float *out, size_t n_out) {
  CUDA_TRY(cudaMemcpyAsync(out, sg.out, n_out * 4, cudaMemcpyDeviceToHost, m->stream));
  return sync_model(m);
}

}  // namespace

extern "C" t0b_status t0b_gguf_validate(const uint8_t *bytes, size_t len, t0b_model_info *out) {
  if (!bytes || !out) return fail(T0B_ERR_INVALID, "t0b_gguf_validate: NULL argument");
  t0b::GgufFile f;
  std::string err;
  if (!t0b::parse_gguf(bytes, len, f, err)) return fail(T0B_ERR_FORMAT, err);
  t0b_model m;
  t0b_status s = parse_config(f, &m);
  if (s != T0B_OK) return s;
  *out = m.info;
  out->total_weight_bytes = 0;
  return T0B_OK;
}

extern "C" t0b_status t0b_model_load_gguf(t0b_engine *e, const uint8_t *bytes, size_t len, t0b_model **out) {
  if (!e || !bytes || !out) return fail(T0B_ERR_INVALID, "t0b_model_load_gguf: NULL argument");
  *out = nullptr;
  CUDA_TRY(cudaSetDevice(e->device));
  std::unique_ptr<t0b_model> m(new t0b_model());
  m->eng = e;
  t0b_status s = load_model(m.get(), bytes, len);
  if (s != T0B_OK) return s;
  CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  m->own_stream = true;
  CUDA_TRY(cudaMalloc(&m->d_err, sizeof(int)));
  CUDA_TRY(cudaMemset(m->d_err, 0, sizeof(int)));
  *out = m.release();
  return T0B_OK;
}

extern "C" void t0b_model_destroy(t0b_model *m) {
  if (!m) return;
  cudaSetDevice(m->eng->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  delete m;
}

extern "C" t0b_status t0b_model_info_get(const t0b_model *m, t0b_model_info *out) {
  if (!m || !out) return fail(T0B_ERR_INVALID, "t0b_model_info_get: NULL argument");
  *out = m->info;
  return T0B_OK;
}

extern "C" t0b_status t0b_model_set_stream(t0b_model *m, void *stream) {
  if (!m) return fail(T0B_ERR_INVALID, "t0b_model_set_stream: NULL model");
  if (stream) {
    if (m->own_stream && m->stream) cudaStreamDestroy(m->stream);
    m->own_stream = false;
    m->stream = (cudaStream_t)stream;
  }
  return T0B_OK;
}

extern "C" void *t0b_model_stream(const t0b_model *m) { return m ? (void *)m->stream : nullptr; }

extern "C" t0b_status t0b_model_set_max_tokens(t0b_model *m, size_t max_tokens) {
  if (!m || max_tokens < 64) return fail(T0B_ERR_INVALID, "t0b_model_set_max_tokens: need >= 64");
  m->max_tokens = max_tokens;
  return T0B_OK;
}

extern "C" t0b_status t0b_model_use_graphs(t0b_model *m, int on) {
  if (!m) return fail(T0B_ERR_INVALID, "t0b_model_use_graphs: NULL model");
  CUDA_TRY(cudaSetDevice(m->eng->device));
  CUDA_TRY(cudaStreamSynchronize(m->stream));
  m->use_graphs = on != 0;
  if (!on) m->drop_graphs();
  return T0B_OK;
}

extern "C" t0b_status t0b_model_profile_enable(t0b_model *m, int on) {
  if (!m) return fail(T0B_ERR_INVALID, "t0b_model_profile_enable: NULL model");
  CUDA_TRY(cudaSetDevice(m->eng->device));
  CUDA_TRY(cudaStreamSynchronize(m->stream));
  fold_records(m);
  std::memset(m->stats, 0, sizeof(m->stats));
  for (int i = 0; i < KC_N; ++i) std::snprintf(m->stats[i].name, sizeof(m->stats[i].name), "%s", kKcNames[i]);
  m->prof = on != 0;
  return T0B_OK;
}

extern "C" t0b_status t0b_model_profile_read(t0b_model *m, t0b_kernel_stats *out, int max_classes, int *n_classes) {
  if (!m || !out || !n_classes) return fail(T0B_ERR_INVALID, "t0b_model_profile_read: NULL argument");
  CUDA_TRY(cudaSetDevice(m->eng->device));
  CUDA_TRY(cudaStreamSynchronize(m->stream));
  fold_records(m);
  const int n = std::min(max_classes, (int)KC_N);
  for (int i = 0; i < n; ++i) {
    out[i] = m->stats[i];
    std::snprintf(out[i].name, sizeof(out[i].name), "%s", kKcNames[i]);
  }
  *n_classes = n;
  return T0B_OK;
}

extern "C" uint64_t t0b_model_launch_count(const t0b_model *m) { return m ? m->launches : 0; }

extern "C" t0b_status t0b_model_sync(t0b_model *m) {
  if (!m) return fail(T0B_ERR_INVALID, "t0b_model_sync: NULL model");
  CUDA_TRY(cudaSetDevice(m->eng->device));
  return sync_model(m);
}

extern "C" t0b_status t0b_forecast_multiseries_device(t0b_model *m, const float *ctx_dev, const int32_t *n_variates,
                                                      size_t n_series, size_t t_ctx, size_t horizon,
                                                      float *out_dev) {
  if (!m || !ctx_dev || !n_variates || !out_dev) return fail(T0B_ERR_INVALID, "t0b_forecast_multiseries: NULL argument");
  t0b_status s = check_horizon(horizon);
  if (s != T0B_OK) return s;
  if (t_ctx == 0) return fail(T0B_ERR_INVALID, "t0b: context length must be >= 1");
  CUDA_TRY(cudaSetDevice(m->eng->device));
  const int pad_left = (int)((32 - t_ctx % 32) % 32);  // data.rs:112
  std::vector<RowSpec> rows;
  std::vector<int> nr;
  int64_t off = 0;
  for (size_t i = 0; i < n_series; ++i) {
    if (n_variates[i] < 1) return fail(T0B_ERR_INVALID, "t0b: every series needs >= 1 variate");
    nr.push_back(n_variates[i]);
    for (int v = 0; v < n_variates[i]; ++v, off += (int64_t)t_ctx) rows.push_back({off, (int)t_ctx});
  }
  return run_series(m, ctx_dev, rows, nr, (int)t_ctx + pad_left, (int)horizon, out_dev, 0);
}

extern "C" t0b_status t0b_forecast_multiseries(t0b_model *m, const float *ctx, const int32_t *n_variates,
                                               size_t n_series, size_t t_ctx, size_t horizon, float *out) {
  if (!m || !ctx || !n_variates || !out) return fail(T0B_ERR_INVALID, "t0b_forecast_multiseries: NULL argument");
  size_t rows = 0;
  for (size_t i = 0; i < n_series; ++i) rows += (size_t)std::max(n_variates[i], 0);
  CUDA_TRY(cudaSetDevice(m->eng->device));
  t0b_status s = check_horizon(horizon);
  if (s != T0B_OK) return s;
  if (t_ctx == 0) return fail(T0B_ERR_INVALID, "t0b: context length must be >= 1");
  CUDA_TRY(m->ctx_stage.reserve(std::max<size_t>(rows * t_ctx, 1) * 4));
  CUDA_TRY(m->out_stage.reserve(std::max<size_t>(rows * horizon * m->nq, 1) * 4));
  const int pad_left = (int)((32 - t_ctx % 32) % 32);  // data.rs:112
  std::vector<RowSpec> rs;
  std::vector<int> nr;
  int64_t off = 0;
  for (size_t i = 0; i < n_series; ++i) {
    if (n_variates[i] < 1) return fail(T0B_ERR_INVALID, "t0b: every series needs >= 1 variate");
    nr.push_back(n_variates[i]);
    for (int v = 0; v < n_variates[i]; ++v, off += (int64_t)t_ctx) rs.push_back({off, (int)t_ctx});
  }
  // contexts up and quantiles down per pass, overlapped with the other passes
  const HostIO hio{ctx, out};
  s = run_series(m, m->ctx_stage.as<float>(), rs, nr, (int)t_ctx + pad_left, (int)horizon, m->out_stage.as<float>(), 0,
                 &hio);
  if (s != T0B_OK) return s;
  return sync_model(m);
}

extern "C" t0b_status t0b_forecast(t0b_model *m, const float *ctx, size_t v, size_t t_ctx, size_t horizon,
                                   float *out) {
  if (v == 0) return fail(T0B_ERR_INVALID, "t0b_forecast: v must be >= 1");
  int32_t nv = (int32_t)v;
  return t0b_forecast_multiseries(m, ctx, &nv, 1, t_ctx, horizon, out);
}

extern "C" t0b_status t0b_forecast_batch(t0b_model *m, const float *ctx, size_t n, size_t t_ctx, size_t horizon,
                                         size_t chunk, float *out) {
  if (!m || !ctx || !out) return fail(T0B_ERR_INVALID, "t0b_forecast_batch: NULL argument");
  t0b_status s = check_horizon(horizon);
  if (s != T0B_OK) return s;
  if (t_ctx == 0) return fail(T0B_ERR_INVALID, "t0b: context length must be >= 1");
  CUDA_TRY(cudaSetDevice(m->eng->device));
  CUDA_TRY(m->ctx_stage.reserve(std::max<size_t>(n * t_ctx, 1) * 4));
  CUDA_TRY(m->out_stage.reserve(std::max<size_t>(n * horizon * m->nq, 1) * 4));
  const int pad_left = (int)((32 - t_ctx % 32) % 32);
  std::vector<RowSpec> rows(n);
  std::vector<int> nr(n, 1);  // data.rs:96-105: a distinct group per signal
  for (size_t i = 0; i < n; ++i) rows[i] = {(int64_t)(i * t_ctx), (int)t_ctx};
  const HostIO hio{ctx, out};
  if ((s = run_series(m, m->ctx_stage.as<float>(), rows, nr, (int)t_ctx + pad_left, (int)horizon,
                      m->out_stage.as<float>(), chunk, &hio)) != T0B_OK)
    return s;
  return sync_model(m);
}

extern "C" t0b_status t0b_forecast_batch_rows(t0b_model *m, const float *ctx, const size_t *lengths, size_t n,
                                              size_t horizon, size_t chunk, float *out) {
  if (!m || !ctx || !lengths || !out) return fail(T0B_ERR_INVALID, "t0b_forecast_batch_rows: NULL argument");
  t0b_status s = check_horizon(horizon);
  if (s != T0B_OK) return s;
  size_t total = 0;
  for (size_t i = 0; i < n; ++i) {
    if (lengths[i] == 0) return fail(T0B_ERR_INVALID, "t0b_forecast_batch_rows: empty row");
    total += lengths[i];
  }
  CUDA_TRY(cudaSetDevice(m->eng->device));
  Staged sg;
  if ((s = stage_io(m, ctx, total, n * horizon * m->nq, &sg)) != T0B_OK) return s;
  // lib.rs:183-240: each chunk is padded to its common patch-aligned width
  const size_t cs = (chunk == 0 || chunk > n) ? n : chunk;
  int64_t off = 0;
  for (size_t start = 0; start < n; start += cs) {
    const size_t k = std::min(cs, n - start);
    int common = 0;
    for (size_t i = 0; i < k; ++i) common = std::max(common, (int)((lengths[start + i] + 31) / 32 * 32));
    std::vector<RowSpec> rows(k);
    std::vector<int> nr(k, 1);
    for (size_t i = 0; i < k; ++i) {
      rows[i] = {off, (int)lengths[start + i]};
      off += (int64_t)lengths[start + i];
    }
    if ((s = run_series(m, sg.ctx, rows, nr, common, (int)horizon, sg.out + start * horizon * m->nq, 0)) != T0B_OK)
      return s;
  }
  return finish_io(m, sg, out, n * horizon * m->nq);
}

cudaError_t t0b_smem_limit(const void *kernel, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void *, int>, size_t> limit;  // (kernel, device) -> bytes set
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  size_t &cur = limit[{kernel, dev}];
  if (bytes <= cur) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) cur = bytes;
  return e;
}

// ================================================== autoregressive rollout
// t0-fast lib.rs:259-345 (port of t0-core model.rs:582-665) over this
// library's own forecast entry points; the quantile reductions are host f32
// code restating t0-core quantile.rs with the same operation order.
namespace {
// indices of key in stable ascending order (Rust's sort_by is stable)
std::vector<int> stable_order(const float *key, int n) {
  std::vector<int> idx(n);
  for (int i = 0; i < n; ++i) idx[i] = i;
  std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return key[a] < key[b]; });
  return idx;
}

// quantile.rs:17-43
void interpolate_quantiles(const float *query, int nq, const float *levels, const float *values, int n, float *out) {
  const std::vector<int> idx = stable_order(levels, n);
  std::vector<float> lv, vv;
  lv.reserve(n + 2);
  vv.reserve(n + 2);
  if (levels[idx[0]] > 0.0f) lv.push_back(0.0f), vv.push_back(values[idx[0]]);
  for (int i : idx) lv.push_back(levels[i]), vv.push_back(values[i]);
  if (lv.back() < 1.0f) lv.push_back(1.0f), vv.push_back(vv.back());
  const int len = (int)lv.size();
  for (int k = 0; k < nq; ++k) {
    const float q = query[k];
    int upper = (int)(std::upper_bound(lv.begin(), lv.end(), q) - lv.begin());  // partition_point(l <= q)
    upper = std::min(upper, len - 1);
    const int lower = upper > 0 ? upper - 1 : 0;
    const float ll = lv[lower], ul = lv[upper], lo = vv[lower], uo = vv[upper];
    const float diff = ul - ll;
    const float w = diff == 0.0f ? 0.0f : (q - ll) / diff;
    const float step = w * (uo - lo);
    out[k] = lo + step;
  }
}

// quantile.rs:47-61
void weighted_quantile(const float *query, int nq, const float *weights, const float *samples, int n, float *out) {
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) sum += weights[i];
  const std::vector<int> idx = stable_order(samples, n);
  std::vector<float> ss(n), cw(n);
  float cum = 0.0f;
  for (int i = 0; i < n; ++i) {
    ss[i] = samples[idx[i]];
    cum += weights[idx[i]] / sum;
    cw[i] = std::min(std::max(cum, 0.0f), 1.0f);
  }
  interpolate_quantiles(query, nq, cw.data(), ss.data(), n, out);
}

// quantile.rs:66-78
std::vector<float> prob_mass(const float *levels, int n) {
  std::vector<float> mass(n);
  for (int i = 0; i < n; ++i) {
    const float lo = i == 0 ? 0.0f : levels[i - 1];
    const float hi = i == n - 1 ? 1.0f : levels[i + 1];
    mass[i] = (hi - lo) / 2.0f;
  }
  float sum = 0.0f;
  for (float v : mass) sum += v;
  for (float &v : mass) v /= sum;
  return mass;
}
}  // namespace

extern "C" t0b_status t0b_forecast_rollout(t0b_model *m, const float *ctx, size_t t_ctx, size_t prediction_length,
                                           const float *query, size_t n_query, float *out) {
  const NvtxRange range("t0b forecast_rollout");
  if (!m || !ctx || !query || !out) return fail(T0B_ERR_INVALID, "t0b_forecast_rollout: NULL argument");
  if (t_ctx == 0 || prediction_length == 0 || n_query == 0 || n_query > 64)
    return fail(T0B_ERR_INVALID, "t0b_forecast_rollout: need t_ctx >= 1, prediction_length >= 1, 1..64 levels");
  for (size_t i = 0; i < n_query; ++i)
    if (!(query[i] > 0.0f && query[i] < 1.0f) || (i && !(query[i] > query[i - 1])))
      return fail(T0B_ERR_INVALID, "t0b_forecast_rollout: query levels must be ascending and inside (0, 1)");
  const size_t P = (size_t)m->P, kMaxH = (size_t)kMaxHorizon;
  const int ntr = m->nq, nq = (int)n_query;
  const float *trained = m->info.quantile_levels;
  const std::vector<float> trained_mass = prob_mass(trained, ntr), query_mass = prob_mass(query, nq);
  const size_t context_width = (t_ctx + P - 1) / P * P;
  const size_t horizon0 = std::min((prediction_length + P - 1) / P * P, kMaxH);

  std::vector<float> block((size_t)horizon0 * ntr);
  t0b_status st = t0b_forecast(m, ctx, 1, t_ctx, horizon0, block.data());
  if (st != T0B_OK) return st;
  std::vector<float> res(horizon0 * nq);  // all blocks, query-level minor
  for (size_t h = 0; h < horizon0; ++h)
    interpolate_quantiles(query, nq, trained, block.data() + h * ntr, ntr, res.data() + h * nq);
  if (prediction_length > horizon0) {
    // each query level is one path: its context plus everything fed back
    std::vector<std::vector<float>> paths(nq, std::vector<float>(ctx, ctx + t_ctx));
    size_t remaining = prediction_length - horizon0, prev_off = 0, prev_width = horizon0;
    std::vector<float> weights((size_t)nq * ntr), samples((size_t)nq * ntr), batch, blocks;
    for (int j = 0; j < nq; ++j)
      for (int pq = 0; pq < ntr; ++pq) weights[(size_t)j * ntr + pq] = trained_mass[pq] * query_mass[j];
    while (remaining > 0) {
      for (int j = 0; j < nq; ++j)
        for (size_t h = 0; h < prev_width; ++h) paths[j].push_back(res[(prev_off + h) * nq + j]);
      const size_t horizon = std::min((remaining + P - 1) / P * P, kMaxH);
      batch.assign((size_t)nq * context_width, 0.0f);
      for (int j = 0; j < nq; ++j) {  // trailing window, right-aligned
        const size_t w = std::min(context_width, paths[j].size());
        std::copy(paths[j].end() - w, paths[j].end(), batch.begin() + (size_t)j * context_width + (context_width - w));
      }
      // the n_query paths are one batch: one device pass per block
      blocks.assign((size_t)nq * horizon * ntr, 0.0f);
      if ((st = t0b_forecast_batch(m, batch.data(), nq, context_width, horizon, nq, blocks.data())) != T0B_OK)
        return st;
      prev_off = res.size() / nq;
      res.resize(res.size() + horizon * nq);
      for (size_t h = 0; h < horizon; ++h) {
        for (int j = 0; j < nq; ++j)
          for (int pq = 0; pq < ntr; ++pq)
            samples[(size_t)j * ntr + pq] = blocks[((size_t)j * horizon + h) * ntr + pq];
        weighted_quantile(query, nq, weights.data(), samples.data(), nq * ntr, res.data() + (prev_off + h) * nq);
      }
      prev_width = horizon;
      remaining = remaining > horizon ? remaining - horizon : 0;  // the last block may overshoot
    }
  }
  std::memcpy(out, res.data(), prediction_length * n_query * sizeof(float));
  return T0B_OK;
}

// ======================================================= standalone GEMMs
namespace {
// Grows engine scratch; growing waits for the stream first, since work
// already queued may still read the old buffers.
t0b_status qm_reserve(DBuf &b, size_t bytes, cudaStream_t st) {
  if (bytes <= b.bytes) return T0B_OK;
  CUDA_TRY(cudaStreamSynchronize(st));
  CUDA_TRY(b.reserve(bytes));
  return T0B_OK;
}

t0b_status split_input(t0b_engine *e, const float *x, size_t n, cudaStream_t st) {
  t0b_status s;
  if ((s = qm_reserve(e->scratch_xh, n * 2, st)) != T0B_OK || (s = qm_reserve(e->scratch_xl, n * 2, st)) != T0B_OK)
    return s;
  CUDA_TRY(t0b_launch_split_f32(x, e->scratch_xh.as<__half>(), e->scratch_xl.as<__half>(), n, st));
  return T0B_OK;
}
int qt_of(int ggml_type) { return ggml_type == T0B_Q8_0 ? 8 : (ggml_type == T0B_Q4_0 ? 4 : 0); }

// Prescale exponent of a device-resident weight matrix (one reduction + copy).
t0b_status device_weight_shift(t0b_engine *e, int qt, const uint8_t *W, size_t n_elements, cudaStream_t st,
                               int *shift) {
  CUDA_TRY(e->scratch_red.reserve(sizeof(unsigned int)));
  const int bpb = qt == 8 ? 34 : 18;
  CUDA_TRY(t0b_launch_absmax_scale(W, n_elements / 32, bpb, e->scratch_red.as<unsigned int>(), st));
  unsigned int bits = 0;
  CUDA_TRY(cudaMemcpyAsync(&bits, e->scratch_red.p, sizeof(bits), cudaMemcpyDeviceToHost, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  float maxd;
  std::memcpy(&maxd, &bits, 4);
  *shift = t0b_weight_shift(maxd, qt);
  return T0B_OK;
}

// The standalone GEMMs take the tensor-core path from 128 tokens, and for
// the small shapes the small-M kernel cannot run.
bool engine_use_tc(int qt, int M, int K, const Epi &epi) { return M >= 128 || !t0b_small_supports(qt, M, K, epi); }

cudaError_t engine_qgemm(t0b_engine *e, int qt, const __half *ah, const __half *al, int M, int K, const uint8_t *W,
                         int wrows, int wshift, Epi &epi, int *err, cudaStream_t st) {
  const bool tc = engine_use_tc(qt, M, K, epi);
  if (tc) return t0b_launch_gemm_tc(qt, ah, al, M, K, W, wrows, wshift, epi, err, st);
  return t0b_launch_gemm_small(qt, ah, al, M, K, W, epi, err, st);
}

// GEMM on f32 activations x [M][K]: where the small-M kernel's K slices are
// 256 wide, it splits them into its f16 planes itself (no separate launch);
// otherwise (whole-K CTAs for 256 < K <= 1024, wider slices, the tensor-core
// kernel) the GEMM reads the planes of one split pass into the engine's
// scratch.
t0b_status engine_qgemm_x(t0b_engine *e, int qt, const float *x, int M, int K, const uint8_t *W, int wrows,
                          int wshift, Epi &epi, int *err, cudaStream_t st) {
  if (!engine_use_tc(qt, M, K, epi) && t0b_small_supports(qt, M, K, epi, true)) {
    CUDA_TRY(t0b_launch_gemm_small(qt, nullptr, nullptr, M, K, W, epi, err, st, x));
    return T0B_OK;
  }
  const t0b_status s = split_input(e, x, (size_t)M * K, st);
  if (s != T0B_OK) return s;
  CUDA_TRY(engine_qgemm(e, qt, e->scratch_xh.as<__half>(), e->scratch_xl.as<__half>(), M, K, W, wrows, wshift, epi,
                        err, st));
  return T0B_OK;
}

t0b_status engine_check(t0b_engine *e, cudaStream_t st) {
  CUDA_TRY(cudaStreamSynchronize(st));
  int herr = 0;
  CUDA_TRY(cudaMemcpy(&herr, e->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (herr) {
    cudaMemset(e->d_err, 0, sizeof(int));
    return fail(T0B_ERR_DEVICE, "t0b: a kernel reported device error code " + std::to_string(herr));
  }
  return T0B_OK;
}
}  // namespace

extern "C" t0b_status t0b_gemm_q(t0b_engine *e, int ggml_type, const void *w_dev, int N, int K, const float *x_dev,
                                 int M, const float *bias_dev, float *y_dev, void *stream) {
  if (!e || !w_dev || !x_dev || !y_dev) return fail(T0B_ERR_INVALID, "t0b_gemm_q: NULL argument");
  const int qt = qt_of(ggml_type);
  if (!qt) return fail(T0B_ERR_UNSUPPORTED, "t0b_gemm_q: weight type must be Q8_0 or Q4_0");
  if (M < 1 || N < 1 || K < 1) return fail(T0B_ERR_INVALID, "t0b_gemm_q: empty shape");
  if (K % 256) return fail(T0B_ERR_UNSUPPORTED, "t0b_gemm_q: K must be a multiple of 256");
  if (N % 256) return fail(T0B_ERR_UNSUPPORTED, "t0b_gemm_q: N must be a multiple of 256");
  CUDA_TRY(cudaSetDevice(e->device));
  cudaStream_t st = (cudaStream_t)stream;
  t0b_status s;
  Epi ep{};
  ep.kind = EPI_PLAIN;
  ep.M = M;
  ep.N = N;
  ep.bias = bias_dev;
  ep.y = y_dev;
  ep.ldy = N;
  int sh = 0;  // tensor-core prescale; the small-M kernel applies block scales in f32 and needs none
  if (engine_use_tc(qt, M, K, ep) &&
      (s = device_weight_shift(e, qt, (const uint8_t *)w_dev, (size_t)N * K, st, &sh)) != T0B_OK)
    return s;
  if ((s = engine_qgemm_x(e, qt, x_dev, M, K, (const uint8_t *)w_dev, N, sh, ep, e->d_err, st)) != T0B_OK) return s;
  return engine_check(e, st);
}

extern "C" t0b_status t0b_swiglu_q(t0b_engine *e, int ggml_type, const void *w0_dev, const void *w2_dev, int F, int K,
                                   int N2, const float *x_dev, int M, const float *b0_dev, const float *b2_dev,
                                   float *z_dev, float *y_dev, void *stream) {
  if (!e || !w0_dev || !w2_dev || !x_dev || !y_dev) return fail(T0B_ERR_INVALID, "t0b_swiglu_q: NULL argument");
  const int qt = qt_of(ggml_type);
  if (!qt) return fail(T0B_ERR_UNSUPPORTED, "t0b_swiglu_q: weight type must be Q8_0 or Q4_0");
  if (M < 1 || F < 1 || K < 1 || N2 < 1) return fail(T0B_ERR_INVALID, "t0b_swiglu_q: empty shape");
  if (K % 256 || F % 256 || N2 % 256)
    return fail(T0B_ERR_UNSUPPORTED, "t0b_swiglu_q: K, F and N2 must be multiples of 256");
  CUDA_TRY(cudaSetDevice(e->device));
  cudaStream_t st = (cudaStream_t)stream;
  t0b_status s;
  if ((s = qm_reserve(e->scratch_zh, (size_t)M * F * 2, st)) != T0B_OK ||
      (s = qm_reserve(e->scratch_zl, (size_t)M * F * 2, st)) != T0B_OK)
    return s;
  Epi sg{};
  sg.kind = EPI_SWIGLU;
  sg.M = M;
  sg.N = 2 * F;
  sg.F = F;
  sg.bias = b0_dev;
  sg.zh = e->scratch_zh.as<__half>();
  sg.zl = e->scratch_zl.as<__half>();
  sg.z32 = z_dev;
  Epi dn{};
  dn.kind = EPI_PLAIN;
  dn.M = M;
  dn.N = N2;
  dn.bias = b2_dev;
  dn.y = y_dev;
  dn.ldy = N2;
  int sh0 = 0, sh2 = 0;  // tensor-core prescales, where that path runs
  if (engine_use_tc(qt, M, K, sg) &&
      (s = device_weight_shift(e, qt, (const uint8_t *)w0_dev, (size_t)2 * F * K, st, &sh0)) != T0B_OK)
    return s;
  if (engine_use_tc(qt, M, F, dn) &&
      (s = device_weight_shift(e, qt, (const uint8_t *)w2_dev, (size_t)N2 * F, st, &sh2)) != T0B_OK)
    return s;
  // the gate / up GEMM reads the planes of a split pass even on the small-M
  // path: launched as the split's programmatic dependent it prefetches its
  // weights while the split runs (M = 16: 23.6 us per call, 26.4 us with
  // the split inside the GEMM, whose CTAs then wait for the previous
  // kernel's to leave the SMs)
  if ((s = split_input(e, x_dev, (size_t)M * K, st)) != T0B_OK) return s;
  CUDA_TRY(engine_qgemm(e, qt, e->scratch_xh.as<__half>(), e->scratch_xl.as<__half>(), M, K, (const uint8_t *)w0_dev,
                        2 * F, sh0, sg, e->d_err, st));
  CUDA_TRY(engine_qgemm(e, qt, e->scratch_zh.as<__half>(), e->scratch_zl.as<__half>(), M, F, (const uint8_t *)w2_dev, N2,
                        sh2, dn, e->d_err, st));
  return engine_check(e, st);
}

// ================================================ resident-weight GEMMs
// A t0b_qmatrix keeps a device weight matrix's tensor-core prescale (found
// once, at creation) and its own error word; the activation scratch is the
// engine's.  Its GEMMs are pure stream work: no host synchronisation, and
// capturable in a CUDA graph once the scratch has reached its size.
struct t0b_qmatrix {
  t0b_engine *eng = nullptr;
  int qt = 0, N = 0, K = 0, shift = 0;
  const uint8_t *W = nullptr;
  int *d_err = nullptr;
  ~t0b_qmatrix() {
    if (d_err) cudaFree(d_err);
  }
};


extern "C" t0b_status t0b_qmatrix_create(t0b_engine *e, int ggml_type, const void *w_dev, int N, int K,
                                         t0b_qmatrix **out) {
  if (!e || !w_dev || !out) return fail(T0B_ERR_INVALID, "t0b_qmatrix_create: NULL argument");
  const int qt = qt_of(ggml_type);
  if (!qt) return fail(T0B_ERR_UNSUPPORTED, "t0b_qmatrix_create: weight type must be Q8_0 or Q4_0");
  if (N < 1 || K < 1) return fail(T0B_ERR_INVALID, "t0b_qmatrix_create: empty shape");
  if (K % 256 || N % 256) return fail(T0B_ERR_UNSUPPORTED, "t0b_qmatrix_create: N and K must be multiples of 256");
  CUDA_TRY(cudaSetDevice(e->device));
  auto q = std::make_unique<t0b_qmatrix>();
  q->eng = e;
  q->qt = qt;
  q->N = N;
  q->K = K;
  q->W = (const uint8_t *)w_dev;
  if (cudaMalloc(&q->d_err, sizeof(int)) != cudaSuccess) return fail(T0B_ERR_OOM, "t0b: out of device memory");
  CUDA_TRY(cudaMemset(q->d_err, 0, sizeof(int)));
  t0b_status s = device_weight_shift(e, qt, q->W, (size_t)N * K, nullptr, &q->shift);
  if (s != T0B_OK) return s;
  *out = q.release();
  return T0B_OK;
}

extern "C" void t0b_qmatrix_destroy(t0b_qmatrix *q) {
  if (!q) return;
  cudaSetDevice(q->eng->device);
  delete q;
}

extern "C" t0b_status t0b_qmatrix_gemm(t0b_qmatrix *q, const float *x_dev, int M, const float *bias_dev, float *y_dev,
                                       void *stream) {
  if (!q || !x_dev || !y_dev) return fail(T0B_ERR_INVALID, "t0b_qmatrix_gemm: NULL argument");
  if (M < 1) return fail(T0B_ERR_INVALID, "t0b_qmatrix_gemm: empty shape");
  CUDA_TRY(cudaSetDevice(q->eng->device));
  cudaStream_t st = (cudaStream_t)stream;
  Epi ep{};
  ep.kind = EPI_PLAIN;
  ep.M = M;
  ep.N = q->N;
  ep.bias = bias_dev;
  ep.y = y_dev;
  ep.ldy = q->N;
  return engine_qgemm_x(q->eng, q->qt, x_dev, M, q->K, q->W, q->N, q->shift, ep, q->d_err, st);
}

extern "C" t0b_status t0b_qmatrix_swiglu(t0b_qmatrix *q0, t0b_qmatrix *q2, const float *x_dev, int M,
                                         const float *b0_dev, const float *b2_dev, float *z_dev, float *y_dev,
                                         void *stream) {
  if (!q0 || !q2 || !x_dev || !y_dev) return fail(T0B_ERR_INVALID, "t0b_qmatrix_swiglu: NULL argument");
  if (M < 1) return fail(T0B_ERR_INVALID, "t0b_qmatrix_swiglu: empty shape");
  if (q0->N % 2 || q2->K != q0->N / 2 || q0->qt != q2->qt || q0->eng != q2->eng)
    return fail(T0B_ERR_INVALID, "t0b_qmatrix_swiglu: need w0 [2F, K] and w2 [N2, F] of one type and engine");
  const int F = q0->N / 2, K = q0->K;
  if (F % 256) return fail(T0B_ERR_UNSUPPORTED, "t0b_qmatrix_swiglu: F must be a multiple of 256");
  CUDA_TRY(cudaSetDevice(q0->eng->device));
  cudaStream_t st = (cudaStream_t)stream;
  t0b_status s;
  t0b_engine *e = q0->eng;
  if ((s = qm_reserve(e->scratch_zh, (size_t)M * F * 2, st)) != T0B_OK ||
      (s = qm_reserve(e->scratch_zl, (size_t)M * F * 2, st)) != T0B_OK)
    return s;
  Epi sg{};
  sg.kind = EPI_SWIGLU;
  sg.M = M;
  sg.N = 2 * F;
  sg.F = F;
  sg.bias = b0_dev;
  sg.zh = e->scratch_zh.as<__half>();
  sg.zl = e->scratch_zl.as<__half>();
  sg.z32 = z_dev;
  // a split pass first, as in t0b_swiglu_q
  if ((s = split_input(e, x_dev, (size_t)M * K, st)) != T0B_OK) return s;
  CUDA_TRY(engine_qgemm(e, q0->qt, e->scratch_xh.as<__half>(), e->scratch_xl.as<__half>(), M, K, q0->W, 2 * F,
                        q0->shift, sg, q0->d_err, st));
  Epi dn{};
  dn.kind = EPI_PLAIN;
  dn.M = M;
  dn.N = q2->N;
  dn.bias = b2_dev;
  dn.y = y_dev;
  dn.ldy = q2->N;
  CUDA_TRY(engine_qgemm(e, q2->qt, e->scratch_zh.as<__half>(), e->scratch_zl.as<__half>(), M, F, q2->W, q2->N,
                        q2->shift, dn, q2->d_err, st));
  return T0B_OK;
}

extern "C" t0b_status t0b_qmatrix_sync(t0b_qmatrix *q, void *stream) {
  if (!q) return fail(T0B_ERR_INVALID, "t0b_qmatrix_sync: NULL argument");
  CUDA_TRY(cudaSetDevice(q->eng->device));
  CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
  int herr = 0;
  CUDA_TRY(cudaMemcpy(&herr, q->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (herr) {
    cudaMemset(q->d_err, 0, sizeof(int));
    return fail(T0B_ERR_DEVICE, "t0b_qmatrix: a kernel reported device error code " + std::to_string(herr));
  }
  return T0B_OK;
}

// ================================================ bounded-wait self-test
extern "C" t0b_status t0b_selftest_bounded_wait(t0b_engine *e, int *device_code, int *outcome) {
  if (!e || !device_code || !outcome) return fail(T0B_ERR_INVALID, "t0b_selftest_bounded_wait: NULL argument");
  CUDA_TRY(cudaSetDevice(e->device));
  *device_code = 0;
  *outcome = 0;
  int *d = nullptr;  // [0] error word, [1] outcome
  CUDA_TRY(cudaMalloc(&d, 2 * sizeof(int)));
  std::unique_ptr<int, decltype(&cudaFree)> guard(d, &cudaFree);
  cudaStream_t st = nullptr;
  CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  std::unique_ptr<CUstream_st, decltype(&cudaStreamDestroy)> sguard(st, &cudaStreamDestroy);
  CUDA_TRY(cudaMemsetAsync(d, 0, 2 * sizeof(int), st));
  CUDA_TRY(t0b_launch_bounded_wait_selftest(d, d + 1, st));
  int h[2] = {0, 0};
  CUDA_TRY(cudaMemcpyAsync(h, d, sizeof(h), cudaMemcpyDeviceToHost, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  *device_code = h[0];
  *outcome = h[1];
  if (h[0])
    return fail(T0B_ERR_DEVICE, "t0b_selftest_bounded_wait: a kernel reported device error code " + std::to_string(h[0]));
  return T0B_OK;
}

// ================================================ no-allocation standalone GEMM
// t0b_gemm_q_noalloc works out of one fixed array that is part of this
// library's device code, so a call allocates nothing.  Layout:
//   bytes [0, 4)              absmax bits of the weight-block scales
//   bytes [4, 8)              kernel error word
//   bytes [256, 256 + 2X)     hi f16 half of x   (X = T0B_NOALLOC_MAX_X_ELEMENTS)
//   bytes [256 + 2X, 256 + 4X) lo f16 half of x
// Both control words must be zero when the kernels that use them start: the
// absmax launcher clears its word on the stream, and the call clears the
// error word first.  The x halves are written in full before they are read.
static __device__ __align__(256) unsigned char g_noalloc_scratch[T0B_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned char *g_noalloc_addr[kNoallocMaxDevices];  // per device ordinal, filled on first use

// Device address of the scratch array on the current device (looked up once
// per device, with that device current).
t0b_status noalloc_scratch(unsigned char **out) {
  int dev = -1;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoallocMaxDevices)
    return fail(T0B_ERR_UNSUPPORTED, "t0b_gemm_q_noalloc: device ordinal " + std::to_string(dev) + " out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    int major = 0, minor = 0;
    CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0)
      return fail(T0B_ERR_UNSUPPORTED, "t0b_gemm_q_noalloc: built for sm_100a (B200); device is sm_" +
                                           std::to_string(major) + std::to_string(minor));
    unsigned char *p = nullptr;
    CUDA_TRY(cudaGetSymbolAddress((void **)&p, g_noalloc_scratch));
    if (!p || (reinterpret_cast<uintptr_t>(p) & 255))
      return fail(T0B_ERR_CUDA, "t0b_gemm_q_noalloc: scratch array address is not 256-byte aligned");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return T0B_OK;
}
}  // namespace

extern "C" t0b_status t0b_gemm_q_noalloc(int ggml_type, const void *w_dev, int N, int K, const float *x_dev, int M,
                                         const float *bias_dev, float *y_dev, void *stream) {
  if (!w_dev || !x_dev || !y_dev) return fail(T0B_ERR_INVALID, "t0b_gemm_q_noalloc: NULL argument");
  const int qt = qt_of(ggml_type);
  if (!qt) return fail(T0B_ERR_UNSUPPORTED, "t0b_gemm_q_noalloc: weight type must be Q8_0 or Q4_0");
  if (M < 1 || N < 1 || K < 1) return fail(T0B_ERR_INVALID, "t0b_gemm_q_noalloc: empty shape");
  if (K % 256) return fail(T0B_ERR_UNSUPPORTED, "t0b_gemm_q_noalloc: K must be a multiple of 256");
  if (N % 256) return fail(T0B_ERR_UNSUPPORTED, "t0b_gemm_q_noalloc: N must be a multiple of 256");
  const size_t n_x = (size_t)M * (size_t)K;
  if (n_x > T0B_NOALLOC_MAX_X_ELEMENTS)
    return fail(T0B_ERR_INVALID, "t0b_gemm_q_noalloc: M*K = " + std::to_string(n_x) + " exceeds the fixed scratch (" +
                                     std::to_string((size_t)T0B_NOALLOC_MAX_X_ELEMENTS) + " elements of x)");
  unsigned char *base = nullptr;
  t0b_status s = noalloc_scratch(&base);
  if (s != T0B_OK) return s;
  unsigned int *red = reinterpret_cast<unsigned int *>(base);
  int *err = reinterpret_cast<int *>(base + 4);
  __half *xh = reinterpret_cast<__half *>(base + 256);
  __half *xl = xh + T0B_NOALLOC_MAX_X_ELEMENTS;
  cudaStream_t st = (cudaStream_t)stream;
  Epi ep{};
  ep.kind = EPI_PLAIN;
  ep.M = M;
  ep.N = N;
  ep.bias = bias_dev;
  ep.y = y_dev;
  ep.ldy = N;
  const bool tc = engine_use_tc(qt, M, K, ep);
  CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), st));
  CUDA_TRY(t0b_launch_split_f32(x_dev, xh, xl, n_x, st));
  if (tc) {
    // weight prescale exponent from the largest block scale (clears `red`
    // first); only the tensor-core kernel uses it
    CUDA_TRY(t0b_launch_absmax_scale((const uint8_t *)w_dev, (size_t)N * K / 32, qt == 8 ? 34 : 18, red, st));
    unsigned int bits = 0;
    CUDA_TRY(cudaMemcpyAsync(&bits, red, sizeof(bits), cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    float maxd;
    std::memcpy(&maxd, &bits, 4);
    const int sh = t0b_weight_shift(maxd, qt);
    CUDA_TRY(t0b_launch_gemm_tc(qt, xh, xl, M, K, (const uint8_t *)w_dev, N, sh, ep, err, st));
  } else {
    CUDA_TRY(t0b_launch_gemm_small(qt, xh, xl, M, K, (const uint8_t *)w_dev, ep, err, st));
  }
  // the error word is read on the call's own stream (no legacy-stream copy)
  int herr = 0;
  CUDA_TRY(cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  if (herr) return fail(T0B_ERR_DEVICE, "t0b_gemm_q_noalloc: a kernel reported device error code " + std::to_string(herr));
  return T0B_OK;
}

// ============================================================ host codecs
extern "C" size_t t0b_row_bytes(int ggml_type, size_t n) { return t0b::row_bytes(ggml_type, n); }

extern "C" t0b_status t0b_quantize(int ggml_type, const float *x, size_t n, uint8_t *out) {
  if (!x || !out) return fail(T0B_ERR_INVALID, "t0b_quantize: NULL argument");
  if (n % 32) return fail(T0B_ERR_INVALID, "t0b_quantize: n must be a multiple of 32");
  if (ggml_type == T0B_Q8_0)
    t0b::quantize_q8_0(x, n, out);
  else if (ggml_type == T0B_Q4_0)
    t0b::quantize_q4_0(x, n, out);
  else
    return fail(T0B_ERR_UNSUPPORTED, "t0b_quantize: type must be Q8_0 or Q4_0");
  return T0B_OK;
}

extern "C" t0b_status t0b_dequantize(int ggml_type, const uint8_t *bytes, size_t n, float *out) {
  if (!bytes || !out) return fail(T0B_ERR_INVALID, "t0b_dequantize: NULL argument");
  if ((ggml_type == T0B_Q8_0 || ggml_type == T0B_Q4_0) && n % 32)
    return fail(T0B_ERR_INVALID, "t0b_dequantize: n must be a multiple of 32");
  if (ggml_type != T0B_F32 && ggml_type != T0B_F16 && ggml_type != T0B_Q8_0 && ggml_type != T0B_Q4_0)
    return fail(T0B_ERR_UNSUPPORTED, "t0b_dequantize: unsupported type");
  t0b::dequantize(ggml_type, bytes, n, out);
  return T0B_OK;
}

extern "C" t0b_status t0b_export_gguf(size_t n, const char *const *names, const int32_t *ndims, const int64_t *shapes,
                                      const float *const *data, int big_type, const t0b_model_info *cfg, uint8_t *out,
                                      size_t *out_len) {
  if (!names || !ndims || !shapes || !data || !cfg || !out_len)
    return fail(T0B_ERR_INVALID, "t0b_export_gguf: NULL argument");
  if (big_type != T0B_F16 && big_type != T0B_Q8_0 && big_type != T0B_Q4_0)
    return fail(T0B_ERR_UNSUPPORTED, "t0b_export_gguf: big_type must be F16, Q8_0 or Q4_0");
  std::vector<t0b::ExportTensor> ts(n);
  for (size_t i = 0; i < n; ++i) {
    if (ndims[i] < 1 || ndims[i] > 2) return fail(T0B_ERR_INVALID, "t0b_export_gguf: tensors must be 1-D or 2-D");
    ts[i].name = names[i];
    ts[i].shape.assign(shapes + 2 * i, shapes + 2 * i + ndims[i]);
    ts[i].data = data[i];
    const bool q = ndims[i] == 2 && (big_type == T0B_Q8_0 || big_type == T0B_Q4_0);
    if (q && ts[i].n_elements() % 32) return fail(T0B_ERR_INVALID, "t0b_export_gguf: quantized tensor size % 32 != 0");
  }
  t0b::ModelMeta mm;
  mm.embed_dim = cfg->embed_dim;
  mm.num_layers = cfg->num_layers;
  mm.num_heads = cfg->num_heads;
  mm.mlp_hidden_dim = cfg->mlp_hidden_dim;
  mm.patch_size = cfg->patch_size;
  mm.group_every_n = cfg->group_every_n;
  mm.dropout = cfg->dropout;
  mm.quantile_levels.assign(cfg->quantile_levels, cfg->quantile_levels + cfg->n_quantiles);
  mm.scaler_use_arcsinh = cfg->scaler_use_arcsinh != 0;
  mm.scaler_eps = cfg->scaler_eps;
  mm.variance_offset = cfg->variance_offset != 0;
  std::vector<uint8_t> b = t0b::export_gguf(ts, big_type, mm);
  if (!out) {
    *out_len = b.size();
    return T0B_OK;
  }
  if (*out_len < b.size()) return fail(T0B_ERR_INVALID, "t0b_export_gguf: output buffer too small");
  std::memcpy(out, b.data(), b.size());
  *out_len = b.size();
  return T0B_OK;
}
