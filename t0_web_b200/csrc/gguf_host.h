// gguf_host.h -- host GGUF v3 subset + Q8_0 / Q4_0 codecs (gguf.rs).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace t0b {

enum { GG_F32 = 0, GG_F16 = 1, GG_Q4_0 = 2, GG_Q8_0 = 8 };

struct MetaValue {
  int type = 0;
  uint32_t u = 0;
  float f = 0.0f;
  bool b = false;
  std::string s;
  std::vector<float> arr;
};

struct GgufTensor {
  std::vector<int64_t> shape;  // row-major
  int type = 0;
  size_t n_elements = 0, nbytes = 0;
  const uint8_t *data = nullptr;  // points into the caller's buffer
};

struct GgufFile {
  std::map<std::string, MetaValue> meta;
  std::map<std::string, GgufTensor> tensors;
};

struct ExportTensor {
  std::string name;
  std::vector<int64_t> shape;
  const float *data;
  size_t n_elements() const {
    size_t n = 1;
    for (auto d : shape) n *= (size_t)d;
    return n;
  }
};

struct ModelMeta {
  uint32_t embed_dim, num_layers, num_heads, mlp_hidden_dim, patch_size, group_every_n;
  float dropout;
  std::vector<float> quantile_levels;
  bool scaler_use_arcsinh;
  float scaler_eps;
  bool variance_offset;
};

uint16_t f32_to_f16(float x);
float f16_to_f32(uint16_t b);
size_t row_bytes(int type, size_t n);
void quantize_q8_0(const float *x, size_t n, uint8_t *out);
void quantize_q4_0(const float *x, size_t n, uint8_t *out);
void dequantize(int type, const uint8_t *in, size_t n, float *out);
bool parse_gguf(const uint8_t *bytes, size_t len, GgufFile &out, std::string &err);
std::vector<uint8_t> export_gguf(const std::vector<ExportTensor> &tensors, int big_type, const ModelMeta &m);

}  // namespace t0b
