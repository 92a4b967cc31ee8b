// gguf_host.cpp -- GGUF v3 container + Q8_0 / Q4_0 block codecs (host).
//
// The subset t0-web writes and reads (crates/t0-core/src/gguf.rs):
//   * header: "GGUF", u32 version 3, u64 tensor count, u64 metadata count;
//   * metadata values: u32 (type 4), f32 (6), bool (7), string (8), array of
//     f32 (9/6) -- anything else is rejected (gguf.rs:271-291);
//   * tensor infos: name, u32 n_dims, ne[] innermost first (reversed
//     row-major shape), u32 ggml type, u64 offset relative to the data blob;
//   * the data blob starts right after the tensor infos with no alignment
//     padding (gguf.rs:333-343, 387-389); offsets inside it are 32-aligned.
// Quantizers follow gguf.rs:100-157 exactly: f32 arithmetic, round half away
// from zero for Q8_0, floor(x*id + 8.5) clamped to [0,15] for Q4_0, the scale
// stored as IEEE binary16 rounded to nearest-even.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "gguf_host.h"

namespace t0b {

uint16_t f32_to_f16(float x) {
  _Float16 h = (_Float16)x;  // IEEE round-to-nearest-even, subnormals kept
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}
float f16_to_f32(uint16_t b) {
  _Float16 h;
  std::memcpy(&h, &b, 2);
  return (float)h;
}

size_t row_bytes(int type, size_t n) {
  switch (type) {
    case GG_F32: return n * 4;
    case GG_F16: return n * 2;
    case GG_Q4_0: return n / 32 * 18;
    case GG_Q8_0: return n / 32 * 34;
  }
  return 0;
}

void quantize_q8_0(const float *x, size_t n, uint8_t *out) {
  for (size_t b = 0; b < n / 32; ++b, x += 32, out += 34) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[i]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const uint16_t dh = f32_to_f16(d);
    std::memcpy(out, &dh, 2);  // little-endian host
    for (int i = 0; i < 32; ++i) {
      float q = std::round(x[i] * id);
      q = std::min(127.0f, std::max(-128.0f, q));
      out[2 + i] = (uint8_t)(int8_t)q;
    }
  }
}

void quantize_q4_0(const float *x, size_t n, uint8_t *out) {
  for (size_t b = 0; b < n / 32; ++b, x += 32, out += 18) {
    float amax = 0.0f, vmax = 0.0f;
    for (int i = 0; i < 32; ++i)
      if (std::fabs(x[i]) > amax) {
        amax = std::fabs(x[i]);
        vmax = x[i];
      }
    const float d = vmax / -8.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const uint16_t dh = f32_to_f16(d);
    std::memcpy(out, &dh, 2);
    for (int j = 0; j < 16; ++j) {
      const float a = x[j] * id, c = x[j + 16] * id;
      int lo = (int)std::floor(a + 8.5f), hi = (int)std::floor(c + 8.5f);
      lo = std::min(15, std::max(0, lo));
      hi = std::min(15, std::max(0, hi));
      out[2 + j] = (uint8_t)(lo | (hi << 4));
    }
  }
}

void dequantize(int type, const uint8_t *in, size_t n, float *out) {
  switch (type) {
    case GG_F32: std::memcpy(out, in, n * 4); return;
    case GG_F16:
      for (size_t i = 0; i < n; ++i) {
        uint16_t b;
        std::memcpy(&b, in + 2 * i, 2);
        out[i] = f16_to_f32(b);
      }
      return;
    case GG_Q8_0:
      for (size_t b = 0; b < n / 32; ++b) {
        uint16_t db;
        std::memcpy(&db, in + 34 * b, 2);
        const float d = f16_to_f32(db);
        for (int i = 0; i < 32; ++i) out[32 * b + i] = d * (float)(int8_t)in[34 * b + 2 + i];
      }
      return;
    case GG_Q4_0:
      for (size_t b = 0; b < n / 32; ++b) {
        uint16_t db;
        std::memcpy(&db, in + 18 * b, 2);
        const float d = f16_to_f32(db);
        for (int j = 0; j < 16; ++j) {
          const uint8_t v = in[18 * b + 2 + j];
          out[32 * b + j] = d * ((float)(v & 15) - 8.0f);
          out[32 * b + 16 + j] = d * ((float)(v >> 4) - 8.0f);
        }
      }
      return;
  }
}

// ------------------------------------------------------------------ reader
namespace {
struct Reader {
  const uint8_t *p;
  size_t n, pos = 0;
  bool bad = false;
  bool take(void *dst, size_t k) {
    if (bad || k > n - pos) {
      bad = true;
      return false;
    }
    std::memcpy(dst, p + pos, k);
    pos += k;
    return true;
  }
  uint32_t u32() {
    uint32_t v = 0;
    take(&v, 4);
    return v;
  }
  uint64_t u64() {
    uint64_t v = 0;
    take(&v, 8);
    return v;
  }
  float f32() {
    float v = 0;
    take(&v, 4);
    return v;
  }
  bool str(std::string &s) {
    uint64_t len = u64();
    if (bad || len > n - pos) {
      bad = true;
      return false;
    }
    s.assign(reinterpret_cast<const char *>(p + pos), len);
    pos += len;
    return true;
  }
};
}  // namespace

bool parse_gguf(const uint8_t *bytes, size_t len, GgufFile &out, std::string &err) {
  Reader r{bytes, len};
  char magic[4];
  if (!r.take(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) {
    err = "not a GGUF file (bad magic)";
    return false;
  }
  const uint32_t version = r.u32();
  if (version != 3) {
    err = "unsupported GGUF version " + std::to_string(version) + ", expected 3";
    return false;
  }
  const uint64_t n_tensors = r.u64(), n_meta = r.u64();
  if (r.bad || n_tensors > (1u << 20) || n_meta > (1u << 20)) {
    err = "gguf: truncated or implausible header";
    return false;
  }
  for (uint64_t i = 0; i < n_meta; ++i) {
    std::string key;
    if (!r.str(key)) break;
    const uint32_t ty = r.u32();
    MetaValue mv;
    mv.type = (int)ty;
    if (ty == 4) {
      mv.u = r.u32();
    } else if (ty == 6) {
      mv.f = r.f32();
    } else if (ty == 7) {
      uint8_t b = 0;
      r.take(&b, 1);
      mv.b = b != 0;
    } else if (ty == 8) {
      r.str(mv.s);
    } else if (ty == 9) {
      const uint32_t et = r.u32();
      const uint64_t cnt = r.u64();
      if (et != 6) {
        err = "gguf: only FLOAT32 arrays are supported by this reader, got type " + std::to_string(et);
        return false;
      }
      if (cnt > (r.n - r.pos) / 4) {
        err = "gguf: truncated metadata array";
        return false;
      }
      mv.arr.resize(cnt);
      for (uint64_t k = 0; k < cnt; ++k) mv.arr[k] = r.f32();
    } else {
      err = "gguf: unsupported metadata value type " + std::to_string(ty);
      return false;
    }
    out.meta[key] = mv;
  }
  struct Info {
    std::string name;
    std::vector<int64_t> shape;
    int type;
    uint64_t off;
  };
  std::vector<Info> infos;
  for (uint64_t i = 0; i < n_tensors && !r.bad; ++i) {
    Info inf;
    r.str(inf.name);
    const uint32_t nd = r.u32();
    if (nd < 1 || nd > 4) {
      err = "gguf: tensor " + inf.name + " has unsupported rank";
      return false;
    }
    inf.shape.resize(nd);
    for (uint32_t d = 0; d < nd; ++d) inf.shape[nd - 1 - d] = (int64_t)r.u64();  // back to row-major
    inf.type = (int)r.u32();
    if (inf.type != GG_F32 && inf.type != GG_F16 && inf.type != GG_Q4_0 && inf.type != GG_Q8_0) {
      err = "unsupported ggml tensor type id " + std::to_string(inf.type);
      return false;
    }
    inf.off = r.u64();
    infos.push_back(inf);
  }
  if (r.bad) {
    err = "gguf: truncated header";
    return false;
  }
  const size_t blob = r.pos;
  for (auto &inf : infos) {
    GgufTensor t;
    t.shape = inf.shape;
    t.type = inf.type;
    size_t ne = 1;
    for (auto d : inf.shape) ne *= (size_t)d;
    if ((t.type == GG_Q4_0 || t.type == GG_Q8_0) && ne % 32) {
      err = "gguf: quantized tensor " + inf.name + " is not a multiple of 32 elements";
      return false;
    }
    t.n_elements = ne;
    t.nbytes = row_bytes(t.type, ne);
    if (inf.off > len - blob || t.nbytes > len - blob - inf.off) {
      err = "gguf: tensor " + inf.name + " out of bounds";
      return false;
    }
    t.data = bytes + blob + inf.off;
    out.tensors[inf.name] = t;
  }
  return true;
}

// ------------------------------------------------------------------ writer
namespace {
struct Writer {
  std::vector<uint8_t> b;
  void put(const void *p, size_t k) {
    const uint8_t *c = (const uint8_t *)p;
    b.insert(b.end(), c, c + k);
  }
  void u32(uint32_t v) { put(&v, 4); }
  void u64(uint64_t v) { put(&v, 8); }
  void f32(float v) { put(&v, 4); }
  void str(const std::string &s) {
    u64(s.size());
    put(s.data(), s.size());
  }
};
bool is_quantizable(const std::string &name) {  // weights.rs:32-37
  return name.find(".attention.wQKV.weight") != std::string::npos ||
         name.find(".attention.wO.weight") != std::string::npos || name.find(".mlp.0.weight") != std::string::npos ||
         name.find(".mlp.2.weight") != std::string::npos;
}
}  // namespace

std::vector<uint8_t> export_gguf(const std::vector<ExportTensor> &tensors, int big_type, const ModelMeta &m) {
  std::vector<size_t> order(tensors.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](size_t a, size_t b) { return tensors[a].name < tensors[b].name; });
  Writer w;
  w.put("GGUF", 4);
  w.u32(3);
  w.u64(tensors.size());
  w.u64(11);
  auto ku32 = [&](const char *k, uint32_t v) {
    w.str(k);
    w.u32(4);
    w.u32(v);
  };
  ku32("t0.embed_dim", m.embed_dim);
  ku32("t0.num_layers", m.num_layers);
  ku32("t0.num_heads", m.num_heads);
  ku32("t0.mlp_hidden_dim", m.mlp_hidden_dim);
  ku32("t0.patch_size", m.patch_size);
  ku32("t0.group_every_n", m.group_every_n);
  w.str("t0.dropout");
  w.u32(6);
  w.f32(m.dropout);
  w.str("t0.quantile_levels");
  w.u32(9);
  w.u32(6);
  w.u64(m.quantile_levels.size());
  for (float q : m.quantile_levels) w.f32(q);
  w.str("t0.scaler_use_arcsinh");
  w.u32(7);
  uint8_t ab = m.scaler_use_arcsinh ? 1 : 0;
  w.put(&ab, 1);
  w.str("t0.scaler_eps");
  w.u32(6);
  w.f32(m.scaler_eps);
  w.str("t0.scaler_eps_mode");
  w.u32(8);
  w.str(m.variance_offset ? "variance_offset" : "std_clamp");

  std::vector<int> types(tensors.size());
  std::vector<uint64_t> offs(tensors.size());
  uint64_t cursor = 0;
  for (size_t oi : order) {
    const auto &t = tensors[oi];
    types[oi] = (t.shape.size() == 2 && is_quantizable(t.name)) ? big_type : GG_F16;
    offs[oi] = cursor;
    cursor += row_bytes(types[oi], t.n_elements());
    cursor = (cursor + 31) / 32 * 32;
  }
  for (size_t oi : order) {
    const auto &t = tensors[oi];
    w.str(t.name);
    w.u32((uint32_t)t.shape.size());
    for (size_t d = t.shape.size(); d-- > 0;) w.u64((uint64_t)t.shape[d]);
    w.u32((uint32_t)types[oi]);
    w.u64(offs[oi]);
  }
  const size_t blob = w.b.size();
  for (size_t oi : order) {
    const auto &t = tensors[oi];
    w.b.resize(blob + offs[oi], 0);
    const size_t n = t.n_elements(), nb = row_bytes(types[oi], n);
    std::vector<uint8_t> enc(nb);
    switch (types[oi]) {
      case GG_F16:
        for (size_t i = 0; i < n; ++i) {
          uint16_t h = f32_to_f16(t.data[i]);
          std::memcpy(&enc[2 * i], &h, 2);
        }
        break;
      case GG_Q8_0: quantize_q8_0(t.data, n, enc.data()); break;
      case GG_Q4_0: quantize_q4_0(t.data, n, enc.data()); break;
      default: std::memcpy(enc.data(), t.data, n * 4);
    }
    w.put(enc.data(), nb);
  }
  return w.b;
}

}  // namespace t0b
