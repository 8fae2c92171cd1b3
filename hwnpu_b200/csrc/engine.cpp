// engine.cpp: hc_model_load / hc_linear_* — the weights of llm.Model (internal/llm/arch.go)
// repacked into integer-MMA tiles and copied to HBM once; the decode step lives in step.cpp.
#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>

namespace hc {

DevLinear::~DevLinear() {
  if (tiles) cudaFree(tiles);
  if (scales) cudaFree(scales);
  if (bias) cudaFree(bias);
}

char *upload(const Packed &p, DevLinear *out, cudaStream_t st) {
  if (char *e = dev_alloc(&out->tiles, p.tiles.size(), "weight tiles")) return e;
  if (char *e = copy_h2d(out->tiles, p.tiles.data(), p.tiles.size(), st)) return e;
  out->bytes = p.tiles.size();
  if (!p.row_scale.empty()) {
    if (char *e = dev_alloc(&out->scales, p.row_scale.size() * 4, "row scales")) return e;
    if (char *e = copy_h2d(out->scales, p.row_scale.data(), p.row_scale.size() * 4, st)) return e;
    out->bytes += p.row_scale.size() * 4;
  }
  if (!p.bias.empty()) {
    if (char *e = dev_alloc(&out->bias, p.bias.size() * 4, "biases")) return e;
    if (char *e = copy_h2d(out->bias, p.bias.data(), p.bias.size() * 4, st)) return e;
    out->bytes += p.bias.size() * 4;
  }
  out->m.kind = p.kind;
  out->m.fmt = p.fmt;
  out->m.rows = p.rows;
  out->m.cols = p.cols;
  out->m.rtiles = p.rtiles;
  out->m.ktiles = p.ktiles;
  out->m.tile_bytes = p.tile_bytes;
  out->m.tiles = static_cast<const uint8_t *>(out->tiles);
  out->m.row_scale = static_cast<const float *>(out->scales);
  out->m.bias = static_cast<const float *>(out->bias);
  // the copies read from p: finish them before p goes away
  HC_TRY_CUDA(cudaStreamSynchronize(st));
  return nullptr;
}

char *load_linear(const std::vector<RowRef> &rows, DevLinear *out, cudaStream_t st) {
  Packed p;
  if (char *e = repack(rows, &p)) return e;
  return upload(p, out, st);
}

}  // namespace hc

hc_model::~hc_model() {
  cudaSetDevice(ordinal);
  layers.clear();
  head.reset();
  for (void *p : allocs) cudaFree(p);
}

namespace {

using hc::f16_bits;
using hc::f16_value;

// A device copy of n fp16 values as float32 (1.0 where p is NULL, the default norm weight).
char *norm_vec(hc_model *m, const uint16_t *p, size_t n, float **out) {
  std::vector<float> v(n, 1.0f);
  if (p)
    for (size_t i = 0; i < n; ++i) v[i] = f16_value(p[i]);
  void *d = nullptr;
  if (char *e = hc::dev_alloc(&d, n * 4, "norm weights")) return e;
  m->allocs.push_back(d);
  if (char *e = hc::copy_h2d(d, v.data(), n * 4, nullptr)) return e;
  HC_TRY_CUDA(cudaStreamSynchronize(nullptr));
  *out = static_cast<float *>(d);
  return nullptr;
}

bool int_format(int f) {
  return f == HC_FMT_INT8_ROW || f == HC_FMT_INT4_SYM_G32 || f == HC_FMT_INT4_ASYM_G32 || f == HC_FMT_MXFP4;
}

char *check_linear(const hc_linear_desc &l, uint32_t rows, uint32_t cols, const char *what) {
  if (l.format == HC_FMT_NONE) return hc::make_error(std::string(what) + ": missing");
  if (l.rows != rows || l.cols != cols)
    return hc::make_error(std::string(what) + ": shape " + std::to_string(l.rows) + "x" + std::to_string(l.cols) +
                          ", expected " + std::to_string(rows) + "x" + std::to_string(cols));
  if (!int_format(l.format))
    return hc::make_error(std::string(what) + ": format " + std::to_string(l.format) +
                          " is not one of this engine's integer formats (int8, int4, MXFP4)");
  return nullptr;
}

// The fp16 constant of an epsilon after the norm's scale (qwen3 build.go:143).
float eps16_of(double eps, double scale) { return f16_value(f16_bits(float(eps / (scale * scale)))); }

// A device array of n floats (zeros where p is NULL).
char *float_vec(hc_model *m, const float *p, size_t n, float **out) {
  std::vector<float> v(n, 0.0f);
  if (p) std::copy(p, p + n, v.begin());
  void *d = nullptr;
  if (char *e = hc::dev_alloc(&d, n * 4, "biases")) return e;
  m->allocs.push_back(d);
  if (char *e = hc::copy_h2d(d, v.data(), n * 4, nullptr)) return e;
  HC_TRY_CUDA(cudaStreamSynchronize(nullptr));
  *out = static_cast<float *>(d);
  return nullptr;
}

// The rows of the parts (bf16 or fp16 [rows][cols], one format) one after another as a device
// matrix of 16-bit floats, with their biases. to_f16: the values rounded to fp16 (gpt-oss's
// programs hold the router's weights and bias as fp16, gptoss/build.go:125-140).
char *load_dense(hc_model *m, const std::vector<const hc_linear_desc *> &parts, bool to_f16, hc::DevDense *out,
                 const char *what) {
  const int fmt = parts[0]->format;
  const uint32_t cols = parts[0]->cols;
  uint32_t rows = 0;
  bool any_bias = false;
  for (auto *d : parts) {
    if (d->format != HC_FMT_BF16 && d->format != HC_FMT_F16)
      return hc::make_error(std::string(what) + ": gpt-oss's attention, router and head take bf16 or fp16");
    if (d->format != fmt || d->cols != cols) return hc::make_error(std::string(what) + ": parts of different formats");
    rows += d->rows;
    any_bias |= d->bias != nullptr;
  }
  if (cols % 8) return hc::make_error(std::string(what) + ": columns not a multiple of 8");
  std::vector<uint16_t> w(size_t(rows) * cols);
  std::vector<float> b(rows, 0.0f);
  size_t r0 = 0;
  for (auto *d : parts) {
    const uint16_t *src = static_cast<const uint16_t *>(d->data);
    const size_t n = size_t(d->rows) * cols;
    for (size_t i = 0; i < n; ++i) {
      uint16_t v = src[i];
      if (to_f16 && fmt == HC_FMT_BF16) {
        uint32_t u = uint32_t(v) << 16;
        float f;
        std::memcpy(&f, &u, 4);
        v = f16_bits(f);
      }
      w[r0 * cols + i] = v;
    }
    if (d->bias)
      for (uint32_t r = 0; r < d->rows; ++r) b[r0 + r] = to_f16 ? f16_value(f16_bits(d->bias[r])) : d->bias[r];
    r0 += d->rows;
  }
  void *dw = nullptr;
  if (char *e = hc::dev_alloc(&dw, w.size() * 2, what)) return e;
  m->allocs.push_back(dw);
  if (char *e = hc::copy_h2d(dw, w.data(), w.size() * 2, nullptr)) return e;
  HC_TRY_CUDA(cudaStreamSynchronize(nullptr));
  out->w = static_cast<const uint16_t *>(dw);
  out->rows = int(rows);
  out->cols = int(cols);
  out->bf16 = fmt == HC_FMT_BF16 && !to_f16;
  out->bias = nullptr;
  if (any_bias) {
    float *db = nullptr;
    if (char *e = float_vec(m, b.data(), b.size(), &db)) return e;
    out->bias = db;
  }
  return nullptr;
}

// gptoss.Config.RopeInvFreq (internal/llm/gptoss/config.go:136-166): YaRN's inverse frequencies and
// the factor its rotary tables are scaled by (0.1 ln(factor) + 1).
void yarn(const hc_model_desc &d, std::vector<double> &inv, float &factor) {
  const int dim = int(d.head_dim), half = dim / 2;
  inv.assign(half, 0.0);
  if (d.yarn_factor <= 1) {
    for (int i = 0; i < half; ++i) inv[i] = 1 / std::pow(d.rope_theta, double(2 * i) / double(dim));
    factor = 1.f;
    return;
  }
  auto corr = [&](double rot) {
    return double(dim) * std::log(double(d.yarn_original) / (rot * 2 * M_PI)) / (2 * std::log(d.rope_theta));
  };
  double low = corr(d.yarn_beta_fast), high = corr(d.yarn_beta_slow);
  if (d.yarn_truncate) {
    low = std::floor(low);
    high = std::ceil(high);
  }
  low = std::max(low, 0.0);
  high = std::min(high, double(dim - 1));
  if (low == high) high += 0.001;
  for (int i = 0; i < half; ++i) {
    const double pos = std::pow(d.rope_theta, double(2 * i) / double(dim));
    const double ramp = std::min(std::max((double(i) - low) / (high - low), 0.0), 1.0);
    const double ef = 1 - ramp;  // the share of extrapolation
    inv[i] = (1 / (d.yarn_factor * pos)) * (1 - ef) + (1 / pos) * ef;
  }
  factor = float(0.1 * std::log(d.yarn_factor) + 1);
}

char *check_shape(const hc_linear_desc &l, uint32_t rows, uint32_t cols, const char *what) {
  if (l.format == HC_FMT_NONE) return hc::make_error(std::string(what) + ": missing");
  if (l.rows != rows || l.cols != cols)
    return hc::make_error(std::string(what) + ": shape " + std::to_string(l.rows) + "x" + std::to_string(l.cols) +
                          ", expected " + std::to_string(rows) + "x" + std::to_string(cols));
  return nullptr;
}

// The weights of a gpt-oss model (HC_ARCH_GPTOSS, internal/llm/gptoss): bf16 q/k/v/o with biases,
// sinks, sliding and full layers, YaRN, a router and MXFP4 experts with biases, an untied bf16 head.
char *load_gptoss(hc_model *m, const hc_model_desc &d) {
  const uint32_t D = d.hidden, hd = d.head_dim, I = d.inter, E = d.experts, K = d.top_k;
  if (!E || !K || K > E || K > 8) return hc::make_error("hc_model_load: gpt-oss needs experts and 1 <= top_k <= 8 of them");
  if (!d.embed) return hc::make_error("hc_model_load: gpt-oss's head is untied: an embedding table is needed");
  if (D % 32 || I % 32) return hc::make_error("hc_model_load: hidden and inter must be multiples of MXFP4's 32");
  m->gptoss = true;
  m->norm_in0 = m->norm_mid = m->norm_head = {1.f, eps16_of(d.norm_eps, 1)};
  uint64_t expert_bytes = 0;
  for (uint32_t i = 0; i < d.layers; ++i) {
    const hc_layer_desc &L = d.layer[i];
    const std::string p = "layer " + std::to_string(i) + " ";
    if (char *e = check_shape(L.q, d.heads * hd, D, (p + "q").c_str())) return e;
    if (char *e = check_shape(L.k, d.kv_heads * hd, D, (p + "k").c_str())) return e;
    if (char *e = check_shape(L.v, d.kv_heads * hd, D, (p + "v").c_str())) return e;
    if (char *e = check_shape(L.o, D, d.heads * hd, (p + "o").c_str())) return e;
    if (char *e = check_shape(L.router, E, D, (p + "router").c_str())) return e;
    if (char *e = check_shape(L.experts_gate_up, E * 2 * I, D, (p + "experts gate_up").c_str())) return e;
    if (char *e = check_shape(L.experts_down, E * D, I, (p + "experts down").c_str())) return e;
    if (L.experts_gate_up.format != HC_FMT_MXFP4 || L.experts_down.format != HC_FMT_MXFP4)
      return hc::make_error(p + "experts: MXFP4 only");
    hc::LayerW w;
    if (char *e = load_dense(m, {&L.q, &L.k, &L.v}, false, &w.qkv16, "qkv")) return e;
    if (char *e = load_dense(m, {&L.o}, false, &w.o16, "o")) return e;
    if (char *e = load_dense(m, {&L.router}, true, &w.router16, "router")) return e;
    // gate rows 2j and up rows 2j + 1 of every expert into GLU tiles, expert after expert
    std::vector<hc::RowRef> gu;
    for (uint32_t x = 0; x < E; ++x) {
      auto r = hc::rows_glu(L.experts_gate_up, x * 2 * I, 2, L.experts_gate_up, x * 2 * I + 1, 2, I);
      gu.insert(gu.end(), r.begin(), r.end());
    }
    w.egu = std::make_unique<hc::DevLinear>();
    w.edown = std::make_unique<hc::DevLinear>();
    if (char *e = hc::load_linear(gu, w.egu.get(), nullptr)) return e;
    w.egu->m.rows = int(E * I);  // the gated unit's outputs
    if (char *e = hc::load_linear(hc::rows_of(L.experts_down), w.edown.get(), nullptr)) return e;
    if (char *e = float_vec(m, L.experts_gate_up.bias, size_t(E) * 2 * I, &w.egb)) return e;
    if (char *e = float_vec(m, L.experts_down.bias, size_t(E) * D, &w.edb)) return e;
    if (char *e = norm_vec(m, L.input_norm, D, &w.in_norm)) return e;
    if (char *e = norm_vec(m, L.post_norm, D, &w.post_norm)) return e;
    if (L.sinks) {
      std::vector<uint16_t> s16(d.heads);
      for (uint32_t h = 0; h < d.heads; ++h) s16[h] = f16_bits(L.sinks[h]);
      if (char *e = norm_vec(m, s16.data(), d.heads, &w.sinks)) return e;
    }
    w.window = int(L.sliding_window);
    expert_bytes = (w.egu->bytes + w.edown->bytes) / E;
    m->weight_bytes += (uint64_t(w.qkv16.rows) + w.o16.rows + w.router16.rows) * D * 2 + K * expert_bytes;
    m->layers.push_back(std::move(w));
  }
  if (char *e = norm_vec(m, d.final_norm, D, &m->final_norm)) return e;
  if (char *e = check_shape(d.head, d.vocab, D, "head")) return e;
  if (char *e = load_dense(m, {&d.head}, false, &m->head16, "head")) return e;
  m->weight_bytes += uint64_t(d.vocab) * D * 2 + uint64_t(D) * 2;
  void *p = nullptr;
  const size_t n = size_t(d.vocab) * D * 2;
  if (char *e = hc::dev_alloc(&p, n, "embedding table")) return e;
  m->allocs.push_back(p);
  if (char *e = hc::copy_h2d(p, d.embed, n, nullptr)) return e;
  HC_TRY_CUDA(cudaStreamSynchronize(nullptr));
  m->embed = static_cast<uint16_t *>(p);
  yarn(d, m->inv_freq, m->rope_factor);
  return nullptr;
}

}  // namespace

extern "C" {

HC_API char *hc_model_load(hc_device *dev, const hc_model_desc *desc, hc_model **out) {
  if (!dev || !desc || !out) return hc::make_error("hc_model_load: NULL argument");
  *out = nullptr;
  const hc_model_desc &d = *desc;
  if (d.abi != HC_ABI) return hc::make_error("hc_model_load: descriptor of ABI " + std::to_string(d.abi));
  if (d.arch != HC_ARCH_QWEN3 && d.arch != HC_ARCH_GPTOSS)
    return hc::make_error("hc_model_load: architecture " + std::to_string(d.arch) + " is not supported by this build");
  if (!d.layers || !d.hidden || !d.heads || !d.kv_heads || !d.vocab || !d.layer)
    return hc::make_error("hc_model_load: empty shape");
  if (d.heads % d.kv_heads) return hc::make_error("hc_model_load: heads not a multiple of kv heads");
  const int rep = int(d.heads / d.kv_heads);
  if (d.head_dim != 64 && d.head_dim != 128) return hc::make_error("hc_model_load: head_dim must be 64 or 128");
  if (rep != 1 && rep != 2 && rep != 4 && rep != 8) return hc::make_error("hc_model_load: heads per kv head must be 1, 2, 4 or 8");
  if (!(d.flags & HC_MODEL_TIED) && !d.embed) return hc::make_error("hc_model_load: untied model without an embedding table");
  HC_TRY_CUDA(cudaSetDevice(hc::device_ordinal(dev)));
  auto m = std::make_unique<hc_model>();
  m->dev = dev;
  m->ordinal = hc::device_ordinal(dev);
  m->sms = hc::device_sms(dev);
  m->d = d;
  m->d.layer = nullptr;
  m->d.embed = nullptr;
  m->d.final_norm = nullptr;
  m->d.head = hc_linear_desc{};
  const uint32_t D = d.hidden, hd = d.head_dim, F = d.inter;
  const bool scaled = d.flags & HC_MODEL_NORM_SCALE;
  m->norm_in0 = {1.f, eps16_of(d.norm_eps, 1)};
  m->norm_mid = scaled ? hc::NormCfg{64.f, eps16_of(d.norm_eps, 64)} : m->norm_in0;
  m->norm_head = m->norm_mid;
  m->score_scale = f16_value(f16_bits(float(1 / std::sqrt(double(hd)))));
  if (d.arch == HC_ARCH_GPTOSS) {
    if (char *e = load_gptoss(m.get(), d)) return e;
    *out = m.release();
    return nullptr;
  }
  for (uint32_t i = 0; i < d.layers; ++i) {
    const hc_layer_desc &L = d.layer[i];
    const std::string p = "layer " + std::to_string(i) + " ";
    if (char *e = check_linear(L.q, d.heads * hd, D, (p + "q").c_str())) return e;
    if (char *e = check_linear(L.k, d.kv_heads * hd, D, (p + "k").c_str())) return e;
    if (char *e = check_linear(L.v, d.kv_heads * hd, D, (p + "v").c_str())) return e;
    if (char *e = check_linear(L.o, D, d.heads * hd, (p + "o").c_str())) return e;
    if (char *e = check_linear(L.gate, F, D, (p + "gate").c_str())) return e;
    if (char *e = check_linear(L.up, F, D, (p + "up").c_str())) return e;
    if (char *e = check_linear(L.down, D, F, (p + "down").c_str())) return e;
    hc::LayerW w;
    w.qkv = std::make_unique<hc::DevLinear>();
    w.o = std::make_unique<hc::DevLinear>();
    w.gu = std::make_unique<hc::DevLinear>();
    w.down = std::make_unique<hc::DevLinear>();
    if (char *e = hc::load_linear(hc::rows_concat({&L.q, &L.k, &L.v}), w.qkv.get(), nullptr)) return e;
    if (char *e = hc::load_linear(hc::rows_of(L.o), w.o.get(), nullptr)) return e;
    if (char *e = hc::load_linear(hc::rows_glu(L.gate, 0, 1, L.up, 0, 1, F), w.gu.get(), nullptr)) return e;
    w.gu->m.rows = int(F);  // the GLU's outputs
    if (char *e = hc::load_linear(hc::rows_of(L.down), w.down.get(), nullptr)) return e;
    if (char *e = norm_vec(m.get(), L.input_norm, D, &w.in_norm)) return e;
    if (char *e = norm_vec(m.get(), L.post_norm, D, &w.post_norm)) return e;
    if (d.flags & HC_MODEL_QK_NORM) {
      if (char *e = norm_vec(m.get(), L.q_norm, hd, &w.q_norm)) return e;
      if (char *e = norm_vec(m.get(), L.k_norm, hd, &w.k_norm)) return e;
    }
    if (L.sinks) {
      std::vector<uint16_t> s16(d.heads);
      for (uint32_t h = 0; h < d.heads; ++h) s16[h] = f16_bits(L.sinks[h]);
      if (char *e = norm_vec(m.get(), s16.data(), d.heads, &w.sinks)) return e;
    }
    w.window = int(L.sliding_window);
    m->weight_bytes += w.qkv->bytes + w.o->bytes + w.gu->bytes + w.down->bytes;
    m->layers.push_back(std::move(w));
  }
  if (char *e = norm_vec(m.get(), d.final_norm, D, &m->final_norm)) return e;
  if (char *e = check_linear(d.head, d.vocab, D, "head")) return e;
  m->head = std::make_unique<hc::DevLinear>();
  if (char *e = hc::load_linear(hc::rows_of(d.head), m->head.get(), nullptr)) return e;
  m->weight_bytes += m->head->bytes + uint64_t(D) * 2;  // + one embedding row
  if (d.embed) {
    void *p = nullptr;
    const size_t n = size_t(d.vocab) * D * 2;
    if (char *e = hc::dev_alloc(&p, n, "embedding table")) return e;
    m->allocs.push_back(p);
    if (char *e = hc::copy_h2d(p, d.embed, n, nullptr)) return e;
    HC_TRY_CUDA(cudaStreamSynchronize(nullptr));
    m->embed = static_cast<uint16_t *>(p);
  }
  // qwen3.Config.RopeInvFreq (internal/llm/qwen3/config.go:152-159)
  m->inv_freq.resize(hd / 2);
  for (uint32_t j = 0; j < hd / 2; ++j) m->inv_freq[j] = 1 / std::pow(d.rope_theta, double(2 * j) / double(hd));
  *out = m.release();
  return nullptr;
}

HC_API void hc_model_free(hc_model *m) { delete m; }

HC_API uint64_t hc_model_weight_bytes(hc_model *m) { return m ? m->weight_bytes : 0; }

}  // extern "C"

// ---- one matrix on its own (tests and the kernel bench) ------------------------------------

struct hc_linear {
  int ordinal = 0;
  hc::DevLinear w;
  uint8_t *act = nullptr;  // activation tiles of up to kMaxChunk tokens
  ~hc_linear() {
    cudaSetDevice(ordinal);
    if (act) cudaFree(act);
  }
};

extern "C" {

HC_API char *hc_linear_load(hc_device *d, const hc_linear_desc *desc, hc_linear **out) {
  if (!d || !desc || !out) return hc::make_error("hc_linear_load: NULL argument");
  *out = nullptr;
  if (!int_format(desc->format)) return hc::make_error("hc_linear_load: not an integer format");
  HC_TRY_CUDA(cudaSetDevice(hc::device_ordinal(d)));
  if (char *e = hc::gemv_prepare()) return e;
  auto l = std::make_unique<hc_linear>();
  l->ordinal = hc::device_ordinal(d);
  if (char *e = hc::load_linear(hc::rows_of(*desc), &l->w, nullptr)) return e;
  void *a = nullptr;
  if (char *e = hc::dev_alloc(&a, size_t(l->w.m.ktiles) * hc::kActTile * hc::kMaxChunk, "activation tiles")) return e;
  l->act = static_cast<uint8_t *>(a);
  *out = l.release();
  return nullptr;
}

HC_API void hc_linear_free(hc_linear *l) { delete l; }

HC_API char *hc_linear_dequant(hc_linear *l, uint32_t row0, uint32_t nrows, float *out) {
  if (!l || !out) return hc::make_error("hc_linear_dequant: NULL argument");
  if (row0 + uint64_t(nrows) > uint64_t(l->w.m.rows)) return hc::make_error("hc_linear_dequant: rows out of range");
  HC_TRY_CUDA(cudaSetDevice(l->ordinal));
  void *buf = nullptr;
  const size_t n = size_t(nrows) * l->w.m.cols * 4;
  if (char *e = hc::dev_alloc(&buf, n, "dequant output")) return e;
  hc::dequant(l->w.m, int(row0), int(nrows), static_cast<float *>(buf), nullptr);
  cudaError_t e1 = cudaGetLastError();
  cudaError_t e2 = cudaMemcpy(out, buf, n, cudaMemcpyDeviceToHost);
  cudaFree(buf);
  if (e1 != cudaSuccess) return hc::make_error(std::string("dequant kernel: ") + cudaGetErrorString(e1));
  if (e2 != cudaSuccess) return hc::make_error(std::string("dequant copy: ") + cudaGetErrorString(e2));
  return nullptr;
}

HC_API char *hc_linear_run(hc_linear *l, const float *x, int32_t ntok, float *y, void *stream) {
  if (!l || !x || !y) return hc::make_error("hc_linear_run: NULL argument");
  if (ntok < 1) return hc::make_error("hc_linear_run: ntok must be at least 1");
  HC_TRY_CUDA(cudaSetDevice(l->ordinal));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const hc::DevMat &W = l->w.m;
  for (int t0 = 0; t0 < ntok; t0 += hc::kMaxChunk) {
    const int n = std::min(hc::kMaxChunk, ntok - t0);
    hc::ActSrc src;
    src.x = x + size_t(t0) * W.cols;
    src.ldx = W.cols;
    src.n = W.cols;
    hc::GemvOut o;
    o.mode = hc::kStore;
    o.y = y + size_t(t0) * W.rows;
    o.ldy = W.rows;
    hc::gemv_x(W, src, n, l->act, o, st);
  }
  HC_TRY_CUDA(cudaGetLastError());
  return nullptr;
}

}  // extern "C"
