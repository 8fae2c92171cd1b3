// model.cpp — TEST INFRASTRUCTURE (see oracle.h): one decode session of a model on the CPU, as
// decode.Session drives milcpu over the program qwen3.Build writes (the wiring of
// internal/llm/qwen3/cache_test.go:43-123): fp16 program inputs and outputs, float32 inside,
// float64 softmax, reduce_mean and rsqrt, an fp16 KV cache written after each step.
#include "oracle.h"
#include "pool.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

using oracle::Pool;

namespace {

inline float float_of(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline float f16v(uint16_t h) { return or_f16_value(h); }
inline float f16r(float x) { return or_f16_value(or_f16_bits(x)); }  // a value through fp16

constexpr int KC = 256;  // sgemm's depth block (internal/sgemm/sgemm.go:5-25)

// A linear layer's weight, dequantised once to float32 as milcpu caches constexpr values
// (internal/milcpu/milcpu.go:163-167), stored transposed [cols][rows] for the product below.
struct Lin {
  int rows = 0, cols = 0, fmt = HC_FMT_NONE;
  std::vector<float> wt;
  std::vector<float> bias;
  bool present() const { return fmt != HC_FMT_NONE; }
};

void dequant_rows(const hc_linear_desc &d, uint32_t r0, uint32_t r1, float *out) {
  const size_t cols = d.cols;
  switch (d.format) {
    case HC_FMT_F16: {
      auto *p = static_cast<const uint16_t *>(d.data) + r0 * cols;
      for (size_t i = 0; i < (r1 - r0) * cols; ++i) out[i] = f16v(p[i]);
      break;
    }
    case HC_FMT_BF16: {
      auto *p = static_cast<const uint16_t *>(d.data) + r0 * cols;
      for (size_t i = 0; i < (r1 - r0) * cols; ++i) out[i] = float_of(uint32_t(p[i]) << 16);
      break;
    }
    case HC_FMT_INT8_ROW:
      or_dequant_linear(static_cast<const uint8_t *>(d.data) + r0 * cols, d.scales + r0, r1 - r0,
                        d.cols, d.cols, 8, out);
      break;
    case HC_FMT_INT4_SYM_G32:
      or_dequant_linear(static_cast<const uint8_t *>(d.data) + r0 * cols / 2,
                        d.scales + r0 * (cols / 32), r1 - r0, d.cols, 32, 4, out);
      break;
    case HC_FMT_INT4_ASYM_G32:
      or_dequant_int4_asym(static_cast<const uint8_t *>(d.data) + r0 * cols / 2,
                           d.scales + r0 * (cols / 32), d.zeros + r0 * (cols / 32), r1 - r0,
                           d.cols, out);
      break;
    case HC_FMT_MXFP4:
      for (uint32_t r = r0; r < r1; ++r)
        or_mxfp4_dequant(static_cast<const uint8_t *>(d.data) + size_t(r) * cols / 2,
                         d.exps + size_t(r) * (cols / 32), d.cols, out + (r - r0) * cols);
      break;
  }
}

Lin load_lin(Pool &pool, const hc_linear_desc &d) {
  Lin L;
  L.fmt = d.format;
  if (d.format == HC_FMT_NONE) return L;
  L.rows = int(d.rows);
  L.cols = int(d.cols);
  L.wt.resize(size_t(d.rows) * d.cols);
  pool.parallel_for(d.rows, 64, [&](long lo, long hi) {
    std::vector<float> tmp(size_t(hi - lo) * d.cols);
    dequant_rows(d, uint32_t(lo), uint32_t(hi), tmp.data());
    for (long r = lo; r < hi; ++r)
      for (size_t c = 0; c < d.cols; ++c) L.wt[c * d.rows + r] = tmp[(r - lo) * d.cols + c];
  });
  if (d.bias) L.bias.assign(d.bias, d.bias + d.rows);
  return L;
}

// milcpu linear (internal/milcpu/ops.go:940-956) over sgemm.MulAdd (sgemm.go:127): y starts as
// the bias (or 0), and every depth block of KC adds its own fused multiply-add chain.
void linear(Pool &pool, const Lin &L, const float *x, int m, float *y) {
  const int rows = L.rows, cols = L.cols;
  pool.parallel_for(rows, 64, [&](long lo, long hi) {
    const long w = hi - lo;
    std::vector<float> blk(size_t(m) * w);
    for (int i = 0; i < m; ++i)
      for (long j = 0; j < w; ++j) y[size_t(i) * rows + lo + j] = L.bias.empty() ? 0.0f : L.bias[lo + j];
    for (int k0 = 0; k0 < cols; k0 += KC) {
      std::fill(blk.begin(), blk.end(), 0.0f);
      const int k1 = std::min(cols, k0 + KC);
      for (int i = 0; i < m; ++i) {
        float *b = blk.data() + size_t(i) * w;
        const float *xi = x + size_t(i) * cols;
        for (int k = k0; k < k1; ++k) {
          const float a = xi[k];
          const float *wk = L.wt.data() + size_t(k) * rows + lo;
          for (long j = 0; j < w; ++j) b[j] = std::fma(a, wk[j], b[j]);
        }
      }
      for (int i = 0; i < m; ++i)
        for (long j = 0; j < w; ++j) y[size_t(i) * rows + lo + j] += blk[size_t(i) * w + j];
    }
  });
}

// qwen3's normScaled (internal/llm/qwen3/build.go:131-151) and blocks.RMSNormWith
// (internal/llm/blocks/blocks.go:351-376) with scale 1: xs = x * f16(1/scale); the mean of xs^2
// summed in float64 (milcpu reduce, ops.go:861-920); r = float32(1 / sqrt(float64(ms) + eps))
// (milcpu rsqrt, ops.go:181-189) with eps the fp16 constant f16(eps / scale^2); y = xs * r * w.
void rms_norm(const float *x, int n, const float *w, float scale, double eps, float *out) {
  const float inv = f16r(1.0f / scale);
  const float eps16 = f16r(float(eps / (double(scale) * scale)));
  double acc = 0;
  std::vector<float> xs(n);
  for (int i = 0; i < n; ++i) {
    xs[i] = scale != 1 ? x[i] * inv : x[i];
    float sq = xs[i] * xs[i];
    acc += double(sq);
  }
  float ms = float(acc / double(n));
  float r = float(1 / std::sqrt(double(ms) + double(eps16)));
  for (int i = 0; i < n; ++i) {
    float y = xs[i] * r;
    out[i] = y * w[i];
  }
}

// blocks.SiLU: x / (1 + exp(-x)), the exp of milcpu (f32.Exp) (blocks.go:395-399).
inline float silu(float x) {
  float neg = x * -1.0f;
  float e = or_exp(neg);
  float den = e + 1.0f;
  return x / den;
}

std::vector<float> f16_vec(const uint16_t *p, size_t n, float fill) {
  std::vector<float> v(n, fill);
  if (p)
    for (size_t i = 0; i < n; ++i) v[i] = f16v(p[i]);
  return v;
}

// One layer's MXFP4 experts as the checkpoint holds them (experts.MXFP4, host.go:62-66): gate_up
// [experts * 2 inter][hidden] with gate rows even and up rows odd, down [experts * hidden][inter],
// blocks of 16 bytes and one e8m0 exponent per 32 columns, float32 biases.
struct Experts {
  const uint8_t *gw = nullptr, *ge = nullptr, *dw = nullptr, *de = nullptr;
  std::vector<float> gb, db;
  bool present() const { return gw != nullptr; }
};

struct Layer {
  std::vector<float> in_norm, post_norm, q_norm, k_norm, sinks;
  Lin q, k, v, o, gate, up, down;
  Lin router;  // gpt-oss: weights and bias as fp16 values (the program's F16s, gptoss/build.go:125-140)
  Experts ex;
  int window = 0;
};

// gptoss.Config.RopeInvFreq (internal/llm/gptoss/config.go:136-166): YaRN's inverse frequencies
// (transformers' _compute_yarn_parameters) and the factor the tables are scaled by.
void yarn_inv_freq(const hc_model_desc &d, std::vector<double> &inv, float &factor) {
  const int dim = int(d.head_dim), half = dim / 2;
  inv.assign(half, 0);
  if (d.yarn_factor <= 1) {
    for (int i = 0; i < half; ++i) inv[i] = 1 / std::pow(d.rope_theta, double(2 * i) / double(dim));
    factor = 1;
    return;
  }
  auto corr = [&](double rot) {
    return double(dim) * std::log(double(d.yarn_original) / (rot * 2 * M_PI)) / (2 * std::log(d.rope_theta));
  };
  double low = corr(d.yarn_beta_fast), high = corr(d.yarn_beta_slow);
  if (d.yarn_truncate) { low = std::floor(low); high = std::ceil(high); }
  low = std::max(low, 0.0);
  high = std::min(high, double(dim - 1));
  if (low == high) high += 0.001;
  for (int i = 0; i < half; ++i) {
    const double pos = std::pow(d.rope_theta, double(2 * i) / double(dim));
    const double extra = 1 / pos, inter = 1 / (d.yarn_factor * pos);
    const double ramp = std::min(std::max((double(i) - low) / (high - low), 0.0), 1.0);
    const double ef = 1 - ramp;
    inv[i] = inter * (1 - ef) + extra * ef;
  }
  factor = float(0.1 * std::log(d.yarn_factor) + 1);
}

}  // namespace

struct or_model {
  hc_model_desc d{};
  std::unique_ptr<Pool> pool;
  std::vector<Layer> layers;
  std::vector<uint16_t> embed;  // fp16 [vocab][hidden]
  std::vector<float> final_norm;
  Lin head;
  std::vector<double> inv_freq;
  float rope_factor = 1;
};

struct or_session {
  or_model *m;
  int cap, pos = 0;
  int kv_format = HC_KV_F16;
  std::vector<std::vector<uint16_t>> kc, vc;  // per layer [kv_heads][cap][head_dim] fp16
  // HC_KV_INT8_PAGED: per layer int8 rows [kv_heads][cap][head_dim] and fp16 scales
  // [kv_heads][pages] for keys and for values
  std::vector<std::vector<int8_t>> kq, vq;
  std::vector<std::vector<uint16_t>> ks, vs;
};

namespace {

constexpr int kOrPage = 16;  // positions a page of the int8 cache
// Tokens of one sequence that one step reads as a program: a step's tokens go in pieces of this
// many (the prompt programs' chunking, decode.go:597-607), each piece reading the earlier positions
// from the cache. The library cuts a call the same way (64-token chunks, a sequence's pieces from
// its first token), so both read the same keys in float32.
constexpr int kOrPiece = 64;

// The round-up of a float32 to fp16 (the page scale, the smallest fp16 not below v; v >= 0 and
// finite here).
float f16_round_up(float v) {
  const uint16_t h = or_f16_bits(v);
  float r = or_f16_value(h);
  if (r < v) r = or_f16_value(uint16_t(h + 1));
  return r;
}

// Writes row `off` of a page of the int8 cache (this library's paged format, which the reference
// does not have: HC_KV_INT8_PAGED in include/hwnpu_cuda.h): the page's scale is the fp16 rounding
// up of max|x| / 127 over its rows; a row that needs more requantises the page's earlier rows to the
// new scale (q' = round_even(q * (s_old / s_new))), then the row is round_even(x * (1 / s)) clamped
// to +-127.
void page_write(int8_t *page_rows, uint16_t *scale, int off, const float *x, int hd) {
  float m = 0;
  for (int e = 0; e < hd; ++e) m = std::max(m, std::fabs(x[e]));
  const float s_old = off == 0 ? 0.0f : or_f16_value(*scale);
  float s_new = s_old;
  if (m / 127.0f > s_old) {
    s_new = f16_round_up(m / 127.0f);
    if (off > 0 && s_old > 0) {
      const float f = s_old / s_new;
      for (int i = 0; i < off * hd; ++i) {
        const float q = float(page_rows[i]);
        page_rows[i] = int8_t(std::min(std::max(std::nearbyint(q * f), -127.0f), 127.0f));
      }
    }
    *scale = or_f16_bits(s_new);
  }
  const float inv = s_new > 0 ? 1.0f / s_new : 0.0f;
  for (int e = 0; e < hd; ++e)
    page_rows[size_t(off) * hd + e] = int8_t(std::min(std::max(std::nearbyint(x[e] * inv), -127.0f), 127.0f));
}

}  // namespace

OR_API or_model *or_model_new(const hc_model_desc *desc, int32_t threads) {
  if (!desc || (desc->arch != HC_ARCH_QWEN3 && desc->arch != HC_ARCH_GPTOSS)) return nullptr;
  const bool gptoss = desc->arch == HC_ARCH_GPTOSS;
  auto *m = new or_model;
  m->d = *desc;
  m->pool = std::make_unique<Pool>(threads);
  const auto &d = *desc;
  const int hd = int(d.head_dim);
  for (uint32_t i = 0; i < d.layers; ++i) {
    const hc_layer_desc &ld = d.layer[i];
    Layer L;
    L.in_norm = f16_vec(ld.input_norm, d.hidden, 1);
    L.post_norm = f16_vec(ld.post_norm, d.hidden, 1);
    if (d.flags & HC_MODEL_QK_NORM) {
      L.q_norm = f16_vec(ld.q_norm, hd, 1);
      L.k_norm = f16_vec(ld.k_norm, hd, 1);
    }
    L.q = load_lin(*m->pool, ld.q);
    L.k = load_lin(*m->pool, ld.k);
    L.v = load_lin(*m->pool, ld.v);
    L.o = load_lin(*m->pool, ld.o);
    if (gptoss) {
      L.router = load_lin(*m->pool, ld.router);
      for (float &w : L.router.wt) w = f16r(w);
      for (float &b : L.router.bias) b = f16r(b);
      const hc_linear_desc &g = ld.experts_gate_up, &dn = ld.experts_down;
      L.ex.gw = static_cast<const uint8_t *>(g.data);
      L.ex.ge = g.exps;
      L.ex.dw = static_cast<const uint8_t *>(dn.data);
      L.ex.de = dn.exps;
      L.ex.gb.assign(size_t(g.rows), 0.0f);
      L.ex.db.assign(size_t(dn.rows), 0.0f);
      if (g.bias) L.ex.gb.assign(g.bias, g.bias + g.rows);
      if (dn.bias) L.ex.db.assign(dn.bias, dn.bias + dn.rows);
    } else {
      L.gate = load_lin(*m->pool, ld.gate);
      L.up = load_lin(*m->pool, ld.up);
      L.down = load_lin(*m->pool, ld.down);
    }
    L.window = int(ld.sliding_window);
    if (ld.sinks) L.sinks.assign(ld.sinks, ld.sinks + d.heads);
    m->layers.push_back(std::move(L));
  }
  m->final_norm = f16_vec(d.final_norm, d.hidden, 1);
  m->head = load_lin(*m->pool, d.head);
  m->embed.resize(size_t(d.vocab) * d.hidden);
  if (d.embed) {
    std::memcpy(m->embed.data(), d.embed, m->embed.size() * 2);
  } else {
    // tied: the head's rows as the format gives them, rounded to fp16 (the program's x input)
    m->pool->parallel_for(d.vocab, 256, [&](long lo, long hi) {
      std::vector<float> tmp(size_t(hi - lo) * d.hidden);
      dequant_rows(d.head, uint32_t(lo), uint32_t(hi), tmp.data());
      for (size_t i = 0; i < tmp.size(); ++i) m->embed[size_t(lo) * d.hidden + i] = or_f16_bits(tmp[i]);
    });
  }
  if (gptoss) {
    yarn_inv_freq(d, m->inv_freq, m->rope_factor);
  } else {
    // qwen3.Config.RopeInvFreq (internal/llm/qwen3/config.go:152-159)
    m->inv_freq.resize(hd / 2);
    for (int j = 0; j < hd / 2; ++j) m->inv_freq[j] = 1 / std::pow(d.rope_theta, double(2 * j) / double(hd));
  }
  return m;
}

OR_API void or_model_free(or_model *m) { delete m; }

OR_API or_session *or_session_new_kv(or_model *m, int32_t max_context, int32_t kv_format) {
  if (kv_format != HC_KV_F16 && kv_format != HC_KV_INT8_PAGED) return nullptr;
  auto *s = new or_session{m, max_context};
  s->kv_format = kv_format;
  const auto &d = m->d;
  const size_t rows = size_t(d.kv_heads) * max_context * d.head_dim;
  if (kv_format == HC_KV_F16) {
    s->kc.resize(d.layers);
    s->vc.resize(d.layers);
    for (uint32_t i = 0; i < d.layers; ++i) {
      s->kc[i].assign(rows, 0);
      s->vc[i].assign(rows, 0);
    }
  } else {
    const size_t pages = size_t(d.kv_heads) * ((max_context + kOrPage - 1) / kOrPage);
    s->kq.resize(d.layers);
    s->vq.resize(d.layers);
    s->ks.resize(d.layers);
    s->vs.resize(d.layers);
    for (uint32_t i = 0; i < d.layers; ++i) {
      s->kq[i].assign(rows, 0);
      s->vq[i].assign(rows, 0);
      s->ks[i].assign(pages, 0);
      s->vs[i].assign(pages, 0);
    }
  }
  return s;
}

OR_API or_session *or_session_new(or_model *m, int32_t max_context) {
  return or_session_new_kv(m, max_context, HC_KV_F16);
}

OR_API void or_session_free(or_session *s) { delete s; }
OR_API int32_t or_session_pos(or_session *s) { return s->pos; }
OR_API void or_truncate(or_session *s, int32_t len) {
  if (len >= 0 && len < s->pos) s->pos = len;
}
OR_API void or_page_write(int8_t *page_rows, uint16_t *scale, int32_t off, const float *x, int32_t hd) {
  page_write(page_rows, scale, off, x, hd);
}

namespace {

// blocks.RopeValues (internal/llm/blocks/blocks.go:412-427): cos/sin of pos * inv_freq in
// float64, as float32, laid out cat(freqs, freqs); passed to the program as fp16 inputs
// (qwen3 StepInputs, internal/llm/qwen3/arch.go:117-137).
void rope_tables(const or_model *m, int pos, int n, std::vector<float> &cs, std::vector<float> &sn) {
  const int hd = int(m->d.head_dim), half = hd / 2;
  cs.assign(size_t(n) * hd, 0);
  sn.assign(size_t(n) * hd, 0);
  for (int i = 0; i < n; ++i) {
    for (int j = 0; j < half; ++j) {
      double a = double(pos + i) * m->inv_freq[j];
      float c = float(std::cos(a)), s = float(std::sin(a));
      if (m->rope_factor != 1) { c *= m->rope_factor; s *= m->rope_factor; }
      cs[size_t(i) * hd + j] = cs[size_t(i) * hd + j + half] = f16r(c);
      sn[size_t(i) * hd + j] = sn[size_t(i) * hd + j + half] = f16r(s);
    }
  }
}

// blocks.ApplyRope (blocks.go:429-443): x*cos + cat(-x2, x1)*sin, in float32.
void apply_rope(float *x, int hd, const float *cs, const float *sn) {
  const int half = hd / 2;
  std::vector<float> r(hd);
  for (int j = 0; j < half; ++j) { r[j] = x[j + half] * -1.0f; r[j + half] = x[j]; }
  for (int j = 0; j < hd; ++j) {
    float a = x[j] * cs[j];
    float b = r[j] * sn[j];
    x[j] = a + b;
  }
}

// experts.Host.runRow (internal/llm/experts/host.go:478-591) of one row x (float32 of the fp16
// moe_x): the row quantised per 32 (mxfp4.Vec.Quantize), each chosen expert's gate and up rows by
// the MXFP4 dot product (mxfp4.Rows = Dot a row, matvec.go) plus their biases, gpt-oss's gated unit
// (host.go:515-524: gate clamped above at limit, up to +-limit, g / (1 + exp(-alpha g)) * (up + 1),
// the exp in float64), the activations quantised again, the down rows, and out += w_k (y + bias)
// added in ascending expert number.
void run_experts(Pool &pool, const hc_model_desc &d, const Experts &ex, const float *x, const int32_t *idx,
                 const float *w, float *out) {
  const int H = int(d.hidden), I = int(d.inter), K = int(d.top_k);
  const float alpha = float(d.swiglu_alpha), limit = float(d.swiglu_limit);
  std::vector<int8_t> xq(H);
  std::vector<float> xs(H / 32);
  or_mxfp4_quantize(x, uint32_t(H), xq.data(), xs.data());
  std::vector<std::vector<float>> y(K, std::vector<float>(H));
  for (int k = 0; k < K; ++k) {
    const int e = idx[k];
    std::vector<float> gu(size_t(2) * I);
    pool.parallel_for(2 * I, 64, [&](long lo, long hi) {
      for (long r = lo; r < hi; ++r) {
        const size_t row = size_t(e) * 2 * I + r;
        gu[r] = or_mxfp4_dot(ex.gw + row * (H / 2), ex.ge + row * (H / 32), uint32_t(H), xq.data(), xs.data()) +
                ex.gb[row];
      }
    });
    std::vector<float> act(I);
    for (int j = 0; j < I; ++j) {
      const float g = std::min(gu[2 * j], limit);
      const float u = std::min(std::max(gu[2 * j + 1], -limit), limit);
      act[j] = g / (1 + float(std::exp(double(-(alpha * g))))) * (u + 1);
    }
    std::vector<int8_t> hq(I);
    std::vector<float> hs(I / 32);
    or_mxfp4_quantize(act.data(), uint32_t(I), hq.data(), hs.data());
    pool.parallel_for(H, 64, [&](long lo, long hi) {
      for (long c = lo; c < hi; ++c) {
        const size_t row = size_t(e) * H + c;
        y[k][c] = or_mxfp4_dot(ex.dw + row * (I / 2), ex.de + row * (I / 32), uint32_t(I), hq.data(), hs.data());
      }
    });
  }
  std::vector<int> order(K);
  for (int k = 0; k < K; ++k) order[k] = k;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return idx[a] < idx[b]; });
  for (int k : order) {
    const float *bias = ex.db.data() + size_t(idx[k]) * H;
    for (int c = 0; c < H; ++c) out[c] += w[k] * (y[k][c] + bias[c]);
  }
}

}  // namespace

OR_API int32_t or_step(or_session *s, const int32_t *tokens, int32_t n, int32_t all_rows,
                       uint16_t *logits) {
  or_model *m = s->m;
  const auto &d = m->d;
  Pool &pool = *m->pool;
  const int D = int(d.hidden), H = int(d.heads), KV = int(d.kv_heads), hd = int(d.head_dim);
  const int rep = H / KV, F = int(d.inter);
  const int pos = s->pos;
  if (n <= 0 || pos + n > s->cap) return -1;
  const bool scaled = d.flags & HC_MODEL_NORM_SCALE;
  std::vector<float> x(size_t(n) * D), hn(size_t(n) * D), q(size_t(n) * H * hd),
      k(size_t(n) * KV * hd), v(size_t(n) * KV * hd), o(size_t(n) * H * hd), a(size_t(n) * D),
      g(size_t(n) * F), u(size_t(n) * F);
  for (int t = 0; t < n; ++t)
    for (int c = 0; c < D; ++c) x[size_t(t) * D + c] = f16v(m->embed[size_t(tokens[t]) * D + c]);
  std::vector<float> cs, sn;
  rope_tables(m, pos, n, cs, sn);
  // the score scale is an fp16 constant (blocks.SDPAScale, blocks.go:497-500)
  const float sscale = f16r(float(1 / std::sqrt(double(hd))));
  for (size_t li = 0; li < m->layers.size(); ++li) {
    const Layer &L = m->layers[li];
    const float sc_in = scaled ? (li == 0 ? 1.0f : 64.0f) : 1.0f, sc = scaled ? 64.0f : 1.0f;
    for (int t = 0; t < n; ++t) rms_norm(&x[size_t(t) * D], D, L.in_norm.data(), sc_in, d.norm_eps, &hn[size_t(t) * D]);
    linear(pool, L.q, hn.data(), n, q.data());
    linear(pool, L.k, hn.data(), n, k.data());
    linear(pool, L.v, hn.data(), n, v.data());
    std::vector<float> tmp(hd);
    for (int t = 0; t < n; ++t) {
      for (int h = 0; h < H; ++h) {
        float *qh = &q[(size_t(t) * H + h) * hd];
        if (!L.q_norm.empty()) { rms_norm(qh, hd, L.q_norm.data(), sc, d.norm_eps, tmp.data()); std::copy(tmp.begin(), tmp.end(), qh); }
        apply_rope(qh, hd, &cs[size_t(t) * hd], &sn[size_t(t) * hd]);
      }
      for (int h = 0; h < KV; ++h) {
        float *kh = &k[(size_t(t) * KV + h) * hd];
        if (!L.k_norm.empty()) { rms_norm(kh, hd, L.k_norm.data(), sc, d.norm_eps, tmp.data()); std::copy(tmp.begin(), tmp.end(), kh); }
        apply_rope(kh, hd, &cs[size_t(t) * hd], &sn[size_t(t) * hd]);
      }
    }
    // blocks.SDPAGrouped (blocks.go:516-539) over the cache (fp16 inputs) followed by the step's
    // own keys and values (float32 inside the program), with gpt-oss's sink column when present
    // (gptoss/build.go:256-285); masked keys weigh exactly 0 in the float64 softmax and are left out.
    const bool paged = s->kv_format == HC_KV_INT8_PAGED;
    const size_t npages = size_t((s->cap + kOrPage - 1) / kOrPage);
    // cache row j of kv head kvh as float32: fp16 values, or int8 codes times the page's fp16 scale
    auto cache_row = [&](bool val, int kvh, int j, float *out) {
      if (!paged) {
        const uint16_t *r = &(val ? s->vc : s->kc)[li][(size_t(kvh) * s->cap + j) * hd];
        for (int e = 0; e < hd; ++e) out[e] = f16v(r[e]);
      } else {
        const int8_t *r = &(val ? s->vq : s->kq)[li][(size_t(kvh) * s->cap + j) * hd];
        const float sc = f16v((val ? s->vs : s->ks)[li][size_t(kvh) * npages + j / kOrPage]);
        for (int e = 0; e < hd; ++e) out[e] = float(r[e]) * sc;
      }
    };
    // The step's tokens in pieces of kOrPiece (hc_step's chunking of one sequence): a piece's
    // tokens read the earlier positions from the cache and the piece's own keys and values in
    // float32; then the piece's rows go into the cache (decode.Session.keep, decode.go:1685-1705):
    // fp16, or the int8 pages in position order.
    for (int c0 = 0; c0 < n; c0 += kOrPiece) {
      const int c1 = std::min(n, c0 + kOrPiece);
      pool.parallel_for(long(c1 - c0) * H, 1, [&](long lo, long hi) {
        std::vector<float> p;
        for (long job = lo; job < hi; ++job) {
          const int t = c0 + int(job / H), h = int(job % H), kvh = h / rep, P = pos + t;
          const int from = L.window > 0 ? std::max(0, P - L.window + 1) : 0;
          const float *qh = &q[(size_t(t) * H + h) * hd];
          int nk = 0;
          std::vector<float> scores;
          std::vector<float> crow(hd);
          for (int j = from; j < pos + c0; ++j) {
            cache_row(false, kvh, j, crow.data());
            float acc = 0;
            for (int e = 0; e < hd; ++e) acc = std::fma(qh[e], crow[e], acc);
            scores.push_back(acc * sscale);
            ++nk;
          }
          const int ncache = nk;
          for (int uu = c0; uu <= t; ++uu) {
            if (L.window > 0 && P - (pos + uu) >= L.window) { scores.push_back(NAN); continue; }
            const float *kr = &k[(size_t(uu) * KV + kvh) * hd];
            float acc = 0;
            for (int e = 0; e < hd; ++e) acc = std::fma(qh[e], kr[e], acc);
            scores.push_back(acc * sscale);
          }
          double mx = -INFINITY;
          for (float z : scores) if (z == z) mx = std::max(mx, double(z));
          const bool sink = !L.sinks.empty();
          const double sk = sink ? double(f16r(L.sinks[h])) : 0;
          if (sink) mx = std::max(mx, sk);
          double zsum = 0;
          for (float z : scores) if (z == z) zsum += std::exp(double(z) - mx);
          if (sink) zsum += std::exp(sk - mx);
          p.assign(scores.size(), 0);
          for (size_t j = 0; j < scores.size(); ++j)
            p[j] = scores[j] == scores[j] ? float(std::exp(double(scores[j]) - mx) / zsum) : 0.0f;
          float *oh = &o[(size_t(t) * H + h) * hd];
          std::fill(oh, oh + hd, 0.0f);
          std::vector<float> blk(hd);
          const size_t nkeys = scores.size();
          for (size_t j0 = 0; j0 < nkeys; j0 += KC) {
            std::fill(blk.begin(), blk.end(), 0.0f);
            for (size_t j = j0; j < std::min(nkeys, j0 + KC); ++j) {
              if (scores[j] != scores[j]) continue;
              if (int(j) < ncache) {
                cache_row(true, kvh, from + int(j), crow.data());
                for (int e = 0; e < hd; ++e) blk[e] = std::fma(p[j], crow[e], blk[e]);
              } else {
                const float *vr = &v[(size_t(c0 + int(j) - ncache) * KV + kvh) * hd];
                for (int e = 0; e < hd; ++e) blk[e] = std::fma(p[j], vr[e], blk[e]);
              }
            }
            for (int e = 0; e < hd; ++e) oh[e] += blk[e];
          }
        }
      });
      for (int t = c0; t < c1; ++t)
        for (int h = 0; h < KV; ++h) {
          if (!paged) {
            for (int e = 0; e < hd; ++e) {
              s->kc[li][(size_t(h) * s->cap + pos + t) * hd + e] = or_f16_bits(k[(size_t(t) * KV + h) * hd + e]);
              s->vc[li][(size_t(h) * s->cap + pos + t) * hd + e] = or_f16_bits(v[(size_t(t) * KV + h) * hd + e]);
            }
          } else {
            const int P = pos + t, page = P / kOrPage, off = P % kOrPage;
            const size_t base = (size_t(h) * s->cap + size_t(page) * kOrPage) * hd;
            page_write(&s->kq[li][base], &s->ks[li][size_t(h) * npages + page], off, &k[(size_t(t) * KV + h) * hd], hd);
            page_write(&s->vq[li][base], &s->vs[li][size_t(h) * npages + page], off, &v[(size_t(t) * KV + h) * hd], hd);
          }
        }
    }
    // o_proj and the residual, then the MLP (qwen3 layerRest, build.go:184-189)
    linear(pool, L.o, o.data(), n, a.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + a[i];
    if (L.ex.present()) {
      // gpt-oss's layer ends at its router (gptoss/build.go:121-140, moeHead): the post-attention
      // norm (moe_x) and the router's logits leave the program as fp16, and so does the residual
      // (the part's y); the host routes (experts.Routing.Choose, chain/moe.go:582-610), runs the
      // experts and returns moe_o as fp16, which the next part adds to y in float32
      const int E = int(d.experts), K = int(d.top_k);
      std::vector<float> mx(size_t(n) * D), lg(size_t(n) * E);
      for (int t = 0; t < n; ++t) {
        rms_norm(&x[size_t(t) * D], D, L.post_norm.data(), 1.0f, d.norm_eps, &mx[size_t(t) * D]);
        for (int c = 0; c < D; ++c) mx[size_t(t) * D + c] = f16r(mx[size_t(t) * D + c]);
      }
      linear(pool, L.router, mx.data(), n, lg.data());
      for (float &v : lg) v = f16r(v);
      for (int t = 0; t < n; ++t) {
        std::vector<int32_t> idx(K);
        std::vector<float> wk(K), mo(D, 0.0f);
        or_route(&lg[size_t(t) * E], E, K, 1, idx.data(), wk.data());
        run_experts(pool, d, L.ex, &mx[size_t(t) * D], idx.data(), wk.data(), mo.data());
        for (int c = 0; c < D; ++c) {
          float &xv = x[size_t(t) * D + c];
          xv = f16r(xv) + f16r(mo[c]);
        }
      }
      continue;
    }
    for (int t = 0; t < n; ++t) rms_norm(&x[size_t(t) * D], D, L.post_norm.data(), sc, d.norm_eps, &hn[size_t(t) * D]);
    linear(pool, L.gate, hn.data(), n, g.data());
    linear(pool, L.up, hn.data(), n, u.data());
    for (size_t i = 0; i < g.size(); ++i) g[i] = silu(g[i]) * u[i];
    linear(pool, L.down, g.data(), n, a.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + a[i];
  }
  // head (qwen3 builder.head, build.go:107-109): the final norm and the logits, fp16 outputs
  const int r0 = all_rows ? 0 : n - 1, nr = n - r0;
  std::vector<float> y(size_t(nr) * d.vocab);
  for (int t = r0; t < n; ++t)
    rms_norm(&x[size_t(t) * D], D, m->final_norm.data(), scaled ? 64.0f : 1.0f, d.norm_eps, &hn[size_t(t - r0) * D]);
  linear(pool, m->head, hn.data(), nr, y.data());
  if (logits)
    for (size_t i = 0; i < y.size(); ++i) logits[i] = or_f16_bits(y[i]);
  s->pos += n;
  return 0;
}

// decode.Session.Speculate (decode.go:1235-1260) with the greedy accept closure of
// chat/engine.go:1044-1058: draft i is kept while the pick from row i equals it.
OR_API int32_t or_speculate(or_session *s, const int32_t *toks, int32_t n, int32_t *next,
                            uint16_t *logits_last) {
  const int V = int(s->m->d.vocab), pos = s->pos;
  std::vector<uint16_t> rows(size_t(n) * V);
  if (or_step(s, toks, n, 1, rows.data()) != 0) return -1;
  int kept = n;
  int picked = 0;
  for (int i = 0; i < n - 1; ++i) {
    picked = or_argmax_f16(&rows[size_t(i) * V], V);
    if (picked != toks[i + 1]) { kept = i + 1; break; }
  }
  if (kept == n) picked = or_argmax_f16(&rows[size_t(n - 1) * V], V);
  *next = picked;
  if (logits_last) std::memcpy(logits_last, &rows[size_t(kept - 1) * V], size_t(V) * 2);
  s->pos = pos + kept;
  return kept;
}

OR_API void or_gemm_nt(int32_t m, int32_t n, int32_t k, const float *a, const float *b, float *c,
                       int32_t threads) {
  Pool pool(threads);
  Lin L;
  L.rows = n;
  L.cols = k;
  L.fmt = HC_FMT_F16;
  L.wt.resize(size_t(n) * k);
  for (int r = 0; r < n; ++r)
    for (int cc = 0; cc < k; ++cc) L.wt[size_t(cc) * n + r] = b[size_t(r) * k + cc];
  std::vector<float> y(size_t(m) * n);
  linear(pool, L, a, m, y.data());
  for (size_t i = 0; i < y.size(); ++i) c[i] += y[i];
}
