// numerics.cpp — TEST INFRASTRUCTURE (see oracle.h): the reference's scalar numerics restated.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <vector>

namespace {

inline uint32_t bits_of(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float float_of(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// math.RoundToEven of a float64.
inline double round_even(double v) { return std::nearbyint(v); }

}  // namespace

// vecops.F16Bits (internal/vecops/vecops.go:297-330).
OR_API uint16_t or_f16_bits(float f) {
  uint32_t x = bits_of(f);
  uint16_t sign = uint16_t(x >> 16) & 0x8000;
  int exp = int((x >> 23) & 0xff) - 127 + 15;
  uint32_t mant = x & 0x7fffff;
  if (((x >> 23) & 0xff) == 0xff) return mant ? (sign | 0x7e00) : (sign | 0x7c00);
  if (exp >= 0x1f) return sign | 0x7c00;
  if (exp <= 0) {
    if (exp < -10) return sign;
    mant |= 0x800000;
    unsigned shift = unsigned(14 - exp);
    uint16_t h = uint16_t(mant >> shift);
    uint32_t rem = mant & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1))) h++;
    return sign | h;
  }
  uint16_t h = sign | uint16_t(exp << 10) | uint16_t(mant >> 13);
  uint32_t rem = mant & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
  return h;
}

// vecops.F16Value (internal/vecops/vecops.go:333-352).
OR_API float or_f16_value(uint16_t h) {
  uint32_t sign = uint32_t(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ff;
  if (exp == 0) {
    if (mant == 0) return float_of(sign);
    uint32_t e = 127 - 15 + 1;
    while (!(mant & 0x400)) { mant <<= 1; e--; }
    return float_of(sign | (e << 23) | ((mant & 0x3ff) << 13));
  }
  if (exp == 0x1f) return float_of(sign | (0xffu << 23) | (mant << 13));
  return float_of(sign | ((exp + 127 - 15) << 23) | (mant << 13));
}

// f32.exp: Cephes' expf, x = n ln2 + r, degree-6 polynomial (internal/f32/f32.go:49-70).
OR_API float or_exp(float x) {
  if (x != x) return x;
  x = std::min(std::max(x, -86.6f), 88.72283f);
  const float log2e = 1.44269504088896341f, c1 = 0.693359375f, c2 = -2.12194440e-4f;
  float n = float(std::floor(double(x * log2e + 0.5f)));
  float r = x - n * c1;
  r = r - n * c2;
  float p = 1.9875691500e-4f;
  p = p * r + 1.3981999507e-3f;
  p = p * r + 8.3334519073e-3f;
  p = p * r + 4.1665795894e-2f;
  p = p * r + 1.6666665459e-1f;
  p = p * r + 5.0000001201e-1f;
  float y = p * r * r + r + 1;
  return (y + y) * float_of(uint32_t(int32_t(n) + 126) << 23);
}

// llm.Synthetic.Get (internal/llm/synth.go:17-36): FNV-1a of the name, then an LCG.
OR_API void or_synth_uniform(const char *name, float *out, uint64_t n) {
  uint64_t seed = 1469598103934665603ull;
  for (const char *p = name; *p; ++p) { seed ^= uint8_t(*p); seed *= 1099511628211ull; }
  for (uint64_t i = 0; i < n; ++i) {
    seed = seed * 6364136223846793005ull + 1442695040888963407ull;
    out[i] = float(int64_t(seed >> 40) - (int64_t(1) << 23)) / float(1 << 23) * 0.2f;
  }
}

namespace {

// vecops quantize: v/s rounded to even and clamped, 0 when s is 0 (vecops.go:172-186).
inline float quant(float v, float s, float qmin, float qmax) {
  if (s == 0) return 0;
  float q = float(round_even(double(v / s)));
  return std::min(std::max(q, qmin), qmax);
}

// vecops.ClipErrors: the sum in order of (v - q s)^2, each step in float32 (vecops.go:142-170).
float clip_error(const float *vals, int n, float s, float qmin, float qmax) {
  float e = 0;
  for (int i = 0; i < n; ++i) {
    float d = vals[i] - float(quant(vals[i], s, qmin, qmax) * s);
    e = float(e + float(d * d));
  }
  return e;
}

const float kClips[] = {1, 0.95f, 0.9f, 0.85f, 0.8f, 0.75f, 0.7f, 0.65f, 0.6f, 0.55f, 0.5f};

}  // namespace

// palette.QuantizeLinear (internal/palette/linear.go:36-114), NaN-free blocks.
OR_API void or_quantize_linear(const float *w, uint32_t rows, uint32_t cols, uint32_t col_block,
                               int32_t bits, int32_t search, uint8_t *data, uint16_t *scales) {
  if (col_block == 0 || col_block > cols) col_block = cols;
  uint32_t nc = cols / col_block;
  float qmax = float((1 << (bits - 1)) - 1), qmin = -qmax - 1;
  if (bits == 4) std::memset(data, 0, (size_t(rows) * cols + 1) / 2);
  std::vector<int8_t> q(col_block);
  for (uint32_t r = 0; r < rows; ++r) {
    for (uint32_t b = 0; b < nc; ++b) {
      const float *blk = w + size_t(r) * cols + size_t(b) * col_block;
      float top = 0;
      for (uint32_t j = 0; j < col_block; ++j) top = std::max(top, std::fabs(blk[j]));
      uint16_t best = or_f16_bits(top / qmax);
      float best_err = INFINITY;
      if (search) {
        for (float c : kClips) {
          uint16_t h = or_f16_bits(top * c / qmax);
          float e = clip_error(blk, int(col_block), or_f16_value(h), qmin, qmax);
          if (e < best_err) { best = h; best_err = e; }
        }
      }
      scales[size_t(r) * nc + b] = best;
      float s = or_f16_value(best);
      for (uint32_t j = 0; j < col_block; ++j) q[j] = int8_t(quant(blk[j], s, qmin, qmax));
      size_t base = size_t(r) * cols + size_t(b) * col_block;
      for (uint32_t j = 0; j < col_block; ++j) {
        size_t i = base + j;
        if (bits == 8) data[i] = uint8_t(q[j]);
        else data[i / 2] |= uint8_t((q[j] & 0xf) << (4 * (i % 2)));
      }
    }
  }
}

// palette.Linear.Dequantize (internal/palette/linear.go:152-169).
OR_API void or_dequant_linear(const uint8_t *data, const uint16_t *scales, uint32_t rows,
                              uint32_t cols, uint32_t col_block, int32_t bits, float *out) {
  if (col_block == 0 || col_block > cols) col_block = cols;
  uint32_t nc = cols / col_block;
  for (size_t i = 0; i < size_t(rows) * cols; ++i) {
    int q;
    if (bits == 8) q = int(int8_t(data[i]));
    else {
      q = int(data[i / 2] >> (4 * (i % 2))) & 0xf;
      if (q >= 8) q -= 16;
    }
    size_t r = i / cols, c = i % cols;
    out[i] = float(q) * or_f16_value(scales[r * nc + c / col_block]);
  }
}

// milcpu shiftScale with an fp16 offset (internal/milcpu/ops.go:1589-1610): v = float32(q);
// v -= offset; out = v * scale; blocks of (1, 32) over unsigned 4-bit codes, low nibble first.
OR_API void or_dequant_int4_asym(const uint8_t *data, const uint16_t *scales,
                                 const uint16_t *zeros, uint32_t rows, uint32_t cols, float *out) {
  uint32_t nc = cols / 32;
  for (size_t i = 0; i < size_t(rows) * cols; ++i) {
    size_t r = i / cols, c = i % cols;
    float v = float(int(data[i / 2] >> (4 * (i % 2))) & 0xf);
    v -= or_f16_value(zeros[r * nc + c / 32]);
    out[i] = v * or_f16_value(scales[r * nc + c / 32]);
  }
}

// The asymmetric quantiser of HC_FMT_INT4_ASYM_G32 (this build's definition; the reference's
// int4 is symmetric): s = f16((max - min) / 15), or f16(max |v|) or 1 for a constant block;
// z = f16(-min / s); q = clamp(round_even(v / s + z), 0, 15).
OR_API void or_quantize_int4_asym(const float *w, uint32_t rows, uint32_t cols, uint8_t *data,
                                  uint16_t *scales, uint16_t *zeros) {
  uint32_t nc = cols / 32;
  std::memset(data, 0, size_t(rows) * cols / 2);
  for (uint32_t r = 0; r < rows; ++r) {
    for (uint32_t b = 0; b < nc; ++b) {
      const float *blk = w + size_t(r) * cols + size_t(b) * 32;
      float mn = blk[0], mx = blk[0];
      for (int j = 1; j < 32; ++j) { mn = std::min(mn, blk[j]); mx = std::max(mx, blk[j]); }
      uint16_t sh = or_f16_bits((mx - mn) / 15.0f);
      if (or_f16_value(sh) == 0) {
        float top = std::max(std::fabs(mn), std::fabs(mx));
        sh = top > 0 ? or_f16_bits(top) : uint16_t(0x3c00);
      }
      float s = or_f16_value(sh);
      uint16_t zh = or_f16_bits(-mn / s);
      float z = or_f16_value(zh);
      scales[size_t(r) * nc + b] = sh;
      zeros[size_t(r) * nc + b] = zh;
      for (int j = 0; j < 32; ++j) {
        float q = float(round_even(double(blk[j] / s + z)));
        q = std::min(std::max(q, 0.0f), 15.0f);
        size_t i = size_t(r) * cols + size_t(b) * 32 + j;
        data[i / 2] |= uint8_t(uint8_t(q) << (4 * (i % 2)));
      }
    }
  }
}

namespace {
// mxfp4.Values and doubled (internal/mxfp4/mxfp4.go:17-21).
const float kE2M1[16] = {0, 0.5f, 1, 1.5f, 2, 3, 4, 6, -0.0f, -0.5f, -1, -1.5f, -2, -3, -4, -6};
const int8_t kDoubled[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
// mxfp4.scale: 2^(e-127) as float32 bits e<<23 (mxfp4.go:77).
inline float e8m0(uint8_t e) { return float_of(uint32_t(e) << 23); }
}  // namespace

// mxfp4.nearest (internal/mxfp4/encode.go:62-78).
OR_API uint8_t or_mxfp4_nearest(double x) {
  uint8_t sign = 0;
  if (x < 0) { sign = 8; x = -x; }
  uint8_t c = 7;
  for (uint8_t k = 0; k < 7; ++k) {
    double mid = double(float(kE2M1[k] + kE2M1[k + 1])) / 2;
    if (x < mid || (x == mid && k % 2 == 0)) { c = k; break; }
    if (x == mid) { c = k + 1; break; }
  }
  if (c == 0) return 0;
  return sign | c;
}

// mxfp4.Encode (internal/mxfp4/encode.go:11-58).
OR_API void or_mxfp4_encode(const float *row, uint32_t n, uint8_t *w, uint8_t *e) {
  uint8_t codes[32];
  for (uint32_t b = 0; b < n / 32; ++b) {
    const float *blk = row + size_t(b) * 32;
    float m = 0;
    for (int j = 0; j < 32; ++j) m = std::max(m, std::fabs(blk[j]));
    uint8_t best = 0;
    double best_err = INFINITY;
    if (m > 0) {
      int ex;
      std::frexp(double(m), &ex);
      int rule = ex - 1 - 2;
      for (int x : {rule - 1, rule, rule + 1}) {
        int eb = x + 127;
        if (eb < 1 || eb > 254) continue;
        double s = double(e8m0(uint8_t(eb)));
        double se = 0;
        for (int j = 0; j < 32; ++j) {
          double d = double(blk[j]) - double(kE2M1[or_mxfp4_nearest(double(blk[j]) / s)]) * s;
          se += d * d;
        }
        if (se < best_err) { best = uint8_t(eb); best_err = se; }
      }
    }
    if (best == 0) {
      std::memset(w + size_t(b) * 16, 0, 16);
      e[b] = 0;
      continue;
    }
    double s = double(e8m0(best));
    for (int j = 0; j < 32; ++j) codes[j] = or_mxfp4_nearest(double(blk[j]) / s);
    for (int j = 0; j < 16; ++j) w[size_t(b) * 16 + j] = uint8_t(codes[2 * j] | (codes[2 * j + 1] << 4));
    e[b] = best;
  }
}

// mxfp4.Dequantize (internal/mxfp4/mxfp4.go:118-128).
OR_API void or_mxfp4_dequant(const uint8_t *w, const uint8_t *e, uint32_t n, float *out) {
  for (uint32_t b = 0; b < n / 32; ++b) {
    float s = e8m0(e[b]);
    for (int j = 0; j < 16; ++j) {
      uint8_t by = w[size_t(b) * 16 + j];
      out[b * 32 + 2 * j] = kE2M1[by & 15] * s;
      out[b * 32 + 2 * j + 1] = kE2M1[by >> 4] * s;
    }
  }
}

// mxfp4.Vec.Quantize (internal/mxfp4/mxfp4.go:33-53): per block of 32, q = round_even(x * (127 /
// max)), the 16 even values then the 16 odd ones; S = max / 127.
OR_API void or_mxfp4_quantize(const float *x, uint32_t n, int8_t *q, float *s) {
  for (uint32_t b = 0; b < n / 32; ++b) {
    const float *blk = x + size_t(b) * 32;
    int8_t *qb = q + size_t(b) * 32;
    float m = 0;
    for (int j = 0; j < 32; ++j) m = std::max(m, std::fabs(blk[j]));
    if (m == 0) { std::memset(qb, 0, 32); s[b] = 0; continue; }
    float inv = 127 / m;
    for (int j = 0; j < 16; ++j) {
      qb[j] = int8_t(round_even(double(blk[2 * j] * inv)));
      qb[16 + j] = int8_t(round_even(double(blk[2 * j + 1] * inv)));
    }
    s[b] = m / 127;
  }
}

// mxfp4.dotGo (internal/mxfp4/mxfp4.go:80-91).
OR_API float or_mxfp4_dot(const uint8_t *w, const uint8_t *e, uint32_t n, const int8_t *q,
                          const float *s) {
  float sum = 0;
  for (uint32_t b = 0; b < n / 32; ++b) {
    int32_t acc = 0;
    const uint8_t *blk = w + size_t(b) * 16;
    const int8_t *qb = q + size_t(b) * 32;
    for (int j = 0; j < 16; ++j) {
      acc += int32_t(kDoubled[blk[j] & 15]) * int32_t(qb[j]) +
             int32_t(kDoubled[blk[j] >> 4]) * int32_t(qb[16 + j]);
    }
    float t = float(acc) * e8m0(e[b]);
    sum += t * s[b];
  }
  return sum / 2;
}

// experts.Routing.Choose, Score "softmax" (internal/llm/experts/weights.go:33-82).
OR_API void or_route(const float *logits, int32_t n, int32_t k, int32_t norm, int32_t *idx,
                     float *w) {
  std::vector<float> score(n);
  float m = -INFINITY;
  for (int e = 0; e < n; ++e) m = std::max(m, logits[e]);
  float sum = 0;
  for (int e = 0; e < n; ++e) {
    score[e] = float(std::exp(double(logits[e] - m)));
    sum += score[e];
  }
  for (int e = 0; e < n; ++e) score[e] /= sum;
  std::vector<int> order(n);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return score[a] > score[b]; });
  float tot = 0;
  for (int j = 0; j < k; ++j) {
    idx[j] = order[j];
    w[j] = score[order[j]];
    tot += w[j];
  }
  if (norm)
    for (int j = 0; j < k; ++j) w[j] /= tot + 1e-6f;
}

// paged.Merge (internal/llm/paged/paged.go:227-310).
struct or_merge {
  int rows, dim;
  std::vector<float> acc, top, sum;
};

OR_API or_merge *or_merge_new(int32_t rows, int32_t dim) {
  auto *m = new or_merge{rows, dim, std::vector<float>(size_t(rows) * dim, 0.0f),
                         std::vector<float>(rows, -INFINITY), std::vector<float>(rows, 0.0f)};
  return m;
}
OR_API void or_merge_free(or_merge *m) { delete m; }

namespace {
void merge_raise(or_merge *c, int r, float mj) {
  if (mj > c->top[r]) {
    if (c->sum[r] > 0) {
      float f = float(std::exp(double(c->top[r] - mj)));
      c->sum[r] *= f;
      for (int i = 0; i < c->dim; ++i) c->acc[size_t(r) * c->dim + i] *= f;
    }
    c->top[r] = mj;
  }
}
}  // namespace

OR_API void or_merge_add(or_merge *c, const float *o, const float *mx, const float *l) {
  for (int r = 0; r < c->rows; ++r) {
    if (l[r] <= 0) continue;
    float mj = mx[r];
    merge_raise(c, r, mj);
    float w = l[r] * float(std::exp(double(mj - c->top[r])));
    c->sum[r] += w;
    for (int i = 0; i < c->dim; ++i) c->acc[size_t(r) * c->dim + i] += w * o[size_t(r) * c->dim + i];
  }
}

OR_API void or_merge_add_sink(or_merge *c, const float *sinks, int32_t tokens) {
  for (int r = 0; r < c->rows; ++r) {
    float mj = sinks[r / tokens];
    merge_raise(c, r, mj);
    c->sum[r] += float(std::exp(double(mj - c->top[r])));
  }
}

OR_API void or_merge_result(or_merge *c, float *out) {
  for (int r = 0; r < c->rows; ++r) {
    float inv = c->sum[r] > 0 ? 1 / c->sum[r] : 0.0f;
    for (int i = 0; i < c->dim; ++i) out[size_t(r) * c->dim + i] = c->acc[size_t(r) * c->dim + i] * inv;
  }
}

// chat.Sampling.pick at temperature 0: strict > so the first largest wins (sample.go:80-88).
OR_API int32_t or_argmax(const float *logits, int32_t n) {
  int32_t best = 0;
  for (int32_t i = 0; i < n; ++i)
    if (logits[i] > logits[best]) best = i;
  return best;
}

OR_API int32_t or_argmax_f16(const uint16_t *logits, int32_t n) {
  int32_t best = 0;
  float bv = or_f16_value(logits[0]);
  for (int32_t i = 0; i < n; ++i) {
    float v = or_f16_value(logits[i]);
    if (v > bv) { best = i; bv = v; }
  }
  return best;
}
