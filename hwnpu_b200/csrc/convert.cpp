// convert.cpp: the converter side on the host's cores: seeded synthetic values, the reference's
// weight quantisers and fp16 conversion. These produce the byte layouts hc_model_load takes.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <string>
#include <thread>
#include <vector>

#include "common.h"
#include "../../include/hwnpu_cuda_synth.h"

namespace {

inline uint32_t fbits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float ffrom(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// Runs f(lo, hi) over [0, n) on the host's cores.
void host_parallel(uint64_t n, uint64_t grain, const std::function<void(uint64_t, uint64_t)> &f) {
  unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  uint64_t chunks = (n + grain - 1) / grain;
  unsigned t = unsigned(std::min<uint64_t>(hw, chunks));
  if (t <= 1) { if (n) f(0, n); return; }
  std::vector<std::thread> th;
  uint64_t per = (n + t - 1) / t;
  for (unsigned i = 0; i < t; ++i) {
    uint64_t lo = i * per, hi = std::min(n, lo + per);
    if (lo >= hi) break;
    th.emplace_back([=, &f] { f(lo, hi); });
  }
  for (auto &x : th) x.join();
}

// PCG32 (O'Neill's pcg32, XSH RR output) on a stream chosen by the caller.
struct Pcg32 {
  uint64_t state = 0, inc = 1;
  Pcg32(uint64_t seed, uint64_t stream) {
    inc = (stream << 1u) | 1u;
    next();
    state += seed;
    next();
  }
  uint32_t next() {
    uint64_t old = state;
    state = old * 6364136223846793005ull + inc;
    uint32_t xs = uint32_t(((old >> 18u) ^ old) >> 27u);
    uint32_t rot = uint32_t(old >> 59u);
    return (xs >> rot) | (xs << ((-rot) & 31));
  }
};

uint64_t fnv1a(const char *s) {
  uint64_t h = 1469598103934665603ull;
  for (; *s; ++s) { h ^= uint8_t(*s); h *= 1099511628211ull; }
  return h;
}

constexpr uint64_t kChunk = 1u << 20;

}  // namespace

namespace hc {

// vecops.F16Bits (internal/vecops/vecops.go:297-330): RNE, overflow to inf, NaN to sign|0x7e00.
uint16_t f16_bits(float f) {
  uint32_t x = fbits(f);
  uint16_t sign = uint16_t(x >> 16) & 0x8000;
  int exp = int((x >> 23) & 0xff) - 127 + 15;
  uint32_t mant = x & 0x7fffff;
  if (((x >> 23) & 0xff) == 0xff) return mant ? (sign | 0x7e00) : (sign | 0x7c00);
  if (exp >= 0x1f) return sign | 0x7c00;
  if (exp <= 0) {
    if (exp < -10) return sign;
    mant |= 0x800000;
    unsigned sh = unsigned(14 - exp);
    uint16_t h = uint16_t(mant >> sh);
    uint32_t rem = mant & ((1u << sh) - 1), half = 1u << (sh - 1);
    if (rem > half || (rem == half && (h & 1))) h++;
    return sign | h;
  }
  uint16_t h = sign | uint16_t(exp << 10) | uint16_t(mant >> 13);
  uint32_t rem = mant & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
  return h;
}

// vecops.F16Value (internal/vecops/vecops.go:333-352): exact.
float f16_value(uint16_t h) {
  uint32_t sign = uint32_t(h >> 15) << 31, exp = (h >> 10) & 0x1f, mant = h & 0x3ff;
  if (exp == 0) {
    if (!mant) return ffrom(sign);
    uint32_t e = 127 - 15 + 1;
    while (!(mant & 0x400)) { mant <<= 1; e--; }
    return ffrom(sign | (e << 23) | ((mant & 0x3ff) << 13));
  }
  if (exp == 0x1f) return ffrom(sign | (0xffu << 23) | (mant << 13));
  return ffrom(sign | ((exp + 127 - 15) << 23) | (mant << 13));
}

}  // namespace hc

using hc::f16_bits;
using hc::f16_value;

extern "C" {

HC_API void hc_f32_to_f16(const float *src, uint16_t *dst, uint64_t n) {
  host_parallel(n, 1 << 16, [&](uint64_t lo, uint64_t hi) {
    for (uint64_t i = lo; i < hi; ++i) dst[i] = f16_bits(src[i]);
  });
}

HC_API void hc_f16_to_f32(const uint16_t *src, float *dst, uint64_t n) {
  host_parallel(n, 1 << 16, [&](uint64_t lo, uint64_t hi) {
    for (uint64_t i = lo; i < hi; ++i) dst[i] = f16_value(src[i]);
  });
}

HC_API char *hc_synth_normal(uint64_t seed, const char *name, const float *std_p, float *out, uint64_t n) {
  if (!name || !std_p || (!out && n)) return hc::make_error("hc_synth_normal: NULL argument");
  const float std_ = *std_p;
  const uint64_t h = fnv1a(name);
  const uint64_t chunks = (n + kChunk - 1) / kChunk;
  host_parallel(chunks, 1, [&](uint64_t c0, uint64_t c1) {
    for (uint64_t c = c0; c < c1; ++c) {
      Pcg32 rng(seed ^ 0x9e3779b97f4a7c15ull, h + c * 0x632be59bd9b4e019ull);
      const uint64_t lo = c * kChunk, hi = std::min(n, lo + kChunk);
      for (uint64_t i = lo; i < hi; i += 2) {
        // Box-Muller on two 32-bit draws: u1 in (0, 1], u2 in [0, 1)
        double u1 = (double(rng.next()) + 1.0) * (1.0 / 4294967296.0);
        double u2 = double(rng.next()) * (1.0 / 4294967296.0);
        double r = std::sqrt(-2.0 * std::log(u1));
        out[i] = float(std_ * r * std::cos(6.283185307179586 * u2));
        if (i + 1 < hi) out[i + 1] = float(std_ * r * std::sin(6.283185307179586 * u2));
      }
    }
  });
  return nullptr;
}

HC_API char *hc_synth_tokens(uint64_t seed, int32_t vocab, int32_t *out, uint64_t n) {
  if (vocab <= 0 || (!out && n)) return hc::make_error("hc_synth_tokens: bad argument");
  Pcg32 rng(seed, 0x70c3a5d1ull);
  for (uint64_t i = 0; i < n; ++i) out[i] = int32_t((uint64_t(rng.next()) * uint64_t(vocab)) >> 32);
  return nullptr;
}

}  // extern "C"

namespace {

// vecops quantize (vecops.go:172-186): v/s rounded to even and clamped, 0 when s is 0.
inline float quant_sym(float v, float s, float qmin, float qmax) {
  if (s == 0) return 0;
  float q = float(std::nearbyint(double(v / s)));
  return std::min(std::max(q, qmin), qmax);
}

const float kClips[] = {1, 0.95f, 0.9f, 0.85f, 0.8f, 0.75f, 0.7f, 0.65f, 0.6f, 0.55f, 0.5f};

}  // namespace

extern "C" {

// palette.QuantizeLinear (internal/palette/linear.go:36-114) for NaN-free weights: a scale
// f16(top * clip / qmax) chosen by the float32 squared error of vecops.ClipErrors
// (vecops.go:142-170), values rounded to even and clamped.
HC_API char *hc_quantize_linear(const float *w, uint32_t rows, uint32_t cols, uint32_t col_block,
                                int32_t bits, int32_t search, uint8_t *data, uint16_t *scales) {
  if (bits != 4 && bits != 8) return hc::make_error("hc_quantize_linear: bits must be 4 or 8");
  if (col_block == 0 || col_block > cols) col_block = cols;
  if (cols % col_block) return hc::make_error("hc_quantize_linear: columns not a multiple of the block");
  if (bits == 4 && (cols % 2)) return hc::make_error("hc_quantize_linear: 4 bits needs even columns");
  const uint32_t nc = cols / col_block;
  const float qmax = float((1 << (bits - 1)) - 1), qmin = -qmax - 1;
  host_parallel(rows, 16, [&](uint64_t r0, uint64_t r1) {
    std::vector<float> q(col_block);
    for (uint64_t r = r0; r < r1; ++r) {
      if (bits == 4) std::memset(data + r * cols / 2, 0, cols / 2);
      for (uint32_t b = 0; b < nc; ++b) {
        const float *blk = w + r * cols + size_t(b) * col_block;
        float top = 0;
        for (uint32_t j = 0; j < col_block; ++j) top = std::max(top, std::fabs(blk[j]));
        uint16_t best = f16_bits(top / qmax);
        float best_err = INFINITY;
        if (search) {
          for (float c : kClips) {
            uint16_t hs = f16_bits(top * c / qmax);
            float s = f16_value(hs), e = 0;
            for (uint32_t j = 0; j < col_block; ++j) {
              float d = blk[j] - float(quant_sym(blk[j], s, qmin, qmax) * s);
              e = float(e + float(d * d));
            }
            if (e < best_err) { best = hs; best_err = e; }
          }
        }
        scales[r * nc + b] = best;
        const float s = f16_value(best);
        for (uint32_t j = 0; j < col_block; ++j) {
          int qv = int(quant_sym(blk[j], s, qmin, qmax));
          size_t i = r * cols + size_t(b) * col_block + j;
          if (bits == 8) data[i] = uint8_t(int8_t(qv));
          else data[i / 2] |= uint8_t((qv & 0xf) << (4 * (i % 2)));
        }
      }
    }
  });
  return nullptr;
}

HC_API char *hc_quantize_int4_asym(const float *w, uint32_t rows, uint32_t cols, uint8_t *data,
                                   uint16_t *scales, uint16_t *zeros) {
  if (cols % 32) return hc::make_error("hc_quantize_int4_asym: columns not a multiple of 32");
  const uint32_t nc = cols / 32;
  host_parallel(rows, 16, [&](uint64_t r0, uint64_t r1) {
    for (uint64_t r = r0; r < r1; ++r) {
      std::memset(data + r * cols / 2, 0, cols / 2);
      for (uint32_t b = 0; b < nc; ++b) {
        const float *blk = w + r * cols + size_t(b) * 32;
        float mn = blk[0], mx = blk[0];
        for (int j = 1; j < 32; ++j) { mn = std::min(mn, blk[j]); mx = std::max(mx, blk[j]); }
        uint16_t sh = f16_bits((mx - mn) / 15.0f);
        if (f16_value(sh) == 0) {
          float top = std::max(std::fabs(mn), std::fabs(mx));
          sh = top > 0 ? f16_bits(top) : uint16_t(0x3c00);
        }
        const float s = f16_value(sh);
        const uint16_t zh = f16_bits(-mn / s);
        const float z = f16_value(zh);
        scales[r * nc + b] = sh;
        zeros[r * nc + b] = zh;
        for (int j = 0; j < 32; ++j) {
          float q = float(std::nearbyint(double(blk[j] / s + z)));
          q = std::min(std::max(q, 0.0f), 15.0f);
          size_t i = r * cols + size_t(b) * 32 + j;
          data[i / 2] |= uint8_t(uint8_t(q) << (4 * (i % 2)));
        }
      }
    }
  });
  return nullptr;
}

}  // extern "C"

namespace {

const float kE2M1[8] = {0, 0.5f, 1, 1.5f, 2, 3, 4, 6};

// The e2m1 code nearest x, clipped to 6, ties to the even code, zero as +0 (mxfp4.nearest,
// internal/mxfp4/encode.go:62-78).
uint8_t e2m1_nearest(double x) {
  uint8_t sign = 0;
  if (x < 0) { sign = 8; x = -x; }
  // the midpoints between neighbouring magnitudes, as the rule computes them
  static const struct Mids {
    double v[7];
    Mids() { for (int k = 0; k < 7; ++k) v[k] = double(float(kE2M1[k] + kE2M1[k + 1])) / 2; }
  } mids;
  // the code is the number of midpoints below x; a tie goes to the even code (k, or k + 1 when k is odd)
  int c = 0;
  for (int k = 0; k < 7; ++k) c += int(x > mids.v[k]) + int(x == mids.v[k] && (k & 1));
  return c == 0 ? 0 : uint8_t(sign | c);
}

inline double e2m1_value(uint8_t code) { return (code & 8) ? -double(kE2M1[code & 7]) : double(kE2M1[code & 7]); }

}  // namespace

extern "C" {

// mxfp4.Encode (internal/mxfp4/encode.go:11-58): per block the exponent of OCP's rule or the one
// above or below it, whichever rounds the block with the least squared error.
HC_API char *hc_mxfp4_encode(const float *w, uint32_t rows, uint32_t cols, uint8_t *blocks,
                             uint8_t *exps) {
  if (cols % 32) return hc::make_error("hc_mxfp4_encode: columns not a multiple of 32");
  const uint32_t nb = cols / 32;
  host_parallel(rows, 8, [&](uint64_t r0, uint64_t r1) {
    uint8_t codes[32];
    for (uint64_t r = r0; r < r1; ++r) {
      for (uint32_t b = 0; b < nb; ++b) {
        const float *blk = w + r * cols + size_t(b) * 32;
        uint8_t *wb = blocks + (r * nb + b) * 16;
        float m = 0;
        for (int j = 0; j < 32; ++j) m = std::max(m, std::fabs(blk[j]));
        uint8_t best = 0;
        double best_err = INFINITY;
        if (m > 0) {
          int ex;
          std::frexp(double(m), &ex);
          const int rule = ex - 1 - 2;
          for (int x : {rule - 1, rule, rule + 1}) {
            const int eb = x + 127;
            if (eb < 1 || eb > 254) continue;
            const double s = double(ffrom(uint32_t(eb) << 23));
            const double inv = 1.0 / s;  // exact: s is a power of two
            double se = 0;
            for (int j = 0; j < 32; ++j) {
              double d = double(blk[j]) - e2m1_value(e2m1_nearest(double(blk[j]) * inv)) * s;
              se += d * d;
            }
            if (se < best_err) { best = uint8_t(eb); best_err = se; }
          }
        }
        if (best == 0) {
          std::memset(wb, 0, 16);
          exps[r * nb + b] = 0;
          continue;
        }
        const double inv = 1.0 / double(ffrom(uint32_t(best) << 23));
        for (int j = 0; j < 32; ++j) codes[j] = e2m1_nearest(double(blk[j]) * inv);
        for (int j = 0; j < 16; ++j) wb[j] = uint8_t(codes[2 * j] | (codes[2 * j + 1] << 4));
        exps[r * nb + b] = best;
      }
    }
  });
  return nullptr;
}

}  // extern "C"
