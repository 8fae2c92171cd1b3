// synth.cpp — TEST INFRASTRUCTURE (see oracle.h): the seeded synthetic inputs of the benchmark
// configurations, generated on the oracle's side so that a CPU run (bench.py --impl reference,
// the cpu_baseline leg) builds its weights and prompts without the product library.
//
// The generator is this build's own (the reference's synthetic values are uniform, synth.go:17-36;
// the benchmark configurations ask for N(0, std^2)): a name's values come in chunks of 2^20, chunk
// c drawn from PCG32 (XSH RR) seeded by (seed ^ golden ratio, FNV-1a(name) + c * odd constant),
// two 32-bit draws a pair of values by Box-Muller in float64. The product library's hc_synth_normal
// follows the same recipe, and tests/test_oracle.py checks that the two agree bit for bit, so the
// GPU arm and the CPU arm of a benchmark read identical weights.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <thread>
#include <vector>

namespace {

struct Pcg32 {
  uint64_t state = 0, inc = 1;
  Pcg32(uint64_t seed, uint64_t stream) {
    inc = (stream << 1u) | 1u;
    step();
    state += seed;
    step();
  }
  uint32_t step() {
    const uint64_t old = state;
    state = old * 6364136223846793005ull + inc;
    const uint32_t xs = uint32_t(((old >> 18u) ^ old) >> 27u);
    const uint32_t rot = uint32_t(old >> 59u);
    return (xs >> rot) | (xs << ((-rot) & 31));
  }
};

uint64_t fnv1a64(const char *s) {
  uint64_t h = 1469598103934665603ull;
  for (; *s; ++s) {
    h ^= uint8_t(*s);
    h *= 1099511628211ull;
  }
  return h;
}

constexpr uint64_t kChunk = uint64_t(1) << 20;

}  // namespace

OR_API void or_synth_normal(uint64_t seed, const char *name, const float *std_, float *out, uint64_t n) {
  const uint64_t h = fnv1a64(name);
  const float sd = *std_;
  const uint64_t chunks = (n + kChunk - 1) / kChunk;
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const unsigned nt = unsigned(std::min<uint64_t>(hw, std::max<uint64_t>(1, chunks)));
  auto body = [&](uint64_t c0, uint64_t c1) {
    for (uint64_t c = c0; c < c1; ++c) {
      Pcg32 rng(seed ^ 0x9e3779b97f4a7c15ull, h + c * 0x632be59bd9b4e019ull);
      const uint64_t lo = c * kChunk, hi = std::min(n, lo + kChunk);
      for (uint64_t i = lo; i < hi; i += 2) {
        const double u1 = (double(rng.step()) + 1.0) * (1.0 / 4294967296.0);
        const double u2 = double(rng.step()) * (1.0 / 4294967296.0);
        const double r = std::sqrt(-2.0 * std::log(u1));
        out[i] = float(sd * r * std::cos(6.283185307179586 * u2));
        if (i + 1 < hi) out[i + 1] = float(sd * r * std::sin(6.283185307179586 * u2));
      }
    }
  };
  if (nt <= 1) {
    body(0, chunks);
    return;
  }
  std::vector<std::thread> th;
  const uint64_t per = (chunks + nt - 1) / nt;
  for (unsigned i = 0; i < nt; ++i) {
    const uint64_t c0 = i * per, c1 = std::min(chunks, c0 + per);
    if (c0 >= c1) break;
    th.emplace_back(body, c0, c1);
  }
  for (auto &t : th) t.join();
}

OR_API void or_synth_tokens(uint64_t seed, int32_t vocab, int32_t *out, uint64_t n) {
  Pcg32 rng(seed, 0x70c3a5d1ull);
  for (uint64_t i = 0; i < n; ++i) out[i] = int32_t((uint64_t(rng.step()) * uint64_t(vocab)) >> 32);
}

OR_API void or_f32_to_f16_n(const float *src, uint16_t *dst, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) dst[i] = or_f16_bits(src[i]);
}
