// mk.cu: the persistent decode kernel (see mk.h). One CTA per SM runs every phase of the step:
//
//   embed -> per layer: [qkv GEMV] -> [attention] -> [o GEMV + residual] -> [gate/up GEMV + SiLU]
//            -> [down GEMV + residual] -> head GEMV + greedy choice
//
// with a grid barrier between phases. A CTA is 8 consumer warps and 1 producer warp. The producer
// walks the same static schedule as the consumers (the CTA's row tiles of every GEMV, its attention
// unit's cached keys and values) and streams it from HBM into a ring of shared-memory stages with
// bulk copies (cp.async.bulk, an mbarrier per stage for "full" and one for "empty"), running ahead
// of the grid barriers the consumers wait at, so HBM keeps streaming while they synchronise.
// No wait is unbounded: a grid barrier or a stage that does not arrive within
// MkParams::spin_limit cycles sets *status and the kernel returns.
//
// Activations reach a GEMV as int8 tiles (common.h's kActTile) written by the phase that produced
// them: the o-proj and down producers own whole groups of 32 output rows, add the residual,
// quantise x times the next norm's weight and store each group's sum of squares, from which
// every consumer forms the norm's 1/rms (qwen3's normScaled, build.go:131-151) and applies it to
// the group scales; the gate/up producer quantises silu(gate)*up; the attention's last split of a
// head quantises the head's output.
#include <algorithm>

#include "device.cuh"
#include "mk.h"

namespace hc {
namespace {

constexpr int kWarps = kMkThreads / 32;

// ---- grid barrier with a deadline ------------------------------------------------------------
// Cycles between two looks at the status word (another CTA's failure) and the deadline in a wait.
constexpr long long kStatusPoll = 20000;

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Synchronises the 8 consumer warps (named barrier 1; the producer warp never joins).
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kMkThreads) : "memory"); }

// The grid barrier of the consumers: returns false when it (or an earlier one) gave up.
// A sub-phase mark of the trace (thread 0): slot 0 when the phase's inputs are in smem, 1 when its
// chunks are consumed.
__device__ __forceinline__ void mark(const MkParams &p, unsigned epoch, int slot) {
  if (p.trace && threadIdx.x == 0)
    p.trace[size_t(2 + slot) * mk_phases(p.layers) * gridDim.x + size_t(epoch) * gridDim.x + blockIdx.x] = global_ns();
}

__device__ bool grid_sync(const MkParams &p, unsigned &epoch) {
  __shared__ int ok;
  csync();
  if (threadIdx.x == 0) {
    if (p.trace) p.trace[size_t(epoch) * gridDim.x + blockIdx.x] = global_ns();
    epoch += 1;
    const unsigned target = epoch * gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
    const long long t0 = clock64();
    long long next = t0 + kStatusPoll;
    int good = 1;
    while (ld_acquire(p.bar) < target) {
      // the status word and the deadline are looked at every kStatusPoll cycles only, so that a
      // poll costs one L2 round trip
      const long long now = clock64();
      if (now < next) continue;
      next = now + kStatusPoll;
      if (*reinterpret_cast<volatile int *>(p.status)) { good = 0; break; }
      if (now - t0 > p.spin_limit) {
        atomicExch(p.status, int(epoch));
        good = 0;
        break;
      }
    }
    if (p.trace) p.trace[size_t(mk_phases(p.layers) + epoch - 1) * gridDim.x + blockIdx.x] = global_ns();
    ok = good;
  }
  csync();
  return ok;
}

// The units [u0, u1) of U that CTA b takes.
__device__ __forceinline__ void my_units(int U, int &u0, int &u1) {
  u0 = int((long long)blockIdx.x * U / gridDim.x);
  u1 = int((long long)(blockIdx.x + 1) * U / gridDim.x);
}

// ---- activation quantisation of one group of 32 (one value a lane) --------------------------
// hi = round_even(v * 127 / max), lo = the residual at 1/256 of the scale (common.h, kActTile).
__device__ __forceinline__ void quant32(float v, uint8_t *tile, int gi, int lane) {
  const float m = warp_max(fabsf(v));
  int8_t hq = 0, lq = 0;
  float S = 0.f;
  int s256 = 0;
  if (m > 0.f) {
    const float inv = 127.0f / m;
    S = m / 127.0f;
    const float h = rintf(v * inv);
    const float r = fmaf(-h, S, v);
    const float l = fminf(fmaxf(rintf(r * (256.0f * inv)), -127.f), 127.f);
    hq = int8_t(h);
    lq = int8_t(l);
    s256 = warp_sum_i(int(hq) * 256 + int(lq));
  }
  tile[gi * 64 + lane] = uint8_t(hq);
  tile[gi * 64 + 32 + lane] = uint8_t(lq);
  if (lane == 0)
    *reinterpret_cast<float2 *>(tile + kGroupsPerTile * 64 + gi * 8) = make_float2(S, float(s256) * (1.0f / 256.0f));
}

// x (one value a lane, the group grp of a row of D) into the activation tiles of the next norm:
// the tiles hold x*w, and sq[grp] the group's sum of (x/scale)^2 (float squares, summed in double
// as milcpu's reduce_mean does, ops.go:861-920).
__device__ __forceinline__ void quant_norm32(float x, float w, float scale, uint8_t *act, double *sq,
                                             int grp, int lane) {
  const float xs = scale == 1.f ? x : x * (1.f / scale);
  double s = double(xs * xs);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) sq[grp] = s;
  quant32(x * w, act + size_t(grp / kGroupsPerTile) * kActTile, grp % kGroupsPerTile, lane);
}

// The factor a consumer applies to the group scales of a normed input: r / scale with
// r = float32(1 / sqrt(float64(mean) + eps16)) (milcpu rsqrt, ops.go:181-189). One warp; the
// group sums (written by other CTAs in this launch) are read past L1.
__device__ float norm_factor_warp(const double *sq, int groups, int n, float scale, float eps16, int lane) {
  double s = 0;
  for (int g = lane; g < groups; g += 32) s += __ldcg(sq + g);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float ms = float(s / double(n));
  const float r = float(1.0 / sqrt(double(ms) + double(eps16)));
  return r * (1.f / scale);
}

// Per-token norm factors into cf[t] (warp t does token t).
template <int NT>
__device__ __forceinline__ void norm_factors(float *cf, const double *sq, int groups, int n, float scale,
                                             float eps16) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < NT) {
    const float f = norm_factor_warp(sq + size_t(warp) * groups, groups, n, scale, eps16, lane);
    if (lane == 0) cf[warp] = f;
  }
}

// ---- the stage ring -----------------------------------------------------------------------------
constexpr int kStageBytes = 16384;  // one chunk: up to 8 column tiles of a row tile, or keys+values
constexpr int kKr = 8;              // column tiles of a weight chunk (one a consumer warp)
constexpr int kProducerWarp = kWarps;

__device__ __forceinline__ uint32_t saddr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b, unsigned count) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred P;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 P, [%1], %2;\n selp.u32 %0, 1, 0, P;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase of parity `parity` of b; false (and *status set) past the deadline or when
// another wait already failed.
__device__ bool mbar_wait(uint64_t *b, unsigned parity, const MkParams &p, int code) {
  if (mbar_try(b, parity)) return true;
  const long long t0 = clock64();
  long long next = t0 + kStatusPoll;
  for (;;) {
    if (mbar_try(b, parity)) return true;
    const long long now = clock64();
    if (now < next) continue;
    next = now + kStatusPoll;
    if (*reinterpret_cast<volatile int *>(p.status)) return false;
    if (now - t0 > p.spin_limit) {
      atomicCAS(p.status, 0, code);
      return false;
    }
  }
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}

struct Ring {
  uint8_t *stages;
  uint64_t *full, *empty;
  int S;
};

// A GEMV phase of a CTA: row tiles [rt0, rt0 + nrt) of a matrix of ktiles column tiles; chunk
// (i, kr), the (kr nrt + i)-th of the phase, holds column tiles [8 kr, 8 kr + 8) of row tile rt0 + i.
struct GemvPhase {
  const uint8_t *tiles;
  int ktiles, rt0, nrt, tb;
  __device__ int nkr() const { return (ktiles + kKr - 1) / kKr; }
  __device__ int chunks() const { return nrt * nkr(); }
};

// The cached keys of an attention unit: positions [k0, kc1) of (slot, kv head), in chunks of kc keys.
struct AttPhase {
  const uint16_t *kbase, *vbase;  // the (slot, kv head) rows of the layer's caches
  int k0, kc1, kc, hd;
  __device__ int chunks() const { return kc1 > k0 ? (kc1 - k0 + kc - 1) / kc : 0; }
};

template <int KIND>
__device__ __forceinline__ int tile_bytes_of() {
  return KIND == kKindInt8 ? kTileInt8 : (KIND == kKindInt4 ? kTileInt4 : kTileMx);
}

// The geometry of everything a CTA streams, in the order both sides walk it.
template <int KIND, int NT>
struct Schedule {
  const MkParams &p;
  __device__ GemvPhase qkv(int l) const {
    int u0, u1;
    my_units(p.rt_qkv, u0, u1);
    return GemvPhase{p.L[l].qkv, p.kt_d, u0, u1 - u0, tile_bytes_of<KIND>()};
  }
  __device__ GemvPhase o(int l) const {
    int u0, u1;
    my_units(p.D / 32, u0, u1);
    return GemvPhase{p.L[l].o, p.kt_o, 4 * u0, 4 * (u1 - u0), tile_bytes_of<KIND>()};
  }
  __device__ GemvPhase gu(int l) const {
    int u0, u1;
    my_units(p.F / 32, u0, u1);
    return GemvPhase{p.L[l].gu, p.kt_d, 8 * u0, 8 * (u1 - u0), tile_bytes_of<KIND>()};
  }
  __device__ GemvPhase down(int l) const {
    int u0, u1;
    my_units(p.D / 32, u0, u1);
    return GemvPhase{p.L[l].down, p.kt_f, 4 * u0, 4 * (u1 - u0), tile_bytes_of<KIND>()};
  }
  __device__ GemvPhase head() const {
    int u0, u1;
    my_units(p.rt_head, u0, u1);
    return GemvPhase{p.head, p.kt_d, u0, u1 - u0, tile_bytes_of<KIND>()};
  }
  __device__ void units(int &a0, int &a1) const { my_units(NT * p.KV * p.splits, a0, a1); }
  __device__ AttPhase att(int l, int u) const {
    const int t = u / (p.KV * p.splits), kvh = (u / p.splits) % p.KV, s = u % p.splits;
    const StepTok tk = p.toks[t];
    const int P = tk.pos;
    const MkLayer &L = p.L[l];
    const int lo = L.window > 0 ? max(0, P - L.window + 1) : 0;
    const int n = P - lo + 1;
    const int chunk = (n + p.splits - 1) / p.splits;
    const int k0 = lo + s * chunk, k1 = min(P + 1, k0 + chunk);
    const size_t base = (size_t(tk.slot) * p.KV + kvh) * size_t(p.cap) * p.hd;
    return AttPhase{L.kc + base, L.vc + base, k0, min(k1, P), kStageBytes / (4 * p.hd), p.hd};
  }
};

// Event k of ring chunk j of CTA 0 (profiled steps).
__device__ __forceinline__ void ctrace(const MkParams &p, int j, int k) {
  if (p.trace && blockIdx.x == 0 && j < kMkChunkTrace)
    p.trace[size_t(4) * (mk_phases(p.layers) + 1) * gridDim.x + size_t(j) * 4 + k] = global_ns();
}
// The consumer-side events: warp 0 saw chunk j full (k = 1) or is done with it (k = 2); warp 7 done (k = 3).
__device__ __forceinline__ void ctrace_c(const MkParams &p, int j, bool done) {
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0 && (warp == 0 || (done && warp == kWarps - 1)))
    ctrace(p, j, done ? (warp == 0 ? 2 : 3) : 1);
}

// Event k (0..7) of the attention unit of CTA 1 in layer li (profiled steps; clock cycles).
__device__ __forceinline__ void utrace(const MkParams &p, int li, int k) {
  if (p.trace && blockIdx.x == 1 && threadIdx.x == 0)
    p.trace[size_t(4) * (mk_phases(p.layers) + 1) * gridDim.x + size_t(4) * kMkChunkTrace + size_t(li) * 8 + k] =
        clock64();
}

// ---- the producer ---------------------------------------------------------------------------
// Cycles the producer spent waiting for free stages (trace runs only).
__device__ __forceinline__ bool produce_slot(const Ring &r, int j, const MkParams &p, long long &waited) {
  const int s = j % r.S;
  if (j < r.S) return true;
  const long long t0 = clock64();
  const bool ok = mbar_wait(&r.empty[s], ((j / r.S) + 1) & 1, p, 1000001);
  waited += clock64() - t0;
  return ok;
}

// Chunks in consume_gemv's order (kr-major), or consume_head's (imajor).
__device__ bool produce_gemv(const Ring &r, int &j, const GemvPhase &g, const MkParams &p, long long &waited,
                             bool imajor = false) {
  const int nkr = g.nkr();
  for (int c = 0; c < g.chunks(); ++c, ++j) {
    const int kr = imajor ? c % nkr : c / g.nrt, i = imajor ? c / nkr : c % g.nrt;
    if (!produce_slot(r, j, p, waited)) return false;
    const int s = j % r.S;
    const int nk = min(kKr, g.ktiles - kr * kKr);
    const unsigned bytes = unsigned(nk * g.tb);
    ctrace(p, j, 0);
    mbar_expect_tx(&r.full[s], bytes);
    bulk_g2s(r.stages + size_t(s) * kStageBytes, g.tiles + (size_t(g.rt0 + i) * g.ktiles + kr * kKr) * g.tb, bytes,
             &r.full[s]);
  }
  return true;
}

__device__ bool produce_att(const Ring &r, int &j, const AttPhase &a, const MkParams &p, long long &waited) {
  const int n = a.chunks();
  for (int c = 0; c < n; ++c, ++j) {
    if (!produce_slot(r, j, p, waited)) return false;
    const int s = j % r.S;
    const int key0 = a.k0 + c * a.kc, nkeys = min(a.kc, a.kc1 - key0);
    const unsigned bytes = unsigned(nkeys * a.hd * 2);
    ctrace(p, j, 0);
    mbar_expect_tx(&r.full[s], 2 * bytes);
    uint8_t *dst = r.stages + size_t(s) * kStageBytes;
    bulk_g2s(dst, a.kbase + size_t(key0) * a.hd, bytes, &r.full[s]);
    bulk_g2s(dst + bytes, a.vbase + size_t(key0) * a.hd, bytes, &r.full[s]);
  }
  return true;
}

template <int KIND, int NT>
__device__ __noinline__ void producer(const Ring r, const MkParams &p) {
  const Schedule<KIND, NT> sc{p};
  const long long t0 = clock64();
  long long waited = 0;
  int j = 0;
  bool ok = true;
  for (int l = 0; l < p.layers && ok; ++l) {
    ok = produce_gemv(r, j, sc.qkv(l), p, waited);
    int a0, a1;
    sc.units(a0, a1);
    for (int u = a0; u < a1 && ok; ++u) ok = produce_att(r, j, sc.att(l, u), p, waited);
    ok = ok && produce_gemv(r, j, sc.o(l), p, waited);
    ok = ok && produce_gemv(r, j, sc.gu(l), p, waited);
    ok = ok && produce_gemv(r, j, sc.down(l), p, waited);
  }
  if (ok) produce_gemv(r, j, sc.head(), p, waited, true);
  if (p.trace) {
    // after the phase planes: [ctas][4] producer waited, producer busy, consumer waited, consumer busy
    unsigned long long *st = p.trace + size_t(4) * mk_phases(p.layers) * gridDim.x + size_t(blockIdx.x) * 4;
    st[0] = waited;
    st[1] = clock64() - t0;
  }
}

// Cycles warp 0 of the consumers waited for stages (trace runs).
__shared__ long long s_cwait;

// The slow path of mbar_wait_warp (kept out of line so the chunk loops stay call-free).
__device__ __noinline__ bool mbar_wait_warp_slow(uint64_t *b, unsigned parity, const MkParams &p, int code) {
  const int lane = threadIdx.x & 31;
  const long long t0 = clock64();
  long long next = t0 + kStatusPoll;
  for (;;) {
    if (__all_sync(0xffffffffu, mbar_try(b, parity))) {
      if (threadIdx.x == 0) s_cwait += clock64() - t0;
      return true;
    }
    const long long now = __shfl_sync(0xffffffffu, clock64(), 0);
    if (now < next) continue;
    next = now + kStatusPoll;
    int bad = 0;
    if (lane == 0) {
      if (*reinterpret_cast<volatile int *>(p.status)) bad = 1;
      else if (now - t0 > p.spin_limit) { atomicCAS(p.status, 0, code); bad = 1; }
    }
    if (__shfl_sync(0xffffffffu, bad, 0)) return false;
  }
}

// mbar_wait for a whole warp: every lane leaves with the same answer (the MMAs that follow need
// the warp converged).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *b, unsigned parity, const MkParams &p, int code) {
  if (__all_sync(0xffffffffu, mbar_try(b, parity))) return true;
  return mbar_wait_warp_slow(b, parity, p, code);
}

// ---- the consumers ----------------------------------------------------------------------------
// Copies NT tokens' activation tiles (ktiles each) from global into smem (the 8 consumer warps).
template <int NT>
__device__ __forceinline__ void load_act(uint8_t *act_s, const uint8_t *act_g, int ktiles) {
  const int n16 = NT * ktiles * kActTile / 16;
  const uint4 *src = reinterpret_cast<const uint4 *>(act_g);
  uint4 *dst = reinterpret_cast<uint4 *>(act_s);
  for (int i = threadIdx.x; i < n16; i += kMkThreads) dst[i] = __ldcg(src + i);
}

// One column tile's B operands for one lane, read out of a stage so that the stage can be released
// before the MMAs run.
template <int KIND>
struct BTile {
  uint32_t w[KIND == kKindInt8 ? 16 : 8];
  uint32_t sz[2];
  __device__ __forceinline__ void load(const uint8_t *tile, int lane) {
    if (KIND == kKindInt8) {
      const uint4 *q = reinterpret_cast<const uint4 *>(tile + lane * 64);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4 v = q[u];
        w[4 * u] = v.x; w[4 * u + 1] = v.y; w[4 * u + 2] = v.z; w[4 * u + 3] = v.w;
      }
    } else {
      const uint4 *q = reinterpret_cast<const uint4 *>(tile + lane * 32);
      const uint4 v0 = q[0], v1 = q[1];
      w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w; w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
      if (KIND == kKindInt4) {
        const uint2 q2 = *reinterpret_cast<const uint2 *>(tile + kTileCodes4 + lane * 8);
        sz[0] = q2.x; sz[1] = q2.y;
      } else {
        sz[0] = *reinterpret_cast<const unsigned short *>(tile + kTileCodes4 + lane * 2);
        sz[1] = 0;
      }
    }
  }
};

// The A fragments of one token's activation tile for the 8 integer MMAs of a column tile: lane
// (g, c) feeds group c (g == c) or group g (g == c + 4) into A's rows, zeros elsewhere; and the
// scale S and sum Xq of the group g the lane's results belong to. hi16: the B codes of groups 4..7
// arrive multiplied by 16 (int4: w & 0xF0 instead of (w >> 4) & 0x0F), so those lanes carry S / 16
// and 16 Xq, which leaves every product exactly as it was (powers of two).
struct AFrag {
  uint32_t a[8][4];
  float S, Xq;
  __device__ __forceinline__ void load(const uint8_t *at, int lane, bool mx, bool hi16) {
    const int gq = lane >> 2, c = lane & 3;
    const bool role0 = gq == c, role1 = gq == c + 4;
    const int agrp = role0 ? c : gq;
    uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0, l0 = h0, l1 = h0;
    if (role0 || role1) {
      const uint4 *ap = reinterpret_cast<const uint4 *>(at + agrp * 64);
      h0 = ap[0]; h1 = ap[1];
      if (!mx) { l0 = ap[2]; l1 = ap[3]; }
    }
    const float2 sx = *reinterpret_cast<const float2 *>(at + kGroupsPerTile * 64 + gq * 8);
    S = sx.x;
    Xq = sx.y;
    if (hi16 && gq >= 4) {
      S *= 0.0625f;
      Xq *= 16.0f;
    }
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      a[u][0] = role0 ? hw[u] : 0u;
      a[u][1] = role0 ? lw[u] : 0u;
      a[u][2] = role1 ? hw[u] : 0u;
      a[u][3] = role1 ? lw[u] : 0u;
    }
  }
  // an inactive column tile: zero A and scales (its B is read from a valid tile, so every
  // product is an exact zero)
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int u = 0; u < 8; ++u) a[u][0] = a[u][1] = a[u][2] = a[u][3] = 0u;
    S = 0.f;
    Xq = 0.f;
  }
};

// The MMAs of one column tile (B read from the stage) with cached A fragments; returns lane
// (g, c)'s two rows' values for group g, scaled to float32.
template <int KIND>
__device__ __forceinline__ void tile_mma_cached(const uint8_t *tile, const AFrag &af, int lane, float &v0, float &v1) {
  BTile<KIND> bt;
  bt.load(tile, lane);
  uint32_t b0[8], b1[8];
  float s0 = 0.f, s1 = 0.f, z0 = 0.f, z1 = 0.f;
  if (KIND == kKindInt8) {
#pragma unroll
    for (int u = 0; u < 8; ++u) { b0[u] = bt.w[2 * u]; b1[u] = bt.w[2 * u + 1]; }
  } else if (KIND == kKindInt4) {
    const __half2 sh = *reinterpret_cast<const __half2 *>(&bt.sz[0]);
    const __half2 zh = *reinterpret_cast<const __half2 *>(&bt.sz[1]);
    s0 = __low2float(sh); s1 = __high2float(sh);
    z0 = __low2float(zh); z1 = __high2float(zh);
#pragma unroll
    for (int u = 0; u < 8; ++u) { b0[u] = bt.w[u] & 0x0F0F0F0Fu; b1[u] = bt.w[u] & 0xF0F0F0F0u; }
  } else {
    s0 = __uint_as_float((bt.sz[0] & 0xff) << 23);
    s1 = __uint_as_float(((bt.sz[0] >> 8) & 0xff) << 23);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const uint32_t wsh = bt.w[u] << 4;
      b0[u] = e2m1x4(bt.w[u], wsh, 0xD9C8u, bt.w[u] & 0x7777u);
      b1[u] = e2m1x4(bt.w[u], wsh, 0xFBEAu, (bt.w[u] >> 16) & 0x7777u);
    }
  }
  int d[4] = {0, 0, 0, 0}, e[4] = {0, 0, 0, 0};
#pragma unroll
  for (int u = 0; u < 8; u += 2) {
    if (KIND == kKindInt4) {
      mma_s8u8(d, af.a[u][0], af.a[u][1], af.a[u][2], af.a[u][3], b0[u], b1[u]);
      mma_s8u8(e, af.a[u + 1][0], af.a[u + 1][1], af.a[u + 1][2], af.a[u + 1][3], b0[u + 1], b1[u + 1]);
    } else {
      mma_s8s8(d, af.a[u][0], af.a[u][1], af.a[u][2], af.a[u][3], b0[u], b1[u]);
      mma_s8s8(e, af.a[u + 1][0], af.a[u + 1][1], af.a[u + 1][2], af.a[u + 1][3], b0[u + 1], b1[u + 1]);
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) d[q] += e[q];
  if (KIND == kKindMx) {
    v0 = float(d[0]) * s0 * af.S;
    v1 = float(d[1]) * s1 * af.S;
  } else {
    const float p0 = fmaf(float(d[2]), 1.0f / 256.0f, float(d[0]));
    const float p1 = fmaf(float(d[3]), 1.0f / 256.0f, float(d[1]));
    if (KIND == kKindInt4) {
      v0 = (s0 * af.S) * fmaf(-z0, af.Xq, p0);
      v1 = (s1 * af.S) * fmaf(-z1, af.Xq, p1);
    } else {
      v0 = af.S * p0;
      v1 = af.S * p1;
    }
  }
}

// Sums lane values over the 8 groups (lanes g = 0..7 of the same c).
__device__ __forceinline__ float group_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// GEMV work split: the 8 consumer warps are 2 teams of 4; team i % 2 takes row tile i, and in a
// chunk (8 column tiles of one row tile) warp q of the team takes column tiles 2q and 2q + 1, so
// each warp runs two independent MMA chains and one group reduction per row tile. A warp arrives
// on the chunk's "empty" barrier with count 2 (4 warps make the 8 the barrier counts).
constexpr int kTeamWarps = 4;

// A warp's pair of column tiles of one chunk for token t: the group-scaled values of its lane
// summed over the 8 groups (lanes (g, c), rows 2c and 2c + 1).
template <int KIND>
__device__ __forceinline__ void pair_mma(const uint8_t *stage, int q4, bool act1, const AFrag &f0, const AFrag &f1,
                                         int lane, float &v0, float &v1) {
  constexpr int TB = KIND == kKindInt8 ? kTileInt8 : (KIND == kKindInt4 ? kTileInt4 : kTileMx);
  const uint8_t *t0 = stage + size_t(2 * q4) * TB;
  const uint8_t *t1 = act1 ? t0 + TB : t0;  // an inactive second tile reads the first (f1 is zero)
  float x0, x1, y0, y1;
  tile_mma_cached<KIND>(t0, f0, lane, x0, x1);
  tile_mma_cached<KIND>(t1, f1, lane, y0, y1);
  v0 = group_sum(x0 + y0);
  v1 = group_sum(x1 + y1);
}

// The column-tile pair (kt0, kt0 + 1) of a warp for token t: fragments from act_s (zero when out of
// range).
template <int KIND>
__device__ __forceinline__ void load_pair(AFrag &f0, AFrag &f1, const uint8_t *act_s, int ktiles, int t, int kt0,
                                          int lane) {
  if (kt0 < ktiles) f0.load(act_s + (size_t(t) * ktiles + kt0) * kActTile, lane, KIND == kKindMx, KIND == kKindInt4);
  else f0.zero();
  if (kt0 + 1 < ktiles) f1.load(act_s + (size_t(t) * ktiles + kt0 + 1) * kActTile, lane, KIND == kKindMx, KIND == kKindInt4);
  else f1.zero();
}

// The chunks of a GEMV phase (kr-major: chunk (i, kr) is the (kr nrt + i)-th), split as above. The
// warp's fragments are built once per kr for a single token and per chunk otherwise. Warp q of
// the team that has row tile i leaves its partial in part[q][i][t][8] (stored at kr = 0, added
// to after); row_value() adds the 4 in order, so results do not depend on timing. Returns the
// ring position after the phase.
template <int KIND, int NT>
__device__ __noinline__ int consume_gemv(const Ring r, int j, const GemvPhase g, const uint8_t *act_s, const MkParams &p,
                                         float *part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int team = warp / kTeamWarps, q4 = warp % kTeamWarps;
  const int c = lane & 3;
  const int nkr = g.nkr();
  bool good = true;
  for (int kr = 0; kr < nkr; ++kr) {
    const int kt0 = kr * kKr + 2 * q4;
    const bool any = kt0 < g.ktiles, act1 = kt0 + 1 < g.ktiles;
    AFrag f0, f1;
    if (NT == 1) load_pair<KIND>(f0, f1, act_s, g.ktiles, 0, kt0, lane);
    for (int i = team; i < g.nrt; i += 2) {
      const int jj = j + kr * g.nrt + i, s = jj % r.S;
      if (good && !mbar_wait_warp(&r.full[s], (jj / r.S) & 1, p, 1000002)) good = false;
      if (!good) continue;
      ctrace_c(p, jj, false);
      float *pw = part + (size_t(q4) * g.nrt + i) * NT * 8;
      const uint8_t *stage = r.stages + size_t(s) * kStageBytes;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float v0 = 0.f, v1 = 0.f;
        if (any) {
          if (NT > 1) load_pair<KIND>(f0, f1, act_s, g.ktiles, t, kt0, lane);
          pair_mma<KIND>(stage, q4, act1, f0, f1, lane, v0, v1);
        }
        if (lane < 4) {
          if (kr == 0) {
            pw[t * 8 + 2 * c] = v0;
            pw[t * 8 + 2 * c + 1] = v1;
          } else {
            pw[t * 8 + 2 * c] += v0;
            pw[t * 8 + 2 * c + 1] += v1;
          }
        }
      }
      ctrace_c(p, jj, true);
      __syncwarp();
      if (lane == 0) mbar_arrive(&r.empty[s], 2);
    }
  }
  (void)good;
  return j + g.chunks();
}

// The value of row r8 of local row tile i for token t: the 4 warps' partials in order.
template <int NT>
__device__ __forceinline__ float row_value(const float *part, int nrt, int i, int t, int r8) {
  float v = 0.f;
#pragma unroll
  for (int q = 0; q < kTeamWarps; ++q) v += part[((size_t(q) * nrt + i) * NT + t) * 8 + r8];
  return v;
}

// The head (i-major: chunk (i, kr) is the (i nkr + kr)-th): split as consume_gemv, into kHeadSlots
// partial slots used round robin; the last of the team's 4 warps to finish row tile i (a shared
// counter) adds the partials in order, writes the fp16 logits and folds them into bmax[t]. Slot
// reuse is safe: no warp runs more than `stages` (<= 16) chunks ahead of the slowest, which
// releases a row tile's last chunk only after that row tile's epilogue.
constexpr int kHeadSlots = 32;
template <int KIND, int NT>
__device__ __noinline__ int consume_head(const Ring r, int j, const GemvPhase g, const uint8_t *act_s, const MkParams &p,
                                         float *part, unsigned *cnt, const float *cf, unsigned long long *bmax) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int team = warp / kTeamWarps, q4 = warp % kTeamWarps;
  const int c = lane & 3;
  const int nkr = g.nkr();
  bool good = true;
  AFrag f0, f1;
  if (nkr == 1 && NT == 1) load_pair<KIND>(f0, f1, act_s, g.ktiles, 0, 2 * q4, lane);
  for (int i = team; i < g.nrt && good; i += 2) {
    const int slot = i % kHeadSlots;
    float *pw = part + (size_t(q4) * kHeadSlots + slot) * NT * 8;
    for (int kr = 0; kr < nkr; ++kr) {
      const int jj = j + i * nkr + kr, s = jj % r.S;
      if (!mbar_wait_warp(&r.full[s], (jj / r.S) & 1, p, 1000004)) { good = false; break; }
      ctrace_c(p, jj, false);
      const int kt0 = kr * kKr + 2 * q4;
      const bool any = kt0 < g.ktiles, act1 = kt0 + 1 < g.ktiles;
      const uint8_t *stage = r.stages + size_t(s) * kStageBytes;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float v0 = 0.f, v1 = 0.f;
        if (any) {
          if (nkr != 1 || NT != 1) load_pair<KIND>(f0, f1, act_s, g.ktiles, t, kt0, lane);
          pair_mma<KIND>(stage, q4, act1, f0, f1, lane, v0, v1);
        }
        if (lane < 4) {
          if (kr == 0) {
            pw[t * 8 + 2 * c] = v0;
            pw[t * 8 + 2 * c + 1] = v1;
          } else {
            pw[t * 8 + 2 * c] += v0;
            pw[t * 8 + 2 * c + 1] += v1;
          }
        }
      }
      if (kr + 1 == nkr) {
        // count this warp in; the team's last adds the partials up
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) {
          __threadfence_block();
          last = atomicAdd(&cnt[slot], 1u) == unsigned(kTeamWarps - 1);
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence_block();
          const int row0 = (g.rt0 + i) * 8;
          for (int q = lane; q < NT * 8; q += 32) {
            const int t = q / 8, row = row0 + q % 8;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kTeamWarps; ++w)
              v += *reinterpret_cast<volatile float *>(part + (size_t(w) * kHeadSlots + slot) * NT * 8 + q);
            v *= cf[t];
            if (p.head_scale) v *= p.head_scale[row];
            const uint16_t hb = __half_as_ushort(__float2half_rn(v));
            if (row < p.V) {
              if (p.logits) p.logits[size_t(t) * p.V + row] = hb;
              atomicMax(&bmax[t], argmax_key(hb, row));
            }
          }
          if (lane == 0) cnt[slot] = 0u;
        }
      }
      ctrace_c(p, jj, true);
      __syncwarp();
      if (lane == 0) mbar_arrive(&r.empty[s], 2);
    }
  }
  (void)good;
  return j + g.chunks();
}

// The attention of one (token, kv head, split) unit (all 8 warps): q/k norms and RoPE of the heads it
// needs (one warp a head; the new key and value of position P in float32, as the reference's step
// rows are, written to the cache as fp16 by the unit that holds P), then an online softmax over its
// cached keys, which arrive from the ring in chunks, by 32 groups of 8 lanes; partials out, and
// the last split of (token, kv head) to arrive merges them (with the sink) and quantises the
// heads' outputs for the o projection. Returns false when a wait gave up.
template <int HD, int REP>
__device__ __noinline__ int attention_unit(const Ring r, int j, const AttPhase a, const MkParams &p, const MkLayer &L, int t,
                               int kvh, int s, uint8_t *scratch, uint8_t *act_next) {
  constexpr int E = HD / 8;
  float *qs = reinterpret_cast<float *>(scratch);  // [REP][HD]
  float *kn = qs + REP * HD;                         // [HD]
  float *vn = kn + HD;                               // [HD]
  float *wm = vn + HD;                               // [8][REP]
  float *wl = wm + kWarps * REP;                     // [8][REP]
  float *wo = wl + kWarps * REP;                     // [8][REP][HD]
  int *flag = reinterpret_cast<int *>(wo + kWarps * REP * HD);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = threadIdx.x >> 3, l8 = threadIdx.x & 7;
  const int li = int(&L - p.L);
  utrace(p, li, 0);
  const StepTok tk = p.toks[t];
  const int P = tk.pos;
  const int lo = L.window > 0 ? max(0, P - L.window + 1) : 0;
  const int n = P - lo + 1;
  const int chunk = (n + p.splits - 1) / p.splits;
  const int k0 = lo + s * chunk, k1 = min(P + 1, k0 + chunk);
  const bool has_new = k0 <= P && P < k1;
  const int W = (p.H + 2 * p.KV) * HD;
  const float *row = p.qkv + size_t(t) * W;
  const size_t base = (size_t(tk.slot) * p.KV + kvh) * size_t(p.cap) * HD;
  for (int task = warp; task < REP + 1; task += kWarps) {
    const bool is_q = task < REP;
    if (!is_q && !has_new) continue;
    const float *src = is_q ? row + size_t(kvh * REP + task) * HD : row + size_t(p.H + kvh) * HD;
    const float *nw = is_q ? L.q_norm : L.k_norm;
    constexpr int E2 = HD / 32;
    float x[E2];
#pragma unroll
    for (int k = 0; k < E2; ++k) x[k] = __ldcg(src + lane + 32 * k);
    if (nw) {
      const float inv = p.sc == 1.f ? 1.f : 1.f / p.sc;
      double ss = 0;
#pragma unroll
      for (int k = 0; k < E2; ++k) {
        x[k] = p.sc == 1.f ? x[k] : __fmul_rn(x[k], inv);
        ss += double(__fmul_rn(x[k], x[k]));
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float ms = float(ss / double(HD));
      const float rr = float(1.0 / sqrt(double(ms) + double(p.eps)));
#pragma unroll
      for (int k = 0; k < E2; ++k) x[k] = __fmul_rn(__fmul_rn(x[k], rr), nw[lane + 32 * k]);
    }
    const uint32_t *rt = p.rope + size_t(P) * (HD / 2);
    float y[E2];
#pragma unroll
    for (int k = 0; k < E2; ++k) {
      const int e = lane + 32 * k;
      const int jr = e < HD / 2 ? e : e - HD / 2;
      const uint32_t cs = rt[jr];
      const float cv = __half2float(__ushort_as_half(uint16_t(cs & 0xffff)));
      const float sv = __half2float(__ushort_as_half(uint16_t(cs >> 16)));
      const int kp = e < HD / 2 ? k + (HD / 64) : k - (HD / 64);
      const float rot = e < HD / 2 ? -x[kp] : x[kp];
      y[k] = __fadd_rn(__fmul_rn(x[k], cv), __fmul_rn(rot, sv));
    }
    if (is_q) {
#pragma unroll
      for (int k = 0; k < E2; ++k) qs[task * HD + lane + 32 * k] = y[k];
    } else {
      const float *vsrc = row + size_t(p.H + p.KV + kvh) * HD;
#pragma unroll
      for (int k = 0; k < E2; ++k) {
        const int e = lane + 32 * k;
        const float v = __ldcg(vsrc + e);
        kn[e] = y[k];
        vn[e] = v;
        L.kc[base + size_t(P) * HD + e] = __half_as_ushort(__float2half_rn(y[k]));
        L.vc[base + size_t(P) * HD + e] = __half_as_ushort(__float2half_rn(v));
      }
    }
  }
  csync();
  utrace(p, li, 1);
  float qv[REP][E], m[REP], l[REP], o[REP][E];
#pragma unroll
  for (int rr = 0; rr < REP; ++rr) {
    m[rr] = -INFINITY;
    l[rr] = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) { qv[rr][k] = qs[rr * HD + l8 * E + k]; o[rr][k] = 0.f; }
  }
  // one step of the online softmax with key kf and value vf, when valid (the shuffles take the
  // whole warp)
  auto step = [&](const float *kf, const float *vf, bool valid) {
#pragma unroll
    for (int rr = 0; rr < REP; ++rr) {
      float d = 0.f;
#pragma unroll
      for (int k = 0; k < E; ++k) d = fmaf(qv[rr][k], kf[k], d);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      if (valid) {
        const float sc = d * p.score_scale;
        const float mn = fmaxf(m[rr], sc);
        const float corr = expf(m[rr] - mn), pr = expf(sc - mn);
        l[rr] = fmaf(l[rr], corr, pr);
#pragma unroll
        for (int k = 0; k < E; ++k) o[rr][k] = fmaf(o[rr][k], corr, pr * vf[k]);
        m[rr] = mn;
      }
    }
  };
  bool good = true;
  const int nch = a.chunks();
  for (int c = 0; c < nch; ++c) {
    const int jj = j + c, st = jj % r.S;
    if (!mbar_wait_warp(&r.full[st], (jj / r.S) & 1, p, 1000003)) { good = false; break; }
    ctrace_c(p, jj, false);
    const uint8_t *stage = r.stages + size_t(st) * kStageBytes;
    const int key0 = a.k0 + c * a.kc, nkeys = min(a.kc, a.kc1 - key0);
    const uint16_t *ks = reinterpret_cast<const uint16_t *>(stage);
    const uint16_t *vs = ks + size_t(nkeys) * HD;
    for (int m0 = 0; m0 < nkeys; m0 += kMkThreads / 8) {
      const int kk = m0 + grp;
      const bool valid = kk < nkeys;
      float kf[E], vf[E];
#pragma unroll
      for (int u = 0; u < E / 8; ++u) {
        uint4 kw4 = make_uint4(0, 0, 0, 0), vw4 = kw4;
        if (valid) {
          kw4 = reinterpret_cast<const uint4 *>(ks + size_t(kk) * HD + l8 * E)[u];
          vw4 = reinterpret_cast<const uint4 *>(vs + size_t(kk) * HD + l8 * E)[u];
        }
        const uint32_t kw[4] = {kw4.x, kw4.y, kw4.z, kw4.w}, vw[4] = {vw4.x, vw4.y, vw4.z, vw4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __half2 k2 = *reinterpret_cast<const __half2 *>(&kw[i]);
          const __half2 v2 = *reinterpret_cast<const __half2 *>(&vw[i]);
          kf[8 * u + 2 * i] = __low2float(k2); kf[8 * u + 2 * i + 1] = __high2float(k2);
          vf[8 * u + 2 * i] = __low2float(v2); vf[8 * u + 2 * i + 1] = __high2float(v2);
        }
      }
      step(kf, vf, valid);
    }
    ctrace_c(p, jj, true);
    __syncwarp();
    if (lane == 0) mbar_arrive(&r.empty[st], 1);
  }
  j += nch;  // the value returned
  utrace(p, li, 2);
  if (has_new) {
    float kf[E], vf[E];
#pragma unroll
    for (int k = 0; k < E; ++k) { kf[k] = kn[l8 * E + k]; vf[k] = vn[l8 * E + k]; }
    step(kf, vf, grp == 0);
  }
  // the 4 groups of a warp, then the 8 warps
#pragma unroll
  for (int rr = 0; rr < REP; ++rr) {
    float M = fmaxf(m[rr], __shfl_xor_sync(0xffffffffu, m[rr], 8));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
    const float f = l[rr] > 0.f ? expf(m[rr] - M) : 0.f;
    float Ls = l[rr] * f;
    Ls += __shfl_xor_sync(0xffffffffu, Ls, 8);
    Ls += __shfl_xor_sync(0xffffffffu, Ls, 16);
#pragma unroll
    for (int k = 0; k < E; ++k) {
      float v = o[rr][k] * f;
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (lane < 8) wo[(warp * REP + rr) * HD + l8 * E + k] = v;
    }
    if (lane == 0) { wm[warp * REP + rr] = M; wl[warp * REP + rr] = Ls; }
  }
  csync();
  utrace(p, li, 3);
  for (int idx = threadIdx.x; idx < REP * HD; idx += kMkThreads) {
    const int rr = idx / HD, e = idx % HD;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w)
      if (wl[w * REP + rr] > 0.f) M = fmaxf(M, wm[w * REP + rr]);
    float Ls = 0.f, acc = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float f = wl[w * REP + rr] > 0.f ? expf(wm[w * REP + rr] - M) : 0.f;
      Ls += wl[w * REP + rr] * f;
      acc = fmaf(wo[(w * REP + rr) * HD + e], f, acc);
    }
    const size_t pi = (size_t(t) * p.H + kvh * REP + rr) * p.splits + s;
    if (e == 0) { p.part_ml[pi * 2] = M; p.part_ml[pi * 2 + 1] = Ls; }
    p.part_o[pi * HD + e] = acc;
  }
  __threadfence();
  csync();
  utrace(p, li, 4);
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(&p.cnt[t * p.KV + kvh], 1u);
    *flag = old == unsigned(p.splits - 1);
  }
  csync();
  utrace(p, li, 5);
  if (!*flag) return j;
  __threadfence();
  float *wsp = wo;               // [REP][64] split weights
  float *invl = wsp + REP * 64;  // [REP]
  float *ov = invl + REP;        // [REP][HD]
  if (warp < REP) {
    const int rr = warp, h = kvh * REP + rr;
    const float *ml = p.part_ml + (size_t(t) * p.H + h) * p.splits * 2;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    if (lane < p.splits) { m0 = __ldcg(ml + 2 * lane); l0 = __ldcg(ml + 2 * lane + 1); }
    if (lane + 32 < p.splits) { m1 = __ldcg(ml + 2 * (lane + 32)); l1 = __ldcg(ml + 2 * (lane + 32) + 1); }
    float M = L.sinks ? L.sinks[h] : -INFINITY;
    M = fmaxf(M, l0 > 0.f ? m0 : -INFINITY);
    M = fmaxf(M, l1 > 0.f ? m1 : -INFINITY);
    M = warp_max(M);
    const float w0 = l0 > 0.f ? expf(m0 - M) : 0.f, w1 = l1 > 0.f ? expf(m1 - M) : 0.f;
    float Ls = warp_sum(l0 * w0 + l1 * w1);
    if (L.sinks) Ls += expf(L.sinks[h] - M);
    if (lane < p.splits) wsp[rr * 64 + lane] = w0;
    if (lane + 32 < p.splits) wsp[rr * 64 + lane + 32] = w1;
    if (lane == 0) invl[rr] = Ls > 0.f ? 1.f / Ls : 0.f;
  }
  csync();
  for (int idx = threadIdx.x; idx < REP * HD; idx += kMkThreads) {
    const int rr = idx / HD, e = idx % HD, h = kvh * REP + rr;
    const float *po = p.part_o + (size_t(t) * p.H + h) * p.splits * HD + e;
    float acc = 0.f;
    for (int sp = 0; sp < p.splits; ++sp) acc = fmaf(__ldcg(po + size_t(sp) * HD), wsp[rr * 64 + sp], acc);
    ov[idx] = acc * invl[rr];
  }
  csync();
  utrace(p, li, 6);
  uint8_t *at = act_next + size_t(t) * p.kt_o * kActTile;
  for (int gq = warp; gq < REP * HD / 32; gq += kWarps) {
    const int grp32 = (kvh * REP * HD) / 32 + gq;
    quant32(ov[gq * 32 + lane], at + size_t(grp32 / kGroupsPerTile) * kActTile, grp32 % kGroupsPerTile, lane);
  }
  if (threadIdx.x == 0) p.cnt[t * p.KV + kvh] = 0u;
  utrace(p, li, 7);
  (void)good;
  return j;
}

template <int KIND, int NT, int HD, int REP>
__global__ void __launch_bounds__(kMkBlock, 1) mk_kernel(const __grid_constant__ MkParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ float cfac[kMkMaxTok];
  __shared__ unsigned long long bmax[kMkMaxTok];
  __shared__ unsigned hcnt[kHeadSlots];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Ring r;
  r.S = p.stages;
  r.stages = smem;
  r.full = reinterpret_cast<uint64_t *>(smem + p.off_bar);
  r.empty = r.full + p.stages;
  uint8_t *act_s = smem + p.off_act;
  float *rows_s = reinterpret_cast<float *>(smem + p.off_rows);
  uint8_t *att_s = smem + p.off_att;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&r.full[s], 1);
      mbar_init(&r.empty[s], kWarps);  // released by arrivals adding up to 8: 1 a warp (attention), 2 a warp of a team (GEMV)
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == kProducerWarp) {
    if (lane == 0) producer<KIND, NT>(r, p);
    return;
  }
  // ---------------- consumers: threads 0..255 ----------------
  const long long c_t0 = clock64();
  if (threadIdx.x == 0) s_cwait = 0;
  unsigned epoch = 0;
  const int Gd = p.D / 32, Gf = p.F / 32;
  const int W = (p.H + 2 * p.KV) * HD;
  const Schedule<KIND, NT> sc{p};
  int j = 0;  // ring position
  int cur = 0;
  // ---- embed: x and its quantised form for layer 0's input norm
  {
    int u0, u1;
    my_units(NT * Gd, u0, u1);
    for (int u = u0 + warp; u < u1; u += kWarps) {
      const int t = u / Gd, gq = u % Gd, col = gq * 32 + lane;
      const int tok = p.toks[t].token;
      float v;
      if (p.embed) {
        v = __half2float(__ushort_as_half(p.embed[size_t(tok) * p.D + col]));
      } else {
        v = tile_value(p.head, p.head_scale, KIND, p.kt_d, tile_bytes_of<KIND>(), tok, col);
        v = __half2float(__float2half_rn(v));
      }
      p.x[size_t(t) * p.D + col] = v;
      quant_norm32(v, p.in_norm0[col], p.sc_in0, p.act[cur] + size_t(t) * p.kt_d * kActTile,
                   p.sq + size_t(t) * Gd, gq, lane);
    }
  }
  if (!grid_sync(p, epoch)) return;
  for (int li = 0; li < p.layers; ++li) {
    const MkLayer &L = p.L[li];
    // ---- qkv
    {
      load_act<NT>(act_s, p.act[cur], p.kt_d);
      norm_factors<NT>(cfac, p.sq, Gd, p.D, li == 0 ? p.sc_in0 : p.sc, li == 0 ? p.eps_in0 : p.eps);
      csync();
      mark(p, epoch, 0);
      const GemvPhase g = sc.qkv(li);
      j = consume_gemv<KIND, NT>(r, j, g, act_s, p, rows_s);
      csync();
      mark(p, epoch, 1);
      for (int idx = threadIdx.x; idx < g.nrt * 8 * NT; idx += kMkThreads) {
        const int t = idx % NT, rr = idx / NT, i = rr / 8, r8 = rr % 8, row = (g.rt0 + i) * 8 + r8;
        if (row >= W) continue;
        float v = row_value<NT>(rows_s, g.nrt, i, t, r8) * cfac[t];
        if (L.qkv_scale) v *= L.qkv_scale[row];
        if (L.qkv_bias) v += L.qkv_bias[row];
        p.qkv[size_t(t) * W + row] = v;
      }
    }
    if (!grid_sync(p, epoch)) return;
    // ---- attention
    {
      int a0, a1;
      sc.units(a0, a1);
      mark(p, epoch, 0);
      for (int u = a0; u < a1; ++u) {
        const int t = u / (p.KV * p.splits), kvh = (u / p.splits) % p.KV, s = u % p.splits;
        j = attention_unit<HD, REP>(r, j, sc.att(li, u), p, L, t, kvh, s, att_s, p.act[cur ^ 1]);
        csync();
      }
      mark(p, epoch, 1);
    }
    if (!grid_sync(p, epoch)) return;
    cur ^= 1;
    // ---- o projection + residual, quantised for the post-attention norm
    {
      load_act<NT>(act_s, p.act[cur], p.kt_o);
      csync();
      mark(p, epoch, 0);
      const GemvPhase g = sc.o(li);
      j = consume_gemv<KIND, NT>(r, j, g, act_s, p, rows_s);
      csync();
      mark(p, epoch, 1);
      const int u0 = g.rt0 / 4, nu = g.nrt / 4;
      for (int wu = warp; wu < nu * NT; wu += kWarps) {
        const int ul = wu / NT, t = wu % NT, row = (u0 + ul) * 32 + lane;
        float v = row_value<NT>(rows_s, g.nrt, ul * 4 + lane / 8, t, lane % 8);
        if (L.o_scale) v *= L.o_scale[row];
        if (L.o_bias) v += L.o_bias[row];
        float *xp = p.x + size_t(t) * p.D + row;
        const float xn = __ldcg(xp) + v;
        *xp = xn;
        quant_norm32(xn, L.post_norm[row], p.sc, p.act[cur ^ 1] + size_t(t) * p.kt_d * kActTile,
                     p.sq + size_t(t) * Gd, u0 + ul, lane);
      }
    }
    if (!grid_sync(p, epoch)) return;
    cur ^= 1;
    // ---- gate/up + SiLU, quantised for down
    {
      load_act<NT>(act_s, p.act[cur], p.kt_d);
      norm_factors<NT>(cfac, p.sq, Gd, p.D, p.sc, p.eps);
      csync();
      mark(p, epoch, 0);
      const GemvPhase g = sc.gu(li);
      j = consume_gemv<KIND, NT>(r, j, g, act_s, p, rows_s);
      csync();
      mark(p, epoch, 1);
      const int u0 = g.rt0 / 8, nu = g.nrt / 8;
      for (int wu = warp; wu < nu * NT; wu += kWarps) {
        const int ul = wu / NT, t = wu % NT;
        const int rtl = ul * 8 + lane / 4, r8 = lane % 4;
        const int grow = (g.rt0 + rtl) * 8 + r8, urow = grow + 4;
        float gv = row_value<NT>(rows_s, g.nrt, rtl, t, r8) * cfac[t];
        float uv = row_value<NT>(rows_s, g.nrt, rtl, t, r8 + 4) * cfac[t];
        if (L.gu_scale) { gv *= L.gu_scale[grow]; uv *= L.gu_scale[urow]; }
        // blocks.SiLU: x / (1 + exp(-x)) (internal/llm/blocks/blocks.go:395-399)
        const float hv = gv / (1.0f + expf(-gv)) * uv;
        const int gq = u0 + ul;
        quant32(hv, p.act[cur ^ 1] + (size_t(t) * p.kt_f + gq / kGroupsPerTile) * kActTile, gq % kGroupsPerTile, lane);
      }
    }
    if (!grid_sync(p, epoch)) return;
    cur ^= 1;
    // ---- down + residual, quantised for the next norm
    {
      load_act<NT>(act_s, p.act[cur], p.kt_f);
      csync();
      mark(p, epoch, 0);
      const GemvPhase g = sc.down(li);
      j = consume_gemv<KIND, NT>(r, j, g, act_s, p, rows_s);
      csync();
      mark(p, epoch, 1);
      const int u0 = g.rt0 / 4, nu = g.nrt / 4;
      for (int wu = warp; wu < nu * NT; wu += kWarps) {
        const int ul = wu / NT, t = wu % NT, row = (u0 + ul) * 32 + lane;
        float v = row_value<NT>(rows_s, g.nrt, ul * 4 + lane / 8, t, lane % 8);
        if (L.down_scale) v *= L.down_scale[row];
        float *xp = p.x + size_t(t) * p.D + row;
        const float xn = __ldcg(xp) + v;
        *xp = xn;
        quant_norm32(xn, L.next_norm[row], p.sc, p.act[cur ^ 1] + size_t(t) * p.kt_d * kActTile,
                     p.sq + size_t(t) * Gd, u0 + ul, lane);
      }
    }
    if (!grid_sync(p, epoch)) return;
    cur ^= 1;
  }
  // ---- head: fp16 logits and the greedy choice (chat/sample.go:80-88)
  {
    load_act<NT>(act_s, p.act[cur], p.kt_d);
    norm_factors<NT>(cfac, p.sq, Gd, p.D, p.sc, p.eps);
    if (threadIdx.x < NT) bmax[threadIdx.x] = 0ull;
    if (threadIdx.x < kHeadSlots) hcnt[threadIdx.x] = 0u;
    csync();
    mark(p, epoch, 0);
    j = consume_head<KIND, NT>(r, j, sc.head(), act_s, p, rows_s, hcnt, cfac, bmax);
    csync();
    mark(p, epoch, 1);
    if (threadIdx.x < NT)
      atomicMax(&p.amax[threadIdx.x * kAmaxSlots + (blockIdx.x % kAmaxSlots)], bmax[threadIdx.x]);
  }
  if (!grid_sync(p, epoch)) return;
  if (p.trace && threadIdx.x == 0) {
    unsigned long long *st = p.trace + size_t(4) * mk_phases(p.layers) * gridDim.x + size_t(blockIdx.x) * 4;
    st[2] = s_cwait;
    st[3] = clock64() - c_t0;
  }
  if (blockIdx.x == 0 && warp == 0) {
    for (int t = 0; t < NT; ++t) {
      unsigned long long k = 0;
      for (int i = lane; i < kAmaxSlots; i += 32) {
        k = max(k, __ldcg(p.amax + t * kAmaxSlots + i));
        p.amax[t * kAmaxSlots + i] = 0ull;  // ready for the next step
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
      if (lane == 0) {
        const int32_t am = int32_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
        p.am[t] = am;
        if (p.gen_out && t == 0) {
          const int i = *p.gen_count;
          p.gen_out[i] = am;
          p.toks[0].token = am;
          p.toks[0].pos += 1;
          *p.gen_count = i + 1;
        }
      }
    }
  }
}

template <int KIND, int NT, int HD, int REP>
cudaError_t launch_t(const MkParams &p, int ctas, size_t smem, cudaStream_t st) {
  auto k = mk_kernel<KIND, NT, HD, REP>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kMkBlock);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, p);
}

template <int KIND, int NT, int HD, int REP>
cudaError_t prepare_t(size_t smem) {
  return cudaFuncSetAttribute(mk_kernel<KIND, NT, HD, REP>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
}

}  // namespace

// Lays out the dynamic shared memory (stages, activations, unit rows, attention scratch, mbarriers)
// and fills p.stages and the offsets; returns the bytes, 0 when it does not fit.
size_t mk_layout(MkParams &p, int ctas) {
  const size_t limit = 225 * 1024;
  const int ktmax = std::max(p.kt_d, std::max(p.kt_f, p.kt_o));
  auto per = [&](int U) { return (U + ctas - 1) / ctas; };
  const int unit_rows = std::max({4 * per(p.D / 32), 8 * per(p.F / 32), per(p.rt_qkv), kHeadSlots});
  const int rep = p.H / p.KV;
  const size_t act = size_t(p.ntok) * ktmax * kActTile;
  const size_t rows = size_t(kTeamWarps) * unit_rows * p.ntok * 8 * 4;
  const size_t att = size_t(rep * p.hd + 2 * p.hd + 2 * kWarps * rep + kWarps * rep * p.hd) * 4 + 16;
  auto al = [](size_t x) { return (x + 127) / 128 * 128; };
  const size_t rest = al(act) + al(rows) + al(att);
  if (rest + 2 * kStageBytes + 64 > limit) return 0;
  int S = int((limit - rest - 16 * 32) / kStageBytes);
  S = std::min(S, 16);
  p.stages = S;
  size_t off = size_t(S) * kStageBytes;
  p.off_act = int(off);
  off += al(act);
  p.off_rows = int(off);
  off += al(rows);
  p.off_att = int(off);
  off += al(att);
  p.off_bar = int(off);
  off += size_t(2) * S * 8;
  return off;
}

size_t mk_smem(const MkParams &p, int ctas) {
  MkParams q = p;
  return mk_layout(q, ctas);
}

cudaError_t mk_prepare(size_t smem) {
  cudaError_t e = cudaSuccess;
#define HC_MK(KD, NTV, HDV, R) \
  if (e == cudaSuccess) e = prepare_t<KD, NTV, HDV, R>(smem);
#define HC_MK_NT(KD, HDV, R) HC_MK(KD, 1, HDV, R) HC_MK(KD, 2, HDV, R) HC_MK(KD, 4, HDV, R) HC_MK(KD, 8, HDV, R)
  HC_MK_NT(kKindInt4, 128, 2)
  HC_MK_NT(kKindInt8, 64, 4)
  HC_MK_NT(kKindInt8, 128, 2)
  HC_MK_NT(kKindInt4, 64, 4)
  HC_MK_NT(kKindInt4, 64, 2)
  HC_MK_NT(kKindInt8, 64, 2)
#undef HC_MK_NT
#undef HC_MK
  return e;
}

cudaError_t mk_launch(const MkParams &p0, int ctas, cudaStream_t st) {
  MkParams p = p0;
  const size_t smem = mk_layout(p, ctas);
  if (!smem) return cudaErrorInvalidConfiguration;
  const int rep = p.H / p.KV;
#define HC_MK(KD, NTV, HDV, R)                                                               \
  if (p.kind == KD && p.ntok == NTV && p.hd == HDV && rep == R)                              \
    return launch_t<KD, NTV, HDV, R>(p, ctas, smem, st);
#define HC_MK_NT(KD, HDV, R) HC_MK(KD, 1, HDV, R) HC_MK(KD, 2, HDV, R) HC_MK(KD, 4, HDV, R) HC_MK(KD, 8, HDV, R)
  HC_MK_NT(kKindInt4, 128, 2)
  HC_MK_NT(kKindInt8, 64, 4)
  HC_MK_NT(kKindInt8, 128, 2)
  HC_MK_NT(kKindInt4, 64, 4)
  HC_MK_NT(kKindInt4, 64, 2)
  HC_MK_NT(kKindInt8, 64, 2)
#undef HC_MK_NT
#undef HC_MK
  return cudaErrorNotSupported;
}

bool mk_supported(int kind, int ntok, int hd, int rep) {
  const bool nt = ntok == 1 || ntok == 2 || ntok == 4 || ntok == 8;
  if (!nt || (kind != kKindInt4 && kind != kKindInt8)) return false;
  return (hd == 128 && rep == 2) || (hd == 64 && (rep == 2 || rep == 4));
}

int mk_max_ctas(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return 0;
  return prop.multiProcessorCount;
}

}  // namespace hc
