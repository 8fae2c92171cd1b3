// pstep.cu: the persistent decode step (pstep.h). One cooperative launch, one CTA per SM, runs a
// whole decode step of up to 8 tokens:
//
//   embedding -> per layer [qkv GEMV] -> [attention splits + merge] -> [o GEMV + residual]
//             -> [gate/up GEMV + SiLU] -> [down GEMV + residual] -> head GEMV + greedy choice
//
// with a grid barrier after each bracket. A CTA is 8 consumer warps and a producer warp. The
// producer walks the step's static schedule for its CTA -- its row tiles of every GEMV and the
// cached keys and values of its attention splits -- and streams them from HBM into a ring of
// shared-memory stages with bulk copies (cp.async.bulk, no multicast; an mbarrier per stage for
// "full" and one for "empty"). Nothing it reads is written during the step, so it runs ahead of
// the grid barriers the consumers wait at, and HBM keeps streaming while they synchronise.
//
// Work split. Each GEMV's row tiles (16 rows) go round robin over the CTAs, continuing where the
// previous GEMV of the step stopped, so that every SM streams about the same bytes over a step; a
// row tile's column tiles are split over the 8 consumer warps (warp w: column tiles w, w + 8, ..)
// and their partial sums added in warp order, so every result has one fixed summation order. The
// attention of a token and kv head is cut into splits of 64 key positions ([64 s, 64 s + 64), so a
// token's splits depend on its position only and a row computes the same in any batch); a CTA
// takes a contiguous run of the step's (token, kv head, split) units, and the last unit of a
// (token, kv head) to finish (a ticket) merges the splits (Flash-Decoding, paged.go:227-310).
// Keys of the step's own tokens are not read from the cache: the unit computes them from the qkv
// rows (norm, RoPE, fp16 rounding), and the unit that holds a token's own position writes its key
// and value into the cache for later steps.
//
// Every wait is bounded (PsParams::spin_limit clock cycles): a grid barrier or a ring stage that
// does not come in time sets *status and the CTA finishes the step without waiting again (its
// results are garbage and the host reports an error); before the CTA exits, the producer waits for
// every bulk copy it issued, so no copy into shared memory outlives the CTA.
#include <algorithm>
#include <mutex>

#include "device.cuh"
#include "pstep.h"

namespace hc {
namespace {

constexpr int kCons = kPsConsumers * 32;  // consumer threads
constexpr int kMaxStages = 16;

__device__ __forceinline__ uint32_t saddr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_n(uint64_t *b, unsigned n) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes)
               : "memory");
}
// try_wait with a suspend-time hint: a waiting thread sleeps in hardware until the phase completes
// (or the hint's time passes) instead of spinning on the issue slots its scheduler's other warps need.
constexpr unsigned kSuspendNs = 2000;
__device__ __forceinline__ bool mbar_try(uint64_t *b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred P;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 P, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, P;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity), "n"(kSuspendNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(saddr(dst)),
      "l"(src), "r"(bytes), "r"(saddr(bar))
      : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// The consumer warps' barrier (named barrier 1; the producer warp never takes part).
__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCons) : "memory"); }

// Loads of data other CTAs wrote during this launch go to L2 (the L1 of this SM may hold an older
// copy of the line).
__device__ __forceinline__ float ldcg(const float *p) { return __ldcg(p); }

// ---- shared state -------------------------------------------------------------------------------
extern __shared__ __align__(1024) uint8_t ps_dyn[];  // activation tiles, then the ring
__shared__ uint64_t s_full[kMaxStages], s_empty[kMaxStages];
__shared__ volatile int s_seq[kMaxStages];  // the stage index each slot was last issued for
__shared__ volatile int s_abort;
__shared__ int s_last;
__shared__ StepTok s_toks[kPsMaxTok];
__shared__ int s_pos0[kPsMaxTok];  // the first position of each token's sequence in this step
__shared__ double s_red[kPsConsumers];
constexpr int kMaxRowGroups = 16 * kGroupsPerTile;  // groups of a normed row: hidden sizes up to 4096
constexpr int kMaxMergeSplits = 256;                 // splits a token may have: positions up to 16384
// scratch of two phases that never overlap: the norms' per-group sums of squares, and the weights of
// the attention merge
union PsScratch {
  double gss[kPsMaxTok][kMaxRowGroups];
  struct {
    float mw[8][kMaxMergeSplits], lw[8][kMaxMergeSplits];
  } mg;
};
__shared__ PsScratch s_x;
__shared__ float s_rn[kPsMaxTok];  // each row's norm factor
__shared__ int s_layer;             // the layer the consumers are in (for the trace)
__shared__ float s_part[2][kPsConsumers][kPsMaxTok][kTileRows];
__shared__ unsigned long long s_bmax[kPsMaxTok];
// attention unit state
__shared__ float s_q[8][128];      // the unit's query heads, normed and rotated
__shared__ float s_sc[8][64];      // scores, then probabilities, of a key block
__shared__ __half s_sk[kPsMaxTok * 128], s_sv[kPsMaxTok * 128];  // the step's own keys and values [i][hd]
__shared__ float s_m[8], s_l[8], s_corr[8];

struct Ring {
  uint8_t *base;
  int S, SB;
};

// Tells every wait of this CTA to give up, and the host which wait it was (the first one only).
__device__ __forceinline__ void give_up(const PsParams &p, int code) {
  if (!s_abort) {
    atomicCAS(p.status, 0, code);
    s_abort = 1;
  }
}

__shared__ unsigned long long s_wait_ns;  // CTA 0, thread 0: time spent waiting for ring stages (trace)

// Waits for a ring stage's phase (bounded). Every lane of a consumer warp calls it.
__device__ __forceinline__ void wait_stage(const PsParams &p, uint64_t *bar, unsigned parity, int code) {
  if (s_abort) return;
  const long long t0 = clock64();
  const unsigned long long w0 = (p.trace && threadIdx.x == 0) ? global_ns() : 0ull;
  while (!mbar_try(bar, parity)) {
    if (s_abort) return;
    if (clock64() - t0 > p.spin_limit) {
      give_up(p, code);
      return;
    }
  }
  if (p.trace && threadIdx.x == 0) s_wait_ns += global_ns() - w0;
}

// A sub-phase mark of CTA 0 in the trace: [phase][0] inputs ready, [1] work done, [2] barrier passed,
// [3] the ns thread 0 waited for ring stages in the phase (recorded with mark 1).
__device__ __forceinline__ void mark(const PsParams &p, int phase, int k) {
  if (p.trace && blockIdx.x == 0 && threadIdx.x == 0) {
    p.trace[phase * 4 + k] = global_ns();
    if (k == 1) {
      p.trace[phase * 4 + 3] = s_wait_ns;
      s_wait_ns = 0;
    }
  }
}

// The consumers' grid barrier (the ordering of cutlass's generic barrier: the CTA's threads
// synchronise, thread 0 releases with an acq_rel fence and a relaxed add, then spins on an
// acquire load): returns false once this CTA has given up.
__device__ __forceinline__ bool grid_sync(const PsParams &p, int &epoch) {
  mark(p, epoch, 1);
  cons_sync();
  ++epoch;
  if (threadIdx.x == 0 && !s_abort) {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
    const unsigned target = unsigned(epoch) * gridDim.x + (epoch == 1 ? unsigned(p.stall_first_barrier) : 0u);
    const long long t0 = clock64();
    int polls = 0;
    while (ld_acquire_u32(p.bar) < target) {
      if (clock64() - t0 > p.spin_limit) {
        give_up(p, epoch);
        break;
      }
      if ((++polls & 63) == 0 && *reinterpret_cast<volatile int *>(p.status)) {
        s_abort = 1;
        break;
      }
    }
  }
  mark(p, epoch - 1, 2);
  cons_sync();
  return !s_abort;
}

// The row tiles of a GEMV that CTA b takes: r = first, first + G, ... < rtiles, where the GEMV's
// row tile r goes to CTA (rr + r) mod G (rr: row tiles of the step's earlier GEMVs, mod G).
__device__ __forceinline__ int first_row_tile(int rr) {
  const int G = gridDim.x;
  return ((int(blockIdx.x) - rr) % G + G) % G;
}

// ---- attention units ------------------------------------------------------------------------------
// Unit u of the step (token-major, then kv head, then split) -> (token, kv head, split index).
struct Unit {
  int t, kvh, s;
  int ka, kb;  // its keys [ka, kb)
};

__device__ __forceinline__ int tok_lo(const PsParams &p, int window, int t) {
  const int P = s_toks[t].pos;
  return window > 0 ? max(0, P - window + 1) : 0;
}

__device__ __forceinline__ int tok_splits(const PsParams &p, int window, int t) {
  return s_toks[t].pos / kPsSplitKeys - tok_lo(p, window, t) / kPsSplitKeys + 1;
}

__device__ __forceinline__ int unit_count(const PsParams &p, int window) {
  int n = 0;
  for (int t = 0; t < p.ntok; ++t) n += p.KV * tok_splits(p, window, t);
  return n;
}

__device__ __forceinline__ Unit unit_of(const PsParams &p, int window, int u) {
  Unit x{0, 0, 0, 0, 0};
  for (int t = 0; t < p.ntok; ++t) {
    const int ns = tok_splits(p, window, t), n = p.KV * ns;
    if (u < n) {
      const int lo = tok_lo(p, window, t), P = s_toks[t].pos;
      x.t = t;
      x.kvh = u / ns;
      x.s = lo / kPsSplitKeys + u % ns;
      x.ka = max(lo, x.s * kPsSplitKeys);
      x.kb = min(P + 1, x.s * kPsSplitKeys + kPsSplitKeys);
      return x;
    }
    u -= n;
  }
  return x;
}

// Keys a ring stage carries (the cached keys of a unit come in blocks of this many).
__device__ __forceinline__ int keys_per_stage(int hd) { return kPsStageAttn / (4 * hd); }

// ---- the producer ------------------------------------------------------------------------------
struct Producer {
  const PsParams &p;
  Ring ring;
  int j = 0;  // stages issued

  __device__ Producer(const PsParams &pp, Ring r) : p(pp), ring(r) {}

  // Claims the next stage (waiting for the consumers to free it); null once giving up.
  __device__ uint8_t *claim(unsigned bytes) {
    const int s = j % ring.S;
    if (j >= ring.S) {
      const unsigned parity = unsigned(j / ring.S - 1) & 1u;
      const long long t0 = clock64();
      while (!mbar_try(&s_empty[s], parity)) {
        if (s_abort) return nullptr;
        if (clock64() - t0 > p.spin_limit) {
          give_up(p, 100000);
          return nullptr;
        }
      }
    }
    if (s_abort) return nullptr;
    s_seq[s] = j;
    mbar_expect_tx(&s_full[s], bytes);
    ++j;
    return ring.base + size_t(s) * ring.SB;
  }

  template <int TB>
  __device__ bool gemv(const uint8_t *tiles, int rtiles, int kt, int &rr) {
    const int G = gridDim.x;
    for (int r = first_row_tile(rr); r < rtiles; r += G) {
      for (int k0 = 0; k0 < kt; k0 += kPsConsumers) {
        const unsigned bytes = unsigned(min(kPsConsumers, kt - k0) * TB);
        uint8_t *dst = claim(bytes);
        if (!dst) return false;
        bulk_g2s(dst, tiles + (size_t(r) * kt + k0) * TB, bytes, &s_full[(j - 1) % ring.S]);
      }
    }
    rr = (rr + rtiles) % G;
    return true;
  }

  __device__ bool attention(const PsLayer &L) {
    const int U = unit_count(p, L.window), G = gridDim.x;
    const int u0 = int((long long)blockIdx.x * U / G), u1 = int((long long)(blockIdx.x + 1) * U / G);
    const int kps = keys_per_stage(p.hd);
    for (int u = u0; u < u1; ++u) {
      const Unit x = unit_of(p, L.window, u);
      const int c1 = min(x.kb, s_pos0[x.t]);
      const size_t base = (size_t(s_toks[x.t].slot) * p.KV + x.kvh) * size_t(p.cap) * p.hd;
      // the cached keys of each block [kps i, kps i + kps) of absolute positions, a stage a block
      for (int c = x.ka; c < c1; c = (c / kps + 1) * kps) {
        const int nk = min((c / kps + 1) * kps, c1) - c;
        const unsigned bytes = unsigned(nk * p.hd * 2);
        uint8_t *dst = claim(2 * bytes);
        if (!dst) return false;
        uint64_t *bar = &s_full[(j - 1) % ring.S];
        bulk_g2s(dst, L.kc + base + size_t(c) * p.hd, bytes, bar);
        bulk_g2s(dst + kPsStageAttn / 2, L.vc + base + size_t(c) * p.hd, bytes, bar);
      }
    }
    return true;
  }

  // Waits (bounded) until every copy issued has landed: the ring's last min(j, S) stages.
  __device__ void drain() {
    for (int k = max(0, j - ring.S); k < j; ++k) {
      const int s = k % ring.S;
      const unsigned parity = unsigned(k / ring.S) & 1u;
      const long long t0 = clock64();
      while (!mbar_try(&s_full[s], parity))
        if (clock64() - t0 > 4 * p.spin_limit) break;  // copies from valid memory always land
    }
  }
};

template <int KIND>
__device__ __forceinline__ void producer_run(const PsParams &p, Ring ring) {
  constexpr int TB = KIND == kKindInt8 ? kTileInt8 : kTileInt4;
  Producer pr(p, ring);
  int rr = 0;
  bool ok = true;
  for (int l = 0; l < p.layers && ok; ++l) {
    const PsLayer &L = p.L[l];
    ok = pr.gemv<TB>(L.qkv, p.rt_qkv, p.kt_d, rr) && pr.attention(L) && pr.gemv<TB>(L.o, p.rt_o, p.kt_o, rr) &&
         pr.gemv<TB>(L.gu, p.rt_gu, p.kt_d, rr) && pr.gemv<TB>(L.down, p.rt_down, p.kt_f, rr);
  }
  if (ok) pr.gemv<TB>(p.head, p.rt_head, p.kt_d, rr);
  pr.drain();
}

// ---- the consumers ------------------------------------------------------------------------------
// The phase bodies (build_act, gemv_phase, attention_phase) are out of line: each exists once in the
// kernel's code instead of once per call site (5 a layer), so that the code one layer runs stays in
// the SM's instruction caches rather than being fetched again from L2 at every phase.
enum Epi { kEpiStore, kEpiGlu, kEpiLogits };

// A quarter (8 values, columns 8 qq .. 8 qq + 7) of one group of 32 quantised by 4 neighbouring lanes
// together (qq = lane & 3): quant_vals' arithmetic value by value, the group's max and its X over the
// 4 lanes. The lanes that run this are whole warps (callers keep their loops warp-uniform).
__device__ __forceinline__ void quant_quarter(const float (&v)[8], uint8_t *act_tile, int gi, int qq) {
  float m = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
  float S = 0.f;
  int acc = 0;
  if (m > 0.f) {
    const float inv = 127.0f / m;
    S = m / 127.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float h = rintf(v[e] * inv);
      const float r = fmaf(-h, S, v[e]);
      const float l = fminf(fmaxf(rintf(r * (256.0f * inv)), -127.f), 127.f);
      const int hq = int(h), lq = int(l);
      acc += hq * 256 + lq;
      hw[e / 4] |= uint32_t(uint8_t(int8_t(hq))) << (8 * (e % 4));
      lw[e / 4] |= uint32_t(uint8_t(int8_t(lq))) << (8 * (e % 4));
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  *reinterpret_cast<uint2 *>(act_tile + gi * 64 + 8 * qq) = make_uint2(hw[0], hw[1]);
  *reinterpret_cast<uint2 *>(act_tile + gi * 64 + 32 + 8 * qq) = make_uint2(lw[0], lw[1]);
  if (qq == 0) *reinterpret_cast<float2 *>(act_tile + kGroupsPerTile * 64 + gi * 8) = make_float2(S, float(acc) * (1.0f / 256.0f));
}

// Loads the 8 values of columns c0 .. c0 + 7 of a row of n (zeros past n).
__device__ __forceinline__ void load8(float (&v)[8], const float *row, int c0, int n, bool global) {
  if (c0 + 7 < n) {
    const float4 *src = reinterpret_cast<const float4 *>(row + c0);
    const float4 a = global ? __ldcg(src) : src[0], b = global ? __ldcg(src + 1) : src[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = c0 + e < n ? (global ? __ldcg(row + c0 + e) : row[c0 + e]) : 0.f;
  }
}

// The activation tiles of ntok rows in dynamic shared memory (token t, column tile k at act +
// (t * KT + k) * kActTile), after the RMS norm of qwen3's normScaled when norm_w is set
// (act_quant_kernel's arithmetic: the squares of x / scale summed in float64, r = 1 / sqrt(mean +
// eps16), y = x / scale * r * w). The rows are the CTA's own copy of the residual stream xl
// ([ntok][n] in shared memory), first updated by dx (a GEMV's output that other CTAs wrote: xl +=
// dx) when dx is set; or, with xl null, src ([ntok][n] that other CTAs wrote). A thread takes a
// (token, group of 32) at a time; a token's squares are added group by group in order, so a row's
// norm does not depend on the other rows of the step.
__device__ __noinline__ void build_act(const float *src, float *xl, const float *dx, int n, int KT, const float *norm_w,
                          float scale, float eps16, uint8_t *act, int ntok) {
  const int GR = KT * kGroupsPerTile;  // groups a row, the zero groups past n included
  const int pairs = ntok * GR;
  const float inv = scale == 1.f ? 1.f : 1.f / scale;
  // pairs * 4 is a multiple of 32 (GR is a multiple of 8) and the loops step by whole warps, so every
  // warp runs the quarter loops' shuffles with all its lanes
  if (!norm_w) {
    for (int qi = threadIdx.x; qi < pairs * 4; qi += kCons) {
      const int pi = qi >> 2, qq = qi & 3;
      const int t = pi / GR, g = pi % GR;
      float v[8];
      load8(v, xl ? xl + size_t(t) * n : src + size_t(t) * n, g * kGroup + 8 * qq, n, !xl);
      quant_quarter(v, act + (size_t(t) * KT + g / kGroupsPerTile) * kActTile, g % kGroupsPerTile, qq);
    }
    cons_sync();
    return;
  }
  // pass 1: xl += dx, and each group's float64 sum of squares (4 threads a group, 8 values each,
  // added in lane order)
  for (int qi = threadIdx.x; qi < pairs * 4; qi += kCons) {
    const int pi = qi >> 2, qq = qi & 3;
    const int t = pi / GR, g = pi % GR;
    float *row = xl + size_t(t) * n;
    const int c0 = g * kGroup + 8 * qq;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = c0 + e < n ? row[c0 + e] : 0.f;
    if (dx) {
      const float *dr = dx + size_t(t) * n;
      float d[8];
      if (c0 + 7 < n) {
        const float4 a = __ldcg(reinterpret_cast<const float4 *>(dr + c0));
        const float4 b = __ldcg(reinterpret_cast<const float4 *>(dr + c0 + 4));
        d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w; d[4] = b.x; d[5] = b.y; d[6] = b.z; d[7] = b.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) d[e] = c0 + e < n ? __ldcg(dr + c0 + e) : 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[e] += d[e];
        if (c0 + e < n) row[c0 + e] = v[e];
      }
    }
    double sum = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xs = scale == 1.f ? v[e] : v[e] * inv;
      const float sq = xs * xs;
      sum += double(sq);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (qq == 0) s_x.gss[t][g] = sum;
  }
  cons_sync();
  // each row's sum over its groups in one fixed order: warp t, lane l adds groups l, l + 32, .. in
  // turn, then a shuffle tree over the lanes
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < ntok; t += kPsConsumers) {
      double a = 0;
      for (int g = lane; g < GR; g += 32) a += s_x.gss[t][g];
#pragma unroll
      for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) {
        const float ms = float(a / double(n));
        s_rn[t] = float(1.0 / sqrt(double(ms) + double(eps16)));
      }
    }
  }
  cons_sync();
  // pass 2: y = x / scale * r * w, quantised (4 threads a group)
  for (int qi = threadIdx.x; qi < pairs * 4; qi += kCons) {
    const int pi = qi >> 2, qq = qi & 3;
    const int t = pi / GR, g = pi % GR;
    const int c0 = g * kGroup + 8 * qq;
    float v[8];
    load8(v, xl + size_t(t) * n, c0, n, false);
    const float r = s_rn[t];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (c0 + e < n) {
        const float xs = scale == 1.f ? v[e] : v[e] * inv;
        v[e] = xs * r * norm_w[c0 + e];
      }
    }
    quant_quarter(v, act + (size_t(t) * KT + g / kGroupsPerTile) * kActTile, g % kGroupsPerTile, qq);
  }
  cons_sync();
}

// The value of row `row` from a raw sum (the int8 row scale, the bias).
template <int KIND>
__device__ __forceinline__ float finish_row(float v, int row, const float *rscale, const float *bias) {
  if (KIND == kKindInt8) v *= rscale[row];
  if (bias) v += bias[row];
  return v;
}

// The epilogue of one output value v of token t, row `row` of row tile r: kEpiStore writes y, kEpiLogits
// writes the fp16 logit and folds the greedy key into s_bmax. (The SwiGLU pairs are handled apart.)
__device__ __forceinline__ void epi_store(const PsParams &p, Epi epi, float *y, int ldy, int t, int row, float v) {
  if (epi == kEpiStore) {
    y[size_t(t) * ldy + row] = v;
  } else {
    const uint16_t hb = __half_as_ushort(__float2half_rn(v));
    if (p.logits) p.logits[size_t(t) * p.V + row] = hb;
    atomicMax(&s_bmax[t], argmax_key(hb, uint32_t(row)));
  }
}

// Waits for ring stage jj in a consumer warp that may be more than a lap of the ring ahead of the
// slot's earlier uses (other warps'): the slot must have been issued for jj (its tag, written before
// the issue) and then the phase of jj must be complete, so the phase parity cannot alias.
__device__ __forceinline__ void wait_stage_any(const PsParams &p, Ring ring, int jj, int code) {
  const int s = jj % ring.S;
  const unsigned parity = unsigned(jj / ring.S) & 1u;
  const unsigned long long w0 = (p.trace && threadIdx.x == 0) ? global_ns() : 0ull;
  if (!s_abort) {
    const long long t0 = clock64();
    while (!(s_seq[s] == jj && mbar_try(&s_full[s], parity))) {
      if (s_abort) break;
      if (clock64() - t0 > p.spin_limit) {
        give_up(p, code);
        break;
      }
    }
  }
  if (p.trace && threadIdx.x == 0) s_wait_ns += global_ns() - w0;
  __syncwarp();
}

// One GEMV over this CTA's row tiles (the producer streams their column tiles, 8 a stage). With at
// least one row tile per CTA on average (rtiles >= G) each warp takes whole row tiles (warp w: the
// CTA's row tiles w, w + 8, ..), summing their column tiles in order and finishing them itself; with
// fewer, a row tile's column tiles are split over the warps (warp w: w, w + 8, ..) and the partial
// sums added in warp order after a barrier of the consumers. Either way one phase has one
// summation order, whatever the tokens of the step.
template <int KIND, int NT>
__device__ __noinline__ void gemv_phase(const PsParams &p, Ring ring, int &j, int &rr, const uint8_t *act, int KT, int rtiles,
                           const float *rscale, const float *bias, Epi epi, float *y, int ldy, int rows) {
  constexpr int TB = KIND == kKindInt8 ? kTileInt8 : kTileInt4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int G = gridDim.x, ntok = p.ntok;
  const int nst = (KT + kPsConsumers - 1) / kPsConsumers;
  const int first = first_row_tile(rr);
  const int nmine = first < rtiles ? (rtiles - 1 - first) / G + 1 : 0;
  if (rtiles >= G) {
    for (int i = warp; i < nmine; i += kPsConsumers) {
      const int r = first + i * G;
      float vg[NT], vg8[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) vg[t] = vg8[t] = 0.f;
      for (int st = 0; st < nst; ++st) {
        const int jj = j + i * nst + st, s = jj % ring.S;
        wait_stage_any(p, ring, jj, 200000 + s);
        const uint8_t *stg = ring.base + size_t(s) * ring.SB;
        const int k1 = min(kPsConsumers, KT - st * kPsConsumers);
        for (int k = 0; k < k1; ++k) {
          WTile<KIND> wt;
          wt.load(stg + size_t(k) * TB, lane);
          const int kk = st * kPsConsumers + k;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
              BFrag<KIND> bf;
              bf.load(act + (size_t(t) * KT + kk) * kActTile, lane);
              wa_mma<KIND>(wt, bf, vg[t], vg8[t]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_n(&s_empty[s], kPsConsumers);
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float a = quad_sum(vg[t]), b = quad_sum(vg8[t]);
        if (c == 0 && t < ntok) {
          const int row0 = r * kTileRows + g, row8 = row0 + kTileRows / 2;
          if (epi == kEpiGlu) {
            const int o = r * (kTileRows / 2) + g;
            if (o < rows) {
              const float gv = finish_row<KIND>(a, row0, rscale, bias), uv = finish_row<KIND>(b, row8, rscale, bias);
              // blocks.SiLU: x / (1 + exp(-x)) (internal/llm/blocks/blocks.go:395-399)
              y[size_t(t) * ldy + o] = gv / (1.0f + expf(-gv)) * uv;
            }
          } else {
            if (row0 < rows) epi_store(p, epi, y, ldy, t, row0, finish_row<KIND>(a, row0, rscale, bias));
            if (row8 < rows) epi_store(p, epi, y, ldy, t, row8, finish_row<KIND>(b, row8, rscale, bias));
          }
        }
      }
    }
    j += nmine * nst;
    rr = (rr + rtiles) % G;
    return;
  }
  const int wk = min(kPsConsumers, KT);  // warps that hold column tiles
  int buf = 0;
  for (int r = first; r < rtiles; r += G) {
    float vg[NT], vg8[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) vg[t] = vg8[t] = 0.f;
    for (int st = 0; st < nst; ++st, ++j) {
      const int s = j % ring.S;
      wait_stage(p, &s_full[s], unsigned(j / ring.S) & 1u, 200000 + s);
      __syncwarp();
      const int kk = st * kPsConsumers + warp;
      if (kk < KT) {
        WTile<KIND> wt;
        wt.load(ring.base + size_t(s) * ring.SB + size_t(warp) * TB, lane);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < ntok) {
            BFrag<KIND> bf;
            bf.load(act + (size_t(t) * KT + kk) * kActTile, lane);
            wa_mma<KIND>(wt, bf, vg[t], vg8[t]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[s]);
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float a = quad_sum(vg[t]), b = quad_sum(vg8[t]);
      if (c == 0 && t < ntok) {
        s_part[buf][warp][t][g] = a;
        s_part[buf][warp][t][g + 8] = b;
      }
    }
    cons_sync();
    for (int i = threadIdx.x; i < ntok * kTileRows; i += kCons) {
      const int t = i / kTileRows, r16 = i % kTileRows;
      auto value = [&](int rr16) {
        float v = 0.f;
        for (int w = 0; w < wk; ++w) v += s_part[buf][w][t][rr16];
        return finish_row<KIND>(v, r * kTileRows + rr16, rscale, bias);
      };
      if (epi == kEpiGlu) {
        if (r16 >= kTileRows / 2) continue;
        const int o = r * (kTileRows / 2) + r16;
        if (o >= rows) continue;
        const float gv = value(r16), uv = value(r16 + kTileRows / 2);
        y[size_t(t) * ldy + o] = gv / (1.0f + expf(-gv)) * uv;
        continue;
      }
      const int row = r * kTileRows + r16;
      if (row < rows) epi_store(p, epi, y, ldy, t, row, value(r16));
    }
    buf ^= 1;
  }
  rr = (rr + rtiles) % G;
}

// q/k RMS norm (qwen3 build.go:283-284, when nw is set) and RoPE (blocks.ApplyRope,
// blocks.go:429-443) of one head of hd = 32 E values, lane l holding elements l + 32 k: the
// arithmetic of qkv_post_kernel.
template <int E>
__device__ __forceinline__ void norm_rope(float (&x)[E], const float *nw, float norm_scale, float eps16,
                                          const uint32_t *rope_row, int lane) {
  constexpr int hd = 32 * E, half = hd / 2;
  if (nw) {
    const float inv = norm_scale == 1.f ? 1.f : 1.f / norm_scale;
    double s = 0;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      x[k] = norm_scale == 1.f ? x[k] : __fmul_rn(x[k], inv);
      s += double(__fmul_rn(x[k], x[k]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float ms = float(s / double(hd));
    const float r = float(1.0 / sqrt(double(ms) + double(eps16)));
#pragma unroll
    for (int k = 0; k < E; ++k) x[k] = __fmul_rn(__fmul_rn(x[k], r), nw[lane + 32 * k]);
  }
  float y[E];
#pragma unroll
  for (int k = 0; k < E; ++k) {
    const int e = lane + 32 * k;
    const int jj = e < half ? e : e - half;
    const uint32_t cs = rope_row[jj];
    const float cv = __half2float(__ushort_as_half(uint16_t(cs & 0xffff)));
    const float sv = __half2float(__ushort_as_half(uint16_t(cs >> 16)));
    const int kp = e < half ? k + (half / 32) : k - (half / 32);
    const float rot = e < half ? -x[kp] : x[kp];
    y[k] = __fadd_rn(__fmul_rn(x[k], cv), __fmul_rn(rot, sv));
  }
#pragma unroll
  for (int k = 0; k < E; ++k) x[k] = y[k];
}

// The keys [ka, kb) of one unit (at most 64, one split) at once: the cached ones from up to two
// ring stages (positions [ka, b1) in Kc0/Vc0, [b1, c1) in Kc1/Vc1, fp16 rows), the step's own from
// s_sk / s_sv (position pos at row pos - sa). Scores by the threads of (key, head) with a rotated
// walk over the row (conflict-free shared-memory reads), the softmax of each head by a warp, then
// o[r][d] = sum_j p_j V[j][d] by the threads of (head, element). The split is fixed by position, so
// a row computes the same whichever of its keys the cache holds.
template <int HD>
__device__ __forceinline__ void attend_unit(const PsParams &p, const __half *Kc0, const __half *Vc0, const __half *Kc1,
                                            const __half *Vc1, int ka, int b1, int c1, int sa, int kb, int rep,
                                            float (&o)[4]) {
  constexpr int H2 = HD / 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = kb - ka;
  auto row = [&](int pos, const __half *C0, const __half *C1, const __half *St) -> const __half * {
    const __half *a = pos < b1 ? C0 + size_t(pos - ka) * HD : C1 + size_t(pos - b1) * HD;
    return pos < c1 ? a : St + size_t(pos - sa) * HD;
  };
  for (int pi = threadIdx.x; pi < nk * rep; pi += kCons) {
    const int jj = pi % nk, r = pi / nk;
    const __half2 *kr = reinterpret_cast<const __half2 *>(row(ka + jj, Kc0, Kc1, s_sk));
    const float2 *qr = reinterpret_cast<const float2 *>(s_q[r]);
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 4
    for (int e = 0; e < H2; e += 4) {
      const int i0 = (e + jj) & (H2 - 1), i1 = (e + 1 + jj) & (H2 - 1), i2 = (e + 2 + jj) & (H2 - 1),
                i3 = (e + 3 + jj) & (H2 - 1);
      const float2 k0 = __half22float2(kr[i0]), k1 = __half22float2(kr[i1]), k2 = __half22float2(kr[i2]),
                   k3 = __half22float2(kr[i3]);
      const float2 q0 = qr[i0], q1 = qr[i1], q2 = qr[i2], q3 = qr[i3];
      d0 = fmaf(q0.y, k0.y, fmaf(q0.x, k0.x, d0));
      d1 = fmaf(q1.y, k1.y, fmaf(q1.x, k1.x, d1));
      d2 = fmaf(q2.y, k2.y, fmaf(q2.x, k2.x, d2));
      d3 = fmaf(q3.y, k3.y, fmaf(q3.x, k3.x, d3));
    }
    s_sc[r][jj] = ((d0 + d1) + (d2 + d3)) * p.score_scale;
  }
  cons_sync();
  if (warp < rep) {
    const int r = warp;
    const float a = lane < nk ? s_sc[r][lane] : -INFINITY;
    const float b = lane + 32 < nk ? s_sc[r][lane + 32] : -INFINITY;
    const float m = warp_max(fmaxf(a, b));
    const float pa = lane < nk ? expf(a - m) : 0.f, pb = lane + 32 < nk ? expf(b - m) : 0.f;
    if (lane < nk) s_sc[r][lane] = pa;
    if (lane + 32 < nk) s_sc[r][lane + 32] = pb;
    const float l = warp_sum(pa + pb);
    if (lane == 0) {
      s_l[r] = l;
      s_m[r] = m;
    }
  }
  cons_sync();
  // keys jj = 4 q + i go to accumulator i, in increasing jj: one order whatever the cache holds
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int idx = threadIdx.x + k * kCons;
    o[k] = 0.f;
    if (idx < rep * HD) {
      const int r = idx / HD, d = idx % HD;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int jj = 0; jj < nk; jj += 4) {
        const float v0 = __half2float(row(ka + jj, Vc0, Vc1, s_sv)[d]);
        const float v1 = jj + 1 < nk ? __half2float(row(ka + jj + 1, Vc0, Vc1, s_sv)[d]) : 0.f;
        const float v2 = jj + 2 < nk ? __half2float(row(ka + jj + 2, Vc0, Vc1, s_sv)[d]) : 0.f;
        const float v3 = jj + 3 < nk ? __half2float(row(ka + jj + 3, Vc0, Vc1, s_sv)[d]) : 0.f;
        a0 = fmaf(s_sc[r][jj], v0, a0);
        if (jj + 1 < nk) a1 = fmaf(s_sc[r][jj + 1], v1, a1);
        if (jj + 2 < nk) a2 = fmaf(s_sc[r][jj + 2], v2, a2);
        if (jj + 3 < nk) a3 = fmaf(s_sc[r][jj + 3], v3, a3);
      }
      o[k] = (a0 + a1) + (a2 + a3);
    }
  }
}

// The attention units of this CTA for layer L.
template <int HD>
__device__ __noinline__ void attention_phase(const PsParams &p, const PsLayer &L, Ring ring, int &j) {
  constexpr int E = HD / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int U = unit_count(p, L.window), G = gridDim.x;
  const int u0 = int((long long)blockIdx.x * U / G), u1 = int((long long)(blockIdx.x + 1) * U / G);
  const int rep = p.H / p.KV, kps = keys_per_stage(HD);
  const int W = (p.H + 2 * p.KV) * HD;
  const int H = p.H;
  for (int u = u0; u < u1; ++u) {
    const Unit x = unit_of(p, L.window, u);
    const StepTok tk = s_toks[x.t];
    const int P = tk.pos, pos0 = s_pos0[x.t];
    unsigned long long tm[6] = {0, 0, 0, 0, 0, 0};  // the unit's marks, kept by thread 0 for the trace
    if (p.trace && threadIdx.x == 0) tm[0] = global_ns();
    // the query heads of the unit, and the step's own keys and values in [max(ka, pos0), kb)
    if (warp < rep) {
      const int h = x.kvh * rep + warp;
      float v[E];
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = ldcg(p.qkv + size_t(x.t) * W + size_t(h) * HD + lane + 32 * e);
      norm_rope<E>(v, L.q_norm, p.sc, p.eps, p.rope + size_t(P) * (HD / 2), lane);
#pragma unroll
      for (int e = 0; e < E; ++e) s_q[warp][lane + 32 * e] = v[e];
    }
    const int sa = max(x.ka, pos0), ns = x.kb - sa;  // ns <= 8: a sequence's tokens in this step
    if (warp < ns) {
      const int pp = sa + warp, t2 = x.t - (P - pp);
      float kv[E], vv[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        kv[e] = ldcg(p.qkv + size_t(t2) * W + size_t(p.H + x.kvh) * HD + lane + 32 * e);
        vv[e] = ldcg(p.qkv + size_t(t2) * W + size_t(p.H + p.KV + x.kvh) * HD + lane + 32 * e);
      }
      norm_rope<E>(kv, L.k_norm, p.sc, p.eps, p.rope + size_t(pp) * (HD / 2), lane);
      const size_t crow = ((size_t(tk.slot) * p.KV + x.kvh) * p.cap + pp) * HD;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const __half kh = __float2half_rn(kv[e]), vh = __float2half_rn(vv[e]);
        s_sk[warp * HD + lane + 32 * e] = kh;
        s_sv[warp * HD + lane + 32 * e] = vh;
        if (pp == P) {  // this token's own key and value go into the cache for later steps
          L.kc[crow + lane + 32 * e] = __half_as_ushort(kh);
          L.vc[crow + lane + 32 * e] = __half_as_ushort(vh);
        }
      }
    }
    // the cached keys [ka, c1) in at most two stages, split at a multiple of kps
    const int c1 = min(x.kb, pos0);
    const int b1 = min(c1, (x.ka / kps + 1) * kps);
    const int nstg = c1 <= x.ka ? 0 : (c1 > b1 ? 2 : 1);
    const uint8_t *stg[2] = {nullptr, nullptr};
    for (int q = 0; q < nstg; ++q) {
      const int jj = j + q, s = jj % ring.S;
      wait_stage(p, &s_full[s], unsigned(jj / ring.S) & 1u, 300000 + s);
      __syncwarp();
      stg[q] = ring.base + size_t(s) * ring.SB;
    }
    if (p.trace && threadIdx.x == 0) tm[1] = global_ns();
    cons_sync();
    if (p.trace && threadIdx.x == 0) tm[2] = global_ns();
    float o[4];
    attend_unit<HD>(p, reinterpret_cast<const __half *>(stg[0]), reinterpret_cast<const __half *>(stg[0] + kPsStageAttn / 2),
                    reinterpret_cast<const __half *>(stg[1]), reinterpret_cast<const __half *>(stg[1] + kPsStageAttn / 2),
                    x.ka, b1, c1, sa, x.kb, rep, o);
    for (int q = 0; q < nstg; ++q) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[(j + q) % ring.S]);
    }
    j += nstg;
    if (p.trace && threadIdx.x == 0) tm[3] = global_ns();
    // the unit's partial: (m, l) and the unnormalised o of each query head
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int idx = threadIdx.x + k * kCons;
      if (idx < rep * HD) {
        const int r = idx / HD, d = idx % HD, h = x.kvh * rep + r;
        const size_t pi = (size_t(x.t) * H + h) * p.max_splits + x.s;
        p.part_o[pi * HD + d] = o[k];
        if (d == 0) {
          p.part_ml[pi * 2] = s_m[r];
          p.part_ml[pi * 2 + 1] = s_l[r];
        }
      }
    }
    // the last unit of (token, kv head) to finish merges the splits (paged.Merge, paged.go:227-310,
    // with the sink logit of Merge.AddSink, paged.go:281-297): release by an acq_rel fence and a
    // relaxed add, the last one acquires with a fence after it
    cons_sync();
    if (threadIdx.x == 0) {
      const int nsp = tok_splits(p, L.window, x.t);
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      const int old = atomicAdd(&p.tickets[x.t * p.KV + x.kvh], 1);
      s_last = old == nsp - 1;
      if (s_last) {
        p.tickets[x.t * p.KV + x.kvh] = 0;
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
      }
      if (p.trace) tm[4] = global_ns();
    }
    cons_sync();
    if (s_last) {
      const int s0 = tok_lo(p, L.window, x.t) / kPsSplitKeys, nsp = P / kPsSplitKeys - s0 + 1;
      // the splits' (m, l) of the unit's heads into shared memory at once, then the weights
      for (int i = threadIdx.x; i < rep * nsp; i += kCons) {
        const int r = i / nsp, sp = i % nsp, h = x.kvh * rep + r;
        const size_t pi = (size_t(x.t) * H + h) * p.max_splits + s0 + sp;
        s_x.mg.mw[r][sp] = ldcg(p.part_ml + pi * 2);
        s_x.mg.lw[r][sp] = ldcg(p.part_ml + pi * 2 + 1);
      }
      cons_sync();
      if (warp < rep) {
        const int r = warp, h = x.kvh * rep + r;
        float M = L.sinks ? L.sinks[h] : -INFINITY;
        for (int sp = lane; sp < nsp; sp += 32)
          if (s_x.mg.lw[r][sp] > 0.f) M = fmaxf(M, s_x.mg.mw[r][sp]);
        M = warp_max(M);
        float Ls = 0.f;
        for (int sp = lane; sp < nsp; sp += 32) {
          const float w = s_x.mg.lw[r][sp] > 0.f ? expf(s_x.mg.mw[r][sp] - M) : 0.f;
          s_x.mg.mw[r][sp] = w;
          Ls = fmaf(s_x.mg.lw[r][sp], w, Ls);
        }
        Ls = warp_sum(Ls);
        if (L.sinks) Ls += expf(L.sinks[h] - M);
        if (lane == 0) s_corr[r] = Ls > 0.f ? 1.f / Ls : 0.f;
      }
      cons_sync();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int idx = threadIdx.x + k * kCons;
        if (idx < rep * HD) {
          const int r = idx / HD, d = idx % HD, h = x.kvh * rep + r;
          const float *po = p.part_o + ((size_t(x.t) * H + h) * p.max_splits + s0) * HD + d;
          float acc = 0.f;
          constexpr int B = 16;  // loads in flight
          for (int s8 = 0; s8 < nsp; s8 += B) {
            float ov[B];
#pragma unroll
            for (int b = 0; b < B; ++b) ov[b] = s8 + b < nsp ? ldcg(po + size_t(s8 + b) * HD) : 0.f;
#pragma unroll
            for (int b = 0; b < B; ++b)
              if (s8 + b < nsp) acc = fmaf(ov[b], s_x.mg.mw[r][s8 + b], acc);
          }
          p.attn[size_t(x.t) * H * HD + size_t(h) * HD + d] = acc * s_corr[r];
        }
      }
    }
    cons_sync();
    // the trace of the unit that merged (token 0, kv head 0): marks since the unit began
    if (p.trace && threadIdx.x == 0 && s_last && x.t == 0 && x.kvh == 0) {
      tm[5] = global_ns();
      unsigned long long *dst = p.trace + 4 * ps_phases(p.layers) + 8 * s_layer;
      for (int k = 0; k < 6; ++k) dst[k] = tm[k];
      dst[6] = blockIdx.x;
      dst[7] = u - u0;
    }
  }
}

template <int KIND, int HD, int NT>
__device__ __forceinline__ void consumer_run(const PsParams &p, Ring ring, float *xl, uint8_t *act) {
  const int G = gridDim.x;
  int j = 0, rr = 0, epoch = 0;
  // the embedding (llm.TokenRow, internal/llm/llm.go:43-60) of every token into this CTA's copy of
  // the residual stream
  for (int t = 0; t < p.ntok; ++t) {
    const int tok = s_toks[t].token;
    for (int cc = int(threadIdx.x); cc < p.D; cc += kCons) {
      float v;
      if (p.embed) {
        v = __half2float(__ushort_as_half(p.embed[size_t(tok) * p.D + cc]));
      } else {
        v = tile_value(p.head, p.head_scale, KIND, p.kt_d, KIND == kKindInt8 ? kTileInt8 : kTileInt4, tok, cc);
        v = __half2float(__float2half_rn(v));
      }
      xl[size_t(t) * p.D + cc] = v;
    }
  }
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < p.ntok * kAmaxSlots; i += kCons) p.amax[i] = 0ull;
  if (threadIdx.x < kPsMaxTok) s_bmax[threadIdx.x] = 0ull;
  cons_sync();
  const int W = (p.H + 2 * p.KV) * HD;
  for (int l = 0; l < p.layers; ++l) {
    const PsLayer &L = p.L[l];
    if (threadIdx.x == 0) s_layer = l;
    // x += the previous layer's down projection, then the input norm
    build_act(nullptr, xl, l ? p.dx_down : nullptr, p.D, p.kt_d, L.in_norm, l == 0 ? p.sc_in0 : p.sc,
                  l == 0 ? p.eps_in0 : p.eps, act, p.ntok);
    mark(p, epoch, 0);
    gemv_phase<KIND, NT>(p, ring, j, rr, act, p.kt_d, p.rt_qkv, L.qkv_scale, L.qkv_bias, kEpiStore, p.qkv, W, W);
    grid_sync(p, epoch);
    mark(p, epoch, 0);
    attention_phase<HD>(p, L, ring, j);
    grid_sync(p, epoch);
    build_act(p.attn, nullptr, nullptr, p.H * HD, p.kt_o, nullptr, 1.f, 0.f, act, p.ntok);
    mark(p, epoch, 0);
    gemv_phase<KIND, NT>(p, ring, j, rr, act, p.kt_o, p.rt_o, L.o_scale, L.o_bias, kEpiStore, p.dx_o, p.D, p.D);
    grid_sync(p, epoch);
    // x += the o projection, then the post-attention norm
    build_act(nullptr, xl, p.dx_o, p.D, p.kt_d, L.post_norm, p.sc, p.eps, act, p.ntok);
    mark(p, epoch, 0);
    gemv_phase<KIND, NT>(p, ring, j, rr, act, p.kt_d, p.rt_gu, L.gu_scale, nullptr, kEpiGlu, p.h, p.F, p.F);
    grid_sync(p, epoch);
    build_act(p.h, nullptr, nullptr, p.F, p.kt_f, nullptr, 1.f, 0.f, act, p.ntok);
    mark(p, epoch, 0);
    gemv_phase<KIND, NT>(p, ring, j, rr, act, p.kt_f, p.rt_down, L.down_scale, nullptr, kEpiStore, p.dx_down, p.D,
                         p.D);
    grid_sync(p, epoch);
  }
  // the head (qwen3 builder.head, build.go:107-109): the final norm, fp16 logits, greedy keys
  build_act(nullptr, xl, p.dx_down, p.D, p.kt_d, p.final_norm, p.sc_head, p.eps_head, act, p.ntok);
  mark(p, epoch, 0);
  gemv_phase<KIND, NT>(p, ring, j, rr, act, p.kt_d, p.rt_head, p.head_scale, nullptr, kEpiLogits, nullptr, p.V, p.V);
  mark(p, epoch, 1);
  cons_sync();
  if (threadIdx.x < p.ntok)
    atomicMax(&p.amax[threadIdx.x * kAmaxSlots + blockIdx.x % kAmaxSlots], s_bmax[threadIdx.x]);
  cons_sync();
  // the last CTA through the head reads the greedy choices (chat/sample.go:80-88: the first
  // largest) and, for hc_generate, feeds the choice back as the next step's token
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(&p.tickets[kPsMaxTok * p.KV], 1);
    s_last = old == G - 1;
    if (s_last) {
      p.tickets[kPsMaxTok * p.KV] = 0;
      __threadfence();
    }
  }
  cons_sync();
  if (s_last && !s_abort && threadIdx.x < 32) {
    const int lane = threadIdx.x;
    for (int t = 0; t < p.ntok; ++t) {
      unsigned long long k = 0;
      for (int i = lane; i < kAmaxSlots; i += 32) k = max(k, __ldcg(p.amax + t * kAmaxSlots + i));
#pragma unroll
      for (int o = 16; o; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
      const int32_t idx = int32_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
      if (lane == 0) {
        p.am[t] = idx;
        if (t == 0 && p.gen_out) {
          const int i = *p.gen_count;
          p.gen_out[i] = idx;
          p.toks[0].token = idx;
          p.toks[0].pos += 1;
          *p.gen_count = i + 1;
        }
      }
    }
  }
}

template <int KIND, int HD, int NT>
__global__ void __launch_bounds__(kPsThreads, 1) ps_kernel(const PsParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    s_wait_ns = 0;
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], kPsConsumers);
      s_seq[s] = -1;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = *reinterpret_cast<volatile int *>(p.status) != 0;
  }
  if (threadIdx.x < p.ntok) s_toks[threadIdx.x] = p.toks[threadIdx.x];
  __syncthreads();
  if (threadIdx.x < p.ntok) {
    int p0 = s_toks[threadIdx.x].pos;
    for (int t = 0; t < p.ntok; ++t)
      if (s_toks[t].slot == s_toks[threadIdx.x].slot) p0 = min(p0, s_toks[t].pos);
    s_pos0[threadIdx.x] = p0;
  }
  const size_t xl_bytes = (size_t(p.ntok) * p.D * 4 + 1023) / 1024 * 1024;
  const size_t act_bytes = (size_t(p.ntok) * max(p.kt_d, max(p.kt_f, p.kt_o)) * kActTile + 1023) / 1024 * 1024;
  Ring ring{ps_dyn + xl_bytes + act_bytes, p.stages, p.stage_bytes};
  __syncthreads();
  if (warp == kPsConsumers) {
    if (lane == 0) producer_run<KIND>(p, ring);
  } else {
    consumer_run<KIND, HD, NT>(p, ring, reinterpret_cast<float *>(ps_dyn), ps_dyn + xl_bytes);
  }
  __syncthreads();
}

template <int KIND, int HD, int NT>
void *kernel_of() {
  return reinterpret_cast<void *>(&ps_kernel<KIND, HD, NT>);
}

void *pick(int kind, int hd, int ntok) {
  const bool one = ntok == 1;
  if (kind == kKindInt4) {
    if (hd == 128) return one ? kernel_of<kKindInt4, 128, 1>() : kernel_of<kKindInt4, 128, kPsMaxTok>();
    return one ? kernel_of<kKindInt4, 64, 1>() : kernel_of<kKindInt4, 64, kPsMaxTok>();
  }
  if (hd == 128) return one ? kernel_of<kKindInt8, 128, 1>() : kernel_of<kKindInt8, 128, kPsMaxTok>();
  return one ? kernel_of<kKindInt8, 64, 1>() : kernel_of<kKindInt8, 64, kPsMaxTok>();
}

size_t g_static_smem = 0;  // the kernels' static shared memory (the largest), from ps_prepare

}  // namespace

bool ps_supported(int kind, int hd, int rep, int cap) {
  return (kind == kKindInt8 || kind == kKindInt4) && (hd == 64 || hd == 128) && rep >= 1 && rep <= 8 &&
         cap <= kMaxMergeSplits * kPsSplitKeys;
}

size_t ps_smem(const PsParams &p) {
  const size_t xl = (size_t(p.ntok) * p.D * 4 + 1023) / 1024 * 1024;
  const size_t act = (size_t(p.ntok) * std::max(p.kt_d, std::max(p.kt_f, p.kt_o)) * kActTile + 1023) / 1024 * 1024;
  return xl + act + size_t(p.stages) * p.stage_bytes;
}

bool ps_layout(PsParams &p, int kind) {
  const int tb = kind == kKindInt8 ? kTileInt8 : kTileInt4;
  p.stage_bytes = std::max(kPsConsumers * tb, kPsStageAttn);
  if (p.kt_d * kGroupsPerTile > kMaxRowGroups) return false;  // the norms' group sums in shared memory
  const size_t limit = 227 * 1024 - (g_static_smem ? g_static_smem : 24 * 1024);
  p.stages = kMaxStages;
  while (p.stages >= 4 && ps_smem(p) > limit) --p.stages;
  return p.stages >= 4 && ps_smem(p) <= limit;
}

cudaError_t ps_prepare() {
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  for (int kind : {int(kKindInt8), int(kKindInt4)})
    for (int hd : {64, 128})
      for (int nt : {1, kPsMaxTok}) {
        void *k = pick(kind, hd, nt);
        cudaFuncAttributes fa{};
        cudaError_t e = cudaFuncGetAttributes(&fa, k);
        if (e != cudaSuccess) return e;
        g_static_smem = std::max(g_static_smem, size_t(fa.sharedSizeBytes));
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(227 * 1024 - fa.sharedSizeBytes));
        if (e != cudaSuccess) return e;
      }
  return cudaSuccess;
}

cudaError_t ps_launch(const PsParams &p, int kind, int ctas, cudaStream_t st) {
  void *k = pick(kind, p.hd, p.ntok);
  void *args[] = {const_cast<PsParams *>(&p)};
  return cudaLaunchCooperativeKernel(k, dim3(ctas), dim3(kPsThreads), args, ps_smem(p), st);
}

int ps_ctas(int device) {
  int sms = 0, coop = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop) return 0;
  int per = 0;
  void *k = pick(kKindInt4, 128, 1);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k, kPsThreads, 64 * 1024) != cudaSuccess || per < 1) return 0;
  return sms;
}

}  // namespace hc
