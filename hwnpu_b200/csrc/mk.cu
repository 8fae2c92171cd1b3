// mk.cu: the persistent decode kernel (see mk.h). One CTA per SM runs every phase of the step:
//
//   per layer: [qkv GEMV] -> [attention units] -> [o GEMV + residual] -> [gate/up GEMV + SiLU]
//              -> [down GEMV + residual];  then the head GEMV + greedy choice
//
// with a grid barrier between phases. A CTA is 8 consumer warps and 1 producer warp. The producer
// walks the same static schedule as the consumers (the CTA's row tiles of every GEMV, its attention
// units' cached keys and values) and streams it from HBM into a ring of shared-memory stages with
// bulk copies (cp.async.bulk, an mbarrier per stage for "full" and one for "empty"), running ahead
// of the grid barriers the consumers wait at, so HBM keeps streaming while they synchronise.
// No wait is unbounded: a grid barrier or a stage that does not arrive within
// MkParams::spin_limit cycles sets *status and the kernel returns.
//
// Every GEMV spreads its 8-row tiles evenly over the CTAs and finishes each row tile where it is
// computed (the last warp of the team that owns it applies the epilogue: the qkv rows, the
// residual add into x, silu(gate) * up into h, or the fp16 logits and greedy key). The inputs of a
// GEMV are built by every CTA for itself at the start of the phase: x (or h) is read back, times
// the norm weight, and quantised to int8 tiles (common.h's kActTile) in shared memory, with the
// norm's 1/rms (qwen3's normScaled, build.go:131-151) applied to the rows' results; the o
// projection's input is the attention output, which every CTA merges from the units' per-split
// partials.
#include <algorithm>

#include "device.cuh"
#include "mk.h"

namespace hc {
namespace {

constexpr int kWarps = kMkThreads / 32;

// Issues the ring's next copies whose stages are free (lane 0 of warp 0; defined with the producer).
__device__ __forceinline__ void try_issue(const MkParams &p);

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

// Synchronises the 8 warps of the CTA (named barrier 1).
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kMkThreads) : "memory"); }

// The grid barrier of the consumers: returns false when it (or an earlier one) gave up.
// A sub-phase mark of the trace (thread 0): slot 0 when the phase's inputs are in smem, 1 when its
// chunks are consumed.
__shared__ unsigned s_epoch;  // grid barriers this CTA passed in the step (thread 0's count)

__device__ __forceinline__ void mark(const MkParams &p, int slot) {
  if (p.trace && threadIdx.x == 0)
    p.trace[size_t(2 + slot) * mk_phases(p.layers) * gridDim.x + size_t(s_epoch) * gridDim.x + blockIdx.x] =
        global_ns();
}

__device__ __forceinline__ bool grid_sync(const MkParams &p) {
  __shared__ int ok;
  csync();
  if (threadIdx.x == 0) {
    unsigned epoch = s_epoch;
    if (p.trace) p.trace[size_t(epoch) * gridDim.x + blockIdx.x] = global_ns();
    epoch += 1;
    const unsigned target = epoch * gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
    const long long t0 = clock64();
    long long next = t0 + kStatusPoll;
    int good = 1;
    try_issue(p);
    while (ld_acquire(p.bar) < target) {
      try_issue(p);  // stages freed by the phase's last chunks
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
    s_epoch = epoch;
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

// ---- the stage ring -----------------------------------------------------------------------------
constexpr int kKr = 8;  // column tiles of a weight chunk (one a consumer warp); a stage holds one chunk
                        // (8 tiles of the model's format, MkParams::stage_bytes) or keys + values

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
// try_wait with a suspend-time hint: a waiting thread sleeps in hardware (woken when the phase
// completes, or after about kSuspendNs) instead of spinning on the issue slots the consumers need.
constexpr unsigned kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_try(uint64_t *b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred P;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 P, [%1], %2, %3;\n selp.u32 %0, 1, 0, P;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity), "n"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// Whether the phase of parity `parity` of b has completed, without waiting.
__device__ __forceinline__ bool mbar_test(uint64_t *b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred P;\n mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 P, [%1], %2;\n selp.u32 %0, 1, 0, P;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}

struct Ring {
  uint8_t *stages;
  uint64_t *full, *empty;
  int S, SB;  // stages, bytes a stage
};

// At most this many stages; the row partials use twice as many slots.
constexpr int kMaxStages = 16;

// The kernel's dynamic shared memory (mk_layout places its parts) and its small shared state. The
// phases find everything from here and from the parameters, so that the kernel body keeps almost
// nothing alive across them.
extern __shared__ __align__(1024) uint8_t mk_smem[];
__shared__ float s_cfac[kMkMaxTok];              // per-token factor of the phase's rows (the norm)
__shared__ unsigned long long s_bmax[kMkMaxTok];  // this CTA's greedy keys in the head
__shared__ unsigned s_rcnt[2 * kMaxStages];       // arrivals at each row partial slot
__shared__ StepTok s_toks[kMkMaxTok];             // the step's tokens
// The row scale and bias of the GEMV phase that runs (set before it; read by its epilogues).
__shared__ const float *s_rscale;
__shared__ const float *s_rbias;

__device__ __forceinline__ Ring ring_of(const MkParams &p) {
  Ring r;
  r.S = p.stages;
  r.SB = p.stage_bytes;
  r.stages = mk_smem;
  r.full = reinterpret_cast<uint64_t *>(mk_smem + p.off_bar);
  r.empty = r.full + p.stages;
  return r;
}

// A GEMV phase of a CTA: row tiles rt0 + i * stride (i < nrt) of a matrix of ktiles column tiles;
// chunk (i, kr), the (i nkr + kr)-th of the phase, holds column tiles [8 kr, 8 kr + 8) of row tile
// rt(i). The CTAs interleave (rt0 = the CTA, stride = the grid), so that at any moment the grid
// reads neighbouring tiles, spread over all of HBM's channels.
struct GemvPhase {
  const uint8_t *tiles;
  int ktiles, rt0, nrt, tb, stride;
  __device__ int nkr() const { return (ktiles + kKr - 1) / kKr; }
  __device__ int chunks() const { return nrt * nkr(); }
  __device__ int rt(int i) const { return rt0 + i * stride; }
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
  // every GEMV deals its row tiles out to the CTAs in turn
  __device__ GemvPhase rows(const uint8_t *tiles, int rtiles, int ktiles) const {
    const int b = blockIdx.x, G = gridDim.x;
    return GemvPhase{tiles, ktiles, b, b < rtiles ? (rtiles - b + G - 1) / G : 0, tile_bytes_of<KIND>(), G};
  }
  __device__ GemvPhase qkv(int l) const { return rows(p.L[l].qkv, p.rt_qkv, p.kt_d); }
  __device__ GemvPhase o(int l) const { return rows(p.L[l].o, p.D / kTileRows, p.kt_o); }
  __device__ GemvPhase gu(int l) const { return rows(p.L[l].gu, 2 * p.F / kTileRows, p.kt_d); }
  __device__ GemvPhase down(int l) const { return rows(p.L[l].down, p.D / kTileRows, p.kt_f); }
  __device__ GemvPhase head() const { return rows(p.head, p.rt_head, p.kt_d); }
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
    return AttPhase{L.kc + base, L.vc + base, k0, min(k1, P), p.stage_bytes / (4 * p.hd), p.hd};
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

// ---- the producer: lane 0 of warp 0 issues the ring's bulk copies, never blocking -------------
// The walker over the step's chunks in the consumers' order: per layer the qkv rows, the attention
// units' keys and values, the o, gate/up and down rows; then the head's rows.
struct Prod {
  int j;      // the next chunk's ring position
  int q;      // its phase: 5 li + (0 qkv, 1 attention, 2 o, 3 gate/up, 4 down); 5 layers: the head
  int i, kr;  // GEMV: row tile and column chunk; attention: unit (from the CTA's first) and key chunk
};
__shared__ Prod s_prod;

__device__ __forceinline__ GemvPhase gemv_rows(const MkParams &p, const uint8_t *tiles, int rtiles, int ktiles) {
  const int b = blockIdx.x, G = gridDim.x;
  const int tb = p.kind == kKindInt8 ? kTileInt8 : (p.kind == kKindInt4 ? kTileInt4 : kTileMx);
  return GemvPhase{tiles, ktiles, b, b < rtiles ? (rtiles - b + G - 1) / G : 0, tb, G};
}

// The cached keys of attention unit u of layer li (as Schedule::att).
__device__ __forceinline__ AttPhase att_phase(const MkParams &p, int li, int u) {
  const int t = u / (p.KV * p.splits), kvh = (u / p.splits) % p.KV, s = u % p.splits;
  const StepTok tk = s_toks[t];
  const int P = tk.pos;
  const MkLayer &L = p.L[li];
  const int lo = L.window > 0 ? max(0, P - L.window + 1) : 0;
  const int n = P - lo + 1;
  const int chunk = (n + p.splits - 1) / p.splits;
  const int k0 = lo + s * chunk, k1 = min(P + 1, k0 + chunk);
  const size_t base = (size_t(tk.slot) * p.KV + kvh) * size_t(p.cap) * p.hd;
  return AttPhase{L.kc + base, L.vc + base, k0, min(k1, P), p.stage_bytes / (4 * p.hd), p.hd};
}

// The next chunk's sources (one or two copies) from the walker's place, which it then passes;
// false when the step has no more.
__device__ __forceinline__ bool prod_next(const MkParams &p, Prod &w, const void *&s0, unsigned &b0, const void *&s1,
                          unsigned &b1) {
  const int L = p.layers;
  for (;;) {
    if (w.q > 5 * L) return false;
    const int li = w.q / 5, ph = w.q % 5;
    if (w.q == 5 * L || ph != 1) {
      const GemvPhase g = w.q == 5 * L ? gemv_rows(p, p.head, p.rt_head, p.kt_d)
                          : ph == 0    ? gemv_rows(p, p.L[li].qkv, p.rt_qkv, p.kt_d)
                          : ph == 2    ? gemv_rows(p, p.L[li].o, p.D / kTileRows, p.kt_o)
                          : ph == 3    ? gemv_rows(p, p.L[li].gu, 2 * p.F / kTileRows, p.kt_d)
                                       : gemv_rows(p, p.L[li].down, p.D / kTileRows, p.kt_f);
      if (w.i < g.nrt) {
        const int nk = min(kKr, g.ktiles - w.kr * kKr);
        s0 = g.tiles + (size_t(g.rt(w.i)) * g.ktiles + w.kr * kKr) * g.tb;
        b0 = unsigned(nk * g.tb);
        s1 = nullptr;
        b1 = 0;
        if (++w.kr == g.nkr()) { w.kr = 0; ++w.i; }
        return true;
      }
    } else {
      int a0, a1;
      my_units(p.ntok * p.KV * p.splits, a0, a1);
      if (a0 + w.i < a1) {
        const AttPhase a = att_phase(p, li, a0 + w.i);
        if (w.kr < a.chunks()) {
          const int key0 = a.k0 + w.kr * a.kc, nkeys = min(a.kc, a.kc1 - key0);
          s0 = a.kbase + size_t(key0) * a.hd;
          s1 = a.vbase + size_t(key0) * a.hd;
          b0 = b1 = unsigned(nkeys * a.hd * 2);
          ++w.kr;
          return true;
        }
        ++w.i;
        w.kr = 0;
        continue;
      }
    }
    ++w.q;
    w.i = 0;
    w.kr = 0;
  }
}

// Issues every chunk whose stage is free (the stage's previous chunk released by all 8 warps), in
// order, without waiting. Lane 0 of warp 0 only: at each of its waits for a chunk, in the grid
// barrier's poll, and when a step starts.
__device__ __forceinline__ void try_issue(const MkParams &p) {
  const Ring r = ring_of(p);
  Prod w = s_prod;
  for (;;) {
    if (w.j >= r.S && !mbar_test(&r.empty[w.j % r.S], ((w.j / r.S) + 1) & 1)) break;
    const void *s0, *s1;
    unsigned b0, b1;
    if (!prod_next(p, w, s0, b0, s1, b1)) break;
    const int s = w.j % r.S;
    ctrace(p, w.j, 0);
    mbar_expect_tx(&r.full[s], b0 + b1);
    uint8_t *dst = r.stages + size_t(s) * r.SB;
    bulk_g2s(dst, s0, b0, &r.full[s]);
    if (b1) bulk_g2s(dst + b0, s1, b1, &r.full[s]);
    ++w.j;
  }
  s_prod = w;
}

// Cycles warp 0 of the consumers waited for stages (trace runs).
__shared__ long long s_cwait;

// The slow path of mbar_wait_warp (kept out of line so the chunk loops stay call-free). Warp 0
// keeps issuing the ring's copies while it waits (so it polls without sleeping); the other warps
// sleep in try_wait.
__device__ __forceinline__ bool mbar_wait_warp_slow(uint64_t *b, unsigned parity, const MkParams &p, int code) {
  const int lane = threadIdx.x & 31;
  const bool issuer = threadIdx.x < 32;
  const long long t0 = clock64();
  long long next = t0 + kStatusPoll;
  for (;;) {
    if (issuer) {
      if (lane == 0) try_issue(p);
      __syncwarp();
    }
    if (__all_sync(0xffffffffu, issuer ? mbar_test(b, parity) : mbar_try(b, parity))) {
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
// the warp converged). Warp 0 first issues what it can.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *b, unsigned parity, const MkParams &p, int code) {
  if (threadIdx.x < 32) {
    if (threadIdx.x == 0) try_issue(p);
    __syncwarp();
  }
  if (__all_sync(0xffffffffu, mbar_test(b, parity))) return true;
  return mbar_wait_warp_slow(b, parity, p, code);
}

// ---- the consumers ----------------------------------------------------------------------------

// The GEMV phases, and what the last warp of a row tile does with its 16 rows x NT tokens.
enum Phase : int {
  kPhQkv = 0,   // qkv[t][row] = v * cf[t] * scale[row] + bias[row]
  kPhO = 1,     // x[t][row] += v * scale[row] + bias[row]       (the residual)
  kPhGu = 2,    // h[t][rt*8 + r] = silu(gate) * up, rows r / r + 8 of tile rt
  kPhDown = 3,  // x[t][row] += v * scale[row]                    (the residual)
  kPhHead = 4,  // fp16 logits and the greedy key of every row below V
};

// The value of row r of partial slot `slot` (of NS) for token t: the 8 warps' partials in order.
template <int NT>
__device__ __forceinline__ float slot_value(const float *part, int NS, int slot, int t, int r) {
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w)
    v += *reinterpret_cast<const volatile float *>(part + ((size_t(w) * NS + slot) * NT + t) * kTileRows + r);
  return v;
}

// The row tiles of a GEMV phase (chunk (i, kr), the (i nkr + kr)-th of the phase, holds column
// tiles [8 kr, 8 kr + 8) of row tile rt(i)). Warp w takes column tile 8 kr + w of every chunk:
// its weights from the stage, its activation fragments built once for the phase when one chunk
// covers the row (nkr == 1) and a single token runs, else per chunk. A warp releases the stage as
// soon as its tile is in registers. The warps leave their rows' partials in 2 S slots (S the ring's
// stages), used round robin (stored at kr = 0, added to after); the last of the 8 to finish row
// tile i (a shared counter) adds them up in warp order (results do not depend on timing) and
// applies the epilogue. Slot reuse is safe: a warp reaches row tile i + 2S only once every warp
// released a chunk of row tile i + S, and the last warp of row tile i finishes its epilogue before
// it goes on to row tile i + 1. Returns the ring position after the phase.
template <int KIND, int NT, int PH>
__device__ __forceinline__ int consume_rows(int j, int li, const MkParams &p) {
  const Schedule<KIND, NT> sc{p};
  const GemvPhase g = PH == kPhQkv ? sc.qkv(li)
                      : PH == kPhO ? sc.o(li)
                      : PH == kPhGu ? sc.gu(li)
                      : PH == kPhDown ? sc.down(li)
                                      : sc.head();
  const Ring r = ring_of(p);
  const uint8_t *act_s = mk_smem + p.off_act;
  float *part = reinterpret_cast<float *>(mk_smem + p.off_rows);
  unsigned *cnt = s_rcnt;
  const float *cf = s_cfac;
  unsigned long long *bmax = s_bmax;
  constexpr int TB = KIND == kKindInt8 ? kTileInt8 : (KIND == kKindInt4 ? kTileInt4 : kTileMx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, c = lane & 3;
  const int nkr = g.nkr();
  const bool cached = nkr == 1 && NT == 1;
  bool good = true;
  BFrag<KIND> bf;
  if (cached) {
    if (warp < g.ktiles) bf.load(act_s + size_t(warp) * kActTile, lane);
    else bf.zero();
  }
  for (int i = 0; i < g.nrt && good; ++i) {
    const int NS = 2 * r.S, slot = i % NS;
    float *pw = part + (size_t(warp) * NS + slot) * NT * kTileRows;
    for (int kr = 0; kr < nkr; ++kr) {
      const int jj = j + i * nkr + kr, s = jj % r.S;
      if (!mbar_wait_warp(&r.full[s], (jj / r.S) & 1, p, 1000004)) { good = false; break; }
      ctrace_c(p, jj, false);
      const int kt = kr * kKr + warp;
      const bool on = kt < g.ktiles;
      float vg[NT], vg8[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) vg[t] = vg8[t] = 0.f;
      WTile<KIND> wt;
      if (on) wt.load(r.stages + size_t(s) * r.SB + size_t(warp) * TB, lane);
      // release the stage as soon as its bytes are in registers
      __syncwarp();
      if (lane == 0) mbar_arrive(&r.empty[s], 1);
      if (on) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (!cached) bf.load(act_s + (size_t(t) * g.ktiles + kt) * kActTile, lane);
          wa_mma<KIND>(wt, bf, vg[t], vg8[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float a = quad_sum(vg[t]), b = quad_sum(vg8[t]);
        if (c == 0) {
          if (kr == 0) {
            pw[t * kTileRows + gq] = a;
            pw[t * kTileRows + gq + 8] = b;
          } else {
            pw[t * kTileRows + gq] += a;
            pw[t * kTileRows + gq + 8] += b;
          }
        }
      }
      if (kr + 1 == nkr) {
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) {
          __threadfence_block();
          last = atomicAdd(&cnt[slot], 1u) == unsigned(kWarps - 1);
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence_block();
          const int rt = g.rt(i);
          const float half = KIND == kKindMx ? 0.5f : 1.f;  // the doubled e2m1 values (mxfp4.go:90)
          if (PH == kPhGu) {
            const float *gsc = *reinterpret_cast<const float *const volatile *>(&s_rscale);
            for (int q = lane; q < NT * 8; q += 32) {
              const int t = q / 8, r8 = q % 8, grow = rt * kTileRows + r8;
              float gv = slot_value<NT>(part, NS, slot, t, r8) * half * cf[t];
              float uv = slot_value<NT>(part, NS, slot, t, r8 + 8) * half * cf[t];
              if (gsc) { gv *= gsc[grow]; uv *= gsc[grow + 8]; }
              // blocks.SiLU: x / (1 + exp(-x)) (internal/llm/blocks/blocks.go:395-399)
              p.h[size_t(t) * p.F + rt * 8 + r8] = gv / (1.0f + expf(-gv)) * uv;
            }
          } else {
            const int W = (p.H + 2 * p.KV) * p.hd;
            const int rows = PH == kPhQkv ? W : PH == kPhHead ? p.V : p.D;
            const float *scale = *reinterpret_cast<const float *const volatile *>(&s_rscale);
            const float *bias = *reinterpret_cast<const float *const volatile *>(&s_rbias);
            for (int q = lane; q < NT * kTileRows; q += 32) {
              const int t = q / kTileRows, row = rt * kTileRows + q % kTileRows;
              if (row >= rows) continue;
              float v = slot_value<NT>(part, NS, slot, t, q % kTileRows) * half * cf[t];
              if (scale) v *= scale[row];
              if (bias) v += bias[row];
              if (PH == kPhHead) {
                const uint16_t hb = __half_as_ushort(__float2half_rn(v));
                if (p.logits) p.logits[size_t(t) * p.V + row] = hb;
                atomicMax(&bmax[t], argmax_key(hb, row));
              } else if (PH == kPhQkv) {
                p.qkv[size_t(t) * W + row] = v;
              } else {
                float *yp = p.x + size_t(t) * p.D + row;
                *yp = __ldcg(yp) + v;
              }
            }
          }
          if (lane == 0) cnt[slot] = 0u;
        }
      }
      ctrace_c(p, jj, true);
    }
  }
  (void)good;
  return j + g.chunks();
}

// ---- activations built by every consumer CTA ------------------------------------------------
// Quantises K groups of 32 at once with quant32's arithmetic (hi = round_even(v * 127 / max), lo
// the residual at 1/256 of the scale, S = max / 127, Xq = sum(hi + lo / 256)): value v[k] of lane
// `lane` is column lane of group `slot` of column tile kt0 + k of token row `at` (act_s + t * ktiles
// tiles); groups with k >= nk are skipped. The K reductions are interleaved.
template <int K>
__device__ __forceinline__ void quant_tiles(const float (&v)[K], uint8_t *at, int kt0, int nk, int slot, int lane) {
  float m[K];
#pragma unroll
  for (int k = 0; k < K; ++k) m[k] = fabsf(v[k]);
#pragma unroll
  for (int o = 16; o; o >>= 1)
#pragma unroll
    for (int k = 0; k < K; ++k) m[k] = fmaxf(m[k], __shfl_xor_sync(0xffffffffu, m[k], o));
  int hq[K], lq[K], s[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    hq[k] = 0;
    lq[k] = 0;
    if (m[k] > 0.f) {
      const float inv = 127.0f / m[k];
      const float S = m[k] / 127.0f;
      const float h = rintf(v[k] * inv);
      const float rr = fmaf(-h, S, v[k]);
      hq[k] = int(h);
      lq[k] = int(fminf(fmaxf(rintf(rr * (256.0f * inv)), -127.f), 127.f));
    }
    s[k] = hq[k] * 256 + lq[k];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
#pragma unroll
    for (int k = 0; k < K; ++k) s[k] += __shfl_xor_sync(0xffffffffu, s[k], o);
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (k >= nk) continue;
    uint8_t *tile = at + size_t(kt0 + k) * kActTile;
    tile[slot * 64 + lane] = uint8_t(int8_t(hq[k]));
    tile[slot * 64 + 32 + lane] = uint8_t(int8_t(lq[k]));
    if (lane == 0)
      *reinterpret_cast<float2 *>(tile + kGroupsPerTile * 64 + slot * 8) =
          make_float2(m[k] > 0.f ? m[k] / 127.0f : 0.f, float(s[k]) * (1.0f / 256.0f));
  }
}

// The embedding of token `tok`, column col, as the reference's fp16 table holds it (the tied case
// decodes the head's tile).
template <int KIND>
__device__ __forceinline__ float embed_value(const MkParams &p, int tok, int col) {
  if (p.embed) return __half2float(__ushort_as_half(p.embed[size_t(tok) * p.D + col]));
  const float v = tile_value(p.head, p.head_scale, KIND, p.kt_d, tile_bytes_of<KIND>(), tok, col);
  return __half2float(__float2half_rn(v));
}

constexpr int kMaxKt = 24;  // column tiles of a GEMV input the step supports (F <= 6144)

// Activation tiles of NT tokens for a GEMV whose input is n columns: x = src[t][col] (EMB: the
// embedding of the step's token, also stored to src for the column tiles this CTA owns), times
// the norm weight nw when there is one, quantised per group of 32 into act_s. Warp w takes group w
// of every column tile, all of a token's loads at once. With a norm, sq_s[t][w] gets the warp's
// sum of (x / scale)^2 in double (the reference sums the squares in float64, milcpu reduce_mean
// ops.go:861-920; only the order differs).
template <int KIND, int NT, bool EMB>
__device__ __forceinline__ void build_act(float *src, int ld, int n, const float *nw, float scale, const MkParams &p) {
  uint8_t *act_s = mk_smem + p.off_act;
  double *sq_s = reinterpret_cast<double *>(mk_smem + p.off_sq);
  const StepTok *toks = s_toks;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = n / kTileCols;
  int own0 = 0, own1 = 0;
  if (EMB) my_units(kt, own0, own1);
  const float inv = scale == 1.f ? 1.f : 1.f / scale;
  for (int t = 0; t < NT; ++t) {
    float x[kMaxKt];
    double ss = 0;
#pragma unroll
    for (int k = 0; k < kMaxKt; ++k) {
      const int col = k * kTileCols + warp * 32 + lane;
      x[k] = 0.f;
      if (k < kt) {
        if (EMB) {
          x[k] = embed_value<KIND>(p, toks[t].token, col);
          if (k >= own0 && k < own1) src[size_t(t) * ld + col] = x[k];
        } else {
          x[k] = __ldcg(src + size_t(t) * ld + col);
        }
      }
    }
    if (nw) {
#pragma unroll
      for (int k = 0; k < kMaxKt; ++k) {
        if (k < kt) {
          const float xs = scale == 1.f ? x[k] : x[k] * inv;
          ss += double(xs * xs);
          x[k] *= nw[k * kTileCols + warp * 32 + lane];
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) sq_s[t * kWarps + warp] = ss;
    }
    uint8_t *at = act_s + size_t(t) * kt * kActTile;
#pragma unroll
    for (int k0 = 0; k0 < kMaxKt; k0 += 8) {
      if (k0 < kt) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = x[k0 + k];
        quant_tiles<8>(v, at, k0, min(8, kt - k0), warp, lane);
      }
    }
  }
}

// cf[t] = r / scale for a normed input of n columns (r = float32(1 / sqrt(float64(mean) + eps16)),
// milcpu's rsqrt, ops.go:181-189), from the warps' sums build_act left in sq_s; 1 without a norm.
template <int NT>
__device__ __forceinline__ void norm_factors_s(const MkParams &p, int n, float scale, float eps16, bool normed) {
  float *cf = s_cfac;
  const double *sq_s = reinterpret_cast<const double *>(mk_smem + p.off_sq);
  if (threadIdx.x < NT) {
    const int t = threadIdx.x;
    float f = 1.f;
    if (normed) {
      double s = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s += sq_s[t * kWarps + w];
      const float ms = float(s / double(n));
      const float r = float(1.0 / sqrt(double(ms) + double(eps16)));
      f = r * (1.f / scale);
    }
    cf[t] = f;
  }
}

// The attention output of NT tokens, merged from the units' per-split partials (Flash-Decoding's
// merge, paged.go:227-310, with gpt-oss's sink in the denominator, gptoss/build.go:256-285) and
// quantised into act_s as the o projection's input. A warp takes one (token, head): lane s holds
// split s's weight, lane l accumulates elements [E l, E l + E) over the splits in split order, and
// each group of 32 columns (32 / E lanes) is quantised with quant32's arithmetic.
template <int NT, int HD>
__device__ __forceinline__ void merge_attn(const MkParams &p, const float *sinks) {
  uint8_t *act_s = mk_smem + p.off_act;
  constexpr int E = HD / 32;   // elements a lane: 4 (hd 128) or 2 (hd 64)
  constexpr int GL = 32 / E;   // lanes of one group of 32 columns
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.splits;      // <= 32 on this path
  for (int th = warp; th < NT * p.H; th += kWarps) {
    const int t = th / p.H, h = th % p.H;
    const float *ml = p.part_ml + (size_t(t) * p.H + h) * S * 2;
    float m0 = -INFINITY, l0 = 0.f;
    if (lane < S) { m0 = __ldcg(ml + 2 * lane); l0 = __ldcg(ml + 2 * lane + 1); }
    const float *po = p.part_o + (size_t(t) * p.H + h) * S * HD + lane * E;
    constexpr int CH = 20;  // splits loaded at once (up to 20: the partials take one round trip)
    float o[CH][E];
    auto load = [&](int s0) {
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        if (s0 + u < S) {
          if constexpr (E == 4) {
            const float4 q = __ldcg(reinterpret_cast<const float4 *>(po + size_t(s0 + u) * HD));
            o[u][0] = q.x; o[u][1] = q.y; o[u][2] = q.z; o[u][3] = q.w;
          } else {
            const float2 q = __ldcg(reinterpret_cast<const float2 *>(po + size_t(s0 + u) * HD));
            o[u][0] = q.x; o[u][1] = q.y;
          }
        }
      }
    };
    load(0);  // before the weights, so both loads are in flight together
    float M = sinks ? sinks[h] : -INFINITY;
    M = fmaxf(M, l0 > 0.f ? m0 : -INFINITY);
    M = warp_max(M);
    const float w0 = l0 > 0.f ? expf(m0 - M) : 0.f;
    float Ls = warp_sum(l0 * w0);
    if (sinks) Ls += expf(sinks[h] - M);
    const float invl = Ls > 0.f ? 1.f / Ls : 0.f;
    float acc[E];
#pragma unroll
    for (int k = 0; k < E; ++k) acc[k] = 0.f;
    for (int s0 = 0; s0 < S; s0 += CH) {
      if (s0 > 0) load(s0);
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        const float ws = __shfl_sync(0xffffffffu, w0, (s0 + u) & 31);
        if (s0 + u < S) {
#pragma unroll
          for (int k = 0; k < E; ++k) acc[k] = fmaf(o[u][k], ws, acc[k]);
        }
      }
    }
    // quantise: the group of 32 columns of this lane is lanes [GL (lane / GL), + GL)
    float v[E], m = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      v[k] = acc[k] * invl;
      m = fmaxf(m, fabsf(v[k]));
    }
#pragma unroll
    for (int o = GL / 2; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int sum = 0;
    int8_t hq[E], lq[E];
    float S32 = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      hq[k] = 0;
      lq[k] = 0;
      if (m > 0.f) {
        const float inv = 127.0f / m;
        S32 = m / 127.0f;
        const float hh = rintf(v[k] * inv);
        const float rr = fmaf(-hh, S32, v[k]);
        hq[k] = int8_t(hh);
        lq[k] = int8_t(fminf(fmaxf(rintf(rr * (256.0f * inv)), -127.f), 127.f));
      }
      sum += int(hq[k]) * 256 + int(lq[k]);
    }
#pragma unroll
    for (int o = GL / 2; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const int col0 = h * HD + lane * E, G = col0 / 32, within = col0 % 32;
    uint8_t *tile = act_s + (size_t(t) * p.kt_o + G / kGroupsPerTile) * kActTile;
    const int gi = G % kGroupsPerTile;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      tile[gi * 64 + within + k] = uint8_t(hq[k]);
      tile[gi * 64 + 32 + within + k] = uint8_t(lq[k]);
    }
    if (within == 0)
      *reinterpret_cast<float2 *>(tile + kGroupsPerTile * 64 + gi * 8) = make_float2(S32, float(sum) * (1.0f / 256.0f));
  }
}

// The attention of one (token, kv head, split) unit (all 8 warps): q/k norms and RoPE of the heads it
// needs (one warp a head; the new key and value of position P in float32, as the reference's step
// rows are, written to the cache as fp16 by the unit that holds P), then an online softmax over its
// cached keys, which arrive from the ring in chunks, by 32 groups of 8 lanes; the split's (m, l, o)
// partials go to global memory, merged by the o projection's consumers (merge_attn).
template <int HD, int REP>
__device__ __forceinline__ int attention_unit(int j, const AttPhase a, const MkParams &p, const MkLayer &L, int t,
                                           int kvh, int s) {
  const Ring r = ring_of(p);
  const StepTok *toks = s_toks;
  uint8_t *scratch = mk_smem + p.off_att;
  constexpr int E = HD / 8;
  float *qs = reinterpret_cast<float *>(scratch);  // [REP][HD]
  float *kn = qs + REP * HD;                         // [HD]
  float *vn = kn + HD;                               // [HD]
  float *wm = vn + HD;                               // [8][REP]
  float *wl = wm + kWarps * REP;                     // [8][REP]
  float *wo = wl + kWarps * REP;                     // [8][REP][HD]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = threadIdx.x >> 3, l8 = threadIdx.x & 7;
  const int li = int(&L - p.L);
  utrace(p, li, 0);
  const StepTok tk = toks[t];
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
    const uint32_t *rt = p.rope + size_t(P) * (HD / 2);
    float x[E2], nwv[E2], vv[E2];
    uint32_t cs[E2];
    // every load of the task first (one round trip)
#pragma unroll
    for (int k = 0; k < E2; ++k) {
      const int e = lane + 32 * k;
      x[k] = __ldcg(src + e);
      nwv[k] = nw ? nw[e] : 1.f;
      cs[k] = rt[e < HD / 2 ? e : e - HD / 2];
      vv[k] = is_q ? 0.f : __ldcg(row + size_t(p.H + p.KV + kvh) * HD + e);
    }
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
      for (int k = 0; k < E2; ++k) x[k] = __fmul_rn(__fmul_rn(x[k], rr), nwv[k]);
    }
    float y[E2];
#pragma unroll
    for (int k = 0; k < E2; ++k) {
      const int e = lane + 32 * k;
      const float cv = __half2float(__ushort_as_half(uint16_t(cs[k] & 0xffff)));
      const float sv = __half2float(__ushort_as_half(uint16_t(cs[k] >> 16)));
      const int kp = e < HD / 2 ? k + (HD / 64) : k - (HD / 64);
      const float rot = e < HD / 2 ? -x[kp] : x[kp];
      y[k] = __fadd_rn(__fmul_rn(x[k], cv), __fmul_rn(rot, sv));
    }
    if (is_q) {
#pragma unroll
      for (int k = 0; k < E2; ++k) qs[task * HD + lane + 32 * k] = y[k];
    } else {
#pragma unroll
      for (int k = 0; k < E2; ++k) {
        const int e = lane + 32 * k;
        kn[e] = y[k];
        vn[e] = vv[k];
        L.kc[base + size_t(P) * HD + e] = __half_as_ushort(__float2half_rn(y[k]));
        L.vc[base + size_t(P) * HD + e] = __half_as_ushort(__float2half_rn(vv[k]));
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
    const uint8_t *stage = r.stages + size_t(st) * r.SB;
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
  csync();  // the scratch is reused by the CTA's next unit
  utrace(p, li, 4);
  (void)good;
  return j;
}

// The row scale and bias of phase ph of layer li for the epilogues (thread 0; a csync follows).
__device__ __forceinline__ void set_rows(const MkParams &p, int ph, int li) {
  if (threadIdx.x != 0) return;
  const MkLayer &L = p.L[li];
  s_rscale = ph == kPhQkv ? L.qkv_scale : ph == kPhO ? L.o_scale : ph == kPhGu ? L.gu_scale
           : ph == kPhDown ? L.down_scale : p.head_scale;
  s_rbias = ph == kPhQkv ? L.qkv_bias : ph == kPhO ? L.o_bias : nullptr;
}

// The phases of the step, each out of line and entered from a kernel loop that keeps only the layer
// and the ring position, so that each is allocated its own registers. Each returns the ring
// position after it; its grid barrier follows in the kernel.
template <int KIND, int NT, int HD, int REP>
__device__ __noinline__ int ph_qkv(const MkParams &p, int li, int j) {
  // the input norm (layer 0: of the embedding, which this phase also stores as x)
  if (li == 0) build_act<KIND, NT, true>(p.x, p.D, p.D, p.in_norm0, p.sc_in0, p);
  else build_act<KIND, NT, false>(p.x, p.D, p.D, p.L[li - 1].next_norm, p.sc, p);
  csync();
  norm_factors_s<NT>(p, p.D, li == 0 ? p.sc_in0 : p.sc, li == 0 ? p.eps_in0 : p.eps, true);
  set_rows(p, kPhQkv, li);
  csync();
  mark(p, 0);
  j = consume_rows<KIND, NT, kPhQkv>(j, li, p);
  mark(p, 1);
  return j;
}

// This CTA's attention units write their partials.
template <int KIND, int NT, int HD, int REP>
__device__ __noinline__ int ph_att(const MkParams &p, int li, int j) {
  const Schedule<KIND, NT> sc{p};
  int a0, a1;
  sc.units(a0, a1);
  mark(p, 0);
  for (int u = a0; u < a1; ++u) {
    const int t = u / (p.KV * p.splits), kvh = (u / p.splits) % p.KV, s = u % p.splits;
    j = attention_unit<HD, REP>(j, sc.att(li, u), p, p.L[li], t, kvh, s);
  }
  mark(p, 1);
  return j;
}

// The o projection + residual: the heads' outputs merged from the units' partials.
template <int KIND, int NT, int HD, int REP>
__device__ __noinline__ int ph_o(const MkParams &p, int li, int j) {
  merge_attn<NT, HD>(p, p.L[li].sinks);
  if (threadIdx.x < NT) s_cfac[threadIdx.x] = 1.f;
  set_rows(p, kPhO, li);
  csync();
  mark(p, 0);
  j = consume_rows<KIND, NT, kPhO>(j, li, p);
  mark(p, 1);
  return j;
}

// gate/up + SiLU after the post-attention norm.
template <int KIND, int NT, int HD, int REP>
__device__ __noinline__ int ph_gu(const MkParams &p, int li, int j) {
  utrace(p, li, 5);
  build_act<KIND, NT, false>(p.x, p.D, p.D, p.L[li].post_norm, p.sc, p);
  utrace(p, li, 6);
  csync();
  norm_factors_s<NT>(p, p.D, p.sc, p.eps, true);
  set_rows(p, kPhGu, li);
  csync();
  utrace(p, li, 7);
  mark(p, 0);
  j = consume_rows<KIND, NT, kPhGu>(j, li, p);
  mark(p, 1);
  return j;
}

// down + residual.
template <int KIND, int NT, int HD, int REP>
__device__ __noinline__ int ph_down(const MkParams &p, int li, int j) {
  build_act<KIND, NT, false>(p.h, p.F, p.F, nullptr, 1.f, p);
  if (threadIdx.x < NT) s_cfac[threadIdx.x] = 1.f;
  set_rows(p, kPhDown, li);
  csync();
  mark(p, 0);
  j = consume_rows<KIND, NT, kPhDown>(j, li, p);
  mark(p, 1);
  return j;
}

// The head: the final norm, fp16 logits and this CTA's greedy keys (chat/sample.go:80-88).
template <int KIND, int NT, int HD, int REP>
__device__ __noinline__ int ph_head(const MkParams &p, int j) {
  build_act<KIND, NT, false>(p.x, p.D, p.D, p.L[p.layers - 1].next_norm, p.sc_head, p);
  if (threadIdx.x < NT) s_bmax[threadIdx.x] = 0ull;
  csync();
  norm_factors_s<NT>(p, p.D, p.sc_head, p.eps_head, true);
  set_rows(p, kPhHead, 0);
  csync();
  mark(p, 0);
  j = consume_rows<KIND, NT, kPhHead>(j, 0, p);
  csync();
  mark(p, 1);
  if (threadIdx.x < NT)
    atomicMax(&p.amax[threadIdx.x * kAmaxSlots + (blockIdx.x % kAmaxSlots)], s_bmax[threadIdx.x]);
  return j;
}

template <int KIND, int NT, int HD, int REP>
__global__ void __launch_bounds__(kMkBlock, 1) mk_kernel(const __grid_constant__ MkParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    const Ring r = ring_of(p);
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&r.full[s], 1);
      mbar_init(&r.empty[s], kWarps);  // released by the 8 consumer warps
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < 2 * kMaxStages) s_rcnt[threadIdx.x] = 0u;
  if (threadIdx.x < NT) s_toks[threadIdx.x] = p.toks[threadIdx.x];
  if (threadIdx.x == 0) s_prod = Prod{0, 0, 0, 0};
  __syncthreads();
  if (threadIdx.x == 0) try_issue(p);
  const long long c_t0 = clock64();
  if (threadIdx.x == 0) { s_cwait = 0; s_epoch = 0; }
  int j = 0;  // ring position
  for (int li = 0; li < p.layers; ++li) {
    j = ph_qkv<KIND, NT, HD, REP>(p, li, j);
    if (!grid_sync(p)) return;
    j = ph_att<KIND, NT, HD, REP>(p, li, j);
    if (!grid_sync(p)) return;
    j = ph_o<KIND, NT, HD, REP>(p, li, j);
    if (!grid_sync(p)) return;
    j = ph_gu<KIND, NT, HD, REP>(p, li, j);
    if (!grid_sync(p)) return;
    j = ph_down<KIND, NT, HD, REP>(p, li, j);
    if (!grid_sync(p)) return;
  }
  j = ph_head<KIND, NT, HD, REP>(p, j);
  if (!grid_sync(p)) return;
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
  const int rep = p.H / p.KV;
  const int tb = p.kind == kKindInt8 ? kTileInt8 : (p.kind == kKindInt4 ? kTileInt4 : kTileMx);
  p.stage_bytes = kKr * tb;
  const size_t act = size_t(p.ntok) * ktmax * kActTile;
  const size_t att = size_t(rep * p.hd + 2 * p.hd + 2 * kWarps * rep + kWarps * rep * p.hd) * 4 + 16;
  const size_t sq = size_t(p.ntok) * kWarps * 8;
  auto al = [](size_t x) { return (x + 127) / 128 * 128; };
  // a stage costs its bytes, two partial slots of every warp and two mbarriers
  const size_t fixed = al(act) + al(att) + al(sq);
  const size_t per_stage = size_t(p.stage_bytes) + size_t(2) * kWarps * p.ntok * kTileRows * 4 + 16;
  if (fixed + 2 * per_stage + 256 > limit) return 0;
  int S = int((limit - fixed - 256) / per_stage);
  S = std::min(S, kMaxStages);
  p.stages = S;
  const size_t rows = size_t(kWarps) * 2 * S * p.ntok * kTileRows * 4;
  size_t off = size_t(S) * p.stage_bytes;
  p.off_act = int(off);
  off += al(act);
  p.off_rows = int(off);
  off += al(rows);
  p.off_att = int(off);
  off += al(att);
  p.off_sq = int(off);
  off += al(sq);
  p.off_bar = int(off);
  off += size_t(2) * S * 8;
  (void)ctas;
  return off <= limit ? off : 0;
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
