// attn_tc.cu: decode attention over the paged int8 cache (HC_KV_INT8_PAGED) on the integer
// tensor cores: blocks.SDPAGrouped's scores and weighted sum (blocks.go:516-539) with an online
// softmax, split over the context and merged by attn_merge (Flash-Decoding, paged.go:227-310).
//
// One CTA per (split, kv head, token) as attn_split_kernel, 4 warps, each warp a run of page pairs
// (32 positions) of the split. Per pair a warp streams the two key pages and the two (transposed)
// value pages into its shared-memory ring with cp.async, then
//   scores  S = Q K^T    mma.sync m16n8k32 s8 x s8 -> s32: rows of A are the kv head's query heads,
//                         each quantised to int8 twice (hi, and the residual lo at 1/256, scale
//                         max|q| / 127), so hi + lo / 256 carries ~15 bits; B is the key rows as
//                         they sit in the page (ldmatrix); the page's key scale comes after
//   weights P            exp(S - m) in float32 (online max m, sum l per head), scaled by the page's
//                         value scale over the pair's larger one, quantised to int8 hi/lo the same
//                         way (P <= 1, scale 1/127)
//   values  O += V^T P   the same MMA: A is the transposed value page (a dimension's 16 positions
//                         contiguous), B is P straight from the score accumulators: the key order of
//                         the score tiles is chosen so that each lane already holds the 4 positions
//                         its B fragment needs
// Everything else is float32: the integer sums are exact, the scales multiply them afterwards. A
// chunk's own keys (StepTok::run0) come from the float32 stage rows on the CUDA cores (16 groups
// of 8 lanes, as attn_split_kernel), as a second partial of each warp.
#include "device.cuh"
#include "kernels.h"

namespace hc {
namespace {

constexpr int kAtWarps = 4;
constexpr int kAtStages = 2;  // page pairs in flight a warp (one ahead of the one computed)

__device__ __forceinline__ uint32_t at_saddr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void at_cp16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(at_saddr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void at_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void at_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void at_ldsm4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
// Four signed bytes (low byte first) from four float codes already in [-127, 127].
__device__ __forceinline__ uint32_t at_pack4(float a, float b, float c, float d) {
  return uint32_t(uint8_t(int8_t(int(a)))) | (uint32_t(uint8_t(int8_t(int(b)))) << 8) |
         (uint32_t(uint8_t(int8_t(int(c)))) << 16) | (uint32_t(uint8_t(int8_t(int(d)))) << 24);
}

// Shared memory of one page pair: the 32 key rows (position-major, each row's 16-byte chunks
// XOR-swizzled by the row so that the 8 rows an ldmatrix reads fall on distinct banks), then the
// two transposed value pages ([hd][16] each, 16-byte rows: contiguous rows read without conflict).
template <int HD>
struct AtPair {
  static constexpr int kChunks = HD / 16;
  static constexpr int kKBytes = 32 * HD;
  static constexpr int kVBytes = HD * 16;
  static constexpr int kBytes = kKBytes + 2 * kVBytes;
  __device__ static __forceinline__ int swz(int r) { return HD == 128 ? (r & 7) : ((r >> 1) & 3); }
  __device__ static __forceinline__ int koff(int r, int chunk) { return r * HD + ((chunk ^ swz(r)) << 4); }
};

size_t at_smem(int hd) { return size_t(kAtWarps) * kAtStages * 4 * 16 * hd; }

// Picks x[i] for a warp-uniform-shaped small array by a runtime index (no local memory).
template <int N>
__device__ __forceinline__ float at_pick(const float (&x)[N], int i) {
  float v = x[0];
#pragma unroll
  for (int k = 1; k < N; ++k)
    if (i == k) v = x[k];
  return v;
}

template <int HD, int REP>
__global__ void __launch_bounds__(kAtWarps * 32) attn_paged_tc_kernel(const float *__restrict__ q,
                                                                     const StepTok *__restrict__ toks, AttnGeom g,
                                                                     PagedKV pk, int splits,
                                                                     float *__restrict__ part_ml,
                                                                     float *__restrict__ part_o,
                                                                     const float *__restrict__ kv_stage) {
  using Pr = AtPair<HD>;
  constexpr int KB = HD / 32;  // K-blocks of the score MMA (32 dimensions each)
  constexpr int DB = HD / 16;  // dimension blocks of the value MMA (16 each)
  extern __shared__ __align__(128) uint8_t at_buf[];
  __shared__ float sm_m[kAtWarps][REP], sm_l[kAtWarps][REP];
  __shared__ float sm_o[kAtWarps][REP][HD];
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, cq = lane & 3;  // the fragment's row group and its lane in the quad
  const StepTok tk = toks[t];
  const int P = tk.pos;
  const int lo = g.window > 0 ? max(0, P - g.window + 1) : 0;
  const int n = P - lo + 1;
  const int chunk = (n + splits - 1) / splits;
  const int k0 = lo + s * chunk, k1 = min(P + 1, k0 + chunk);
  // positions from p0 on are this token's piece (float32 stage rows); cached keys are [k0, kc1)
  const int p0 = tk.run0 >= 0 ? P - (t - tk.run0) : P + 1;
  const int kc1 = min(k1, max(k0, p0));
  int pairs = 0, pg0 = 0, pg_last = -1;
  if (kc1 > k0) {
    pg0 = k0 / kPage;
    pg_last = (kc1 - 1) / kPage;
    pairs = (pg_last - pg0 + 2) / 2;
  }
  const int per = (pairs + kAtWarps - 1) / kAtWarps;
  const int w0 = min(pairs, warp * per), w1 = min(pairs, w0 + per);

  // The query heads as int8 hi/lo rows of the score MMA's A operand: row r < REP is head r's hi
  // codes, row REP + r its lo codes (the residual at 1/256), rows from 2 REP on are zero.
  const float *qh = q + (size_t(t) * g.heads + size_t(kvh) * REP) * HD;
  float qs[REP];
#pragma unroll
  for (int h = 0; h < REP; ++h) {
    float mx = 0.f;
#pragma unroll
    for (int d = lane; d < HD; d += 32) mx = fmaxf(mx, fabsf(qh[h * HD + d]));
    qs[h] = warp_max(mx) / 127.0f;
  }
  const int hr = gq % REP;
  const bool row_hi = gq < REP, row_used = gq < 2 * REP;
  const float qsr = at_pick(qs, hr);
  const float qinv = qsr > 0.f ? 1.0f / qsr : 0.f;
  uint32_t qa[KB][2];
#pragma unroll
  for (int J = 0; J < KB; ++J) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const float4 v = *reinterpret_cast<const float4 *>(qh + hr * HD + 32 * J + 16 * half + 4 * cq);
      const float x[4] = {v.x * qinv, v.y * qinv, v.z * qinv, v.w * qinv};
      float c[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float hi = rintf(x[i]);
        c[i] = row_hi ? hi : fminf(fmaxf(rintf((x[i] - hi) * 256.0f), -127.f), 127.f);
      }
      qa[J][half] = row_used ? at_pack4(c[0], c[1], c[2], c[3]) : 0u;
    }
  }

  uint8_t *ring = at_buf + size_t(warp) * kAtStages * Pr::kBytes;
  const int32_t *bt = pk.btab + size_t(tk.slot) * pk.max_pages;
  // the warp's page ids, 32 a register (lane i: page base + i) with the next 32 preloaded, so that
  // issuing a pair reads no global memory before its copies
  const int pgw = pg0 + 2 * w0;
  int bt_base = pgw;
  int bt_cur = pgw + lane <= pg_last ? bt[pgw + lane] : 0;
  int bt_nxt = pgw + 32 + lane <= pg_last ? bt[pgw + 32 + lane] : 0;
  auto page_id = [&](int pg) {  // pg is never below a page asked for before
    while (pg - bt_base >= 32) {
      bt_base += 32;
      bt_cur = bt_nxt;
      bt_nxt = bt_base + 32 + lane <= pg_last ? bt[bt_base + 32 + lane] : 0;
    }
    return __shfl_sync(0xffffffffu, bt_cur, pg - bt_base);
  };
  // the pages of pair pi into ring stage st: key rows (swizzled) and transposed values
  auto issue = [&](int pi, int st) {
    uint8_t *dst = ring + st * Pr::kBytes;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int pg = pg0 + 2 * pi + half;
      if (pg > pg_last) continue;
      const size_t ph = size_t(page_id(pg)) * g.kv_heads + kvh;
      const int8_t *ksrc = pk.k + ph * kPage * HD;
      const int8_t *vsrc = pk.v + ph * kPage * HD;
#pragma unroll
      for (int i = lane; i < kPage * Pr::kChunks; i += 32) {
        const int r = i / Pr::kChunks, ch = i % Pr::kChunks;
        at_cp16(dst + Pr::koff(16 * half + r, ch), ksrc + r * HD + ch * 16);
      }
#pragma unroll
      for (int i = lane; i < HD; i += 32) at_cp16(dst + Pr::kKBytes + half * Pr::kVBytes + i * 16, vsrc + i * 16);
    }
  };
#pragma unroll
  for (int st = 0; st < kAtStages - 1; ++st) {
    if (w0 + st < w1) issue(w0 + st, st);
    at_commit();
  }

  float m_r = -INFINITY, l_r = 0.f;  // this lane's row's head: running max and sum
  float o[DB][4];                     // values: rows (dims 16b + gq, + 8) x columns (2 cq, 2 cq + 1)
#pragma unroll
  for (int b = 0; b < DB; ++b) o[b][0] = o[b][1] = o[b][2] = o[b][3] = 0.f;
  // columns 2 cq, 2 cq + 1 of the value MMA: hi weights of head col (< REP), lo weights (< 2 REP)
  const int col0 = 2 * cq, col1 = 2 * cq + 1;
  const float cs0 = col0 < REP ? 1.0f / 127.0f : (col0 < 2 * REP ? 1.0f / (127.0f * 256.0f) : 0.f);
  const float cs1 = col1 < REP ? 1.0f / 127.0f : (col1 < 2 * REP ? 1.0f / (127.0f * 256.0f) : 0.f);

  // the pair's (key, value) scales of both pages, loaded a pair ahead of their use
  uint16_t sc_cur[4] = {0, 0, 0, 0}, sc_nxt[4] = {0, 0, 0, 0};
  auto load_scales = [&](int pi, uint16_t (&sc)[4]) {
    const int pa = pg0 + 2 * pi;
    const size_t pha = size_t(page_id(pa)) * g.kv_heads + kvh;
    sc[0] = pk.kscale[pha];
    sc[1] = pk.vscale[pha];
    if (pa + 1 <= pg_last) {
      const size_t phb = size_t(page_id(pa + 1)) * g.kv_heads + kvh;
      sc[2] = pk.kscale[phb];
      sc[3] = pk.vscale[phb];
    } else {
      sc[2] = sc[3] = 0;
    }
  };
  if (w0 < w1) load_scales(w0, sc_cur);
  for (int pi = w0; pi < w1; ++pi) {
    const int i = pi - w0;
    if (pi + kAtStages - 1 < w1) issue(pi + kAtStages - 1, (i + kAtStages - 1) % kAtStages);
    at_commit();
    if (pi + 1 < w1) load_scales(pi + 1, sc_nxt);
    at_wait<kAtStages - 1>();
    __syncwarp();
    const uint8_t *buf = ring + (i % kAtStages) * Pr::kBytes;
    const int pa = pg0 + 2 * pi;
    const float ksa = __half2float(__ushort_as_half(sc_cur[0]));
    const float vsa = __half2float(__ushort_as_half(sc_cur[1]));
    const float ksb = __half2float(__ushort_as_half(sc_cur[2]));
    const float vsb = __half2float(__ushort_as_half(sc_cur[3]));
#pragma unroll
    for (int k = 0; k < 4; ++k) sc_cur[k] = sc_nxt[k];
    // scores: tiles 0, 1 (page a) and 2, 3 (page b) of 8 positions; tile column n of tile tt of a
    // page is position 4 (n >> 1) + (n & 1) + 2 tt, so that the lane of quad position cq ends up
    // with positions 4 cq .. 4 cq + 3 of each page
    int d[4][4];
#pragma unroll
    for (int tl = 0; tl < 4; ++tl) d[tl][0] = d[tl][1] = d[tl][2] = d[tl][3] = 0;
#pragma unroll
    for (int J = 0; J < KB; ++J) {
#pragma unroll
      for (int pg = 0; pg < 2; ++pg) {
        const int m = lane >> 3, r8 = lane & 7;
        const int key = 16 * pg + 4 * (r8 >> 1) + (r8 & 1) + 2 * (m >> 1);
        uint32_t b00, b01, b10, b11;
        at_ldsm4(at_saddr(buf + Pr::koff(key, 2 * J + (m & 1))), b00, b01, b10, b11);
        mma_s8s8(d[2 * pg], qa[J][0], 0u, qa[J][1], 0u, b00, b01);
        mma_s8s8(d[2 * pg + 1], qa[J][0], 0u, qa[J][1], 0u, b10, b11);
      }
    }
    // A head's hi-row lane and lo-row lane (4 REP lanes apart) share the head's scores: the hi lane
    // takes page a's 4 positions, the lo lane page b's, each combining hi + lo / 256 from its own
    // sum and the partner's; the softmax sums and the weights' codes are then exchanged, so each lane
    // does half of the per-position work. Only a pair that reaches outside [k0, kc1) masks
    // positions (uniform over the warp).
    constexpr int PX = 4 * REP;
    float sc[4];
    const float sa = qsr * ksa * g.score_scale, sb = qsr * ksb * g.score_scale;
    const bool full = 16 * pa >= k0 && 16 * (pa + 2) <= kc1;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int mine = row_hi ? d[u][e] : d[2 + u][e];
        const int give = row_hi ? d[2 + u][e] : d[u][e];
        const int got = __shfl_xor_sync(0xffffffffu, give, PX);
        const float v = row_hi ? float(mine) + float(got) * (1.0f / 256.0f) : float(got) + float(mine) * (1.0f / 256.0f);
        sc[2 * u + e] = v * (row_hi ? sa : sb);
      }
    }
    const int my_page = pa + (row_hi ? 0 : 1);
    if (!full) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int pos = 16 * my_page + 4 * cq + k;
        if (pos < k0 || pos >= kc1) sc[k] = -INFINITY;
      }
    }
    // the online softmax of this row's head over the pair's 32 positions (the quad and its partner)
    float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, PX));
    // every pair holds a position of [k0, kc1), so m_new is finite: exp(-inf) gives the zeros
    const float m_new = fmaxf(m_r, mx);
    const float corr = __expf(m_r - m_new);
    float p[4], psum = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      p[k] = __expf(sc[k] - m_new);
      psum += p[k];
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    psum += __shfl_xor_sync(0xffffffffu, psum, PX);
    l_r = l_r * corr + psum;
    m_r = m_new;
    // the weights times each page's value scale over the pair's larger one, as int8 hi/lo (B of
    // the value MMA: column gq, positions 4 cq .. 4 cq + 3 of page a in b0, of page b in b1): each
    // lane codes its page's 4 weights both ways and hands the partner the half it needs
    const float vsm = fmaxf(vsa, vsb);
    const float fa = vsm > 0.f ? vsa / vsm * 127.0f : 0.f, fb = vsm > 0.f ? vsb / vsm * 127.0f : 0.f;
    const float f = row_hi ? fa : fb;
    float wh[4], wl[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = p[k] * f;
      wh[k] = rintf(x);
      wl[k] = fminf(fmaxf(rintf((x - wh[k]) * 256.0f), -127.f), 127.f);
    }
    const uint32_t my_hi = at_pack4(wh[0], wh[1], wh[2], wh[3]), my_lo = at_pack4(wl[0], wl[1], wl[2], wl[3]);
    const uint32_t got_codes = __shfl_xor_sync(0xffffffffu, row_hi ? my_lo : my_hi, PX);
    const uint32_t pb0 = row_used ? (row_hi ? my_hi : got_codes) : 0u;
    const uint32_t pb1 = row_used ? (row_hi ? got_codes : my_lo) : 0u;
    // each column's head's rescale (from the score row of that head: lane 4 h)
    const float c0 = __shfl_sync(0xffffffffu, corr, 4 * (col0 % REP));
    const float c1 = __shfl_sync(0xffffffffu, corr, 4 * (col1 % REP));
    const float s0 = cs0 * vsm, s1 = cs1 * vsm;
#pragma unroll
    for (int b = 0; b < DB; ++b) {
      const int m = lane >> 3;
      const int dim = 16 * b + 8 * (m & 1) + (lane & 7);
      uint32_t a0, a1, a2, a3;
      at_ldsm4(at_saddr(buf + Pr::kKBytes + (m >> 1) * Pr::kVBytes + dim * 16), a0, a1, a2, a3);
      int dd[4] = {0, 0, 0, 0};
      mma_s8s8(dd, a0, a1, a2, a3, pb0, pb1);
      o[b][0] = o[b][0] * c0 + float(dd[0]) * s0;
      o[b][1] = o[b][1] * c1 + float(dd[1]) * s1;
      o[b][2] = o[b][2] * c0 + float(dd[2]) * s0;
      o[b][3] = o[b][3] * c1 + float(dd[3]) * s1;
    }
    __syncwarp();  // the stage is refilled at the next pair
  }
  at_wait<0>();

  // The chunk's own keys and values (float32 stage rows) on the CUDA cores: 16 groups of 8 lanes,
  // a key a group at a time, E = HD / 8 dimensions a lane; merged into the warp's second partial
  // (kept in the ring's shared memory, free once every warp is past its pages).
  constexpr int E = HD / 8;
  const bool has_stage = kc1 < k1;  // uniform over the CTA
  __syncthreads();
  float *st_o = reinterpret_cast<float *>(at_buf);  // [warps][REP][HD]
  float *st_ml = st_o + kAtWarps * REP * HD;        // [warps][REP][2]
  if (has_stage) {
    const int grp = threadIdx.x >> 3, l8 = threadIdx.x & 7;
    float qv[REP][E], gm[REP], gl[REP], go[REP][E];
#pragma unroll
    for (int h = 0; h < REP; ++h) {
      gm[h] = -INFINITY;
      gl[h] = 0.f;
#pragma unroll
      for (int k = 0; k < E; ++k) {
        qv[h][k] = qh[h * HD + l8 * E + k];
        go[h][k] = 0.f;
      }
    }
    for (int j0 = kc1; j0 < k1; j0 += kAtWarps * 4) {  // 16 groups; the same trip count on every lane
      const int j = j0 + grp;
      const bool valid = j < k1;
      float kf[E], vf[E];
#pragma unroll
      for (int k = 0; k < E; ++k) kf[k] = vf[k] = 0.f;
      if (valid) {
        const float4 *kp = reinterpret_cast<const float4 *>(
            kv_stage + ((size_t(t - (P - j)) * 2) * g.kv_heads + kvh) * HD + l8 * E);
        const float4 *vp = kp + size_t(g.kv_heads) * HD / 4;
#pragma unroll
        for (int k = 0; k < E / 4; ++k) {
          const float4 x = kp[k], y = vp[k];
          kf[4 * k] = x.x; kf[4 * k + 1] = x.y; kf[4 * k + 2] = x.z; kf[4 * k + 3] = x.w;
          vf[4 * k] = y.x; vf[4 * k + 1] = y.y; vf[4 * k + 2] = y.z; vf[4 * k + 3] = y.w;
        }
      }
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        float dsum = 0.f;
#pragma unroll
        for (int k = 0; k < E; ++k) dsum = fmaf(qv[h][k], kf[k], dsum);
        dsum += __shfl_xor_sync(0xffffffffu, dsum, 1);
        dsum += __shfl_xor_sync(0xffffffffu, dsum, 2);
        dsum += __shfl_xor_sync(0xffffffffu, dsum, 4);
        if (valid) {
          const float sc = dsum * g.score_scale;
          const float mn = fmaxf(gm[h], sc);
          const float corr = gm[h] == -INFINITY ? 0.f : expf(gm[h] - mn), pp = expf(sc - mn);
          gl[h] = fmaf(gl[h], corr, pp);
#pragma unroll
          for (int k = 0; k < E; ++k) go[h][k] = fmaf(go[h][k], corr, pp * vf[k]);
          gm[h] = mn;
        }
      }
    }
    // the warp's 4 groups (lanes differing in bits 3 and 4)
#pragma unroll
    for (int h = 0; h < REP; ++h) {
      float M = gm[h];
      M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 8));
      M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
      const float f = gl[h] > 0.f ? expf(gm[h] - M) : 0.f;
      float L = gl[h] * f;
      L += __shfl_xor_sync(0xffffffffu, L, 8);
      L += __shfl_xor_sync(0xffffffffu, L, 16);
#pragma unroll
      for (int k = 0; k < E; ++k) {
        float v = go[h][k] * f;
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (lane < 8) st_o[(warp * REP + h) * HD + l8 * E + k] = v;
      }
      if (lane == 0) {
        st_ml[(warp * REP + h) * 2] = M;
        st_ml[(warp * REP + h) * 2 + 1] = L;
      }
    }
  }

  // this warp's (m, l) per head (score row h: lane 4 h) and its values: the hi columns, then the
  // lo columns added (already in the same units)
  if (cq == 0 && gq < REP) {
    sm_m[warp][gq] = m_r;
    sm_l[warp][gq] = l_r;
  }
#pragma unroll
  for (int b = 0; b < DB; ++b) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = 2 * cq + (e & 1), dim = 16 * b + gq + 8 * (e >> 1);
      if (col < REP) sm_o[warp][col][dim] = o[b][e];
    }
  }
  __syncwarp();
#pragma unroll
  for (int b = 0; b < DB; ++b) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = 2 * cq + (e & 1), dim = 16 * b + gq + 8 * (e >> 1);
      if (col >= REP && col < 2 * REP) sm_o[warp][col - REP][dim] += o[b][e];
    }
  }
  __syncthreads();
  // the warps' partials (and the stage keys' ones) into the split's (m, l) and unnormalised o, as
  // attn_split_kernel
  for (int r = 0; r < REP; ++r) {
    float pm[2 * kAtWarps], pl[2 * kAtWarps];
#pragma unroll
    for (int w = 0; w < kAtWarps; ++w) {
      pm[w] = sm_m[w][r];
      pl[w] = sm_l[w][r];
      pm[kAtWarps + w] = has_stage ? st_ml[(w * REP + r) * 2] : -INFINITY;
      pl[kAtWarps + w] = has_stage ? st_ml[(w * REP + r) * 2 + 1] : 0.f;
    }
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 2 * kAtWarps; ++w)
      if (pl[w] > 0.f) M = fmaxf(M, pm[w]);
    float fw[2 * kAtWarps], L = 0.f;
#pragma unroll
    for (int w = 0; w < 2 * kAtWarps; ++w) {
      fw[w] = pl[w] > 0.f ? expf(pm[w] - M) : 0.f;
      L += pl[w] * fw[w];
    }
    const size_t pi = (size_t(t) * g.heads + kvh * REP + r) * splits + s;
    if (threadIdx.x == 0) {
      part_ml[pi * 2] = M;
      part_ml[pi * 2 + 1] = L;
    }
    for (int e = threadIdx.x; e < HD; e += blockDim.x) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kAtWarps; ++w) {
        acc = fmaf(sm_o[w][r][e], fw[w], acc);
        if (has_stage) acc = fmaf(st_o[(w * REP + r) * HD + e], fw[kAtWarps + w], acc);
      }
      part_o[pi * HD + e] = acc;
    }
  }
}

}  // namespace

char *attn_tc_prepare() {
#define HC_AT(D, R)                                                                                   \
  HC_TRY_CUDA(cudaFuncSetAttribute(attn_paged_tc_kernel<D, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   int(at_smem(D))));
  HC_AT(128, 1) HC_AT(128, 2) HC_AT(128, 4) HC_AT(64, 1) HC_AT(64, 2) HC_AT(64, 4)
#undef HC_AT
  return nullptr;
}

bool attn_paged_tc(const float *q, const StepTok *toks, int ntok, const AttnGeom &g, const PagedKV &pk, int splits,
                   float *part_ml, float *part_o, const float *kv_stage, cudaStream_t st) {
  const int rep = g.heads / g.kv_heads;
  if ((g.hd != 64 && g.hd != 128) || (rep != 1 && rep != 2 && rep != 4)) return false;
  const dim3 grid(splits, g.kv_heads, ntok);
#define HC_AT(D, R)                                                                                         \
  if (g.hd == D && rep == R) {                                                                              \
    launch_pdl(attn_paged_tc_kernel<D, R>, grid, dim3(kAtWarps * 32), at_smem(D), st, q, toks, g, pk, splits, \
               part_ml, part_o, kv_stage);                                                                  \
    return true;                                                                                            \
  }
  HC_AT(128, 1) HC_AT(128, 2) HC_AT(128, 4) HC_AT(64, 1) HC_AT(64, 2) HC_AT(64, 4)
#undef HC_AT
  return false;
}

}  // namespace hc
