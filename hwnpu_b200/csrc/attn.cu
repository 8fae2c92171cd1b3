// attn.cu: the attention side of a decode step: per-head RMS norm, RoPE and the KV-cache append
// (qwen3 builder.qkv, internal/llm/qwen3/build.go:261-289; blocks.ApplyRope, blocks.go:429-443),
// then split-K decode attention over the fp16 cache (blocks.SDPAGrouped blocks.go:516-539 with
// the online merge of paged.Merge, paged.go:227-310).
#include "device.cuh"
#include "kernels.h"

namespace hc {
namespace {


// One warp a head: E = hd / 32 values a lane, element e = lane + 32 k (so that RoPE's partner
// e +- hd/2 stays in the lane).
template <int E>
__global__ void __launch_bounds__(128) qkv_post_kernel(const float *__restrict__ qkv,
                                                       const StepTok *__restrict__ toks, int ntok,
                                                       AttnGeom g, const float *__restrict__ qn,
                                                       const float *__restrict__ kn,
                                                       float norm_scale, float eps16,
                                                       const uint32_t *__restrict__ rope,
                                                       float *__restrict__ q_out,
                                                       uint16_t *__restrict__ kcache,
                                                       uint16_t *__restrict__ vcache,
                                                       float *__restrict__ kv_stage) {
  pdl_trigger();
  pdl_wait();
  const int hd = E * 32, half = hd / 2;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int per_tok = g.heads + g.kv_heads;
  if (gw >= ntok * per_tok) return;
  const int t = gw / per_tok, hh = gw % per_tok;
  const StepTok tk = toks[t];
  const int width = (g.heads + 2 * g.kv_heads) * hd;
  const bool is_q = hh < g.heads;
  const int kvh = hh - g.heads;
  const float *src = qkv + size_t(t) * width + size_t(is_q ? hh : g.heads + kvh) * hd;
  const float *nw = is_q ? qn : kn;
  float x[E];
#pragma unroll
  for (int k = 0; k < E; ++k) x[k] = src[lane + 32 * k];
  if (nw) {
    // qwen3's norm over the head (build.go:283-284): the squares of x/scale, eps16
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
  {
    // RoPE: x*cos + rotate_half(x)*sin with the fp16 tables of position pos
    const uint32_t *rt = rope + size_t(tk.pos) * half;
    float y[E];
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const int e = lane + 32 * k;
      const int j = e < half ? e : e - half;
      const uint32_t cs = rt[j];
      const float c = __half2float(__ushort_as_half(uint16_t(cs & 0xffff)));
      const float s = __half2float(__ushort_as_half(uint16_t(cs >> 16)));
      const int kp = e < half ? k + (half / 32) : k - (half / 32);
      const float rot = e < half ? -x[kp] : x[kp];
      y[k] = __fadd_rn(__fmul_rn(x[k], c), __fmul_rn(rot, s));
    }
    if (is_q) {
      float *dst = q_out + (size_t(t) * g.heads + hh) * hd;
#pragma unroll
      for (int k = 0; k < E; ++k) dst[lane + 32 * k] = y[k];
      return;
    }
    const float *vs = qkv + size_t(t) * width + size_t(g.heads + g.kv_heads + kvh) * hd;
    // the stage rows ([t][k|v][kv head][hd] float32): the chunk's attention and kv_append_int8
    float *kd = kv_stage + ((size_t(t) * 2) * g.kv_heads + kvh) * hd;
    float *vd = kd + size_t(g.kv_heads) * hd;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      kd[lane + 32 * k] = y[k];
      vd[lane + 32 * k] = vs[lane + 32 * k];
    }
    if (!kcache) return;
    const size_t row = ((size_t(tk.slot) * g.kv_heads + kvh) * g.cap + tk.pos) * hd;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      kcache[row + lane + 32 * k] = __half_as_ushort(__float2half_rn(y[k]));
      vcache[row + lane + 32 * k] = __half_as_ushort(__float2half_rn(vs[lane + 32 * k]));
    }
  }
}

// One CTA per (split, kv head, token). Its 16 groups of 8 lanes each take a key at a time (8 lanes
// cover the key's head_dim in 16-byte loads, so a warp has 4 keys in flight), keeping an online
// softmax for every query head of the kv head's group (GQA: heads kvh*REP .. kvh*REP+REP-1);
// the groups then merge, first within a warp by shuffles, then across the 4 warps in smem.
template <int HD, int REP, bool PAGED>
__global__ void __launch_bounds__(128) attn_split_kernel(const float *__restrict__ q,
                                                         const StepTok *__restrict__ toks,
                                                         AttnGeom g,
                                                         const uint16_t *__restrict__ kcache,
                                                         const uint16_t *__restrict__ vcache,
                                                         PagedKV pk,
                                                         int splits, float *__restrict__ part_ml,
                                                         float *__restrict__ part_o,
                                                         const float *__restrict__ kv_stage) {
  pdl_trigger();
  pdl_wait();
  constexpr int E = HD / 8;  // elements a lane: 16 (hd 128) or 8 (hd 64)
  __shared__ float sm_m[4][REP], sm_l[4][REP];
  __shared__ float sm_o[4][REP][HD];
  const int s = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = threadIdx.x >> 3, l8 = threadIdx.x & 7;
  const StepTok tk = toks[t];
  const int P = tk.pos;
  const int lo = g.window > 0 ? max(0, P - g.window + 1) : 0;
  const int n = P - lo + 1;
  const int chunk = (n + splits - 1) / splits;
  const int k0 = lo + s * chunk, k1 = min(P + 1, k0 + chunk);
  // positions from p0 on are this token's piece: float32 stage rows (row t - (P - j) for key j)
  const int p0 = tk.run0 >= 0 ? P - (t - tk.run0) : P + 1;
  const int kc1 = min(k1, max(k0, p0));  // cached keys [k0, kc1), stage keys [kc1, k1)
  float qv[REP][E];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    const float4 *qp = reinterpret_cast<const float4 *>(q + (size_t(t) * g.heads + kvh * REP + r) * HD + l8 * E);
#pragma unroll
    for (int k = 0; k < E / 4; ++k) {
      const float4 v = qp[k];
      qv[r][4 * k] = v.x; qv[r][4 * k + 1] = v.y; qv[r][4 * k + 2] = v.z; qv[r][4 * k + 3] = v.w;
    }
  }
  float m[REP], l[REP], o[REP][E];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) o[r][k] = 0.f;
  }
  const size_t base = (size_t(tk.slot) * g.kv_heads + kvh) * size_t(g.cap) * HD;
  // key j sits at slot j mod cap: the slot itself in a linear cache (every key below cap), a ring
  // otherwise; the split's keys span less than cap, so one wrap at most
  const int slot0 = k0 % g.cap;
  // the trip count is the same for every lane (the shuffles below take the whole warp); a group
  // whose key is past the chunk's end loads nothing and leaves its softmax as it is. The loads of
  // a group's next key are issued before the current key's arithmetic (one key in flight ahead).
  constexpr int KW = PAGED ? E / 4 : E / 2;  // 32-bit words of a lane's part of a K (or V) row
  struct Raw {
    uint32_t k[KW], v[KW];
    float ks, vs;
  };
  auto fetch = [&](int j, Raw &r) {
#pragma unroll
    for (int i = 0; i < KW; ++i) r.k[i] = r.v[i] = 0u;
    r.ks = r.vs = 0.f;
    if (j >= kc1) return;
    const uint32_t *kp, *vp;
    if (PAGED) {
      // key j of the sequence: row j % 16 of its page, int8 times the (page, head) scale
      const int page = pk.btab[size_t(tk.slot) * pk.max_pages + j / kPage];
      const size_t ph = size_t(page) * g.kv_heads + kvh;
      r.ks = __half2float(__ushort_as_half(pk.kscale[ph]));
      r.vs = __half2float(__ushort_as_half(pk.vscale[ph]));
      kp = reinterpret_cast<const uint32_t *>(pk.k + (ph * kPage + j % kPage) * HD + l8 * E);
      // the page's values are transposed ([dim][position]): this lane's E dims of key j, a byte each
      const int8_t *vb = pk.v + ph * kPage * HD + size_t(l8 * E) * kPage + j % kPage;
#pragma unroll
      for (int i = 0; i < KW; ++i)
        r.v[i] = uint32_t(uint8_t(vb[(4 * i) * kPage])) | (uint32_t(uint8_t(vb[(4 * i + 1) * kPage])) << 8) |
                 (uint32_t(uint8_t(vb[(4 * i + 2) * kPage])) << 16) | (uint32_t(uint8_t(vb[(4 * i + 3) * kPage])) << 24);
      vp = nullptr;
    } else {
      int sl = slot0 + (j - k0);
      if (sl >= g.cap) sl -= g.cap;
      kp = reinterpret_cast<const uint32_t *>(kcache + base + size_t(sl) * HD + l8 * E);
      vp = reinterpret_cast<const uint32_t *>(vcache + base + size_t(sl) * HD + l8 * E);
    }
    if (KW % 4 == 0) {
#pragma unroll
      for (int i = 0; i < KW / 4; ++i) {
        const uint4 a = reinterpret_cast<const uint4 *>(kp)[i];
        r.k[4 * i] = a.x; r.k[4 * i + 1] = a.y; r.k[4 * i + 2] = a.z; r.k[4 * i + 3] = a.w;
        if (!PAGED) {
          const uint4 b = reinterpret_cast<const uint4 *>(vp)[i];
          r.v[4 * i] = b.x; r.v[4 * i + 1] = b.y; r.v[4 * i + 2] = b.z; r.v[4 * i + 3] = b.w;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < KW / 2; ++i) {
        const uint2 a = reinterpret_cast<const uint2 *>(kp)[i];
        r.k[2 * i] = a.x; r.k[2 * i + 1] = a.y;
        if (!PAGED) {
          const uint2 b = reinterpret_cast<const uint2 *>(vp)[i];
          r.v[2 * i] = b.x; r.v[2 * i + 1] = b.y;
        }
      }
    }
  };
  // one key of the online softmax for every query head of the group
  auto step = [&](const float (&kf)[E], const float (&vf)[E], bool valid) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float d = 0.f;
#pragma unroll
      for (int k = 0; k < E; ++k) d = fmaf(qv[r][k], kf[k], d);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      if (valid) {
        const float sc = d * g.score_scale;
        const float mn = fmaxf(m[r], sc);
        const float corr = expf(m[r] - mn), p = expf(sc - mn);
        l[r] = fmaf(l[r], corr, p);
#pragma unroll
        for (int k = 0; k < E; ++k) o[r][k] = fmaf(o[r][k], corr, p * vf[k]);
        m[r] = mn;
      }
    }
  };
  Raw cur;
  fetch(k0 + grp, cur);
  for (int j0 = k0; j0 < kc1; j0 += 16) {
    const int j = j0 + grp;
    const bool valid = j < kc1;
    Raw nxt;
    fetch(j + 16, nxt);
    float kf[E], vf[E];
    if (PAGED) {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        kf[i] = float(int8_t((cur.k[i / 4] >> (8 * (i % 4))) & 0xff)) * cur.ks;
        vf[i] = float(int8_t((cur.v[i / 4] >> (8 * (i % 4))) & 0xff)) * cur.vs;
      }
    } else {
#pragma unroll
      for (int i = 0; i < E / 2; ++i) {
        const __half2 k2 = *reinterpret_cast<const __half2 *>(&cur.k[i]);
        const __half2 v2 = *reinterpret_cast<const __half2 *>(&cur.v[i]);
        kf[2 * i] = __low2float(k2); kf[2 * i + 1] = __high2float(k2);
        vf[2 * i] = __low2float(v2); vf[2 * i + 1] = __high2float(v2);
      }
    }
    step(kf, vf, valid);
    cur = nxt;
  }
  // the piece's own keys and values, float32 from the stage rows
  for (int j0 = kc1; j0 < k1; j0 += 16) {
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
        const float4 a = kp[k], b = vp[k];
        kf[4 * k] = a.x; kf[4 * k + 1] = a.y; kf[4 * k + 2] = a.z; kf[4 * k + 3] = a.w;
        vf[4 * k] = b.x; vf[4 * k + 1] = b.y; vf[4 * k + 2] = b.z; vf[4 * k + 3] = b.w;
      }
    }
    step(kf, vf, valid);
  }
  // merge the 4 groups of the warp (lanes differing in bits 3 and 4)
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float M = m[r];
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 8));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
    const float f = l[r] > 0.f ? expf(m[r] - M) : 0.f;
    float L = l[r] * f;
    L += __shfl_xor_sync(0xffffffffu, L, 8);
    L += __shfl_xor_sync(0xffffffffu, L, 16);
#pragma unroll
    for (int k = 0; k < E; ++k) {
      float v = o[r][k] * f;
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      o[r][k] = v;
    }
    if (lane < 8) {
#pragma unroll
      for (int k = 0; k < E; ++k) sm_o[warp][r][l8 * E + k] = o[r][k];
    }
    if (lane == 0) { sm_m[warp][r] = M; sm_l[warp][r] = L; }
  }
  __syncthreads();
  // merge the 4 warps: thread e of the CTA takes element e of every head of the group
  for (int r = 0; r < REP; ++r) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w)
      if (sm_l[w][r] > 0.f) M = fmaxf(M, sm_m[w][r]);
    float fw[4], L = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      fw[w] = sm_l[w][r] > 0.f ? expf(sm_m[w][r] - M) : 0.f;
      L += sm_l[w][r] * fw[w];
    }
    const size_t pi = (size_t(t) * g.heads + kvh * REP + r) * splits + s;
    if (threadIdx.x == 0) {
      part_ml[pi * 2] = M;
      part_ml[pi * 2 + 1] = L;
    }
    for (int e = threadIdx.x; e < HD; e += blockDim.x) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) acc = fmaf(sm_o[w][r][e], fw[w], acc);
      part_o[pi * HD + e] = acc;
    }
  }
}

}  // namespace

void qkv_post(const float *qkv, const StepTok *toks, int ntok, const AttnGeom &g, const float *qn,
              const float *kn, float norm_scale, float eps16, const uint32_t *rope, float *q_out,
              uint16_t *kcache, uint16_t *vcache, float *kv_stage, cudaStream_t st) {
  const int warps = ntok * (g.heads + g.kv_heads);
  const int grid = (warps + 3) / 4;
  if (g.hd == 128)
    launch_pdl(qkv_post_kernel<4>, dim3(grid), dim3(128), 0, st, qkv, toks, ntok, g, qn, kn, norm_scale, eps16, rope,
               q_out, kcache, vcache, kv_stage);
  else
    launch_pdl(qkv_post_kernel<2>, dim3(grid), dim3(128), 0, st, qkv, toks, ntok, g, qn, kn, norm_scale, eps16, rope,
               q_out, kcache, vcache, kv_stage);
}

void attn_split(const float *q, const StepTok *toks, int ntok, const AttnGeom &g,
                const uint16_t *kcache, const uint16_t *vcache, int splits, float *part_ml,
                float *part_o, cudaStream_t st, const PagedKV *paged, const float *kv_stage) {
  if (paged && attn_paged_tc(q, toks, ntok, g, *paged, splits, part_ml, part_o, kv_stage, st)) return;
  dim3 grid(splits, g.kv_heads, ntok);
  const int rep = g.heads / g.kv_heads;
  const PagedKV pk = paged ? *paged : PagedKV{};
#define HC_ATT(D, R)                                                                          \
  if (g.hd == D && rep == R) {                                                                \
    if (paged)                                                                                \
      launch_pdl(attn_split_kernel<D, R, true>, grid, dim3(128), 0, st, q, toks, g, kcache,   \
                 vcache, pk, splits, part_ml, part_o, kv_stage);                              \
    else                                                                                      \
      launch_pdl(attn_split_kernel<D, R, false>, grid, dim3(128), 0, st, q, toks, g, kcache,  \
                 vcache, pk, splits, part_ml, part_o, kv_stage);                              \
    return;                                                                                   \
  }
  HC_ATT(128, 1) HC_ATT(128, 2) HC_ATT(128, 4) HC_ATT(128, 8)
  HC_ATT(64, 1) HC_ATT(64, 2) HC_ATT(64, 4) HC_ATT(64, 8)
#undef HC_ATT
}

// Appends the chunk's new key and value rows (float32 from qkv_post) to the paged int8 cache. The
// tokens of one sequence are consecutive in a chunk (a sequence is listed once a call), so the
// chunk splits into runs of tokens that write the same page; one CTA a (run, kv head, key | value)
// (the CTA of the run's first token; the others return at once). The cache's rule is sequential: a
// page's scale is the fp16 rounding up of max|x| / 127 over its rows; when a new row needs a larger
// scale, the rows already in the page are requantised to it (q' = round_even(q * s_old / s_new)),
// so every value stays within [-127, 127]. Rows interact only through that sequence of scales, so
// the CTA takes the run's row maxima, walks them once for the scale each row is written at and the
// requantisations that follow it, and then every value takes its own chain at once: an earlier row
// of the page through all of the run's requantisations, a new row through those after it. The
// result is the row-by-row one exactly.
template <int HD>
__global__ void __launch_bounds__(128) kv_append_int8_kernel(const float *__restrict__ stage,
                                                            const StepTok *__restrict__ toks, int ntok,
                                                            int kv_heads, PagedKV pk) {
  constexpr int E = HD / 32;
  __shared__ float s_max[kPage], s_sr[kPage], s_ef[kPage];
  __shared__ int s_er[kPage], s_nev;
  __shared__ float s_final;
  pdl_trigger();
  pdl_wait();
  const int t0 = blockIdx.x / (2 * kv_heads), kvh = (blockIdx.x >> 1) % kv_heads, is_v = blockIdx.x & 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto same_page = [&](const StepTok &a, const StepTok &b) { return a.slot == b.slot && a.pos / kPage == b.pos / kPage; };
  if (t0 > 0 && same_page(toks[t0 - 1], toks[t0])) return;  // not the first token of its run (uniform)
  const StepTok tk0 = toks[t0];
  int R = 1;
  while (t0 + R < ntok && R < kPage && same_page(tk0, toks[t0 + R])) ++R;
  const int off0 = tk0.pos % kPage;
  const int page = pk.btab[size_t(tk0.slot) * pk.max_pages + tk0.pos / kPage];
  const size_t ph = size_t(page) * kv_heads + kvh;
  int8_t *pg = const_cast<int8_t *>(is_v ? pk.v : pk.k) + ph * kPage * HD;
  uint16_t *scales = const_cast<uint16_t *>(is_v ? pk.vscale : pk.kscale);
  // warp w holds rows w, w + 4, w + 8, w + 12 of the run (E values a lane) and their maxima
  float x[kPage / 4][E];
#pragma unroll
  for (int i = 0; i < kPage / 4; ++i) {
    const int r = warp + 4 * i;
    float m = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      x[i][k] = r < R ? stage[((size_t(t0 + r) * 2 + is_v) * kv_heads + kvh) * HD + lane + 32 * k] : 0.f;
      m = fmaxf(m, fabsf(x[i][k]));
    }
    m = warp_max(m);
    if (lane == 0 && r < R) s_max[r] = m;
  }
  __syncthreads();
  const float s_first = off0 == 0 ? 0.f : __half2float(__ushort_as_half(scales[ph]));
  if (threadIdx.x == 0) {
    float sc = s_first;
    int nev = 0;
    for (int r = 0; r < R; ++r) {
      const float m = s_max[r];
      if (m / 127.0f > sc) {
        const float s_new = __half2float(__float2half_ru(m / 127.0f));
        if (off0 + r > 0 && sc > 0.f) {
          s_ef[nev] = sc / s_new;
          s_er[nev] = r;
          ++nev;
        }
        sc = s_new;
      }
      s_sr[r] = sc;
    }
    s_nev = nev;
    s_final = sc;
  }
  __syncthreads();
  const int nev = s_nev;
  auto requant = [](float q, float f) { return fminf(fmaxf(rintf(q * f), -127.f), 127.f); };
  if (off0 > 0 && nev > 0) {
    // the page's earlier rows through every requantisation of the run: keys rows 0..off0-1
    // (contiguous), values the whole 16-byte row of each dimension (bytes past off0 are written below)
    uint4 *rows = reinterpret_cast<uint4 *>(pg);
    const int n16 = is_v ? HD : off0 * HD / 16;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) {
      uint4 w = rows[i];
      uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t o = 0;
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          float q = float(int8_t((u[k] >> (8 * bb)) & 0xff));
          for (int e = 0; e < nev; ++e) q = requant(q, s_ef[e]);
          o |= uint32_t(uint8_t(int8_t(q))) << (8 * bb);
        }
        u[k] = o;
      }
      rows[i] = make_uint4(u[0], u[1], u[2], u[3]);
    }
    __syncthreads();
  }
  // the new rows: each at its own scale, then through the requantisations after it
#pragma unroll
  for (int i = 0; i < kPage / 4; ++i) {
    const int r = warp + 4 * i;
    if (r >= R) continue;
    const float sr = s_sr[r];
    const float inv = sr > 0.f ? 1.0f / sr : 0.f;
    const int off = off0 + r;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      float q = fminf(fmaxf(rintf(x[i][k] * inv), -127.f), 127.f);
      for (int e = 0; e < nev; ++e)
        if (s_er[e] > r) q = requant(q, s_ef[e]);
      // keys row-major [position][dim]; values transposed [dim][position]
      if (is_v) pg[(lane + 32 * k) * kPage + off] = int8_t(q);
      else pg[off * HD + lane + 32 * k] = int8_t(q);
    }
  }
  if (threadIdx.x == 0 && s_final != s_first) scales[ph] = __half_as_ushort(__float2half_rn(s_final));
}

void kv_append_int8(const float *stage, const StepTok *toks, int ntok, int kv_heads, int hd, const PagedKV &pk,
                    cudaStream_t st) {
  const int grid = 2 * kv_heads * ntok;  // a CTA a (token, kv head, key | value)
  if (hd == 128)
    launch_pdl(kv_append_int8_kernel<128>, dim3(grid), dim3(128), 0, st, stage, toks, ntok, kv_heads, pk);
  else
    launch_pdl(kv_append_int8_kernel<64>, dim3(grid), dim3(128), 0, st, stage, toks, ntok, kv_heads, pk);
}

}  // namespace hc
