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
                                                       uint16_t *__restrict__ vcache) {
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
    const size_t row = ((size_t(tk.slot) * g.kv_heads + kvh) * g.cap + tk.pos) * hd;
    const float *vs = qkv + size_t(t) * width + size_t(g.heads + g.kv_heads + kvh) * hd;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      kcache[row + lane + 32 * k] = __half_as_ushort(__float2half_rn(y[k]));
      vcache[row + lane + 32 * k] = __half_as_ushort(__float2half_rn(vs[lane + 32 * k]));
    }
  }
}

// One CTA per (split, kv head, token), 4 warps over its keys; each warp keeps an online softmax
// per query head of the group (GQA: heads kvh*rep .. kvh*rep+rep-1 read kv head kvh).
template <int E, int REP>
__global__ void __launch_bounds__(128) attn_split_kernel(const float *__restrict__ q,
                                                         const StepTok *__restrict__ toks,
                                                         AttnGeom g,
                                                         const uint16_t *__restrict__ kcache,
                                                         const uint16_t *__restrict__ vcache,
                                                         int splits, float *__restrict__ part_ml,
                                                         float *__restrict__ part_o) {
  constexpr int hd = E * 32;
  constexpr int rep = REP;
  __shared__ float sm_m[4][REP], sm_l[4][REP];
  __shared__ float sm_o[4][REP][hd];
  const int s = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const StepTok tk = toks[t];
  const int P = tk.pos;
  const int lo = g.window > 0 ? max(0, P - g.window + 1) : 0;
  const int n = P - lo + 1;
  const int chunk = (n + splits - 1) / splits;
  const int k0 = lo + s * chunk, k1 = min(P + 1, k0 + chunk);
  float qv[REP][E];
#pragma unroll
  for (int r = 0; r < rep; ++r)
#pragma unroll
    for (int k = 0; k < E; ++k)
      qv[r][k] = q[(size_t(t) * g.heads + kvh * rep + r) * hd + lane * E + k];
  float m[REP], l[REP], o[REP][E];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) o[r][k] = 0.f;
  }
  const size_t base = (size_t(tk.slot) * g.kv_heads + kvh) * size_t(g.cap) * hd;
  for (int j = k0 + warp; j < k1; j += 4) {
    const uint16_t *kr = kcache + base + size_t(j) * hd + lane * E;
    const uint16_t *vr = vcache + base + size_t(j) * hd + lane * E;
    float kf[E], vf[E];
    if constexpr (E == 4) {
      const uint2 kk = *reinterpret_cast<const uint2 *>(kr);
      const uint2 vv = *reinterpret_cast<const uint2 *>(vr);
      const __half2 k01 = *reinterpret_cast<const __half2 *>(&kk.x), k23 = *reinterpret_cast<const __half2 *>(&kk.y);
      const __half2 v01 = *reinterpret_cast<const __half2 *>(&vv.x), v23 = *reinterpret_cast<const __half2 *>(&vv.y);
      kf[0] = __low2float(k01); kf[1] = __high2float(k01); kf[2] = __low2float(k23); kf[3] = __high2float(k23);
      vf[0] = __low2float(v01); vf[1] = __high2float(v01); vf[2] = __low2float(v23); vf[3] = __high2float(v23);
    } else {
#pragma unroll
      for (int k = 0; k < E; ++k) {
        kf[k] = __half2float(__ushort_as_half(kr[k]));
        vf[k] = __half2float(__ushort_as_half(vr[k]));
      }
    }
#pragma unroll
    for (int r = 0; r < rep; ++r) {
      float d = 0.f;
#pragma unroll
      for (int k = 0; k < E; ++k) d = fmaf(qv[r][k], kf[k], d);
      d = warp_sum(d);
      const float sc = d * g.score_scale;
      if (sc > m[r]) {
        const float corr = expf(m[r] - sc);
        l[r] *= corr;
#pragma unroll
        for (int k = 0; k < E; ++k) o[r][k] *= corr;
        m[r] = sc;
      }
      const float p = expf(sc - m[r]);
      l[r] += p;
#pragma unroll
      for (int k = 0; k < E; ++k) o[r][k] = fmaf(p, vf[k], o[r][k]);
    }
  }
#pragma unroll
  for (int r = 0; r < rep; ++r) {
    if (lane == 0) { sm_m[warp][r] = m[r]; sm_l[warp][r] = l[r]; }
#pragma unroll
    for (int k = 0; k < E; ++k) sm_o[warp][r][lane * E + k] = o[r][k];
  }
  __syncthreads();
  // warp r' merges head r' of the group (4 warps, rep up to 8: loop)
  for (int r = warp; r < rep; r += 4) {
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w)
      if (sm_l[w][r] > 0.f) M = fmaxf(M, sm_m[w][r]);
    float L = 0.f;
    for (int w = 0; w < 4; ++w)
      if (sm_l[w][r] > 0.f) L += sm_l[w][r] * expf(sm_m[w][r] - M);
    const int h = kvh * rep + r;
    const size_t pi = (size_t(t) * g.heads + h) * splits + s;
    if (lane == 0) {
      part_ml[pi * 2] = M;
      part_ml[pi * 2 + 1] = L;
    }
    for (int e = lane; e < hd; e += 32) {
      float acc = 0.f;
      for (int w = 0; w < 4; ++w)
        if (sm_l[w][r] > 0.f) acc += sm_o[w][r][e] * expf(sm_m[w][r] - M);
      part_o[pi * hd + e] = acc;
    }
  }
}

}  // namespace

void qkv_post(const float *qkv, const StepTok *toks, int ntok, const AttnGeom &g, const float *qn,
              const float *kn, float norm_scale, float eps16, const uint32_t *rope, float *q_out,
              uint16_t *kcache, uint16_t *vcache, cudaStream_t st) {
  const int warps = ntok * (g.heads + g.kv_heads);
  const int grid = (warps + 3) / 4;
  if (g.hd == 128)
    qkv_post_kernel<4><<<grid, 128, 0, st>>>(qkv, toks, ntok, g, qn, kn, norm_scale, eps16, rope, q_out, kcache, vcache);
  else
    qkv_post_kernel<2><<<grid, 128, 0, st>>>(qkv, toks, ntok, g, qn, kn, norm_scale, eps16, rope, q_out, kcache, vcache);
}

void attn_split(const float *q, const StepTok *toks, int ntok, const AttnGeom &g,
                const uint16_t *kcache, const uint16_t *vcache, int splits, float *part_ml,
                float *part_o, cudaStream_t st) {
  dim3 grid(splits, g.kv_heads, ntok);
  const int rep = g.heads / g.kv_heads;
#define HC_ATT(E, R)                                                                         \
  if (g.hd == E * 32 && rep == R) {                                                          \
    attn_split_kernel<E, R><<<grid, 128, 0, st>>>(q, toks, g, kcache, vcache, splits, part_ml, \
                                                  part_o);                                   \
    return;                                                                                  \
  }
  HC_ATT(4, 1) HC_ATT(4, 2) HC_ATT(4, 4) HC_ATT(4, 8)
  HC_ATT(2, 1) HC_ATT(2, 2) HC_ATT(2, 4) HC_ATT(2, 8)
#undef HC_ATT
}

}  // namespace hc
