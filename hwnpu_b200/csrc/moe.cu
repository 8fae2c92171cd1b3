// moe.cu: the gpt-oss side of a decode step (internal/llm/gptoss, internal/llm/experts): RMS norms
// to float32 rows, the 16-bit-float GEMV of its bf16 attention, router and head (and the router's
// fp16 weights), and the mixture of experts on the device -- the token-grouped MXFP4 expert GEMVs
// (mxfp4.Run reads an expert's rows once for all the rows that chose it, matvec.go:33-160), gpt-oss's
// gated unit, and the ascending-expert combine of experts.Host.runRow (host.go:478-591).
#include <cuda_bf16.h>

#include "device.cuh"
#include "kernels.h"

namespace hc {
namespace {

__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }

// milcpu's RMS norm with a scale of 1 (act_quant_kernel's arithmetic: the squares summed in float64,
// r = float32(1 / sqrt(mean + eps16)), y = x r w), one CTA a row; round16: y rounded to fp16 (the
// program's fp16 output moe_x, gptoss/build.go:121-124).
__global__ void __launch_bounds__(256) rms_rows_kernel(const float *__restrict__ x, int ldx, int n,
                                                       const float *__restrict__ w, float eps16,
                                                       float *__restrict__ y, int ldy, int round16,
                                                       const StepTok *__restrict__ rows) {
  __shared__ double red[8];
  pdl_trigger();
  pdl_wait();
  const float *xt = x + size_t(rows ? rows[blockIdx.x].head_src : blockIdx.x) * ldx;
  double s = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xt[i];
    const float sq = v * v;
    s += double(sq);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  double tot = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += red[k];
  const float ms = float(tot / double(n));
  const float r = float(1.0 / sqrt(double(ms) + double(eps16)));
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = xt[i] * r;
    v = v * w[i];
    y[size_t(blockIdx.x) * ldy + i] = round16 ? f16_round(v) : v;
  }
}

template <bool BF16>
__device__ __forceinline__ void unpack8(const uint4 q, float (&f)[8]) {
  const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (BF16) {
      f[2 * i] = __uint_as_float(u[i] << 16);
      f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    } else {
      const __half2 h = *reinterpret_cast<const __half2 *>(&u[i]);
      f[2 * i] = __low2float(h);
      f[2 * i + 1] = __high2float(h);
    }
  }
}

// y = x W^T (+ bias) for up to NT tokens of float32 x, W 16-bit floats [rows][cols] (bf16 or fp16,
// cols a multiple of 8): a warp takes 2 rows, its lanes 16-byte pieces of them, each product in
// float32 (the weights' values are exact in it). Modes: 0 store, 1 add into y, 2 store rounded to
// fp16, 3 fp16 logits and the greedy key (argmax_key) folded into amax.
template <bool BF16, int NT>
__global__ void __launch_bounds__(256) gemv16_kernel(const uint16_t *__restrict__ W, int rows, int cols,
                                                     const float *__restrict__ x, int ldx, int ntok,
                                                     const float *__restrict__ bias, int mode,
                                                     float *__restrict__ y, int ldy, uint16_t *__restrict__ logits,
                                                     unsigned long long *__restrict__ amax) {
  __shared__ unsigned long long bmax[NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = (blockIdx.x * 8 + warp) * 2;
  if (threadIdx.x < NT) bmax[threadIdx.x] = 0ull;
  pdl_trigger();
  float acc[NT][2];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = 0.f;
  const int chunks = cols / 8;
  const uint4 *w0 = reinterpret_cast<const uint4 *>(W + size_t(r0) * cols);
  const uint4 *w1 = reinterpret_cast<const uint4 *>(W + size_t(r0 + 1) * cols);
  const bool has0 = r0 < rows, has1 = r0 + 1 < rows;
  pdl_wait();
  for (int c = lane; c < chunks; c += 32) {
    float a[8], b[8];
    const uint4 qa = has0 ? w0[c] : make_uint4(0, 0, 0, 0);
    const uint4 qb = has1 ? w1[c] : make_uint4(0, 0, 0, 0);
    unpack8<BF16>(qa, a);
    unpack8<BF16>(qb, b);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < ntok) {
        const float4 *xp = reinterpret_cast<const float4 *>(x + size_t(t) * ldx + size_t(c) * 8);
        const float4 u = __ldg(xp), v = __ldg(xp + 1);
        const float xv[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          acc[t][0] = fmaf(a[e], xv[e], acc[t][0]);
          acc[t][1] = fmaf(b[e], xv[e], acc[t][1]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    acc[t][0] = warp_sum(acc[t][0]);
    acc[t][1] = warp_sum(acc[t][1]);
  }
  if (lane < 2 && (lane ? has1 : has0)) {
    const int r = r0 + lane;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t >= ntok) continue;
      float v = acc[t][lane];
      if (bias) v += bias[r];
      float *dst = y ? y + size_t(t) * ldy + r : nullptr;
      if (mode == 0) {
        *dst = v;
      } else if (mode == 1) {
        *dst = *dst + v;
      } else if (mode == 2) {
        *dst = f16_round(v);
      } else {
        const uint16_t hb = __half_as_ushort(__float2half_rn(v));
        if (logits) logits[size_t(t) * ldy + r] = hb;
        atomicMax(&bmax[t], argmax_key(hb, uint32_t(r)));
      }
    }
  }
  if (mode == 3) {
    __syncthreads();
    if (threadIdx.x < NT && threadIdx.x < ntok)
      atomicMax(&amax[threadIdx.x * kAmaxSlots + (blockIdx.x % kAmaxSlots)], bmax[threadIdx.x]);
  }
}

// The rows of a step that chose each expert: pair p = t K + k (token t's k-th choice) goes to
// list[idx[p]][..]; cnt[e] is their number. One CTA.
__global__ void moe_group_kernel(const int32_t *__restrict__ idx, int npairs, int E, int *__restrict__ cnt,
                                 int *__restrict__ list, int maxp) {
  extern __shared__ int c[];
  pdl_trigger();
  pdl_wait();
  for (int e = threadIdx.x; e < E; e += blockDim.x) c[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
    const int e = idx[p];
    const int slot = atomicAdd(&c[e], 1);
    list[size_t(e) * maxp + slot] = p;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = c[e];
}

// The experts' MXFP4 GEMV, token-grouped: CTA (row tiles, expert e) reads e's rows once for every
// pair that chose e (8 at a time), each pair's activation tiles (the token's for gate/up, the pair's
// own for down: act_row = p / K or p) against the doubled e2m1 codes with integer block sums
// (wa_mma<kKindMx>, mxfp4.Vec.Quantize / dotGo's arithmetic). 8 warps; wpr of them split a row
// tile's column tiles. MODE 0: tiles of 8 gate then 8 up rows (gate_up's even and odd rows), plus
// their biases, through gpt-oss's gated unit (host.go:515-524) into out[p][o]; MODE 1: out[p][row].
template <int MODE>
__global__ void __launch_bounds__(256) moe_gemv_kernel(const uint8_t *__restrict__ tiles, int rt_e, int ktiles,
                                                       const int *__restrict__ cnt, const int *__restrict__ list,
                                                       int maxp, int K, const uint8_t *__restrict__ act,
                                                       const float *__restrict__ bias, int rows_e, float alpha,
                                                       float limit, int wpr, float *__restrict__ out, int ldo) {
  constexpr int NT = 8;
  __shared__ float part[8][NT][kTileRows];
  __shared__ int pairs[NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rpc = 8 / wpr, lrt = warp / wpr, ks = warp % wpr;
  const int e = blockIdx.y, rt = blockIdx.x * rpc + lrt;
  pdl_trigger();
  pdl_wait();
  const int n = cnt[e];
  const uint8_t *etiles = tiles + size_t(e) * rt_e * ktiles * kTileMx;
  for (int p0 = 0; p0 < n; p0 += NT) {
    const int np = min(NT, n - p0);
    if (threadIdx.x < NT) pairs[threadIdx.x] = threadIdx.x < np ? list[size_t(e) * maxp + p0 + threadIdx.x] : 0;
    __syncthreads();
    float vg[NT], vg8[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) vg[t] = vg8[t] = 0.f;
    if (rt < rt_e) {
      for (int kt = ks; kt < ktiles; kt += wpr) {
        WTile<kKindMx> wt;
        wt.load(etiles + (size_t(rt) * ktiles + kt) * kTileMx, lane);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < np) {
            const int arow = MODE == 0 ? pairs[t] / K : pairs[t];
            BFrag<kKindMx> bf;
            bf.load(act + (size_t(arow) * ktiles + kt) * kActTile, lane);
            wa_mma<kKindMx>(wt, bf, vg[t], vg8[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float a = quad_sum(vg[t]), b = quad_sum(vg8[t]);
      if (c == 0) {
        part[warp][t][g] = a;
        part[warp][t][g + 8] = b;
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < rpc * NT * kTileRows; i += blockDim.x) {
      const int l2 = i / (NT * kTileRows), t = (i / kTileRows) % NT, r16 = i % kTileRows;
      const int trow = blockIdx.x * rpc + l2;
      if (trow >= rt_e || t >= np) continue;
      auto value = [&](int rr) {
        float v = 0.f;
        for (int k = 0; k < wpr; ++k) v += part[l2 * wpr + k][t][rr];
        return v * 0.5f;  // the doubled e2m1 values (mxfp4.go:90)
      };
      const int p = pairs[t];
      if (MODE == 0) {
        if (r16 >= kTileRows / 2) continue;
        const int o = trow * (kTileRows / 2) + r16;
        if (o >= rows_e / 2) continue;
        const float *be = bias + size_t(e) * rows_e;
        const float gate = value(r16) + be[2 * o], up = value(r16 + kTileRows / 2) + be[2 * o + 1];
        const float gg = fminf(gate, limit);
        const float uu = fminf(fmaxf(up, -limit), limit);
        out[size_t(p) * ldo + o] = gg / (1.0f + float(exp(double(-(alpha * gg))))) * (uu + 1.0f);
      } else {
        const int row = trow * kTileRows + r16;
        if (row < rows_e) out[size_t(p) * ldo + row] = value(r16);
      }
    }
    __syncthreads();
  }
}

// The experts' weighted sum of one token (host.go:578-590: added in ascending expert number, each
// out += w_k (y + down bias)), its fp16 rounding (moe_o), and the next part's residual
// x = f16(h) + moe_o, the residual h rounded as the part's fp16 output (gptoss/build.go:60-88).
__global__ void moe_combine_kernel(const float *__restrict__ y, const int32_t *__restrict__ idx,
                                   const float *__restrict__ w, int K, const float *__restrict__ dbias, int H,
                                   float *__restrict__ x) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.y;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= H) return;
  int order[8];
  for (int k = 0; k < K; ++k) order[k] = k;
  for (int a = 1; a < K; ++a)  // a stable insertion sort by expert number
    for (int b = a; b > 0 && idx[t * K + order[b - 1]] > idx[t * K + order[b]]; --b) {
      const int tmp = order[b];
      order[b] = order[b - 1];
      order[b - 1] = tmp;
    }
  float out = 0.f;
  for (int i = 0; i < K; ++i) {
    const int k = order[i], e = idx[t * K + k];
    out += w[t * K + k] * (y[(size_t(t) * K + k) * H + col] + dbias[size_t(e) * H + col]);
  }
  float *xp = x + size_t(t) * H + col;
  *xp = f16_round(*xp) + f16_round(out);
}

}  // namespace

void rms_rows(const float *x, int ldx, int n, int ntok, const float *w, float eps16, float *y, int ldy, bool round16,
              cudaStream_t st, const StepTok *rows) {
  launch_pdl(rms_rows_kernel, dim3(ntok), dim3(256), 0, st, x, ldx, n, w, eps16, y, ldy, int(round16), rows);
}

void gemv16(const DevDense &W, const float *x, int ldx, int ntok, int mode, float *y, int ldy, uint16_t *logits,
            unsigned long long *amax, cudaStream_t st) {
  const int grid = (W.rows + 15) / 16;
  for (int t0 = 0; t0 < ntok; t0 += 8) {
    const int n = std::min(8, ntok - t0);
    const float *xt = x + size_t(t0) * ldx;
    float *yt = y ? y + size_t(t0) * ldy : nullptr;
    uint16_t *lt = logits ? logits + size_t(t0) * ldy : nullptr;
    unsigned long long *at = amax ? amax + size_t(t0) * kAmaxSlots : nullptr;
#define HC_G16(B, N)                                                                                     \
  launch_pdl(gemv16_kernel<B, N>, dim3(grid), dim3(256), 0, st, W.w, W.rows, W.cols, xt, ldx, n, W.bias, \
             mode, yt, ldy, lt, at)
    if (W.bf16) {
      if (n == 1) HC_G16(true, 1); else if (n <= 4) HC_G16(true, 4); else HC_G16(true, 8);
    } else {
      if (n == 1) HC_G16(false, 1); else if (n <= 4) HC_G16(false, 4); else HC_G16(false, 8);
    }
#undef HC_G16
  }
}

void moe_group(const int32_t *idx, int npairs, int E, int *cnt, int *list, int maxp, cudaStream_t st) {
  launch_pdl(moe_group_kernel, dim3(1), dim3(256), size_t(E) * sizeof(int), st, idx, npairs, E, cnt, list, maxp);
}

void moe_gemv(const DevMat &W, int experts, int mode, const int *cnt, const int *list, int maxp, int K,
              const uint8_t *act, const float *bias, float alpha, float limit, float *out, int ldo, cudaStream_t st) {
  const int rt_e = W.rtiles / experts;
  const int rows_e = mode == 0 ? 2 * (W.rows / experts) : W.rows / experts;  // gate_up: 2 inter rows an expert
  const int wpr = W.ktiles >= 8 ? 8 : (W.ktiles >= 4 ? 4 : (W.ktiles >= 2 ? 2 : 1));
  const int rpc = 8 / wpr;
  const dim3 grid((rt_e + rpc - 1) / rpc, experts);
  if (mode == 0)
    launch_pdl(moe_gemv_kernel<0>, grid, dim3(256), 0, st, W.tiles, rt_e, W.ktiles, cnt, list, maxp, K, act, bias,
               rows_e, alpha, limit, wpr, out, ldo);
  else
    launch_pdl(moe_gemv_kernel<1>, grid, dim3(256), 0, st, W.tiles, rt_e, W.ktiles, cnt, list, maxp, K, act, bias,
               rows_e, alpha, limit, wpr, out, ldo);
}

void moe_combine(const float *y, const int32_t *idx, const float *w, int K, const float *dbias, int H, int ntok,
                 float *x, cudaStream_t st) {
  launch_pdl(moe_combine_kernel, dim3((H + 255) / 256, ntok), dim3(256), 0, st, y, idx, w, K, dbias, H, x);
}

}  // namespace hc
