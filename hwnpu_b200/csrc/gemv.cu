// gemv.cu: the decode GEMV over repacked integer tiles, and the activation quantiser it reads.
//
// One CTA (8 warps) owns 8 / wpr row tiles; the wpr warps of a row tile split its column tiles.
// Per column tile a warp issues 8 integer MMAs (m16n8k32): B is the tile's 8 rows (codes straight
// from HBM, unpacked in registers), A carries the activation of the 8 groups of 32 columns on
// its 8 rows ("hi" bytes) and 8 more rows ("lo" bytes, the residual at 1/256), so that every
// A row holds one group: after the 8 MMAs lane (g, c) holds group g's exact integer dot products
// for output rows 2c and 2c+1, which it scales by the group's weight scale (and zero point) and
// by the activation's group scale in float32.
#include "device.cuh"
#include "kernels.h"

namespace hc {
namespace {

template <int KIND, int NT>
__global__ void __launch_bounds__(256) gemv_kernel(const uint8_t *__restrict__ tiles,
                                                   const float *__restrict__ row_scale,
                                                   const float *__restrict__ bias,
                                                   const uint8_t *__restrict__ act, int rtiles,
                                                   int ktiles, int rows, int wpr, GemvOut out) {
  constexpr int TB = KIND == kKindInt8 ? kTileInt8 : (KIND == kKindInt4 ? kTileInt4 : kTileMx);
  __shared__ float part[8][NT][8];
  __shared__ unsigned long long bmax[NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rpc = 8 / wpr;
  const int lrt = warp / wpr, ks = warp % wpr;
  const int rt = blockIdx.x * rpc + lrt;
  const bool role0 = g == c, role1 = g == c + 4;
  const int agrp = role0 ? c : g;  // the group whose activation bytes this lane puts in A
  if (threadIdx.x < NT) bmax[threadIdx.x] = 0ull;
  float acc[NT][2];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = 0.f;

  if (rt < rtiles) {
    for (int kt = ks; kt < ktiles; kt += wpr) {
      const uint8_t *tile = tiles + (size_t(rt) * ktiles + kt) * TB;
      uint32_t b0[8], b1[8];
      float s0 = 0.f, s1 = 0.f, z0 = 0.f, z1 = 0.f;
      if (KIND == kKindInt8) {
        const uint4 *p = reinterpret_cast<const uint4 *>(tile + lane * 64);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v = __ldg(p + q);
          b0[2 * q] = v.x; b1[2 * q] = v.y; b0[2 * q + 1] = v.z; b1[2 * q + 1] = v.w;
        }
      } else {
        const uint4 *p = reinterpret_cast<const uint4 *>(tile + lane * 32);
        uint4 v0 = __ldg(p), v1 = __ldg(p + 1);
        uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        if (KIND == kKindInt4) {
          const uint2 sz = __ldg(reinterpret_cast<const uint2 *>(tile + kTileCodes4 + lane * 8));
          const __half2 sh = *reinterpret_cast<const __half2 *>(&sz.x);
          const __half2 zh = *reinterpret_cast<const __half2 *>(&sz.y);
          s0 = __low2float(sh); s1 = __high2float(sh);
          z0 = __low2float(zh); z1 = __high2float(zh);
#pragma unroll
          for (int i = 0; i < 8; ++i) { b0[i] = w[i] & 0x0F0F0F0Fu; b1[i] = (w[i] >> 4) & 0x0F0F0F0Fu; }
        } else {
          const uint16_t e2 = __ldg(reinterpret_cast<const unsigned short *>(tile + kTileCodes4 + lane * 2));
          s0 = __uint_as_float(uint32_t(e2 & 0xff) << 23);  // 2^(e-127)
          s1 = __uint_as_float(uint32_t(e2 >> 8) << 23);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t wsh = w[i] << 4;
            b0[i] = e2m1x4(w[i], wsh, 0xD9C8u, w[i] & 0x7777u);
            b1[i] = e2m1x4(w[i], wsh, 0xFBEAu, (w[i] >> 16) & 0x7777u);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint8_t *at = act + (size_t(t) * ktiles + kt) * kActTile;
        uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0, l0 = h0, l1 = h0;
        if (role0 || role1) {
          const uint4 *ap = reinterpret_cast<const uint4 *>(at + agrp * 64);
          h0 = ap[0]; h1 = ap[1];
          if (KIND != kKindMx) { l0 = ap[2]; l1 = ap[3]; }
        }
        const float2 sx = *reinterpret_cast<const float2 *>(at + kGroupsPerTile * 64 + g * 8);
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        int d[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t a0 = role0 ? hw[i] : 0u, a1 = role0 ? lw[i] : 0u;
          const uint32_t a2 = role1 ? hw[i] : 0u, a3 = role1 ? lw[i] : 0u;
          if (KIND == kKindInt4) mma_s8u8(d, a0, a1, a2, a3, b0[i], b1[i]);
          else mma_s8s8(d, a0, a1, a2, a3, b0[i], b1[i]);
        }
        // d[0], d[1]: group g's dot with rows 2c, 2c+1 on the hi bytes; d[2], d[3]: on the lo
        const float S = sx.x, Xq = sx.y;
        if (KIND == kKindMx) {
          acc[t][0] = fmaf(float(d[0]) * s0, S, acc[t][0]);
          acc[t][1] = fmaf(float(d[1]) * s1, S, acc[t][1]);
        } else {
          const float p0 = fmaf(float(d[2]), 1.0f / 256.0f, float(d[0]));
          const float p1 = fmaf(float(d[3]), 1.0f / 256.0f, float(d[1]));
          if (KIND == kKindInt4) {
            acc[t][0] = fmaf(s0 * S, fmaf(-z0, Xq, p0), acc[t][0]);
            acc[t][1] = fmaf(s1 * S, fmaf(-z1, Xq, p1), acc[t][1]);
          } else {
            acc[t][0] = fmaf(S, p0, acc[t][0]);
            acc[t][1] = fmaf(S, p1, acc[t][1]);
          }
        }
      }
    }
  }
  // sum the 8 groups (lanes g = 0..7 of the same c)
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v = acc[t][j];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      acc[t][j] = v;
    }
  if (g == 0) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      part[warp][t][2 * c] = acc[t][0];
      part[warp][t][2 * c + 1] = acc[t][1];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < rpc * NT * 8; idx += blockDim.x) {
    const int l2 = idx / (NT * 8), t = (idx / 8) % NT, r8 = idx % 8;
    const int tile_r = blockIdx.x * rpc + l2;
    if (tile_r >= rtiles) continue;
    auto value = [&](int rr) {
      float v = 0.f;
      for (int k = 0; k < wpr; ++k) v += part[l2 * wpr + k][t][rr];
      const int row = tile_r * 8 + rr;
      if (KIND == kKindInt8) v *= row_scale[row];
      if (KIND == kKindMx) v *= 0.5f;  // the doubled e2m1 values (mxfp4.go:90)
      if (bias) v += bias[row];
      return v;
    };
    if (out.mode == kGlu) {
      if (r8 >= 4) continue;
      const int o = tile_r * 4 + r8;
      if (o >= rows) continue;
      const float gv = value(r8), uv = value(r8 + 4);
      // blocks.SiLU: x / (1 + exp(-x)) (internal/llm/blocks/blocks.go:395-399)
      out.y[size_t(t) * out.ldy + o] = gv / (1.0f + expf(-gv)) * uv;
      continue;
    }
    const int row = tile_r * 8 + r8;
    if (row >= rows) continue;
    const float v = value(r8);
    if (out.mode == kStore) {
      out.y[size_t(t) * out.ldy + row] = v;
    } else if (out.mode == kAdd) {
      float *p = out.y + size_t(t) * out.ldy + row;
      *p = *p + v;
    } else {
      const __half h = __float2half_rn(v);
      const uint16_t hb = __half_as_ushort(h);
      if (out.logits) out.logits[size_t(t) * out.ldy + row] = hb;
      atomicMax(&bmax[t], argmax_key(hb, uint32_t(row)));
    }
  }
  if (out.mode == kLogits) {
    __syncthreads();
    if (threadIdx.x < NT)
      atomicMax(&out.amax[threadIdx.x * kAmaxSlots + (blockIdx.x % kAmaxSlots)], bmax[threadIdx.x]);
  }
}

template <int KIND>
void launch_kind(const DevMat &W, const uint8_t *act, int ntok, const GemvOut &out, int wpr,
                 int grid, cudaStream_t st) {
  switch (ntok) {
#define HC_NT(n)                                                                          \
  case n:                                                                                 \
    gemv_kernel<KIND, n><<<grid, 256, 0, st>>>(W.tiles, W.row_scale, W.bias, act, W.rtiles, \
                                              W.ktiles, W.rows, wpr, out);               \
    break;
    HC_NT(1) HC_NT(2) HC_NT(3) HC_NT(4) HC_NT(5) HC_NT(6) HC_NT(7) HC_NT(8)
#undef HC_NT
  }
}

// ---- the activation quantiser --------------------------------------------------------------

__device__ double block_sum_d(double v, double *sh) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  double t = 0;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) sh[0] = t;
  }
  __syncthreads();
  t = sh[0];
  __syncthreads();
  return t;
}

// One warp quantises one group of 32 values (v is this lane's): hi = round_even(v * 127 / max),
// the residual in lo at 1/256 of the scale (see common.h's kActTile).
__device__ __forceinline__ void quant_group(float v, uint8_t *act_tile, int gi, int lane) {
  const float m = warp_max(fabsf(v));
  int8_t hq = 0, lq = 0;
  float S = 0.f;
  int s256 = 0;
  if (m > 0.f) {
    const float inv = 127.0f / m;  // mxfp4.Vec.Quantize's inv (mxfp4.go:44)
    S = m / 127.0f;
    const float h = rintf(v * inv);
    const float r = fmaf(-h, S, v);
    const float l = fminf(fmaxf(rintf(r * (256.0f * inv)), -127.f), 127.f);
    hq = int8_t(h);
    lq = int8_t(l);
    s256 = warp_sum_i(int(hq) * 256 + int(lq));
  }
  act_tile[gi * 64 + lane] = uint8_t(hq);
  act_tile[gi * 64 + 32 + lane] = uint8_t(lq);
  if (lane == 0) {
    float2 *sx = reinterpret_cast<float2 *>(act_tile + kGroupsPerTile * 64 + gi * 8);
    *sx = make_float2(S, float(s256) * (1.0f / 256.0f));
  }
}

// One CTA per (token, column tile): the RMS norm's sum of squares is taken over the whole row by
// every CTA (the row is a few KB in L2), then the CTA quantises its tile's 8 groups, one warp each.
__global__ void __launch_bounds__(256) act_quant_kernel(const float *__restrict__ x, int ldx,
                                                        int n, const float *__restrict__ norm_w,
                                                        float scale, float eps16,
                                                        uint8_t *__restrict__ act, int ktiles) {
  __shared__ double red[32];
  const int t = blockIdx.y, kt = blockIdx.x;
  const float *xt = x + size_t(t) * ldx;
  const float inv = scale == 1.f ? 1.f : 1.f / scale;
  float r = 1.f;
  if (norm_w) {
    double s = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float xs = scale == 1.f ? xt[i] : xt[i] * inv;
      const float sq = xs * xs;
      s += double(sq);
    }
    s = block_sum_d(s, red);
    const float ms = float(s / double(n));
    r = float(1.0 / sqrt(double(ms) + double(eps16)));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = (kt * kGroupsPerTile + warp) * kGroup + lane;
  float v = 0.f;
  if (col < n) {
    v = xt[col];
    if (norm_w) {
      const float xs = scale == 1.f ? v : v * inv;
      const float y = xs * r;
      v = y * norm_w[col];
    }
  }
  quant_group(v, act + (size_t(t) * ktiles + kt) * kActTile, warp, lane);
}

// Merges the attention partials of one (token, head) (Flash-Decoding; with a sink logit when
// given, paged.Merge.AddSink, paged.go:281-297) and quantises the head's groups of 32 (a group
// never crosses a head: head_dim is 64 or 128).
__global__ void __launch_bounds__(128) attn_merge_kernel(const float *__restrict__ part_ml,
                                                         const float *__restrict__ part_o,
                                                         const float *__restrict__ sinks,
                                                         int heads, int hd, int splits,
                                                         uint8_t *__restrict__ act, int ktiles,
                                                         float *__restrict__ o_out) {
  __shared__ float wsh[64];
  __shared__ float stat[2];
  const int h = blockIdx.x, t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float *ml = part_ml + (size_t(t) * heads + h) * splits * 2;
  if (warp == 0) {
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    if (lane < splits) { m0 = ml[2 * lane]; l0 = ml[2 * lane + 1]; }
    if (lane + 32 < splits) { m1 = ml[2 * (lane + 32)]; l1 = ml[2 * (lane + 32) + 1]; }
    float M = sinks ? sinks[h] : -INFINITY;
    M = fmaxf(M, l0 > 0.f ? m0 : -INFINITY);
    M = fmaxf(M, l1 > 0.f ? m1 : -INFINITY);
    M = warp_max(M);
    const float w0 = l0 > 0.f ? expf(m0 - M) : 0.f, w1 = l1 > 0.f ? expf(m1 - M) : 0.f;
    float L = warp_sum(l0 * w0 + l1 * w1);
    if (sinks) L += expf(sinks[h] - M);
    if (lane < splits) wsh[lane] = w0;
    if (lane + 32 < splits) wsh[lane + 32] = w1;
    if (lane == 0) stat[0] = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  const float invL = stat[0];
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    const float *po = part_o + ((size_t(t) * heads + h) * splits) * hd + d;
    float o = 0.f;
#pragma unroll 8
    for (int s = 0; s < splits; ++s) o = fmaf(po[size_t(s) * hd], wsh[s], o);
    o *= invL;
    if (o_out) o_out[(size_t(t) * heads + h) * hd + d] = o;
    // one warp a group of 32: warp w of this head holds columns h*hd + 32w .. + 31
    const int gcol = h * hd + d;
    const int grp = gcol / kGroup;
    quant_group(o, act + (size_t(t) * ktiles + grp / kGroupsPerTile) * kActTile, grp % kGroupsPerTile, lane);
  }
}

// Values of repacked rows with the format's own arithmetic: int8 q * s
// (palette Linear.Dequantize), int4 (float(q) - z) * s (milcpu shiftScale), e2m1 * 2^(e-127)
// (mxfp4.Dequantize).
__global__ void dequant_kernel(const uint8_t *__restrict__ tiles, const float *__restrict__ row_scale,
                               int kind, int ktiles, int tile_bytes, int cols, int row0, int nrows,
                               float *__restrict__ out) {
  const long total = long(nrows) * cols;
  for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < total; i += long(gridDim.x) * blockDim.x) {
    const int r = row0 + int(i / cols), col = int(i % cols);
    const int rt = r / 8, g = r % 8, kt = col / kTileCols, cc = col % kTileCols;
    const int grp = cc / 32, e = cc % 32, i4 = e / 4, p = e % 4;
    const int c = grp & 3, hi = grp >> 2;  // group grp sits with lane c's low (grp < 4) or high part
    const int lane = g * 4 + c;
    const uint8_t *tile = tiles + (size_t(rt) * ktiles + kt) * tile_bytes;
    float v;
    if (kind == kKindInt8) {
      const int8_t q = int8_t(tile[lane * 64 + i4 * 8 + hi * 4 + p]);
      v = float(q) * row_scale[r];
    } else {
      // the scale data of (row r, group grp) sits with lane (grp, r%8 / 2)
      const int sl = grp * 4 + g / 2;
      if (kind == kKindInt4) {
        const uint8_t by = tile[lane * 32 + i4 * 4 + p];
        const int q = hi ? (by >> 4) : (by & 15);
        const uint16_t *sz = reinterpret_cast<const uint16_t *>(tile + kTileCodes4 + sl * 8);
        const float s = __half2float(__ushort_as_half(sz[g & 1]));
        const float z = __half2float(__ushort_as_half(sz[2 + (g & 1)]));
        float x = float(q);
        x = __fsub_rn(x, z);
        v = __fmul_rn(x, s);
      } else {
        const uint8_t by = tile[lane * 32 + i4 * 4 + hi * 2 + p / 2];
        const int code = (p & 1) ? (by >> 4) : (by & 15);
        const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
        const float val = (code & 8) ? -mag[code & 7] : mag[code & 7];
        const uint8_t ee = tile[kTileCodes4 + sl * 2 + (g & 1)];
        v = __fmul_rn(val, __uint_as_float(uint32_t(ee) << 23));
      }
    }
    out[i] = v;
  }
}

}  // namespace

void gemv(const DevMat &W, const uint8_t *act, int ntok, const GemvOut &out, cudaStream_t st) {
  const int wpr = W.ktiles >= 8 ? 8 : (W.ktiles >= 4 ? 4 : (W.ktiles >= 2 ? 2 : 1));
  const int rpc = 8 / wpr;
  const int grid = (W.rtiles + rpc - 1) / rpc;
  switch (W.kind) {
    case kKindInt8: launch_kind<kKindInt8>(W, act, ntok, out, wpr, grid, st); break;
    case kKindInt4: launch_kind<kKindInt4>(W, act, ntok, out, wpr, grid, st); break;
    case kKindMx: launch_kind<kKindMx>(W, act, ntok, out, wpr, grid, st); break;
  }
}

void act_quant(const float *x, int ldx, int n, int ntok, const float *norm_w, float scale,
               float eps16, uint8_t *act, int ktiles, cudaStream_t st) {
  act_quant_kernel<<<dim3(ktiles, ntok), 256, 0, st>>>(x, ldx, n, norm_w, scale, eps16, act, ktiles);
}

void attn_merge_quant(const float *part_ml, const float *part_o, const float *sinks, int ntok,
                      int heads, int hd, int splits, uint8_t *act, int ktiles, float *o_out,
                      cudaStream_t st) {
  // columns past heads*hd in the last tile are zero groups
  const int n = heads * hd;
  if (n % kTileCols) {
    for (int t = 0; t < ntok; ++t)
      cudaMemsetAsync(act + (size_t(t) * ktiles + ktiles - 1) * kActTile, 0, kActTile, st);
  }
  attn_merge_kernel<<<dim3(heads, ntok), hd, 0, st>>>(part_ml, part_o, sinks, heads, hd, splits, act,
                                                     ktiles, o_out);
}

void dequant(const DevMat &W, int row0, int nrows, float *out, cudaStream_t st) {
  const long total = long(nrows) * W.cols;
  const int grid = int(std::min<long>((total + 255) / 256, 4096));
  dequant_kernel<<<grid, 256, 0, st>>>(W.tiles, W.row_scale, W.kind, W.ktiles, W.tile_bytes,
                                       W.cols, row0, nrows, out);
}

}  // namespace hc
