// device.cuh: device helpers shared by the kernels.
#ifndef HWNPU_DEVICE_CUH
#define HWNPU_DEVICE_CUH

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.h"

namespace hc {

// ---- programmatic dependent launch -----------------------------------------------------------
// The step's kernels are launched with programmatic stream serialization (launch_pdl): a kernel
// lets the next one start as soon as all of its CTAs run (pdl_trigger), and waits for the
// previous one's results (pdl_wait) only right before it reads them, so that a GEMV's weight
// loads overlap the tail of the kernel before it. Every kernel waits (before its first dependent
// read, or before it ends), which keeps the whole sequence ordered.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// mma.sync m16n8k32 with int32 accumulation: A (16x32, row), B (32x8, col), signed or unsigned
// bytes as the name says (A first).
__device__ __forceinline__ void mma_s8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A (weights) unsigned bytes: int4 codes 0..15, or 16x them (see common.h).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Four e2m1 codes (the low 16 bits of w, a code a nibble) to their doubled values as signed
// bytes: {0,1,2,3,4,6,8,12} and their negatives (mxfp4's doubled, internal/mxfp4/mxfp4.go:21).
// `signs` selects, per output byte, the sign bit of its nibble from (w << 4, w).
__device__ __forceinline__ uint32_t e2m1x4(uint32_t w, uint32_t wsh, uint32_t sign_sel,
                                           uint32_t mag_sel) {
  const uint32_t pos = prmt(0x03020100u, 0x0C080604u, mag_sel);
  const uint32_t neg = prmt(0xFDFEFF00u, 0xF4F8FAFCu, mag_sel);
  const uint32_t m = prmt(wsh, w, sign_sel);
  return (pos & ~m) | (neg & m);
}

// Byte offset of token t's value of column k in the tensor-core GEMV's fp16 operand (kActF16,
// npad rows): per column tile npad x 512 bytes; in it per 16 columns (one MMA's K) npad x 32 bytes
// of core matrices, 8 tokens x 16 bytes each, the two 8-column halves 128 bytes apart, the 8-token
// groups 256 bytes apart (tcgemm.cu's descriptors: LBO 128, SBO 256).
__device__ __forceinline__ size_t f16op_offset(int t, int k, int npad) {
  const int cc = k & (kTileCols - 1);
  return size_t(k / kTileCols) * npad * (kTileCols * 2) + (cc >> 4) * (npad * 32) + (t >> 3) * 256 +
         ((cc >> 3) & 1) * 128 + (t & 7) * 16 + (cc & 7) * 2;
}

// fp16 bits as a key whose unsigned order is the value order (-0 as +0), for argmax.
__device__ __forceinline__ uint32_t f16_order(uint16_t h) {
  if (h == 0x8000) h = 0;
  return (h & 0x8000) ? uint32_t(uint16_t(~h)) : uint32_t(h | 0x8000);
}

// The argmax key of (fp16 value, index): larger value first, then the smaller index
// (chat/sample.go:80-88 keeps the first of equal maxima).
__device__ __forceinline__ unsigned long long argmax_key(uint16_t h, uint32_t idx) {
  return (static_cast<unsigned long long>(f16_order(h)) << 32) | (0xFFFFFFFFu - idx);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The float32 value of (row, col) of a repacked matrix, with the format's own arithmetic: int8
// q * s (palette Linear.Dequantize), int4 (float(q) - z) * s (milcpu shiftScale), e2m1 *
// 2^(e-127) (mxfp4.Dequantize).
__device__ __forceinline__ float tile_value(const uint8_t *tiles, const float *row_scale, int kind, int ktiles,
                                            int tile_bytes, int r, int col) {
  const int rt = r / kTileRows, kt = col / kTileCols;
  const TilePos tp = tile_pos(kind != kKindInt8, kind == kKindMx, r % kTileRows, col % kTileCols);
  const uint8_t *tile = tiles + (size_t(rt) * ktiles + kt) * tile_bytes;
  if (kind == kKindInt8) return float(int8_t(tile[tp.byte])) * row_scale[r];
  const int code = (tile[tp.byte] >> tp.shift) & 15;
  if (kind == kKindInt4) {
    const uint16_t *sz = reinterpret_cast<const uint16_t *>(tile + kTileCodes4 + tp.lane * 16);
    const float s = __half2float(__ushort_as_half(sz[tp.sidx]));
    const float z = __half2float(__ushort_as_half(sz[4 + tp.sidx]));
    return __fmul_rn(__fsub_rn(float(code), z), s);
  }
  const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float val = (code & 8) ? -mag[code & 7] : mag[code & 7];
  return __fmul_rn(val, __uint_as_float(uint32_t(tile[kTileCodes4 + tp.lane * 4 + tp.sidx]) << 23));
}

// ---- one column tile of a GEMV (common.h's tile layout) -------------------------------------
// The weight operand of one tile for one lane: the code words (int8: 8 MMAs x 4 registers; int4 /
// mxfp4: 4 words, each two MMAs' registers) and the scale data of rows g, g+8 x groups c, 4+c.
template <int KIND>
struct WTile {
  static constexpr int NW = KIND == kKindInt8 ? 32 : 16;
  uint32_t w[NW];
  uint32_t sd[4];  // int4: s,s,s,s,z,z,z,z as fp16 pairs; mxfp4: 4 exponent bytes in sd[0]
  __device__ __forceinline__ void load(const uint8_t *tile, int lane) {
    const uint4 *q = reinterpret_cast<const uint4 *>(tile) + lane;
#pragma unroll
    for (int i = 0; i < NW / 4; ++i) {
      const uint4 v = q[32 * i];
      w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
    if (KIND == kKindInt4) {
      const uint4 v = *reinterpret_cast<const uint4 *>(tile + kTileCodes4 + lane * 16);
      sd[0] = v.x; sd[1] = v.y; sd[2] = v.z; sd[3] = v.w;
    } else if (KIND == kKindMx) {
      sd[0] = *reinterpret_cast<const uint32_t *>(tile + kTileCodes4 + lane * 4);
      sd[1] = sd[2] = sd[3] = 0u;
    }
  }
};

// The activation operand of one tile for one token and lane (g, c): B registers of the 8 MMAs
// (lane (g, c) with g / 2 == c carries group 4h + c's hi (g even) or lo (g odd) bytes, the others
// zeros; mxfp4 reads hi only, as mxfp4.Vec.Quantize has no residual), and the scale S and sum Xq
// of the lane's groups c (h = 0) and 4 + c (h = 1). For int4 the h = 1 group carries S / 16 and
// 16 Xq, undoing the 16x codes exactly (powers of two).
template <int KIND>
struct BFrag {
  uint32_t b[8][2];
  float S[2], Xq[2];
  __device__ __forceinline__ void load(const uint8_t *at, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const bool on = (g >> 1) == c && !(KIND == kKindMx && (g & 1));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int G = 4 * h + c;
      uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
      if (on) {
        const uint4 *ap = reinterpret_cast<const uint4 *>(at + G * 64 + (g & 1) * 32);
        q0 = ap[0];
        q1 = ap[1];
      }
      b[4 * h + 0][0] = q0.x; b[4 * h + 0][1] = q0.y;
      b[4 * h + 1][0] = q0.z; b[4 * h + 1][1] = q0.w;
      b[4 * h + 2][0] = q1.x; b[4 * h + 2][1] = q1.y;
      b[4 * h + 3][0] = q1.z; b[4 * h + 3][1] = q1.w;
      const float2 sx = *reinterpret_cast<const float2 *>(at + kGroupsPerTile * 64 + G * 8);
      S[h] = sx.x;
      Xq[h] = sx.y;
      if (KIND == kKindInt4 && h == 1) {
        S[h] *= 0.0625f;
        Xq[h] *= 16.0f;
      }
    }
  }
  // an inactive tile: zero operands and scales, so every product is an exact zero
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int u = 0; u < 8; ++u) b[u][0] = b[u][1] = 0u;
    S[0] = S[1] = Xq[0] = Xq[1] = 0.f;
  }
};

// The 8 MMAs of one tile and their group scaling: adds to vg / vg8 this lane's values of rows g and
// g + 8 over its groups c and 4 + c (int8: before the row scale; mxfp4: doubled, before the 1/2).
template <int KIND>
__device__ __forceinline__ void wa_mma(const WTile<KIND> &wt, const BFrag<KIND> &bf, float &vg, float &vg8) {
  int D[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
  for (int o = 0; o < 4; ++o) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int u = 4 * h + o;
      uint32_t a[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (KIND == kKindInt8) {
          a[j] = wt.w[4 * u + j];
        } else if (KIND == kKindInt4) {
          a[j] = h ? (wt.w[4 * o + j] & 0xF0F0F0F0u) : (wt.w[4 * o + j] & 0x0F0F0F0Fu);
        } else {
          const uint32_t x = wt.w[4 * o + j], xs = x << 4;
          a[j] = h ? e2m1x4(x, xs, 0xFBEAu, (x >> 16) & 0x7777u) : e2m1x4(x, xs, 0xD9C8u, x & 0x7777u);
        }
      }
      if (KIND == kKindInt4) mma_u8s8(D[h], a[0], a[1], a[2], a[3], bf.b[u][0], bf.b[u][1]);
      else mma_s8s8(D[h], a[0], a[1], a[2], a[3], bf.b[u][0], bf.b[u][1]);
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (KIND == kKindMx) {
      const uint32_t e4 = wt.sd[0];
      const float sg = __uint_as_float(((e4 >> (16 * h)) & 0xffu) << 23);
      const float sg8 = __uint_as_float(((e4 >> (16 * h + 8)) & 0xffu) << 23);
      vg = fmaf(float(D[h][0]) * sg, bf.S[h], vg);
      vg8 = fmaf(float(D[h][2]) * sg8, bf.S[h], vg8);
    } else {
      const float pg = fmaf(float(D[h][1]), 1.0f / 256.0f, float(D[h][0]));
      const float pg8 = fmaf(float(D[h][3]), 1.0f / 256.0f, float(D[h][2]));
      if (KIND == kKindInt4) {
        const __half2 s2 = *reinterpret_cast<const __half2 *>(&wt.sd[h]);
        const __half2 z2 = *reinterpret_cast<const __half2 *>(&wt.sd[2 + h]);
        vg = fmaf(__low2float(s2) * bf.S[h], fmaf(-__low2float(z2), bf.Xq[h], pg), vg);
        vg8 = fmaf(__high2float(s2) * bf.S[h], fmaf(-__high2float(z2), bf.Xq[h], pg8), vg8);
      } else {
        vg = fmaf(bf.S[h], pg, vg);
        vg8 = fmaf(bf.S[h], pg8, vg8);
      }
    }
  }
}

// One warp quantises one group of 32 values (v is this lane's): hi = round_even(v * 127 / max),
// the residual in lo at 1/256 of the scale (see common.h's kActTile); X is the group's sum of
// (hi + lo / 256), the same on every lane.
struct QGroup {
  int8_t hq, lq;
  float S, X;
};
__device__ __forceinline__ QGroup quant_vals(float v) {
  const float m = warp_max(fabsf(v));
  QGroup q{0, 0, 0.f, 0.f};
  if (m > 0.f) {
    const float inv = 127.0f / m;  // mxfp4.Vec.Quantize's inv (mxfp4.go:44)
    q.S = m / 127.0f;
    const float h = rintf(v * inv);
    const float r = fmaf(-h, q.S, v);
    const float l = fminf(fmaxf(rintf(r * (256.0f * inv)), -127.f), 127.f);
    q.hq = int8_t(h);
    q.lq = int8_t(l);
    q.X = float(warp_sum_i(int(q.hq) * 256 + int(q.lq))) * (1.0f / 256.0f);
  }
  return q;
}

// Token-major tiles (up to 8 tokens): group gi of the tile at act_tile.
__device__ __forceinline__ void quant_group(float v, uint8_t *act_tile, int gi, int lane) {
  const QGroup q = quant_vals(v);
  act_tile[gi * 64 + lane] = uint8_t(q.hq);
  act_tile[gi * 64 + 32 + lane] = uint8_t(q.lq);
  if (lane == 0) *reinterpret_cast<float2 *>(act_tile + kGroupsPerTile * 64 + gi * 8) = make_float2(q.S, q.X);
}

// Sums a lane value over the 4 lanes of one g (the groups c = 0..3): lane 4g ends with rows g, g+8.
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

}  // namespace hc

#endif
