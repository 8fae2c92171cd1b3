// device.cuh: device helpers shared by the kernels.
#ifndef HWNPU_DEVICE_CUH
#define HWNPU_DEVICE_CUH

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.h"

namespace hc {

// mma.sync m16n8k32 with int32 accumulation: A (16x32, row) signed bytes, B (32x8, col)
// unsigned (int4 codes 0..15) or signed (int8 codes, doubled e2m1 values) bytes.
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

// The float32 value of (row, col) of a repacked matrix, as dequant_kernel computes it.
__device__ __forceinline__ float tile_value(const uint8_t *tiles, const float *row_scale, int kind, int ktiles,
                            int tile_bytes, int r, int col) {
  const int rt = r / 8, g = r % 8, kt = col / kTileCols, cc = col % kTileCols;
  const int grp = cc / 32, e = cc % 32, i4 = e / 4, p = e % 4;
  const int c = grp & 3, hi = grp >> 2, lane = g * 4 + c, sl = grp * 4 + g / 2;
  const uint8_t *tile = tiles + (size_t(rt) * ktiles + kt) * tile_bytes;
  if (kind == kKindInt8) return float(int8_t(tile[lane * 64 + i4 * 8 + hi * 4 + p])) * row_scale[r];
  if (kind == kKindInt4) {
    const uint8_t by = tile[lane * 32 + i4 * 4 + p];
    const int q = hi ? (by >> 4) : (by & 15);
    const uint16_t *sz = reinterpret_cast<const uint16_t *>(tile + kTileCodes4 + sl * 8);
    const float s = __half2float(__ushort_as_half(sz[g & 1]));
    const float z = __half2float(__ushort_as_half(sz[2 + (g & 1)]));
    return __fmul_rn(__fsub_rn(float(q), z), s);
  }
  const uint8_t by = tile[lane * 32 + i4 * 4 + hi * 2 + p / 2];
  const int code = (p & 1) ? (by >> 4) : (by & 15);
  const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float val = (code & 8) ? -mag[code & 7] : mag[code & 7];
  return __fmul_rn(val, __uint_as_float(uint32_t(tile[kTileCodes4 + sl * 2 + (g & 1)]) << 23));
}

}  // namespace hc

#endif
