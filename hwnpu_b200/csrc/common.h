// common.h: internal definitions shared by the host runtime and the kernels of libhwnpu_cuda.so.
#ifndef HWNPU_COMMON_H
#define HWNPU_COMMON_H

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/hwnpu_cuda.h"

namespace hc {

// ---- repacked tile geometry -------------------------------------------------------------
// A linear layer is stored as tiles of 16 output rows x 256 input columns (8 groups of 32), laid
// out for integer MMAs (m16n8k32) whose A operand is the weights and whose B operand is the
// activation. MMA u = 4h + o (h = 0, 1; o = 0..3) covers groups 4h..4h+3, columns 8o..8o+7 of each:
// lane L = 4g + c holds, for rows g and g + 8, group 4h + c's columns 8o..8o+3 (A registers a0, a1)
// and 8o+4..8o+7 (a2, a3). So every lane's results belong to the rows g, g + 8 and the groups c,
// 4 + c, and the 8 columns of one group never mix with another group's inside an MMA.
// A lane's code words come in 16-byte pieces, piece i of lane L at (32 i + L) * 16, so that the
// warp's 16-byte loads of one piece read 512 contiguous bytes (no shared-memory bank conflicts).
//   int8  codes: 8 pieces a lane: piece u holds MMA u's registers a0..a3.
//   int4  codes: 4 pieces a lane: word j of piece o holds MMA (0, o)'s register a_j in its low
//         nibbles and MMA (1, o)'s in its high nibbles (w & 0x0F0F0F0F, w & 0xF0F0F0F0: the
//         second reads 16x the code, which the group's scale takes back exactly).
//         Then lane L's fp16 s and z at 2048 + L * 16: s of (g, c), (g+8, c), (g, 4+c), (g+8, 4+c),
//         then z in the same order.
//   mxfp4 codes: as int4, but word j of piece o holds e2m1 nibbles a0 a1 a2 a3 b0 b1 b2 b3 from
//         the lowest (a: MMA (0, o)'s bytes, b: MMA (1, o)'s), the order e2m1x4 reads. Then lane
//         L's 4 exponents at 2048 + L * 4, in the order of the int4 scales.
constexpr int kTileRows = 16;
constexpr int kTileCols = 256;
constexpr int kGroup = 32;
constexpr int kGroupsPerTile = kTileCols / kGroup;  // 8

// Bytes of one tile by format (codes, then the per-lane scale data).
constexpr int kTileCodes4 = kTileRows * kTileCols / 2;  // 2048: two codes a byte
constexpr int kTileCodes8 = kTileRows * kTileCols;      // 4096: one code a byte
constexpr int kTileInt4 = kTileCodes4 + 32 * 16;        // + s,s,s,s,z,z,z,z fp16 per lane = 2560
constexpr int kTileMx = kTileCodes4 + 32 * 4;           // + 4 exponents per lane = 2176
constexpr int kTileInt8 = kTileCodes8;                  // row scales live apart: 4096

#ifdef __CUDACC__
#define HC_HD __host__ __device__
#else
#define HC_HD
#endif

// Where (row r, column cc) of a tile (r < 16, cc < 256) sits: the byte of its code and, for the
// 4-bit formats, the nibble (0 low, 4 high); and the index (0..3) of its group's scale data within
// the lane's scale block (int4: s at 2048 + lane * 16 + 2 * idx, z 8 bytes further; mxfp4: the
// exponent byte at 2048 + lane * 4 + idx).
struct TilePos {
  int byte, shift, lane, sidx;
};
HC_HD inline TilePos tile_pos(int kind4, int mx, int r, int cc) {
  const int G = cc / kGroup, e = cc % kGroup;
  const int h = G / 4, c = G % 4, o = e / 8, e8 = e % 8;
  const int g = r % 8, hi = r / 8;
  const int j = (e8 >= 4 ? 2 : 0) + hi, p = e8 % 4;
  TilePos t;
  t.lane = 4 * g + c;
  t.sidx = 2 * h + hi;
  if (!kind4) {  // int8: piece u = 4h + o, register j, byte p
    t.byte = ((4 * h + o) * 32 + t.lane) * 16 + j * 4 + p;
    t.shift = 0;
  } else if (!mx) {  // int4: piece o, word j, byte p, nibble h
    t.byte = (o * 32 + t.lane) * 16 + j * 4 + p;
    t.shift = 4 * h;
  } else {  // mxfp4: piece o, word j, byte 2h + p / 2, nibble p % 2
    t.byte = (o * 32 + t.lane) * 16 + j * 4 + 2 * h + p / 2;
    t.shift = 4 * (p % 2);
  }
  return t;
}

// The activation of one token for one tile's 256 columns: per group 32 int8 "hi" and 32 int8
// "lo" values, then per group the float scale S and the float sum Xq of (hi + lo/256); the
// value of column k is S * (hi + lo / 256).
constexpr int kActTile = kGroupsPerTile * 64 + kGroupsPerTile * 8;  // 576

// Slots over which one token's argmax atomics are spread (the head GEMV has ~19k CTAs).
constexpr int kAmaxSlots = 64;

inline int pad_to(int x, int m) { return (x + m - 1) / m * m; }

// Kernel-side kinds of a repacked matrix.
enum Kind : int {
  kKindInt8 = 0,   // signed codes, one float scale a row
  kKindInt4 = 1,   // unsigned codes with fp16 s and z per (row, group): w = (q - z) s
  kKindMx = 2,     // e2m1 codes, doubled to integers, with an e8m0 exponent per (row, group)
};

// ---- errors ------------------------------------------------------------------------------
// A heap string for the C ABI's error protocol (NULL is success), freed by hc_free_error.
char *make_error(const std::string &msg);

#define HC_TRY_CUDA(call)                                                                   \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess)                                                                  \
      return ::hc::make_error(std::string(#call) + ": " + cudaGetErrorString(e_));          \
  } while (0)

// ---- host-side fault injection (hc_set_fault) ----------------------------------------------
enum FaultPoint { kFaultAlloc = 0, kFaultH2D = 1, kFaultStep = 2 };
// True when the armed fault of this point fires on this call.
bool fault_fires(FaultPoint p);
// The armed device stall in milliseconds (hc_set_fault "stall:MS"), cleared by the call; 0: none.
long take_stall_ms();

// cudaMalloc that honours the alloc fault and returns an error string.
char *dev_alloc(void **p, size_t n, const char *what);
// cudaMemcpy host to device that honours the h2d fault.
char *copy_h2d(void *dst, const void *src, size_t n, cudaStream_t st);

}  // namespace hc

#endif
