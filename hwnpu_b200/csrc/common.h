// common.h: internal definitions shared by the host runtime and the kernels of libhwnpu_cuda.so.
#ifndef HWNPU_COMMON_H
#define HWNPU_COMMON_H

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/hwnpu_cuda.h"

namespace hc {

// ---- repacked tile geometry -------------------------------------------------------------
// A linear layer is stored as tiles of 8 output rows x 256 input columns (8 groups of 32). In a
// tile, lane L = 4g + c of a warp holds, for each of the 8 integer MMAs (m16n8k32) that cover the
// tile, the B fragment of row g: 4 columns of group c and 4 of group c + 4 (k interleaved: the 8
// groups are the 8 rows of the MMA's A, so one MMA adds one group's dot product per A row).
constexpr int kTileRows = 8;
constexpr int kTileCols = 256;
constexpr int kGroup = 32;
constexpr int kGroupsPerTile = kTileCols / kGroup;  // 8

// Bytes of one tile by format (codes, then the per-lane scale data).
constexpr int kTileCodes4 = kTileRows * kTileCols / 2;  // 1024: two codes a byte
constexpr int kTileCodes8 = kTileRows * kTileCols;      // 2048: one code a byte
constexpr int kTileInt4 = kTileCodes4 + 32 * 8;         // + s,s,z,z fp16 per lane = 1280
constexpr int kTileMx = kTileCodes4 + 32 * 2;           // + e,e per lane = 1088
constexpr int kTileInt8 = kTileCodes8;                  // row scales live apart: 2048

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

// cudaMalloc that honours the alloc fault and returns an error string.
char *dev_alloc(void **p, size_t n, const char *what);
// cudaMemcpy host to device that honours the h2d fault.
char *copy_h2d(void *dst, const void *src, size_t n, cudaStream_t st);

}  // namespace hc

#endif
