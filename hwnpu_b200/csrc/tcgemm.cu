// tcgemm.cu: the batched GEMV of the int8 and int4 formats (9..64 tokens: prompt chunks, ragged
// decode batches, speculative verify chunks past 8 rows) on the 5th-generation tensor cores.
//
// Y[t][r] = sum_k X[t][k] W[r][k] for n <= 64 tokens. A CTA owns a tile of 128 weight rows (8 of
// the 16-row repacked tiles) over a range of column tiles (all of them, or a split of them when
// there are too few row tiles to fill the SMs), and all n tokens: one tcgen05.mma of M = 128,
// N = n rounded up to 16, K = 16 (kind::f16, float32 accumulator in tensor memory) per 16 columns.
//
//   warp 0      bulk-copies (cp.async.bulk, no multicast) each column tile's 8 weight tiles into a
//               ring of up to 6 stages (an mbarrier with complete_tx per stage), from the kernel's
//               start: the weights do not depend on the kernel before
//   warp 18     bulk-copies the tokens' fp16 operand into a ring of 2, once the kernel before is done
//   warp 1      allocates the tensor memory; one lane issues the MMAs and their commits
//   warps 2..17 warps 2 + 2i and 3 + 2i dequantise row tile i of each half column tile from the ring
//               into the MMA's A operand (fp16, K-major, no swizzle), then, with the
//               accumulator's lane quarter (warp % 4) and 16 of its columns, run the epilogue
//
// Arithmetic. A weight is dequantised with its format's float32 arithmetic (int4: (q - z) s,
// milcpu shiftScale) and rounded to fp16; int8 codes go in as exact integers and their row scale is
// applied to the float32 sum. The tokens' values are rounded to fp16 once (act_quant's fp16
// operand). Products and sums are exact/float32 in the tensor core. So a row of a 9..64-token chunk
// differs from the same row computed by the one-token GEMV (int8 hi/lo activations) by the fp16
// roundings, about 2^-12 of a product; both are within the model tolerance of the oracle.
//
// With splits > 1 the splits of a row tile run as one thread block cluster: each CTA leaves its
// float32 partial sums in its own shared memory, and after a cluster barrier CTA r adds a share
// of the rows over all the splits, in split order, through distributed shared memory, and runs
// the epilogue on them: the result does not depend on which CTA finishes first.
//
// Every mbarrier wait is bounded (about a second of SM clocks): a wait that runs out records an
// error code in *status and proceeds, so that no thread waits forever; the kernel still waits for
// its own bulk copies and MMAs before it frees the tensor memory and exits.
#include <algorithm>

#include "device.cuh"
#include "kernels.h"

namespace hc {
namespace {

constexpr int kTcRows = 128;                       // rows of a CTA tile: 8 row tiles (the MMA's M)
constexpr int kTcTiles = kTcRows / kTileRows;      // 8
constexpr int kTcMaxW = 6;                         // most weight ring stages (a column tile's 8 tiles each)
constexpr int kTcBStages = 2;                      // tokens' operand ring stages (the operand sits in L2)
constexpr int kTcSmem = 230400;                    // dynamic shared memory a CTA may take
constexpr int kTcDeq = 16;                         // dequantising warps: two a row tile
constexpr int kTcBWarp = 2 + kTcDeq;                // the warp that copies the tokens' operand
constexpr int kTcThreads = (3 + kTcDeq) * 32;
constexpr int kTcHalf = kTileCols / 2;             // columns of one A buffer
// bytes of A per 16 columns (one MMA's K): 128 rows x 32 bytes, and 16 more so that the 4 K-steps
// a warp's store instruction touches fall on different banks
constexpr int kTcStepA = kTcRows * 16 * 2 + 16;
constexpr int kTcABytes = (kTcHalf / 16) * kTcStepA;
constexpr int kTcMaxN = 64;
constexpr long long kTcSpin = 2000000000ll;        // clock cycles a wait may take

__device__ __forceinline__ uint32_t tc_saddr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void tc_bar_init(uint64_t *b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc_saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void tc_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(tc_saddr(b)) : "memory");
}
__device__ __forceinline__ void tc_expect_tx(uint64_t *b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(tc_saddr(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool tc_try(uint64_t *b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred P;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 P, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, P;\n}\n"
      : "=r"(ok)
      : "r"(tc_saddr(b)), "r"(parity), "n"(1000)
      : "memory");
  return ok != 0;
}
// Waits for the phase of the given parity to complete, at most kTcSpin cycles; on running out it
// records code in *status (the first one) and returns.
__device__ __forceinline__ void tc_wait(uint64_t *b, unsigned parity, int *status, int code) {
  if (tc_try(b, parity)) return;
  const long long t0 = clock64();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (tc_try(b, parity)) return;
    if (clock64() - t0 > kTcSpin) {
      atomicCAS(status, 0, code);
      return;
    }
  }
}
__device__ __forceinline__ void tc_bulk(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(tc_saddr(dst)),
      "l"(src), "r"(bytes), "r"(tc_saddr(bar))
      : "memory");
}

// ---- tcgen05 --------------------------------------------------------------------------------
// Shared-memory matrix descriptor of a K-major operand without swizzle: core matrices of 8 rows x
// 16 bytes (128 contiguous bytes); lbo: bytes between the two core matrices of one MMA's 16
// columns, sbo: bytes between core matrices 8 rows apart; version 1 (bits 46-47).
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
// Instruction descriptor of kind::f16: fp16 A and B, K-major both, float32 D, M = 128, N = n.
__host__ __device__ constexpr uint32_t tc_idesc(int n) {
  return (1u << 4) | (uint32_t(n >> 3) << 17) | (uint32_t(kTcRows >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrives on b once every MMA this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t *b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(tc_saddr(b))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// Makes this thread's shared-memory stores visible to the tensor core (the async proxy).
__device__ __forceinline__ void tc_fence_proxy() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 16 columns of the accumulator for this warp's 32 lanes (rows) into v.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- dequantisation into the A operand --------------------------------------------------------
// Byte offset, in one half buffer (128 rows x 128 columns), of the 16-byte run of 8 columns
// kl..kl+7 (kl a multiple of 8) of row r: K-steps of 16 columns (kTcStepA bytes), in a step the core
// matrices of 8 rows (256 bytes a row group: the two 8-column halves, 128 bytes apart).
__device__ __forceinline__ int tc_aoff(int r, int kl) {
  return (kl >> 4) * kTcStepA + (r >> 3) * 256 + ((kl >> 3) & 1) * 128 + (r & 7) * 16;
}

// Four byte codes (or nibbles, already shifted into the low half of each byte) of w as two fp16
// pairs 1024 + code (the exponent trick: fp16 0x6400 | u is 1024 + u for u < 1024).
__device__ __forceinline__ void tc_magic4(uint32_t w, __half2 &lo, __half2 &hi) {
  const uint32_t a = prmt(w, 0x64646464u, 0x5140u), b = prmt(w, 0x64646464u, 0x7362u);
  lo = *reinterpret_cast<const __half2 *>(&a);
  hi = *reinterpret_cast<const __half2 *>(&b);
}
__device__ __forceinline__ uint32_t tc_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// Half h (columns 128h .. 128h + 127) of one repacked 16 x 256 tile into the A buffer at rows
// 16 i .. 16 i + 15, by one warp. The tile's 16-byte pieces (common.h's tile_pos): piece (o, lane =
// 4 g + c) holds rows g and g + 8 (words 0, 2 and 1, 3), elements 8o .. 8o + 7 of group c (and, int4,
// group c + 4 in the high nibbles; int8: pieces 4h + o). Lane (g, c) takes pieces o0 and o0 + 1 and
// writes 8 fp16 values a row a piece. int4: (q - z) s with fp16 arithmetic (q exact, then two roundings);
// int8: the code itself (exact), the row scale comes in the epilogue.
template <int KIND>
__device__ __forceinline__ void tc_dequant_half(const uint8_t *__restrict__ tile, int h, uint8_t *abuf, int i,
                                                int lane, int o0, bool present) {
  const int g = lane >> 2, c = lane & 3;
  const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));  // 1024
  const __half2 k1152 = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1024 + 128
  __half2 s0 = k1024, s1 = k1024, z0 = k1024, z1 = k1024;
  if (KIND == kKindInt4 && present) {
    const uint4 sz = *reinterpret_cast<const uint4 *>(tile + kTileCodes4 + lane * 16);
    const uint32_t sw = h ? sz.y : sz.x, zw = h ? sz.w : sz.z;  // (s of row g, row g + 8) at half h
    s0 = __half2half2(__ushort_as_half(uint16_t(sw & 0xFFFF)));
    s1 = __half2half2(__ushort_as_half(uint16_t(sw >> 16)));
    z0 = __half2half2(__ushort_as_half(uint16_t(zw & 0xFFFF)));
    z1 = __half2half2(__ushort_as_half(uint16_t(zw >> 16)));
  }
#pragma unroll
  for (int o = o0; o < o0 + 2; ++o) {
    uint4 out0 = make_uint4(0, 0, 0, 0), out1 = make_uint4(0, 0, 0, 0);
    if (present) {
      const int piece = KIND == kKindInt8 ? 4 * h + o : o;
      const uint4 w = *reinterpret_cast<const uint4 *>(tile + (piece * 32 + lane) * 16);
      const uint32_t words[4] = {w.x, w.z, w.y, w.w};  // row g: e8 0-3, 4-7; row g + 8: e8 0-3, 4-7
      uint32_t r[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __half2 lo, hi;
        if (KIND == kKindInt8) {
          tc_magic4(words[k] ^ 0x80808080u, lo, hi);  // 1024 + (code + 128)
          lo = __hsub2(lo, k1152);
          hi = __hsub2(hi, k1152);
        } else {
          tc_magic4((words[k] >> (4 * h)) & 0x0F0F0F0Fu, lo, hi);
          const __half2 zz = k < 2 ? z0 : z1, ss = k < 2 ? s0 : s1;
          lo = __hmul2(__hsub2(__hsub2(lo, k1024), zz), ss);
          hi = __hmul2(__hsub2(__hsub2(hi, k1024), zz), ss);
        }
        r[2 * k] = tc_bits(lo);
        r[2 * k + 1] = tc_bits(hi);
      }
      out0 = make_uint4(r[0], r[1], r[2], r[3]);
      out1 = make_uint4(r[4], r[5], r[6], r[7]);
    }
    const int kl = 32 * c + 8 * o;
    *reinterpret_cast<uint4 *>(abuf + tc_aoff(16 * i + g, kl)) = out0;
    *reinterpret_cast<uint4 *>(abuf + tc_aoff(16 * i + g + 8, kl)) = out1;
  }
}

struct TcArgs {
  const uint8_t *tiles;
  const float *row_scale, *bias;
  const uint8_t *xop;  // the tokens' fp16 operand: per column tile npad x 256 values (act_quant)
  int rtiles, ktiles, rows, tile_bytes, ntok, npad, splits, wstages;
  GemvOut out;
  int *status;
};

__device__ int tc_status_word;  // the first wait that ran out in any launch (0: none)

// The thread block cluster of a row tile's splits: every thread of every CTA of the cluster
// arrives and waits (release / acquire: shared-memory writes before it are seen by the cluster
// after it).
__device__ __forceinline__ void tc_cluster_sync() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A float of cluster CTA `rank`'s shared memory at this CTA's address p of the same variable.
__device__ __forceinline__ float tc_ld_cluster(const float *p, int rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(tc_saddr(p)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// The last steps of 16 tokens t0 .. t0 + 15 of tile row `row` (this thread's row; the lanes of a
// warp hold 32 consecutive rows): row scale, bias, and the output mode.
template <int KIND>
__device__ __forceinline__ void tc_finish(const TcArgs &a, int row, int lane, int mt, int t0, float (&v)[16]) {
  const GemvOut &out = a.out;
  const bool valid = row < a.rtiles * kTileRows;
  float scale = 1.f, bias = 0.f;
  if (valid && KIND == kKindInt8) scale = a.row_scale[row];
  if (valid && a.bias) bias = a.bias[row];
#pragma unroll
  for (int e = 0; e < 16; ++e) v[e] = v[e] * scale + bias;
  if (out.mode == kGlu) {
    // tile rows 0-7 gate, 8-15 up: lane l (l % 16 < 8) pairs with lane l + 8
    const int r16 = lane & 15, o = (row >> 4) * (kTileRows / 2) + r16;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float u = __shfl_down_sync(0xffffffffu, v[e], 8);
      if (t0 + e < a.ntok && valid && r16 < 8 && o < a.rows) {
        const float gv = v[e];
        // blocks.SiLU: x / (1 + exp(-x)) (internal/llm/blocks/blocks.go:395-399)
        out.y[size_t(t0 + e) * out.ldy + o] = gv / (1.0f + expf(-gv)) * u;
      }
    }
  } else if (out.mode == kLogits) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      unsigned long long key = 0ull;
      if (t0 + e < a.ntok && valid && row < a.rows) {
        const uint16_t hb = __half_as_ushort(__float2half_rn(v[e]));
        if (out.logits) out.logits[size_t(t0 + e) * out.ldy + row] = hb;
        key = argmax_key(hb, uint32_t(row));
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) {
        const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, key, off);
        key = o2 > key ? o2 : key;
      }
      if (lane == 0 && key) atomicMax(&out.amax[(t0 + e) * kAmaxSlots + (mt % kAmaxSlots)], key);
    }
  } else if (valid && row < a.rows) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      if (t0 + e >= a.ntok) continue;
      float *p = out.y + size_t(t0 + e) * out.ldy + row;
      *p = out.mode == kAdd ? *p + v[e] : v[e];
    }
  }
}

template <int KIND>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t tc_smem[];
  __shared__ uint64_t wfull[kTcMaxW], wempty[kTcMaxW], bfull[kTcBStages], bempty[kTcBStages];
  __shared__ uint64_t afull[2], aempty[2], done;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x / a.splits, sp = blockIdx.x % a.splits;
  const int per = a.ktiles / a.splits, rem = a.ktiles % a.splits;
  const int kt0 = sp * per + min(sp, rem), nkt = per + (sp < rem ? 1 : 0);
  const int WS = a.wstages;
  const int raw_bytes = kTcTiles * a.tile_bytes, b_bytes = a.npad * kTileCols * 2;
  uint8_t *raw = tc_smem;
  uint8_t *bop = raw + WS * raw_bytes;
  uint8_t *aop = bop + kTcBStages * b_bytes;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < WS; ++s) {
      tc_bar_init(&wfull[s], 1);
      tc_bar_init(&wempty[s], kTcDeq);  // the dequantising warps have read the stage
    }
    for (int s = 0; s < kTcBStages; ++s) {
      tc_bar_init(&bfull[s], 1);
      tc_bar_init(&bempty[s], 1);  // the MMA commit
    }
    for (int h = 0; h < 2; ++h) {
      tc_bar_init(&afull[h], kTcDeq);
      tc_bar_init(&aempty[h], 1);
    }
    tc_bar_init(&done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_saddr(&tmem_base)),
                 "r"(kTcMaxN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // the weights: the 8 tiles of each column tile, WS column tiles ahead
      int present = 0;
      for (int i = 0; i < kTcTiles; ++i) present += mt * kTcTiles + i < a.rtiles;
      for (int j = 0; j < nkt; ++j) {
        const int s = j % WS, kt = kt0 + j;
        if (j >= WS) tc_wait(&wempty[s], ((j / WS) - 1) & 1, a.status, 1);
        tc_expect_tx(&wfull[s], unsigned(present * a.tile_bytes));
        for (int i = 0; i < kTcTiles; ++i) {
          const int rt = mt * kTcTiles + i;
          if (rt < a.rtiles)
            tc_bulk(raw + s * raw_bytes + i * a.tile_bytes, a.tiles + (size_t(rt) * a.ktiles + kt) * a.tile_bytes,
                    unsigned(a.tile_bytes), &wfull[s]);
        }
      }
    }
  } else if (warp == kTcBWarp) {
    if (lane == 0) {
      // the tokens' operand (the previous kernel's output), two column tiles ahead; a warp of its
      // own, so that waiting for the previous kernel holds back none of the weight copies
      pdl_wait();
      for (int j = 0; j < nkt; ++j) {
        const int s = j % kTcBStages, kt = kt0 + j;
        if (j >= kTcBStages) tc_wait(&bempty[s], ((j / kTcBStages) - 1) & 1, a.status, 7);
        tc_expect_tx(&bfull[s], unsigned(b_bytes));
        tc_bulk(bop + s * b_bytes, a.xop + size_t(kt) * b_bytes, unsigned(b_bytes), &bfull[s]);
      }
    }
  } else if (warp == 1) {
    // MMA issue: 8 MMAs (K = 16 each) per half column tile
    if (lane == 0) {
      const uint32_t idesc = tc_idesc(a.npad);
      int acc = 0;
      for (int j = 0; j < nkt; ++j) {
        const int s = j % kTcBStages;
        tc_wait(&bfull[s], (j / kTcBStages) & 1, a.status, 2);
        for (int h = 0; h < 2; ++h) {
          tc_wait(&afull[h], j & 1, a.status, 3);
          tc_fence_after();
          const uint32_t abase = tc_saddr(aop + h * kTcABytes);
          const uint32_t bbase = tc_saddr(bop + s * b_bytes);
#pragma unroll
          for (int st = 0; st < 8; ++st) {
            const uint64_t ad = tc_desc(abase + st * kTcStepA, 128, 256);
            const uint64_t bd = tc_desc(bbase + (h * 8 + st) * a.npad * 32, 128, 256);
            tc_mma(tmem, ad, bd, idesc, acc);
            acc = 1;
          }
          tc_commit(&aempty[h]);
        }
        tc_commit(&bempty[s]);
      }
      tc_commit(&done);
    }
  } else {
    // dequantisation (warps 2 + 2i and 3 + 2i: row tile i, pieces 0-1 and 2-3), then the epilogue
    const int dw = warp - 2, ti = dw >> 1;
    const bool present = mt * kTcTiles + ti < a.rtiles;
    for (int j = 0; j < nkt; ++j) {
      const int s = j % WS;
      tc_wait(&wfull[s], (j / WS) & 1, a.status, 4);
      const uint8_t *tile = raw + s * raw_bytes + ti * a.tile_bytes;
      for (int h = 0; h < 2; ++h) {
        if (j >= 1) tc_wait(&aempty[h], (j - 1) & 1, a.status, 5);
        tc_dequant_half<KIND>(tile, h, aop + h * kTcABytes, ti, lane, 2 * (dw & 1), present);
        tc_fence_proxy();
        __syncwarp();
        if (lane == 0) tc_arrive(&afull[h]);
      }
      __syncwarp();
      if (lane == 0) tc_arrive(&wempty[s]);
    }
    tc_wait(&done, 0, a.status, 6);
    tc_fence_after();
    pdl_wait();
    // this warp's quarter of the accumulator (rows 32 q + lane) and 16 of its columns (tokens)
    const int q = warp & 3, t0 = 16 * (dw >> 2);
    const int row = mt * kTcRows + 32 * q + lane;  // tile row index (16 rows a tile)
    const uint32_t taddr = tmem + (uint32_t(32 * q) << 16) + uint32_t(t0);
    const bool mine = t0 < a.npad;  // uniform over the warp
    if (a.splits == 1) {
      if (mine) {
        float v[16];
        tc_ld16(taddr, v);
        tc_finish<KIND>(a, row, lane, mt, t0, v);
      }
    } else if (mine) {
      // this split's partial sums into the CTA's own shared memory (the A buffers, free now),
      // [token][128 rows], for the cluster's reduction below
      float v[16];
      tc_ld16(taddr, v);
      float *red = reinterpret_cast<float *>(aop);
#pragma unroll
      for (int e = 0; e < 16; ++e) red[(t0 + e) * kTcRows + 32 * q + lane] = v[e];
    }
  }
  if (a.splits > 1) {
    // the splits of a row tile are one thread block cluster: split r adds rows [r RR, r RR + RR) of
    // every split's partials, in split order, through distributed shared memory, and runs the
    // epilogue on them (RR = 128 / splits: one or more 16-row tiles, whose GLU pairs and argmax
    // lanes stay in one warp)
    tc_cluster_sync();
    if (warp >= 2 && warp < 2 + kTcDeq) {
      const int dw = warp - 2;
      const int RR = kTcRows / a.splits;
      const int rgs = (RR + 31) / 32;  // row groups of 32 lanes
      const float *red = reinterpret_cast<const float *>(aop);
      for (int u = dw; u < rgs * 4; u += kTcDeq) {
        const int rg = u >> 2, t0 = 16 * (u & 3);
        if (t0 >= a.npad) continue;
        const int rl = sp * RR + 32 * rg + lane;  // the tile-local row
        const bool mine = 32 * rg + lane < RR;
        // split by split, its 16 values loaded together (one remote round trip a split)
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0.f;
        for (int k = 0; k < a.splits; ++k) {
          float u[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) u[e] = mine ? tc_ld_cluster(red + (t0 + e) * kTcRows + rl, k) : 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] += u[e];
        }
        // rows outside this split's share take part in the warp's shuffles with nothing to write
        tc_finish<KIND>(a, mine ? mt * kTcRows + rl : 0x7fffffff, lane, mt, t0, v);
      }
    }
    tc_cluster_sync();  // no CTA leaves (or reuses its shared memory) while others still read it
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcMaxN) : "memory");
  }
}

// The weight stages that fit beside the operand ring and the A buffers, and the shared memory.
int tc_wstages(int tile_bytes, int npad) {
  const int room = kTcSmem - kTcBStages * npad * kTileCols * 2 - 2 * kTcABytes;
  return std::min(kTcMaxW, room / (kTcTiles * tile_bytes));
}
size_t tc_smem_bytes(int tile_bytes, int npad) {
  return size_t(tc_wstages(tile_bytes, npad)) * kTcTiles * tile_bytes + size_t(kTcBStages) * npad * kTileCols * 2 +
         2 * kTcABytes;
}

}  // namespace

namespace {
int *g_tc_status[64];  // each device's tc_status_word (tc_gemm_prepare, outside any capture)
}  // namespace

char *tc_gemm_prepare() {
  int dev = 0;
  HC_TRY_CUDA(cudaGetDevice(&dev));
  HC_TRY_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(&g_tc_status[dev & 63]), tc_status_word));
  const int mx = kTcSmem;
  HC_TRY_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<kKindInt8>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx));
  HC_TRY_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<kKindInt4>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx));
  return nullptr;
}

// Column-tile splits of a row tile (one thread block cluster, so 1, 2, 4 or 8): the fewest waves
// of CTAs times the column tiles a CTA walks, plus a CTA's fixed cost of about two column tiles'.
int tc_splits(const DevMat &W, int sms) {
  const int mtiles = (W.rtiles + kTcTiles - 1) / kTcTiles;
  int best = 1;
  long best_cost = -1;
  for (int s = 1; s <= 8 && s <= W.ktiles; s *= 2) {
    const long waves = (long(mtiles) * s + sms - 1) / sms;
    const long cost = waves * ((W.ktiles + s - 1) / s + 2);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

void tc_gemm(const DevMat &W, const uint8_t *xop, int ntok, const GemvOut &out, int sms, cudaStream_t st) {
  const int npad = (ntok + 15) / 16 * 16;
  const int mtiles = (W.rtiles + kTcTiles - 1) / kTcTiles;
  const int splits = tc_splits(W, sms);
  int dev = 0;
  cudaGetDevice(&dev);
  int *status = g_tc_status[dev & 63];
  const TcArgs a{W.tiles, W.row_scale, W.bias, xop, W.rtiles, W.ktiles, W.rows, W.tile_bytes, ntok, npad, splits,
                 tc_wstages(W.tile_bytes, npad), out, status};
  const size_t smem = tc_smem_bytes(W.tile_bytes, npad);
  // programmatic stream serialization (as launch_pdl) and the splits of a row tile as one cluster
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(mtiles * splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = unsigned(splits);
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  if (W.kind == kKindInt8)
    cudaLaunchKernelEx(&cfg, tc_gemm_kernel<kKindInt8>, a);
  else
    cudaLaunchKernelEx(&cfg, tc_gemm_kernel<kKindInt4>, a);
}

int tc_status_take() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, tc_status_word, sizeof(int)) != cudaSuccess) return 0;
  if (v) cudaMemcpyToSymbol(tc_status_word, &zero, sizeof(int));
  return v;
}

}  // namespace hc
