// gemv.cu: the decode GEMV over repacked integer tiles, and the activation quantiser it reads.
//
// One CTA (8 warps) owns 8 / wpr row tiles of 16 rows; the wpr warps of a row tile split its column
// tiles. Per column tile a warp issues 8 integer MMAs (m16n8k32) whose A operand is the tile's codes
// (unpacked in registers from HBM) and whose B operand is the activation: the hi bytes and the lo
// bytes (the residual at 1/256) of one group on two of B's columns, so that each MMA adds, for 16
// rows, the exact integer dot products of 8 columns of 4 groups at once (common.h). Lane (g, c)
// then scales its rows g, g+8 by the weight scale (and zero point) and the activation's scale of
// its groups c and 4 + c in float32; 2 shuffles add the 4 lanes of a row.
#include <algorithm>
#include <mutex>

#include "device.cuh"
#include "kernels.h"

namespace hc {
namespace {

// The batched activation layout (9..64 tokens in nb blocks of 8): per (k-tile kt, group G, block
// b) 576 bytes at act_tn_offset: lane (g, c) of the MMA reads its B registers as the 16 bytes at
// 16 (4g + c) -- token 8b + g's hi bytes 4c..4c+3 and 16+4c..19+4c of the group, then its lo bytes
// likewise -- and the (S, X) of tokens 8b + 2c, 8b + 2c + 1 as the 16 bytes at 512 + 16c.
__device__ __forceinline__ size_t act_tn_offset(int kt, int G, int b, int nb) {
  return (size_t(kt * kGroupsPerTile + G) * nb + b) * kActTile;
}

// The end of both GEMV kernels: part[w][t][r] holds warp w's sum for token t and row r of its row
// tile, of row-tile block blk (default blockIdx.x); the wpr warps of a row tile are added, scaled and written as out.mode says, for tokens
// t < nt. Ends with the argmax atomics of kLogits (bmax is the CTA's per-token key, zeroed before).
template <int KIND, int NT>
__device__ __forceinline__ void gemv_finish(float (*part)[NT][kTileRows], unsigned long long *bmax, int nt,
                                            const float *__restrict__ row_scale, const float *__restrict__ bias,
                                            int rtiles, int rows, int wpr, const GemvOut &out, int warps = 8,
                                            int blk = -1) {
  const int rpc = warps / wpr;
  if (blk < 0) blk = blockIdx.x;
  __syncthreads();
  for (int idx = threadIdx.x; idx < rpc * NT * kTileRows; idx += blockDim.x) {
    const int l2 = idx / (NT * kTileRows), t = (idx / kTileRows) % NT, r16 = idx % kTileRows;
    const int tile_r = blk * rpc + l2;
    if (tile_r >= rtiles || t >= nt) continue;
    auto value = [&](int rr) {
      float v = 0.f;
      for (int k = 0; k < wpr; ++k) v += part[l2 * wpr + k][t][rr];
      const int row = tile_r * kTileRows + rr;
      if (KIND == kKindInt8) v *= row_scale[row];
      if (KIND == kKindMx) v *= 0.5f;  // the doubled e2m1 values (mxfp4.go:90)
      if (bias) v += bias[row];
      return v;
    };
    if (out.mode == kGlu) {
      if (r16 >= kTileRows / 2) continue;
      const int o = tile_r * (kTileRows / 2) + r16;
      if (o >= rows) continue;
      const float gv = value(r16), uv = value(r16 + kTileRows / 2);
      // blocks.SiLU: x / (1 + exp(-x)) (internal/llm/blocks/blocks.go:395-399)
      out.y[size_t(t) * out.ldy + o] = gv / (1.0f + expf(-gv)) * uv;
      continue;
    }
    const int row = tile_r * kTileRows + r16;
    if (row >= rows) continue;
    const float v = value(r16);
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
    if (threadIdx.x < nt)
      atomicMax(&out.amax[threadIdx.x * kAmaxSlots + (blockIdx.x % kAmaxSlots)], bmax[threadIdx.x]);
  }
}

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

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Shared memory of the fused one-token GEMV: the activation tiles [NT][ktiles].
__host__ __device__ constexpr size_t gv_smem(int nt, int ktiles) { return size_t(nt) * ktiles * kActTile; }

// The RMS norm's column order, shared by act_quant_kernel and act_build so that both add the same
// per-thread partial sums: in round k, lane (sub = lane / 8, i = lane % 8) of warp w holds the 4
// columns 32 G + 4i .. + 3 of group G = 32k + 4w + sub (groups: ktiles x 8, a multiple of 8, so a
// warp's 4 groups are all in range or all past the end).
__device__ __forceinline__ int act_group(int k, int warp, int lane) { return k * 32 + warp * 4 + (lane >> 3); }

// Four columns of a row, 0 past n; a 16-byte load when the row allows it.
__device__ __forceinline__ void load4(const float *p, int c0, int n, bool vec, float v[4]) {
  if (vec && c0 + 3 < n) {
    const float4 q = *reinterpret_cast<const float4 *>(p + c0);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = c0 + e < n ? p[c0 + e] : 0.f;
  }
}

// Quantises group G from its 8 lanes' 4 values each (quant_vals' arithmetic: the maximum and the
// integer sum are order-free, the rest per element) into the token-major tiles at tt.
__device__ __forceinline__ void quant4(const float v[4], uint8_t *tt, int G, int lane) {
  const int i4 = (lane & 7) * 4;
  float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const bool nz = m > 0.f;
  const float qi = nz ? 127.0f / m : 0.f;  // quant_vals' inv and S
  const float S = nz ? m / 127.0f : 0.f;
  uint32_t hw = 0, lw = 0;
  int xs = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float h = rintf(v[e] * qi);
    const float rr = fmaf(-h, S, v[e]);
    const float l = fminf(fmaxf(rintf(rr * (256.0f * qi)), -127.f), 127.f);
    const int hq = int(int8_t(h)), lq = int(int8_t(l));
    hw |= uint32_t(uint8_t(hq)) << (8 * e);
    lw |= uint32_t(uint8_t(lq)) << (8 * e);
    xs += hq * 256 + lq;
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) xs += __shfl_xor_sync(0xffffffffu, xs, o);
  uint8_t *tile = tt + size_t(G / kGroupsPerTile) * kActTile;
  const int gi = G % kGroupsPerTile;
  *reinterpret_cast<uint32_t *>(tile + gi * 64 + i4) = hw;
  *reinterpret_cast<uint32_t *>(tile + gi * 64 + 32 + i4) = lw;
  if ((lane & 7) == 0)
    *reinterpret_cast<float2 *>(tile + kGroupsPerTile * 64 + gi * 8) =
        make_float2(S, nz ? float(xs) * (1.0f / 256.0f) : 0.f);
}

// The normed value of a column: act_quant_kernel's arithmetic.
__device__ __forceinline__ float norm_val(float x, float inv, float unit, float r, float w) {
  const float xs = unit ? x : x * inv;
  const float y = xs * r;
  return y * w;
}

// The activation tiles of NT rows into shared memory, by a CTA of 256 threads, with the bytes of
// act_quant_kernel. Rows of up to RM rounds (2 x 1024 columns) are read once, into registers,
// with their norm weights, and quantised from there after the sum of squares; longer rows are
// read again for the quantisation.
template <int NT>
__device__ void act_build(const ActSrc &src, int ktiles, uint8_t *sm) {
  __shared__ double red[32];
  constexpr int RM = 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i4 = (lane & 7) * 4;
  const float inv = src.scale == 1.f ? 1.f : 1.f / src.scale;
  const bool unit = src.scale == 1.f;
  const int n = src.n, groups = ktiles * kGroupsPerTile, rounds = (groups + 31) / 32;
  const bool wvec = (reinterpret_cast<uintptr_t>(src.norm_w) & 15) == 0;
#pragma unroll 1
  for (int t = 0; t < NT; ++t) {
    const float *xt = src.x + size_t(src.rows ? src.rows[t].head_src : t) * src.ldx;
    const bool vec = (reinterpret_cast<uintptr_t>(xt) & 15) == 0;
    uint8_t *tt = sm + size_t(t) * ktiles * kActTile;
    if (rounds <= RM) {
      float v[RM][4], w[RM][4];
#pragma unroll
      for (int k = 0; k < RM; ++k) {
        const int G = act_group(k, warp, lane);
        const bool in = k < rounds && G < groups;
        float z[4] = {0.f, 0.f, 0.f, 0.f};
        if (in) load4(xt, G * kGroup + i4, n, vec, v[k]);
        else for (int e = 0; e < 4; ++e) v[k][e] = 0.f;
        if (in && src.norm_w) load4(src.norm_w, G * kGroup + i4, n, wvec, w[k]);
        else for (int e = 0; e < 4; ++e) w[k][e] = z[e];
      }
      float r = 1.f;
      if (src.norm_w) {
        double s = 0;
#pragma unroll
        for (int k = 0; k < RM; ++k) {
          const int c0 = act_group(k, warp, lane) * kGroup + i4;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (k < rounds && c0 + e < n && act_group(k, warp, lane) < groups) {
              const float xs = unit ? v[k][e] : v[k][e] * inv;
              const float sq = xs * xs;
              s += double(sq);
            }
          }
        }
        s = block_sum_d(s, red);
        const float ms = float(s / double(n));
        r = float(1.0 / sqrt(double(ms) + double(src.eps16)));
      }
#pragma unroll
      for (int k = 0; k < RM; ++k) {
        const int G = act_group(k, warp, lane);
        if (k >= rounds || k * 32 + warp * 4 >= groups) break;  // uniform over the warp
        float q[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          q[e] = src.norm_w && G * kGroup + i4 + e < n ? norm_val(v[k][e], inv, unit, r, w[k][e]) : v[k][e];
        quant4(q, tt, G, lane);
      }
    } else {
      float r = 1.f;
      if (src.norm_w) {
        double s = 0;
#pragma unroll 1
        for (int k = 0; k < rounds; ++k) {
          const int G = act_group(k, warp, lane);
          if (G >= groups) break;
          float x[4];
          load4(xt, G * kGroup + i4, n, vec, x);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (G * kGroup + i4 + e < n) {
              const float xs = unit ? x[e] : x[e] * inv;
              const float sq = xs * xs;
              s += double(sq);
            }
          }
        }
        s = block_sum_d(s, red);
        const float ms = float(s / double(n));
        r = float(1.0 / sqrt(double(ms) + double(src.eps16)));
      }
#pragma unroll 2
      for (int k = 0; k < rounds; ++k) {
        const int G = act_group(k, warp, lane);
        if (k * 32 + warp * 4 >= groups) break;  // uniform over the warp
        float x[4], w[4];
        load4(xt, G * kGroup + i4, n, vec, x);
        if (src.norm_w) {
          load4(src.norm_w, G * kGroup + i4, n, wvec, w);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (G * kGroup + i4 + e < n) x[e] = norm_val(x[e], inv, unit, r, w[e]);
        }
        quant4(x, tt, G, lane);
      }
    }
  }
  __syncthreads();
}

// One token-a-column GEMV. A CTA takes the row-tile blocks blockIdx.x, + gridDim.x, ... (a block:
// 8 / wpr row tiles): one when the activation tiles come from act (the grid covers them all),
// several when act is null and the CTA builds the tiles from src once, into shared memory, for
// all its blocks (the grid is then capped at the CTAs the SMs hold at once).
template <int KIND, int NT>
__global__ void __launch_bounds__(256) gemv_kernel(const uint8_t *__restrict__ tiles,
                                                   const float *__restrict__ row_scale,
                                                   const float *__restrict__ bias,
                                                   const uint8_t *__restrict__ act, int rtiles,
                                                   int ktiles, int rows, int wpr, GemvOut out, ActSrc src) {
  constexpr int TB = KIND == kKindInt8 ? kTileInt8 : (KIND == kKindInt4 ? kTileInt4 : kTileMx);
  extern __shared__ __align__(16) uint8_t gv_act[];  // the activation tiles when act is null
  __shared__ float part[8][NT][kTileRows];
  __shared__ unsigned long long bmax[NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rpc = 8 / wpr;
  const int lrt = warp / wpr, ks = warp % wpr;
  const int nblk = (rtiles + rpc - 1) / rpc;
  pdl_trigger();
  if (threadIdx.x < NT) bmax[threadIdx.x] = 0ull;
  // the first weight tile does not depend on the kernels before: load it before waiting for them
  int blk = blockIdx.x;
  bool mine = blk * rpc + lrt < rtiles && ks < ktiles;
  WTile<KIND> wt;
  if (mine) wt.load(tiles + (size_t(blk * rpc + lrt) * ktiles + ks) * TB, lane);
  pdl_wait();
  if (!act) {  // uniform: build the activation tiles from the rows (while the first tile loads)
    act_build<NT>(src, ktiles, gv_act);
    act = gv_act;
  }
#pragma unroll 1
  for (;;) {
    const int rt = blk * rpc + lrt;
    float vg[NT], vg8[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) vg[t] = vg8[t] = 0.f;
    if (mine) {
      for (int kt = ks; kt < ktiles; kt += wpr) {
        WTile<KIND> nx;  // the next tile in flight while this one computes
        if (kt + wpr < ktiles) nx.load(tiles + (size_t(rt) * ktiles + kt + wpr) * TB, lane);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          BFrag<KIND> bf;
          bf.load(act + (size_t(t) * ktiles + kt) * kActTile, lane);
          wa_mma<KIND>(wt, bf, vg[t], vg8[t]);
        }
        wt = nx;
      }
    }
    // the next block's first tile in flight during this block's reduction
    const int nb = blk + gridDim.x;
    const bool nmine = nb < nblk && nb * rpc + lrt < rtiles && ks < ktiles;
    if (nmine) wt.load(tiles + (size_t(nb * rpc + lrt) * ktiles + ks) * TB, lane);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float a = quad_sum(vg[t]), b = quad_sum(vg8[t]);
      if (c == 0) {
        part[warp][t][g] = a;
        part[warp][t][g + 8] = b;
      }
    }
    gemv_finish<KIND, NT>(part, bmax, NT, row_scale, bias, rtiles, rows, wpr, out, 8, blk);
    if (nb >= nblk) break;
    __syncthreads();  // part is rewritten by the next block
    blk = nb;
    mine = nmine;
  }
}

// ---- the batched GEMV: tokens on the MMA's n ----------------------------------------------
// For 9..64 tokens the same tiles are read once for all of them. Per group G of a tile a warp
// gathers the m16n8k32 A operand whose k is G's 32 columns (tile_pos: lane (g, c) takes rows g,
// g + 8 and columns 4c..4c+3, 16+4c..19+4c, which lane 4g + G % 4 of the tile layout holds as the
// two words j = 2 (c & 1), +1 of pieces c / 2 and 2 + c / 2; int8 pieces 4 (G / 4) + those), and
// B is 8 tokens' hi (then lo) bytes of G. D is then, exactly, the group's integer dot product of
// 16 rows x 8 tokens, which lane (g, c) scales for rows g, g + 8 and tokens 2c, 2c + 1 with the
// same float32 arithmetic as the token-a-column GEMV (wa_mma): s S (hi + lo/256 - z Xq) for int4,
// S (hi + lo/256) for int8, 2^(e-127) S hi for mxfp4.

// Dynamic shared memory of gemm_tn_kernel<KIND, nb, warps, ..>: warps x 2 stages of nb x 576 bytes
// (the larger of that and the warps x 8nb x 16 float partials).
constexpr int gemm_tn_smem(int nb, int warps = 8) { return warps * 2 * nb * kActTile; }
constexpr int kTnNarrowRows = 512;  // row tiles below which the batched GEMV takes 16-warp CTAs

__device__ __forceinline__ uint32_t ldg32(const uint8_t *p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }
__device__ __forceinline__ uint2 ldg64(const uint8_t *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }

// WARPS warps a CTA; GS: the warps that share one k-tile's 8 groups (1, or 2 for the narrow
// matrices, so that each warp walks fewer steps). A warp's units are u = ks, ks + wpr, ... of the
// row tile's ktiles x GS units, unit u being groups (u % GS) * 8 / GS .. of k-tile u / GS.
template <int KIND, int NB, int WARPS, int GS>
__global__ void __launch_bounds__(WARPS * 32) gemm_tn_kernel(const uint8_t *__restrict__ tiles,
                                                      const float *__restrict__ row_scale,
                                                      const float *__restrict__ bias,
                                                      const uint8_t *__restrict__ act, int ntok,
                                                      int rtiles, int ktiles, int rows, int wpr,
                                                      GemvOut out) {
  constexpr int TB = KIND == kKindInt8 ? kTileInt8 : (KIND == kKindInt4 ? kTileInt4 : kTileMx);
  constexpr int NT = 8 * NB;
  constexpr int SB = NB * kActTile;  // one (k-tile, group)'s B operands of all the tokens
  // dynamic shared memory (gemm_tn_smem): each warp's two stages of B, later the CTA's partials
  extern __shared__ __align__(16) uint8_t tn_smem[];
  float (*part)[NT][kTileRows] = reinterpret_cast<float (*)[NT][kTileRows]>(tn_smem);
  __shared__ unsigned long long bmax[NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  constexpr int SPU = kGroupsPerTile / GS;  // steps (groups) a unit
  const int rpc = WARPS / wpr;
  const int lrt = warp / wpr, ks = warp % wpr;
  const int rt = blockIdx.x * rpc + lrt;
  const int units = ktiles * GS;
  uint8_t *stage = tn_smem + warp * 2 * SB;
  pdl_trigger();
  if (threadIdx.x < NT) bmax[threadIdx.x] = 0ull;
  float acc[NB][4];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
  const bool mine = rt < rtiles && ks < units;
  // the first weight tile does not depend on the kernels before: bring it towards L2 meanwhile
  constexpr int kLines = (TB + 127) / 128;
  if (mine && lane < kLines)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(tiles + (size_t(rt) * ktiles + ks / GS) * TB + lane * 128));
  pdl_wait();
  // The warp walks its (k-tile, group) steps in order; the B operands of step i + 1 are copied
  // into the other stage (cp.async, 16 bytes a lane a copy) while step i computes.
  auto issue = [&](int kt, int G, int buf) {
    const uint8_t *src = act + act_tn_offset(kt, G, 0, NB);
    uint8_t *dst = stage + buf * SB;
    for (int i = lane; i < SB / 16; i += 32) cp_async16(dst + 16 * i, src + 16 * i);
  };
  auto unit_kt = [&](int u) { return u / GS; };
  auto unit_g0 = [&](int u) { return (u % GS) * SPU; };
  if (mine) {
    const int steps = ((units - ks + wpr - 1) / wpr) * SPU;
    issue(unit_kt(ks), unit_g0(ks), 0);
    cp_async_commit();
    const uint8_t *tile = nullptr;
    int u = ks - wpr, G = 0;
#pragma unroll 1
    for (int it = 0; it < steps; ++it) {
      const int buf = it & 1;
      if (it % SPU == 0) {
        u += wpr;
        G = unit_g0(u);
        tile = tiles + (size_t(rt) * ktiles + unit_kt(u)) * TB;
        if (u + wpr < units && lane < kLines)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(tiles + (size_t(rt) * ktiles + unit_kt(u + wpr)) * TB + lane * 128));
      } else {
        ++G;
      }
      if (it + 1 < steps) {
        const int u1 = ks + ((it + 1) / SPU) * wpr;
        issue(unit_kt(u1), unit_g0(u1) + (it + 1) % SPU, buf ^ 1);
      }
      cp_async_commit();
      cp_async_wait_1();  // this step's copies (all groups but the newest) are in
      __syncwarp();
      const uint8_t *sb = stage + buf * SB;
      {
        const int h = G >> 2, Ls = 4 * g + (G & 3);
        const int piece0 = (KIND == kKindInt8 ? 4 * h : 0) + (c >> 1);
        const uint2 w01 = ldg64(tile + (piece0 * 32 + Ls) * 16 + 8 * (c & 1));
        const uint2 w23 = ldg64(tile + ((piece0 + 2) * 32 + Ls) * 16 + 8 * (c & 1));
        uint32_t a[4];
        float s0 = 1.f, s8 = 1.f, z0 = 0.f, z8 = 0.f;
        if (KIND == kKindInt8) {
          a[0] = w01.x; a[1] = w01.y; a[2] = w23.x; a[3] = w23.y;
        } else if (KIND == kKindInt4) {
          const int sh = 4 * h;
          a[0] = (w01.x >> sh) & 0x0F0F0F0Fu; a[1] = (w01.y >> sh) & 0x0F0F0F0Fu;
          a[2] = (w23.x >> sh) & 0x0F0F0F0Fu; a[3] = (w23.y >> sh) & 0x0F0F0F0Fu;
          const uint32_t sz = ldg32(tile + kTileCodes4 + Ls * 16 + 4 * h);      // s(g), s(g+8)
          const uint32_t zz = ldg32(tile + kTileCodes4 + Ls * 16 + 8 + 4 * h);  // z(g), z(g+8)
          const __half2 s2 = *reinterpret_cast<const __half2 *>(&sz);
          const __half2 z2 = *reinterpret_cast<const __half2 *>(&zz);
          s0 = __low2float(s2); s8 = __high2float(s2);
          z0 = __low2float(z2); z8 = __high2float(z2);
        } else {
          const uint32_t w[4] = {w01.x, w01.y, w23.x, w23.y};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t x = w[j], xs = x << 4;
            a[j] = h ? e2m1x4(x, xs, 0xFBEAu, (x >> 16) & 0x7777u) : e2m1x4(x, xs, 0xD9C8u, x & 0x7777u);
          }
          const uint32_t e4 = ldg32(tile + kTileCodes4 + Ls * 4);
          s0 = __uint_as_float(((e4 >> (16 * h)) & 0xffu) << 23);
          s8 = __uint_as_float(((e4 >> (16 * h + 8)) & 0xffu) << 23);
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          // B registers of token 8b + g and the (S, X) of tokens 8b + 2c, 8b + 2c + 1 (the lane's D
          // columns); the padding tokens of the last block are zero groups
          const uint8_t *blk = sb + b * kActTile;
          const uint4 bq = reinterpret_cast<const uint4 *>(blk)[lane];
          const float4 sx = reinterpret_cast<const float4 *>(blk + 512)[c];
          const uint32_t bh0 = bq.x, bh1 = bq.y, bl0 = bq.z, bl1 = bq.w;
          const float2 x0 = make_float2(sx.x, sx.y), x1 = make_float2(sx.z, sx.w);
          int dh[4] = {0, 0, 0, 0};
          if (KIND == kKindInt4) mma_u8s8(dh, a[0], a[1], a[2], a[3], bh0, bh1);
          else mma_s8s8(dh, a[0], a[1], a[2], a[3], bh0, bh1);
          if (KIND == kKindMx) {
            // d: (row g, t0), (g, t0+1), (g+8, t0), (g+8, t0+1)
            acc[b][0] = fmaf(float(dh[0]) * s0, x0.x, acc[b][0]);
            acc[b][1] = fmaf(float(dh[1]) * s0, x1.x, acc[b][1]);
            acc[b][2] = fmaf(float(dh[2]) * s8, x0.x, acc[b][2]);
            acc[b][3] = fmaf(float(dh[3]) * s8, x1.x, acc[b][3]);
          } else {
            int dl[4] = {0, 0, 0, 0};
            if (KIND == kKindInt4) mma_u8s8(dl, a[0], a[1], a[2], a[3], bl0, bl1);
            else mma_s8s8(dl, a[0], a[1], a[2], a[3], bl0, bl1);
            const float p0 = fmaf(float(dl[0]), 1.0f / 256.0f, float(dh[0]));
            const float p1 = fmaf(float(dl[1]), 1.0f / 256.0f, float(dh[1]));
            const float p2 = fmaf(float(dl[2]), 1.0f / 256.0f, float(dh[2]));
            const float p3 = fmaf(float(dl[3]), 1.0f / 256.0f, float(dh[3]));
            if (KIND == kKindInt4) {
              acc[b][0] = fmaf(s0 * x0.x, fmaf(-z0, x0.y, p0), acc[b][0]);
              acc[b][1] = fmaf(s0 * x1.x, fmaf(-z0, x1.y, p1), acc[b][1]);
              acc[b][2] = fmaf(s8 * x0.x, fmaf(-z8, x0.y, p2), acc[b][2]);
              acc[b][3] = fmaf(s8 * x1.x, fmaf(-z8, x1.y, p3), acc[b][3]);
            } else {
              acc[b][0] = fmaf(x0.x, p0, acc[b][0]);
              acc[b][1] = fmaf(x1.x, p1, acc[b][1]);
              acc[b][2] = fmaf(x0.x, p2, acc[b][2]);
              acc[b][3] = fmaf(x1.x, p3, acc[b][3]);
            }
          }
        }
      }
      __syncwarp();  // every lane is done with this stage before step it + 2 copies into it
    }
    cp_async_wait_0();
  }
  __syncthreads();  // the partials overwrite the stages of every warp
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int t0 = 8 * b + 2 * c;
    part[warp][t0][g] = acc[b][0];
    part[warp][t0 + 1][g] = acc[b][1];
    part[warp][t0][g + 8] = acc[b][2];
    part[warp][t0 + 1][g + 8] = acc[b][3];
  }
  gemv_finish<KIND, NT>(part, bmax, ntok, row_scale, bias, rtiles, rows, wpr, out, WARPS);
}

int dev_sms();
constexpr int kGvSlab = 128 * 1024;  // the activation tiles a CTA builds, at most
template <int KIND>
int gemv_occupancy(int ntok, int smem);

// The token-a-column GEMV of 1..8 tokens: a CTA a block when the activation tiles come from act;
// when the CTAs build them (act null), as many CTAs as the SMs hold, each over several blocks.
template <int KIND>
void gv_launch(const DevMat &W, const uint8_t *act, int ntok, const GemvOut &out, const ActSrc &src,
               cudaStream_t st) {
  const int wpr = W.ktiles >= 8 ? 8 : (W.ktiles >= 4 ? 4 : (W.ktiles >= 2 ? 2 : 1));
  const int rpc = 8 / wpr;
  const int nblk = (W.rtiles + rpc - 1) / rpc;
  const size_t smem = act ? 0 : gv_smem(ntok, W.ktiles);
  const int grid = act ? nblk : std::min(nblk, dev_sms() * gemv_occupancy<KIND>(ntok, int(smem)));
  switch (ntok) {
#define HC_NT(n)                                                                                     \
  case n:                                                                                            \
    launch_pdl(gemv_kernel<KIND, n>, dim3(grid), dim3(256), smem, st, W.tiles, W.row_scale, W.bias, act, \
               W.rtiles, W.ktiles, W.rows, wpr, out, src);                                           \
    break;
    HC_NT(1) HC_NT(2) HC_NT(3) HC_NT(4) HC_NT(5) HC_NT(6) HC_NT(7) HC_NT(8)
#undef HC_NT
  }
}

// The batched GEMV of 9..64 tokens.
template <int KIND>
void launch_kind(const DevMat &W, const uint8_t *act, int ntok, const GemvOut &out, int wpr,
                 int grid, cudaStream_t st) {
  switch (ntok) {
    default: {
      // narrow matrices (few row tiles): 16 warps a row tile, two to a k-tile's groups
      const bool narrow = W.rtiles < kTnNarrowRows;
      int twpr = wpr, tgrid = grid;
      if (narrow) {
        const int units = 2 * W.ktiles;
        twpr = units >= 16 ? 16 : (units >= 8 ? 8 : (units >= 4 ? 4 : 2));
        tgrid = (W.rtiles + 16 / twpr - 1) / (16 / twpr);
      }
      switch ((ntok + 7) / 8) {
#define HC_NB(b)                                                                                           \
  case b:                                                                                                  \
    if (narrow)                                                                                            \
      launch_pdl(gemm_tn_kernel<KIND, b, 16, 2>, dim3(tgrid), dim3(512), gemm_tn_smem(b, 16), st, W.tiles, \
                 W.row_scale, W.bias, act, ntok, W.rtiles, W.ktiles, W.rows, twpr, out);                   \
    else                                                                                                   \
      launch_pdl(gemm_tn_kernel<KIND, b, 8, 1>, dim3(tgrid), dim3(256), gemm_tn_smem(b), st, W.tiles,     \
                 W.row_scale, W.bias, act, ntok, W.rtiles, W.ktiles, W.rows, twpr, out);                   \
    break;
        HC_NB(2) HC_NB(3) HC_NB(4) HC_NB(5) HC_NB(6) HC_NB(7) HC_NB(8)
#undef HC_NB
      }
    }
  }
}

// ---- the activation quantiser --------------------------------------------------------------

// The batched layout: group G of k-tile kt for token t.
__device__ __forceinline__ void quant_group_tn(float v, uint8_t *act, int kt, int G, int t, int nb, int lane) {
  const QGroup q = quant_vals(v);
  uint8_t *blk = act + act_tn_offset(kt, G, t / 8, nb);
  const int g = t % 8, c = (lane % 16) / 4, at = (4 * g + c) * 16 + (lane / 16) * 4 + lane % 4;
  blk[at] = uint8_t(q.hq);
  blk[at + 8] = uint8_t(q.lq);
  if (lane == 0) *reinterpret_cast<float2 *>(blk + 512 + g * 8) = make_float2(q.S, q.X);
}

// One CTA per (token, column tile): the RMS norm's sum of squares is taken over the whole row by
// every CTA (the row is a few KB in L2), then the CTA quantises its tile's 8 groups, one warp each.
// With nb > 0 the tiles take the batched layout, and the rows past ntok of the last block of 8
// are written as zero groups.
__global__ void __launch_bounds__(256) act_quant_kernel(const float *__restrict__ x, int ldx,
                                                        int n, const float *__restrict__ norm_w,
                                                        float scale, float eps16,
                                                        uint8_t *__restrict__ act, int ktiles,
                                                        int ntok, int nb, const StepTok *__restrict__ rows,
                                                        int f16pad) {
  __shared__ double red[32];
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.y, kt = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (t >= ntok) {  // padding of the batched layouts (uniform over the CTA)
    if (f16pad) {
      const int col = (kt * kGroupsPerTile + warp) * kGroup + lane;
      *reinterpret_cast<__half *>(act + f16op_offset(t, col, f16pad)) = __float2half_rn(0.f);
    } else {
      quant_group_tn(0.f, act, kt, warp, t, nb, lane);
    }
    return;
  }
  const float *xt = x + size_t(rows ? rows[t].head_src : t) * ldx;
  const float inv = scale == 1.f ? 1.f : 1.f / scale;
  float r = 1.f;
  if (norm_w) {  // act_build's per-thread column order (act_group)
    double s = 0;
    const int groups = ktiles * kGroupsPerTile, i4 = (lane & 7) * 4;
    for (int k = 0; k * 32 < groups; ++k) {
      const int G = act_group(k, warp, lane);
      if (G >= groups) break;
      for (int e = 0; e < 4; ++e) {
        const int i = G * kGroup + i4 + e;
        if (i < n) {
          const float xs = scale == 1.f ? xt[i] : xt[i] * inv;
          const float sq = xs * xs;
          s += double(sq);
        }
      }
    }
    s = block_sum_d(s, red);
    const float ms = float(s / double(n));
    r = float(1.0 / sqrt(double(ms) + double(eps16)));
  }
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
  if (f16pad) *reinterpret_cast<__half *>(act + f16op_offset(t, col, f16pad)) = __float2half_rn(v);
  else if (nb) quant_group_tn(v, act, kt, warp, t, nb, lane);
  else quant_group(v, act + (size_t(t) * ktiles + kt) * kActTile, warp, lane);
}

// Merges the attention partials of one (token, head) (Flash-Decoding; with a sink logit when
// given, paged.Merge.AddSink, paged.go:281-297) and quantises the head's groups of 32 (a group
// never crosses a head: head_dim is 64 or 128).
__global__ void __launch_bounds__(128) attn_merge_kernel(const float *__restrict__ part_ml,
                                                         const float *__restrict__ part_o,
                                                         const float *__restrict__ sinks,
                                                         int heads, int hd, int splits,
                                                         uint8_t *__restrict__ act, int ktiles,
                                                         int nb, float *__restrict__ o_out, int f16pad) {
  __shared__ float wsh[64];
  __shared__ float stat[2];
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float *ml = part_ml + (size_t(t) * heads + h) * splits * 2;
  // the partials of this thread's element first (independent of the weights: one round trip)
  constexpr int kPre = 32;
  float pv[kPre];
  const int d0 = threadIdx.x;
  const float *po0 = part_o + ((size_t(t) * heads + h) * splits) * hd + d0;
#pragma unroll
  for (int s = 0; s < kPre; ++s) pv[s] = (s < splits && d0 < hd) ? po0[size_t(s) * hd] : 0.f;
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
    if (d == d0) {
#pragma unroll
      for (int s = 0; s < kPre; ++s)
        if (s < splits) o = fmaf(pv[s], wsh[s], o);
      for (int s = kPre; s < splits; ++s) o = fmaf(po[size_t(s) * hd], wsh[s], o);
    } else {
      for (int s = 0; s < splits; ++s) o = fmaf(po[size_t(s) * hd], wsh[s], o);
    }
    o *= invL;
    if (o_out) o_out[(size_t(t) * heads + h) * hd + d] = o;
    // one warp a group of 32: warp w of this head holds columns h*hd + 32w .. + 31
    const int gcol = h * hd + d;
    const int grp = gcol / kGroup;
    if (f16pad) *reinterpret_cast<__half *>(act + f16op_offset(t, gcol, f16pad)) = __float2half_rn(o);
    else if (nb) quant_group_tn(o, act, grp / kGroupsPerTile, grp % kGroupsPerTile, t, nb, lane);
    else quant_group(o, act + (size_t(t) * ktiles + grp / kGroupsPerTile) * kActTile, grp % kGroupsPerTile, lane);
  }
}

// Values of repacked rows with the format's own arithmetic (tile_value).
__global__ void dequant_kernel(const uint8_t *__restrict__ tiles, const float *__restrict__ row_scale,
                               int kind, int ktiles, int tile_bytes, int cols, int row0, int nrows,
                               float *__restrict__ out) {
  const long total = long(nrows) * cols;
  for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < total; i += long(gridDim.x) * blockDim.x) {
    const int r = row0 + int(i / cols), col = int(i % cols);
    out[i] = tile_value(tiles, row_scale, kind, ktiles, tile_bytes, r, col);
  }
}

}  // namespace

namespace {
int g_sms[64];  // SMs of each device (gemv_prepare)
constexpr int kGvSmem = 160 * 1024;  // the one-token GEMV's dynamic shared memory, at most
int dev_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  return g_sms[dev & 63] ? g_sms[dev & 63] : 148;
}
}  // namespace

char *gemv_prepare() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  HC_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return make_error("gemv_prepare: device ordinal beyond 64");
  std::lock_guard<std::mutex> lk(mu);
  if (done[dev]) return nullptr;
#define HC_SET(K, b)                                                                                  \
  HC_TRY_CUDA(cudaFuncSetAttribute(gemm_tn_kernel<K, b, 8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   gemm_tn_smem(b)));                                                   \
  HC_TRY_CUDA(cudaFuncSetAttribute(gemm_tn_kernel<K, b, 16, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   gemm_tn_smem(b, 16)));
#define HC_SET_K(K) HC_SET(K, 2) HC_SET(K, 3) HC_SET(K, 4) HC_SET(K, 5) HC_SET(K, 6) HC_SET(K, 7) HC_SET(K, 8)
  HC_SET_K(kKindInt8) HC_SET_K(kKindInt4) HC_SET_K(kKindMx)
#undef HC_SET_K
#undef HC_SET
#define HC_SETG(K, n)                                                                                \
  HC_TRY_CUDA(cudaFuncSetAttribute(gemv_kernel<K, n>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGvSmem));
#define HC_SETG_K(K) HC_SETG(K, 1) HC_SETG(K, 2) HC_SETG(K, 3) HC_SETG(K, 4) HC_SETG(K, 5) HC_SETG(K, 6) \
  HC_SETG(K, 7) HC_SETG(K, 8)
  HC_SETG_K(kKindInt8) HC_SETG_K(kKindInt4) HC_SETG_K(kKindMx)
#undef HC_SETG_K
#undef HC_SETG
  if (char *e = tc_gemm_prepare()) return e;
  if (char *e = attn_tc_prepare()) return e;
  HC_TRY_CUDA(cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev));
  done[dev] = true;
  return nullptr;
}

namespace {
// CTAs of gemv_kernel<KIND, ntok> one SM holds with smem bytes of activation tiles.
template <int KIND>
int gemv_occupancy(int ntok, int smem) {
  static std::mutex mu;
  static int cache[9][64];  // [ntok][smem / 4 KB] + 1, 0 = not asked yet
  const int key = smem >> 12;
  std::lock_guard<std::mutex> lk(mu);
  if (key < 64 && cache[ntok][key]) return cache[ntok][key] - 1;
  int b = 0;
  switch (ntok) {
#define HC_NT(n) \
  case n: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, gemv_kernel<KIND, n>, 256, smem); break;
    HC_NT(1) HC_NT(2) HC_NT(3) HC_NT(4) HC_NT(5) HC_NT(6) HC_NT(7) HC_NT(8)
#undef HC_NT
  }
  if (b < 1) b = 1;
  if (key < 64) cache[ntok][key] = b + 1;
  return b;
}

}  // namespace

int gemv_x(const DevMat &W, const ActSrc &src, int ntok, uint8_t *act, const GemvOut &out, cudaStream_t st) {
  // one token: the CTAs build the tiles themselves; for 2..8 the build's per-token norm passes
  // would run one after another in every CTA, and one act_quant launch (a CTA a token and column
  // tile) is faster
  if (ntok == 1 && gv_smem(ntok, W.ktiles) <= size_t(kGvSlab)) {
    switch (W.kind) {
      case kKindInt8: gv_launch<kKindInt8>(W, nullptr, ntok, out, src, st); break;
      case kKindInt4: gv_launch<kKindInt4>(W, nullptr, ntok, out, src, st); break;
      case kKindMx: gv_launch<kKindMx>(W, nullptr, ntok, out, src, st); break;
    }
    return 1;
  }
  act_quant(src.x, src.ldx, src.n, ntok, src.norm_w, src.scale, src.eps16, act, W.ktiles, st, src.rows,
            act_layout(W, ntok));
  gemv(W, act, ntok, out, st);
  return 2;
}

void gemv(const DevMat &W, const uint8_t *act, int ntok, const GemvOut &out, cudaStream_t st) {
  if (act_layout(W, ntok) == kActF16) {
    tc_gemm(W, act, ntok, out, dev_sms(), st);
    return;
  }
  if (ntok <= 8) {
    switch (W.kind) {
      case kKindInt8: gv_launch<kKindInt8>(W, act, ntok, out, ActSrc{}, st); break;
      case kKindInt4: gv_launch<kKindInt4>(W, act, ntok, out, ActSrc{}, st); break;
      case kKindMx: gv_launch<kKindMx>(W, act, ntok, out, ActSrc{}, st); break;
    }
    return;
  }
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
               float eps16, uint8_t *act, int ktiles, cudaStream_t st, const StepTok *rows, ActLayout layout) {
  const int f16pad = layout == kActF16 ? tc_npad(ntok) : 0;
  const int nb = layout == kActAuto ? act_tn_blocks(ntok) : 0;
  launch_pdl(act_quant_kernel, dim3(ktiles, f16pad ? f16pad : (nb ? 8 * nb : ntok)), dim3(256), 0, st, x, ldx, n,
             norm_w, scale, eps16, act, ktiles, ntok, nb, rows, f16pad);
}

void attn_merge_quant(const float *part_ml, const float *part_o, const float *sinks, int ntok,
                      int heads, int hd, int splits, uint8_t *act, int ktiles, float *o_out,
                      cudaStream_t st, ActLayout layout) {
  const int nb = layout == kActAuto ? act_tn_blocks(ntok) : 0;
  const int f16pad = layout == kActF16 ? tc_npad(ntok) : 0;
  // columns past heads*hd in the last tile are zero groups; so are the padding tokens of a batch
  const int n = heads * hd;
  if (f16pad) {
    cudaMemsetAsync(act, 0, size_t(ktiles) * f16pad * kTileCols * 2, st);
  } else if (nb) {
    cudaMemsetAsync(act, 0, size_t(ktiles) * kGroupsPerTile * nb * kActTile, st);
  } else if (n % kTileCols) {
    for (int t = 0; t < ntok; ++t)
      cudaMemsetAsync(act + (size_t(t) * ktiles + ktiles - 1) * kActTile, 0, kActTile, st);
  }
  launch_pdl(attn_merge_kernel, dim3(heads, ntok), dim3(hd), 0, st, part_ml, part_o, sinks, heads, hd, splits, act,
             ktiles, nb, o_out, f16pad);
}

void dequant(const DevMat &W, int row0, int nrows, float *out, cudaStream_t st) {
  const long total = long(nrows) * W.cols;
  const int grid = int(std::min<long>((total + 255) / 256, 4096));
  dequant_kernel<<<grid, 256, 0, st>>>(W.tiles, W.row_scale, W.kind, W.ktiles, W.tile_bytes,
                                       W.cols, row0, nrows, out);
}

}  // namespace hc
