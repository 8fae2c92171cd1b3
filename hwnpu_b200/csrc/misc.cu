// misc.cu: embedding rows, greedy choice, MoE routing and the speculative accept on the device.
#include "device.cuh"
#include "kernels.h"

namespace hc {
namespace {

// The float32 value of (row, col) of a repacked matrix, as dequant_kernel computes it.
__device__ float tile_value(const uint8_t *tiles, const float *row_scale, int kind, int ktiles,
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

// llm.TokenRow (internal/llm/llm.go:43-60): the token's row of the embedding table, the program's
// fp16 input x; a tied table is the head's rows in its format, rounded to fp16.
__global__ void embed_kernel(const StepTok *__restrict__ toks, const uint16_t *__restrict__ table,
                             const uint8_t *__restrict__ tiles, const float *__restrict__ row_scale,
                             int kind, int ktiles, int tile_bytes, int hidden,
                             float *__restrict__ x, unsigned long long *__restrict__ amax) {
  const int t = blockIdx.x;
  const int tok = toks[t].token;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    float v;
    if (table) {
      v = __half2float(__ushort_as_half(table[size_t(tok) * hidden + c]));
    } else {
      v = tile_value(tiles, row_scale, kind, ktiles, tile_bytes, tok, c);
      v = __half2float(__float2half_rn(v));
    }
    x[size_t(t) * hidden + c] = v;
  }
  if (amax)
    for (int i = threadIdx.x; i < kAmaxSlots; i += blockDim.x) amax[t * kAmaxSlots + i] = 0ull;
}

__global__ void amax_index_kernel(const unsigned long long *__restrict__ amax, int ntok,
                                  int32_t *__restrict__ out) {
  const int t = blockIdx.x, lane = threadIdx.x;
  unsigned long long k = 0;
  for (int i = lane; i < kAmaxSlots; i += 32) k = max(k, amax[t * kAmaxSlots + i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
  if (lane == 0) out[t] = int32_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
}

__global__ void argmax_kernel(const uint16_t *__restrict__ logits, int vocab,
                              int32_t *__restrict__ out) {
  __shared__ unsigned long long best;
  if (threadIdx.x == 0) best = 0ull;
  __syncthreads();
  const uint16_t *row = logits + size_t(blockIdx.x) * vocab;
  unsigned long long k = 0;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) k = max(k, argmax_key(row[i], uint32_t(i)));
#pragma unroll
  for (int o = 16; o; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
  if ((threadIdx.x & 31) == 0) atomicMax(&best, k);
  __syncthreads();
  if (threadIdx.x == 0) out[blockIdx.x] = int32_t(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFull));
}

// experts.Routing.Choose with Score "softmax" and Norm (internal/llm/experts/weights.go:33-82):
// exp in float64 from the largest logit, the float32 sum in order, a stable descending choice
// of k, renormalised by the float32 sum of the chosen plus 1e-6. One thread a row.
__global__ void route_kernel(const float *__restrict__ logits, int rows, int n, int k,
                             int32_t *__restrict__ idx, float *__restrict__ w) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const float *lg = logits + size_t(r) * n;
  float m = -INFINITY;
  for (int e = 0; e < n; ++e) m = fmaxf(m, lg[e]);
  float score[256];
  float sum = 0.f;
  for (int e = 0; e < n; ++e) {
    score[e] = float(exp(double(lg[e] - m)));
    sum += score[e];
  }
  for (int e = 0; e < n; ++e) score[e] /= sum;
  uint32_t taken[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float tot = 0.f;
  for (int j = 0; j < k; ++j) {
    int best = -1;
    for (int e = 0; e < n; ++e) {
      if (taken[e >> 5] & (1u << (e & 31))) continue;
      if (best < 0 || score[e] > score[best]) best = e;
    }
    taken[best >> 5] |= 1u << (best & 31);
    idx[size_t(r) * k + j] = best;
    w[size_t(r) * k + j] = score[best];
    tot += score[best];
  }
  for (int j = 0; j < k; ++j) w[size_t(r) * k + j] /= tot + 1e-6f;
}

// chat/engine.go:1044-1058: keep draft i while the greedy pick after token i equals it.
__global__ void spec_accept_kernel(const int32_t *__restrict__ am, const StepTok *__restrict__ toks,
                                   int n, int32_t *__restrict__ res) {
  int kept = n, next = am[n - 1];
  for (int i = 0; i + 1 < n; ++i) {
    if (am[i] != toks[i + 1].token) { kept = i + 1; next = am[i]; break; }
  }
  res[0] = kept;
  res[1] = next;
}

__global__ void advance_kernel(StepTok *__restrict__ toks, const int32_t *__restrict__ am,
                               int32_t *__restrict__ out, int32_t *__restrict__ count) {
  const int i = *count;
  out[i] = am[0];
  toks[0].token = am[0];
  toks[0].pos += 1;
  *count = i + 1;
}

}  // namespace

void advance(StepTok *toks, const int32_t *am, int32_t *out, int32_t *count, cudaStream_t st) {
  advance_kernel<<<1, 1, 0, st>>>(toks, am, out, count);
}

void embed(const StepTok *toks, int ntok, const uint16_t *table, const DevMat *head, int hidden,
           float *x, unsigned long long *amax, cudaStream_t st) {
  embed_kernel<<<ntok, 256, 0, st>>>(toks, table, head ? head->tiles : nullptr,
                                     head ? head->row_scale : nullptr, head ? head->kind : 0,
                                     head ? head->ktiles : 0, head ? head->tile_bytes : 0, hidden,
                                     x, amax);
}

void amax_to_index(const unsigned long long *amax, int ntok, int32_t *out, cudaStream_t st) {
  amax_index_kernel<<<ntok, 32, 0, st>>>(amax, ntok, out);
}

void argmax_rows(const uint16_t *logits, int rows, int vocab, int32_t *out, cudaStream_t st) {
  argmax_kernel<<<rows, 1024, 0, st>>>(logits, vocab, out);
}

void route(const float *logits, int rows, int n, int k, int32_t *idx, float *w, cudaStream_t st) {
  route_kernel<<<(rows + 63) / 64, 64, 0, st>>>(logits, rows, n, k, idx, w);
}

void spec_accept(const int32_t *amax_idx, const StepTok *toks, int n, int32_t *res,
                 cudaStream_t st) {
  spec_accept_kernel<<<1, 1, 0, st>>>(amax_idx, toks, n, res);
}

}  // namespace hc
