// misc.cu: embedding rows, greedy choice, MoE routing and the speculative accept on the device.
#include "device.cuh"
#include "kernels.h"

namespace hc {
namespace {

// llm.TokenRow (internal/llm/llm.go:43-60): the token's row of the embedding table, the program's
// fp16 input x; a tied table is the head's rows in its format, rounded to fp16.
__global__ void embed_kernel(const StepTok *__restrict__ toks, const uint16_t *__restrict__ table,
                             const uint8_t *__restrict__ tiles, const float *__restrict__ row_scale,
                             int kind, int ktiles, int tile_bytes, int hidden,
                             float *__restrict__ x, unsigned long long *__restrict__ amax) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.y;
  const int tok = toks[t].token;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < hidden; c += blockDim.x * gridDim.x) {
    float v;
    if (table) {
      v = __half2float(__ushort_as_half(table[size_t(tok) * hidden + c]));
    } else {
      v = tile_value(tiles, row_scale, kind, ktiles, tile_bytes, tok, c);
      v = __half2float(__float2half_rn(v));
    }
    x[size_t(t) * hidden + c] = v;
  }
  if (amax && blockIdx.x == 0)
    for (int i = threadIdx.x; i < kAmaxSlots; i += blockDim.x) amax[t * kAmaxSlots + i] = 0ull;
}

__global__ void amax_index_kernel(const unsigned long long *__restrict__ amax, int ntok,
                                  int32_t *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x, lane = threadIdx.x;
  unsigned long long k = 0;
  for (int i = lane; i < kAmaxSlots; i += 32) k = max(k, amax[t * kAmaxSlots + i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
  if (lane == 0) out[t] = int32_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
}

__global__ void argmax_kernel(const uint16_t *__restrict__ logits, int vocab,
                              int32_t *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
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
  pdl_trigger();
  pdl_wait();
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
  pdl_trigger();
  pdl_wait();
  int kept = n, next = am[n - 1];
  for (int i = 0; i + 1 < n; ++i) {
    if (am[i] != toks[i + 1].token) { kept = i + 1; next = am[i]; break; }
  }
  res[0] = kept;
  res[1] = next;
}

__global__ void advance_kernel(StepTok *__restrict__ toks, const int32_t *__restrict__ am,
                               int32_t *__restrict__ out, int32_t *__restrict__ count) {
  pdl_trigger();
  pdl_wait();
  const int i = *count;
  out[i] = am[0];
  toks[0].token = am[0];
  toks[0].pos += 1;
  *count = i + 1;
}

// One thread waits until ns nanoseconds of the global timer have passed (capped at 2 s).
__global__ void stall_kernel(unsigned long long ns) {
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  if (ns > 2000000000ull) ns = 2000000000ull;
  do {
    __nanosleep(100000);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  } while (t - t0 < ns);
}

}  // namespace

void device_stall(long ms, cudaStream_t st) {
  if (ms > 0) stall_kernel<<<1, 1, 0, st>>>((unsigned long long)ms * 1000000ull);
}

void advance(StepTok *toks, const int32_t *am, int32_t *out, int32_t *count, cudaStream_t st) {
  launch_pdl(advance_kernel, dim3(1), dim3(1), 0, st, toks, am, out, count);
}

void embed(const StepTok *toks, int ntok, const uint16_t *table, const DevMat *head, int hidden,
           float *x, unsigned long long *amax, cudaStream_t st) {
  launch_pdl(embed_kernel, dim3((hidden + 255) / 256, ntok), dim3(256), 0, st, toks, table,
             head ? head->tiles : nullptr, head ? head->row_scale : nullptr, head ? head->kind : 0,
             head ? head->ktiles : 0, head ? head->tile_bytes : 0, hidden, x, amax);
}

void amax_to_index(const unsigned long long *amax, int ntok, int32_t *out, cudaStream_t st) {
  launch_pdl(amax_index_kernel, dim3(ntok), dim3(32), 0, st, amax, ntok, out);
}

void argmax_rows(const uint16_t *logits, int rows, int vocab, int32_t *out, cudaStream_t st) {
  launch_pdl(argmax_kernel, dim3(rows), dim3(1024), 0, st, logits, vocab, out);
}

void route(const float *logits, int rows, int n, int k, int32_t *idx, float *w, cudaStream_t st) {
  route_kernel<<<(rows + 63) / 64, 64, 0, st>>>(logits, rows, n, k, idx, w);
}

void spec_accept(const int32_t *amax_idx, const StepTok *toks, int n, int32_t *res,
                 cudaStream_t st) {
  launch_pdl(spec_accept_kernel, dim3(1), dim3(1), 0, st, amax_idx, toks, n, res);
}

}  // namespace hc
