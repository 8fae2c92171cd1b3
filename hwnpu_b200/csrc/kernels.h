// kernels.h: launch wrappers of the sm_100a kernels (gemv.cu, attn.cu, misc.cu).
#ifndef HWNPU_KERNELS_H
#define HWNPU_KERNELS_H

#include "common.h"

#include <algorithm>
#include <utility>

namespace hc {

// Launches k on st with programmatic stream serialization (device.cuh's pdl_trigger/pdl_wait): the
// kernel may start while the one before it in the stream finishes.
template <typename... KArgs, typename... Args>
void launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}


// A repacked matrix on the device (repack.h's Packed after the copy).
struct DevMat {
  Kind kind = kKindInt8;
  int fmt = HC_FMT_NONE;
  int rows = 0, cols = 0, rtiles = 0, ktiles = 0, tile_bytes = 0;
  const uint8_t *tiles = nullptr;
  const float *row_scale = nullptr;  // kKindInt8
  const float *bias = nullptr;       // or nullptr
};

// What the GEMV does with each output value v of token t and output row r.
enum GemvMode : int {
  kStore = 0,     // y[t][r] = v
  kAdd = 1,       // y[t][r] += v (the residual stream)
  kGlu = 2,       // tile rows 0-7 gate, 8-15 up: y[t][o] = silu(gate) * up, o = 8 * rtile + j
  kLogits = 3,    // fp16 logits[t][r] and the greedy choice folded into amax[t]
};

struct GemvOut {
  GemvMode mode = kStore;
  float *y = nullptr;
  int ldy = 0;
  uint16_t *logits = nullptr;           // kLogits: [t][ldy] fp16 bits, or nullptr
  unsigned long long *amax = nullptr;   // kLogits: [t], see argmax_key in misc.cu
};

// The activation operand a GEMV of ntok tokens reads (act_quant, attn_merge_quant):
//  kActAuto        int8 hi/lo tiles, token-major up to 8 tokens, the batched layout above (the
//                  MMA-sync GEMV kernels)
//  kActTokenMajor  int8 hi/lo tiles, token-major at any count (the expert GEMVs)
//  kActF16         fp16 values in the tensor-core GEMV's operand layout (tcgemm.cu): per column tile
//                  npad x 256 values, npad = ntok rounded up to 16, padding rows zero
enum ActLayout : int { kActAuto = 0, kActTokenMajor = 1, kActF16 = 2 };
// The layout gemv() reads for W at ntok tokens: 9..64 tokens of int8 / int4 matrices of at least
// kTcMinRows rows go to the tensor cores. Below that a matrix has too few 128-row tiles to fill
// the SMs without splitting its columns over a cluster, and the split's fixed costs outweigh what
// the tensor cores save (measured on B200 at 64 tokens: 2,048 x 2,048 takes 11.7 us on the MMA-sync
// GEMV against 22.0 us; 4,096 x 2,048 takes 12.3 us on the tensor cores against 19.3 us).
constexpr int kTcMinRows = 4096;
inline ActLayout act_layout(const DevMat &W, int ntok) {
  return ntok > 8 && W.kind != kKindMx && W.rows >= kTcMinRows ? kActF16 : kActAuto;
}
inline int tc_npad(int ntok) { return (ntok + 15) / 16 * 16; }

// Sets, once a device (call it with the device current, outside stream capture), the shared
// memory the batched GEMV asks for; hc_session_new and hc_linear_load call it.
char *gemv_prepare();

// y = x W^T for ntok (1..64) tokens whose activations act_quant wrote into act (in the layout
// act_layout(W, ntok) names): up to 8 tokens a token per MMA column group (gemv_kernel); 9..64
// tokens on the tensor cores (tc_gemm, int8 and int4) or on the MMA's n (gemm_tn_kernel, MXFP4).
void gemv(const DevMat &W, const uint8_t *act, int ntok, const GemvOut &out, cudaStream_t st);
// The tensor-core GEMV (tcgemm.cu) of 9..64 tokens: xop in kActF16 layout; sms: the device's SMs.
void tc_gemm(const DevMat &W, const uint8_t *xop, int ntok, const GemvOut &out, int sms, cudaStream_t st);
char *tc_gemm_prepare();
// The error code of the first tensor-core GEMV wait that ran out on the current device since the
// last call (0: none), cleared.
int tc_status_take();

// Per-token position data of a step, in device memory so that a captured graph replays it.
struct StepTok {
  int32_t token;  // id
  int32_t slot;   // sequence slot
  int32_t pos;    // position of this token
  int32_t head_src;  // entry j < the chunk's head rows: the chunk token whose logits are row j
  // the chunk index of the first token of this token's piece (its sequence's consecutive tokens
  // in the chunk): the keys and values of the piece's positions are read in float32 from the
  // chunk's stage rows, the earlier ones from the cache; -1: every key from the cache
  int32_t run0 = -1;
};

// The rows a GEMV's activation is made from (act_quant's arguments): ntok rows of x (stride ldx, n
// columns; row t is rows[t].head_src when rows is set), normed with norm_w (when set) as act_quant.
struct ActSrc {
  const float *x = nullptr;
  int ldx = 0, n = 0;
  const float *norm_w = nullptr;
  float scale = 1.f, eps16 = 0.f;
  const StepTok *rows = nullptr;
};
// y = x W^T from the rows themselves: for one token the GEMV builds its activation tiles in
// shared memory first (one launch, no act_quant); otherwise act_quant into act (sized for ntok
// tokens of W) and gemv. Returns the kernels launched.
int gemv_x(const DevMat &W, const ActSrc &src, int ntok, uint8_t *act, const GemvOut &out, cudaStream_t st);

// Blocks of 8 tokens of the batched activation layout that 9..64 tokens take (0: token-major).
inline int act_tn_blocks(int ntok) { return ntok > 8 ? (ntok + 7) / 8 : 0; }

// Quantises ntok rows of x (float32, stride ldx, n columns) into the GEMV's activation tiles
// (ktiles of kActTile bytes a token; for 9..64 tokens the batched layout of 8 act_tn_blocks(ntok)
// token rows, padding included), after an optional RMS norm: when norm_w is set,
// x is normed as qwen3's normScaled with scale (1 or 64) and epsilon eps16 (the fp16 constant
// f16(eps / scale^2)) and multiplied by norm_w (float32 values of fp16 weights).
// With rows set, token t's input is row rows[t].head_src of x (the head's rows of a chunk);
// layout: see ActLayout (the normed values are the same in all three).
void act_quant(const float *x, int ldx, int n, int ntok, const float *norm_w, float scale,
               float eps16, uint8_t *act, int ktiles, cudaStream_t st, const StepTok *rows = nullptr,
               ActLayout layout = kActAuto);

// Attention partials -> merged o (float32 [ntok][heads*hd]) -> activation operand of the output
// projection in the given layout (Flash-Decoding's merge with gpt-oss's sinks, paged.go:252-310).
void attn_merge_quant(const float *part_ml, const float *part_o, const float *sinks, int ntok,
                      int heads, int hd, int splits, uint8_t *act, int ktiles, float *o_out,
                      cudaStream_t st, ActLayout layout = kActTokenMajor);


struct AttnGeom {
  int heads, kv_heads, hd, cap, window;  // cap: positions a slot's cache holds
  float score_scale;                     // the fp16 score scale 1/sqrt(hd), as float
};

// The rows of the fused q|k|v projection (float32 [ntok][(heads + 2 kv_heads) hd]) -> per-head
// RMS norm of q and k (when qn/kn are set), RoPE with the fp16 tables rope[pos][hd/2] (cos, sin
// pairs as fp16 bits), q into q_out (float32 [ntok][heads][hd]) and k, v as fp16 into the
// cache at (slot, kv_head, pos).
// The paged int8 KV cache of one layer (HC_KV_INT8_PAGED): pages of kPage positions, per (page,
// kv head) the keys [kPage][hd] int8 (a position's row contiguous) and the values transposed,
// [hd][kPage] (a dimension's 16 positions contiguous: the operand the attention's P.V integer MMA
// reads), an fp16 scale per (page, head) for each, and the block table [slots][max_pages].
constexpr int kPage = 16;
struct PagedKV {
  const int8_t *k = nullptr, *v = nullptr;
  const uint16_t *kscale = nullptr, *vscale = nullptr;
  const int32_t *btab = nullptr;
  int max_pages = 0;
};

// Every token's rotated key and its value also go to kv_stage ([ntok][2][kv_heads][hd] float32),
// where the attention of the chunk reads its own pieces' keys (StepTok::run0); with kcache NULL (the
// paged int8 cache) nothing else is written, and kv_append_int8 quantises the rows into the pages
// after the chunk's attention.
void qkv_post(const float *qkv, const StepTok *toks, int ntok, const AttnGeom &g,
              const float *qn, const float *kn, float norm_scale, float eps16,
              const uint32_t *rope, float *q_out, uint16_t *kcache, uint16_t *vcache,
              float *kv_stage, cudaStream_t st);
void kv_append_int8(const float *stage, const StepTok *toks, int ntok, int kv_heads, int hd, const PagedKV &pk,
                    cudaStream_t st);

// Split-K decode attention over the fp16 cache: token t attends keys [lo, pos] of its slot
// (lo = pos - window + 1 with a window); `splits` partials of (m, l) and unnormalised o. The keys of
// a token's own piece come from kv_stage (float32, as qkv_post wrote them), the others from the cache.
void attn_split(const float *q, const StepTok *toks, int ntok, const AttnGeom &g,
                const uint16_t *kcache, const uint16_t *vcache, int splits, float *part_ml,
                float *part_o, cudaStream_t st, const PagedKV *paged = nullptr,
                const float *kv_stage = nullptr);

// attn_split over the paged int8 cache on the integer tensor cores (attn_tc.cu), for head_dim 64 or
// 128 and 1, 2 or 4 heads a kv head; false (nothing launched) for other shapes.
bool attn_paged_tc(const float *q, const StepTok *toks, int ntok, const AttnGeom &g, const PagedKV &pk, int splits,
                   float *part_ml, float *part_o, const float *kv_stage, cudaStream_t st);
char *attn_tc_prepare();

// Embedding rows of the step's tokens into x (float32 [ntok][hidden]): from an fp16 table, or
// (table nullptr) from the tied head's tiles, dequantised and rounded to fp16. Also resets amax.
void embed(const StepTok *toks, int ntok, const uint16_t *table, const DevMat *head, int hidden,
           float *x, unsigned long long *amax, cudaStream_t st);

// Reads the greedy choice out of amax keys.
void amax_to_index(const unsigned long long *amax, int ntok, int32_t *out, cudaStream_t st);

// ---- gpt-oss (moe.cu) -------------------------------------------------------------------------
// A dense matrix of 16-bit floats on the device: bf16 (the checkpoint's attention and head) or fp16
// (the router, whose weights gpt-oss's programs hold as fp16), row-major [rows][cols], cols a
// multiple of 8; float32 biases or null.
struct DevDense {
  const uint16_t *w = nullptr;
  int rows = 0, cols = 0;
  bool bf16 = true;
  const float *bias = nullptr;
};

// RMS norm (scale 1) of ntok rows of x into float32 y, rounded to fp16 when round16; with rows set,
// row t of y is row rows[t].head_src of x.
void rms_rows(const float *x, int ldx, int n, int ntok, const float *w, float eps16, float *y, int ldy, bool round16,
              cudaStream_t st, const StepTok *rows = nullptr);
// y = x W^T (+ bias) of ntok float32 rows; mode 0 store, 1 add into y, 2 store rounded to fp16,
// 3 fp16 logits (stride ldy) and greedy keys into amax.
void gemv16(const DevDense &W, const float *x, int ldx, int ntok, int mode, float *y, int ldy, uint16_t *logits,
            unsigned long long *amax, cudaStream_t st);
// The pairs (token, k) of each expert from the routing's idx ([npairs]): cnt[E], list[E][maxp].
void moe_group(const int32_t *idx, int npairs, int E, int *cnt, int *list, int maxp, cudaStream_t st);
// The experts' MXFP4 GEMV grouped by expert (W: all experts' tiles, experts row blocks of equal
// size): mode 0 gate/up (GLU tiles) + bias through gpt-oss's gated unit into out[pair][inter],
// act = the tokens' activation tiles; mode 1 down into out[pair][hidden], act = the pairs' tiles.
void moe_gemv(const DevMat &W, int experts, int mode, const int *cnt, const int *list, int maxp, int K,
              const uint8_t *act, const float *bias, float alpha, float limit, float *out, int ldo, cudaStream_t st);
// x[t] = f16(x[t]) + f16(sum over token t's experts in ascending number of w (y + down bias)).
void moe_combine(const float *y, const int32_t *idx, const float *w, int K, const float *dbias, int H, int ntok,
                 float *x, cudaStream_t st);

// Float32 values of rows [row0, row0+nrows) of a repacked matrix (the format's arithmetic).
void dequant(const DevMat &W, int row0, int nrows, float *out, cudaStream_t st);

// Argmax over fp16 rows (first largest wins); MoE softmax top-k routing.
void argmax_rows(const uint16_t *logits, int rows, int vocab, int32_t *out, cudaStream_t st);
void route(const float *logits, int rows, int n, int k, int32_t *idx, float *w, cudaStream_t st);

// Greedy speculative accept on the device: given the argmax of each of n rows and the n tokens
// read, writes kept (1..n) and next into res[0], res[1].
void spec_accept(const int32_t *amax_idx, const StepTok *toks, int n, int32_t *res,
                 cudaStream_t st);

// A bounded device-side wait of ms milliseconds (at most 2 s) on st: the injected stall that makes
// a step outlast its timeout in the failure tests, with nothing hung or faulted.
void device_stall(long ms, cudaStream_t st);

// The device-side token feedback of hc_generate: out[*count] = am[0], the next step reads that
// token at the next position.
void advance(StepTok *toks, const int32_t *am, int32_t *out, int32_t *count, cudaStream_t st);

}  // namespace hc

#endif
