// mk.h: the persistent decode kernel — one cooperative launch runs a whole decode step of a dense
// Qwen3/Llama model for up to 8 sequences that read one token each.
#ifndef HWNPU_MK_H
#define HWNPU_MK_H

#include "kernels.h"

namespace hc {

constexpr int kMkThreads = 256;         // 8 warps (lane 0 of warp 0 also issues the copies)
constexpr int kMkBlock = kMkThreads;
constexpr int kMkMaxTok = 8;
constexpr int kMkMaxSplits = 32;  // attention splits of a (token, kv head): one a lane in the merge
constexpr int kMkChunkTrace = 4096;  // ring chunks of CTA 0 a profiled step records

struct MkLayer {
  const uint8_t *qkv, *o, *gu, *down;  // repacked tiles
  const float *qkv_scale, *o_scale, *gu_scale, *down_scale;  // int8 row scales or null
  const float *qkv_bias, *o_bias;
  const float *post_norm;  // this layer's post-attention norm (gate/up's input)
  const float *next_norm;  // the next layer's input norm (or the final norm)
  const float *q_norm, *k_norm, *sinks;
  uint16_t *kc, *vc;       // this layer's caches [slots][kv_heads][cap][hd]
  int window;
};

struct MkParams {
  int layers, D, F, H, KV, hd, V, cap, ntok, kind;
  int kt_d, kt_f, kt_o;             // column tiles of D, F and H*hd inputs
  int rt_qkv, rt_head;              // row tiles of the fused qkv and of the head
  int splits;                       // attention splits per (token, kv head)
  float sc_in0, eps_in0, sc, eps;   // norm scales and fp16 epsilons: layer 0's input, the others,
  float sc_head, eps_head;          // and the final norm
  float score_scale;
  const MkLayer *L;                 // [layers], device memory
  const uint8_t *head;              // head tiles
  const float *head_scale;
  const uint16_t *embed;            // fp16 table or null (tied: the head's rows)
  const float *in_norm0;            // layer 0's input norm
  const uint32_t *rope;
  StepTok *toks;
  float *x;                         // [ntok][D] the residual stream
  float *h;                         // [ntok][F] silu(gate) * up
  float *qkv;                       // [ntok][(H + 2 KV) hd]
  float *part_ml, *part_o;          // attention partials [ntok][H][splits] (m, l) and [.][hd]
  uint16_t *logits;                 // [ntok][V] or null
  unsigned long long *amax;         // [ntok][kAmaxSlots]
  int32_t *am;                      // [ntok] greedy choices
  int32_t *gen_out, *gen_count;     // device feedback for hc_generate (null: none)
  unsigned *bar;                    // grid barrier counter (zeroed before each launch)
  int *status;                      // 0, or the code of a barrier that timed out
  long long spin_limit;             // clock cycles a barrier waits before it gives up
  unsigned long long *trace;        // null, or [4][phases][ctas] globaltimer ns: arrivals, releases,
                                    // inputs ready, chunks consumed; then [ctas][4] cycle counts
                                    // (0, 0, warp 0 waited, busy); then
                                    // [kMkChunkTrace][4] ns of CTA 0's ring chunks (copy issued,
                                    // warp 0 saw it full, warp 0 done, warp 7 done); then
                                    // [layers][8] clock64 events of CTA 1's attention unit
  int stages, stage_bytes, off_act, off_rows, off_att, off_sq, off_bar;  // shared-memory layout (mk_layout)
};

// Barriers of one step (the phases a trace records): 5 a layer (qkv, attention, o, gate/up,
// down), then the head.
#ifdef __CUDACC__
__host__ __device__
#endif
inline int mk_phases(int layers) { return 5 * layers + 1; }

// Whether a step of ntok tokens of this kind and attention shape has a compiled kernel.
bool mk_supported(int kind, int ntok, int hd, int rep);
// Dynamic shared memory the kernel needs for p on a grid of ctas (0: it does not fit).
size_t mk_smem(const MkParams &p, int ctas);
// mk_smem that also fills p's stage count and offsets.
size_t mk_layout(MkParams &p, int ctas);
// Allows every instantiation smem bytes of dynamic shared memory (once, outside a capture).
cudaError_t mk_prepare(size_t smem);
// Launches one step on st (cooperatively, one CTA per SM). Returns the error of the launch.
cudaError_t mk_launch(const MkParams &p, int ctas, cudaStream_t st);
// The largest co-resident grid of the kernel (CTAs), 0 when it cannot run.
int mk_max_ctas(int device);

}  // namespace hc

#endif
