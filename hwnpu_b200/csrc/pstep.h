// pstep.h: the persistent decode step — one cooperative launch runs a whole decode step of a dense
// Qwen3/Llama model for up to 8 tokens (any mix of sequences and positions) over the fp16 cache.
#ifndef HWNPU_PSTEP_H
#define HWNPU_PSTEP_H

#include "kernels.h"

namespace hc {

constexpr int kPsMaxTok = 8;        // tokens a launch reads
constexpr int kPsConsumers = 8;     // consumer warps
constexpr int kPsThreads = 32 * (kPsConsumers + 1);  // + the producer warp
constexpr int kPsSplitKeys = 64;    // keys of one attention split (fixed by position: [64 s, 64 s + 64))
constexpr int kPsStageAttn = 16384; // bytes of cached keys + values a ring stage carries

// One layer's device data.
struct PsLayer {
  const uint8_t *qkv, *o, *gu, *down;                        // repacked tiles
  const float *qkv_scale, *o_scale, *gu_scale, *down_scale;  // int8 row scales, or null
  const float *qkv_bias, *o_bias;                            // or null
  const float *in_norm, *post_norm, *q_norm, *k_norm;        // float32 norm weights (q/k: or null)
  const float *sinks;                                        // [heads] or null
  uint16_t *kc, *vc;                                         // the layer's cache [slots][kv][cap][hd]
  int window;                                                // 0: full attention
};

struct PsParams {
  int layers, D, F, H, KV, hd, V, cap, ntok;
  int kt_d, kt_f, kt_o;                 // column tiles of the D, F and H*hd inputs
  int rt_qkv, rt_o, rt_gu, rt_down, rt_head;
  int max_splits;                       // cap / kPsSplitKeys rounded up: the partials' stride
  float sc_in0, eps_in0, sc, eps, sc_head, eps_head;  // norm scales and fp16 epsilons
  float score_scale;
  const PsLayer *L;                     // [layers], device memory
  const uint8_t *head;
  const float *head_scale;
  const uint16_t *embed;                // fp16 table, or null (tied: the head's rows)
  const float *final_norm;
  const uint32_t *rope;                 // [cap][hd / 2] (cos, sin) fp16 pairs
  StepTok *toks;                        // [ntok]
  float *dx_o, *dx_down;                // [ntok][D] the o and down projections (the residual's deltas)
  float *qkv;                           // [ntok][(H + 2 KV) hd]
  float *attn;                          // [ntok][H hd] the merged attention output
  float *h;                             // [ntok][F] silu(gate) * up
  float *part_ml, *part_o;              // [ntok][H][max_splits] (m, l) and [..][hd]
  int *tickets;                         // [ntok][KV] merge tickets, then the head's ticket
  uint16_t *logits;                     // [ntok][V] or null
  unsigned long long *amax;             // [ntok][kAmaxSlots]
  int32_t *am;                          // [ntok] greedy choices
  int32_t *gen_out, *gen_count;         // hc_generate's device feedback, or null
  unsigned *bar;                        // grid barrier counter (zeroed before each launch)
  int *status;                          // 0, or the phase + 1 of the wait that gave up
  long long spin_limit;                 // clock cycles any wait may take before it gives up
  int stall_first_barrier;              // 1: the first grid barrier waits for one arrival more than
                                        // the grid has, so it runs out (the failure tests)
  unsigned long long *trace;            // null, or [phases][3] global-timer ns of CTA 0: inputs ready,
                                        // work done, barrier passed
  int stages, stage_bytes;              // the ring
};

// Phases of one step: 5 a layer (qkv, attention, o, gate/up, down), each ended by a grid barrier,
// then the head.
#ifdef __CUDACC__
__host__ __device__
#endif
inline int ps_phases(int layers) { return 5 * layers + 1; }

// Whether the step of this model shape has a compiled kernel (kind int8 or int4 throughout,
// head_dim 64 or 128, heads per kv head <= 8, contexts up to 16384 positions).
bool ps_supported(int kind, int hd, int rep, int cap);
// Dynamic shared memory of a launch of ntok tokens with the given ring (0: does not fit).
size_t ps_smem(const PsParams &p);
// Chooses the ring (stages, stage bytes) for p.ntok tokens; false when nothing fits.
bool ps_layout(PsParams &p, int kind);
// Allows the kernels their shared memory (once a device, outside a capture).
cudaError_t ps_prepare();
// Launches one step on st cooperatively, one CTA per SM (ctas of them).
cudaError_t ps_launch(const PsParams &p, int kind, int ctas, cudaStream_t st);
// The CTAs of the launch: the SM count when one CTA fits on every SM, else 0.
int ps_ctas(int device);

}  // namespace hc

#endif
