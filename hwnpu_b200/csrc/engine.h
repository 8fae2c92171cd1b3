// engine.h: the device-resident model and session behind hc_model_* / hc_session_* / hc_step.
#ifndef HWNPU_ENGINE_H
#define HWNPU_ENGINE_H

#include <map>
#include <memory>
#include <vector>

#include "kernels.h"
#include "repack.h"

namespace hc {

int device_ordinal(const hc_device *d);
int device_sms(const hc_device *d);

constexpr int kMaxChunk = 64;  // tokens one pass of the GEMVs reads the weights for

// One repacked matrix in HBM.
struct DevLinear {
  DevMat m;
  void *tiles = nullptr, *scales = nullptr, *bias = nullptr;
  uint64_t bytes = 0;  // bytes a pass reads: tiles, row scales, biases
  ~DevLinear();
};

char *upload(const Packed &p, DevLinear *out, cudaStream_t st);
char *load_linear(const std::vector<RowRef> &rows, DevLinear *out, cudaStream_t st);

struct LayerW {
  std::unique_ptr<DevLinear> qkv, o, gu, down;
  float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  float *sinks = nullptr;  // fp16-rounded sink logits, or nullptr
  int window = 0;
  // gpt-oss: 16-bit-float attention and router, the experts' MXFP4 tiles (gate/up as GLU tiles of
  // each expert's even and odd rows, down) and their float32 biases
  DevDense qkv16, o16, router16;
  std::unique_ptr<DevLinear> egu, edown;
  float *egb = nullptr, *edb = nullptr;
};

// Norm settings of one RMS norm: the scale of qwen3's normScaled and its fp16 epsilon.
struct NormCfg {
  float scale = 1.f, eps16 = 0.f;
};

}  // namespace hc

struct hc_model {
  hc_device *dev = nullptr;
  int ordinal = 0, sms = 148;
  hc_model_desc d{};
  std::vector<hc::LayerW> layers;
  float *final_norm = nullptr;
  std::unique_ptr<hc::DevLinear> head;
  uint16_t *embed = nullptr;  // fp16 [vocab][hidden], or nullptr when tied
  bool gptoss = false;
  hc::DevDense head16;        // gpt-oss's bf16 head
  std::vector<double> inv_freq;
  float rope_factor = 1.f;
  hc::NormCfg norm_in0, norm_mid, norm_head;
  float score_scale = 1.f;
  uint64_t weight_bytes = 0;
  std::vector<void *> allocs;  // small device arrays (norms, sinks, embedding)
  ~hc_model();
};

struct hc_session {
  hc_model *m = nullptr;
  hc_session_opts o{};
  cudaStream_t st = nullptr;
  int cap = 0, splits = 1;
  uint16_t *kc = nullptr, *vc = nullptr;  // [layers][slots][kv_heads][cap][hd] fp16
  size_t layer_kv = 0;                    // elements of one layer's cache
  // HC_KV_INT8_PAGED: page pools of int8 keys [layers][pages][kv_heads][16][hd] and values stored
  // transposed [layers][pages][kv_heads][hd][16], scales [layers][pages][kv_heads] fp16, the block
  // table [slots][max_pages] (device, and its host copy) and the free pages
  bool paged = false;
  int8_t *kp = nullptr, *vp = nullptr;
  uint16_t *kps = nullptr, *vps = nullptr;
  int32_t *btab_dev = nullptr;
  std::vector<int32_t> btab;
  std::vector<int32_t> free_pages;
  int max_pages = 0, n_pages = 0;
  float *kv_stage = nullptr;              // [max_step][2][kv_heads][hd] the new rows before quantisation
  uint32_t *rope = nullptr;               // [cap][hd/2] (cos, sin) fp16 pairs
  std::vector<int> pos;                   // per slot
  std::vector<bool> poisoned;             // per slot: a failed step may have half written it
  // work buffers for one chunk of up to kMaxChunk tokens
  float *x = nullptr, *qkv = nullptr, *q = nullptr, *h = nullptr;
  uint8_t *act = nullptr;
  float *part_ml = nullptr, *part_o = nullptr;
  // gpt-oss: normed rows (moe_x), the attention output, router logits, the routing (indices and
  // weights [tokens][top_k]), each expert's pairs, the pairs' activation tiles, gated rows and outputs
  float *xn = nullptr, *oatt = nullptr, *mlog = nullptr, *mw = nullptr, *hh = nullptr, *ey = nullptr;
  int32_t *midx = nullptr;
  int *mcnt = nullptr, *mlist = nullptr;
  uint8_t *act2 = nullptr;
  hc::StepTok *toks_dev = nullptr, *toks_host = nullptr;
  uint16_t *logits_dev = nullptr;
  unsigned long long *amax = nullptr;
  int32_t *am_dev = nullptr, *am_host = nullptr, *res_dev = nullptr, *res_host = nullptr;
  int32_t *gen_out = nullptr, *gen_count = nullptr;  // hc_generate's tokens [cap] and counter
  cudaGraphExec_t gen_graph = nullptr;
  // captured step graphs by (tokens, accept kernel)
  std::map<int, cudaGraphExec_t> graphs;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  hc_stats stats{};
  uint64_t launches_per_chunk[hc::kMaxChunk + 1] = {};
  std::map<int, uint64_t> launches_per_key;
  ~hc_session();
};

#endif
