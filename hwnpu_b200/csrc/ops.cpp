// ops.cpp: kernel entry points on caller-owned device memory (include/hwnpu_cuda.h), for parity
// tests and kernel timing: decode attention, greedy choice, MoE routing.
#include <string>
#include <vector>

#include "kernels.h"

namespace {
template <typename T>
char *tmp_alloc(T **p, size_t n, const char *what) {
  void *v = nullptr;
  if (char *e = hc::dev_alloc(&v, n * sizeof(T), what)) return e;
  *p = static_cast<T *>(v);
  return nullptr;
}
}  // namespace

extern "C" {

HC_API char *hc_attention_run(const float *q, const uint16_t *kcache, const uint16_t *vcache,
                              const float *sinks, float *o, int32_t ntok, int32_t heads,
                              int32_t kv_heads, int32_t head_dim, int32_t pos, int32_t cap,
                              int32_t window, const float *scale, void *stream) {
  if (!q || !kcache || !vcache || !o || !scale) return hc::make_error("hc_attention_run: NULL argument");
  if (ntok < 1 || heads < 1 || kv_heads < 1 || heads % kv_heads) return hc::make_error("hc_attention_run: bad heads");
  const int rep = heads / kv_heads;
  if (head_dim != 64 && head_dim != 128) return hc::make_error("hc_attention_run: head_dim must be 64 or 128");
  if (rep != 1 && rep != 2 && rep != 4 && rep != 8) return hc::make_error("hc_attention_run: heads per kv head must be 1, 2, 4 or 8");
  if (pos < 0 || cap < 1) return hc::make_error("hc_attention_run: bad positions");
  if (pos + ntok > cap && !(window > 0 && cap >= window + ntok - 1))
    return hc::make_error("hc_attention_run: positions beyond the cache (a ring needs window > 0 and cap >= window + ntok - 1)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int splits = 16;
  std::vector<hc::StepTok> toks(ntok);
  for (int t = 0; t < ntok; ++t) toks[t] = hc::StepTok{0, 0, pos + t, 0};
  hc::StepTok *dt = nullptr;
  float *ml = nullptr, *po = nullptr;
  uint8_t *act = nullptr;
  const int ktiles = (heads * head_dim + hc::kTileCols - 1) / hc::kTileCols;
  char *e = nullptr;
  if (!e) e = tmp_alloc(&dt, ntok, "step tokens");
  if (!e) e = tmp_alloc(&ml, size_t(ntok) * heads * splits * 2, "attention partials");
  if (!e) e = tmp_alloc(&po, size_t(ntok) * heads * splits * head_dim, "attention partials");
  if (!e) e = tmp_alloc(&act, size_t(ntok) * ktiles * hc::kActTile, "activation tiles");
  if (!e) e = hc::copy_h2d(dt, toks.data(), sizeof(hc::StepTok) * ntok, st);
  if (!e) {
    hc::AttnGeom g{heads, kv_heads, head_dim, cap, window, *scale};
    hc::attn_split(q, dt, ntok, g, kcache, vcache, splits, ml, po, st);
    hc::attn_merge_quant(ml, po, sinks, ntok, heads, head_dim, splits, act, ktiles, o, st);
    cudaError_t ce = cudaGetLastError();
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
    if (ce != cudaSuccess) e = hc::make_error(std::string("attention: ") + cudaGetErrorString(ce));
  }
  cudaFree(dt);
  cudaFree(ml);
  cudaFree(po);
  cudaFree(act);
  return e;
}

HC_API char *hc_argmax_run(const uint16_t *logits, int32_t rows, int32_t vocab, int32_t *out,
                           void *stream) {
  if (!logits || !out || rows < 1 || vocab < 1) return hc::make_error("hc_argmax_run: bad argument");
  hc::argmax_rows(logits, rows, vocab, out, static_cast<cudaStream_t>(stream));
  HC_TRY_CUDA(cudaGetLastError());
  return nullptr;
}

HC_API char *hc_route_run(const float *logits, int32_t rows, int32_t n, int32_t k, int32_t *idx,
                          float *w, void *stream) {
  if (!logits || !idx || !w || rows < 1) return hc::make_error("hc_route_run: bad argument");
  if (n < 1 || n > 256 || k < 1 || k > n) return hc::make_error("hc_route_run: n must be 1..256 and k 1..n");
  hc::route(logits, rows, n, k, idx, w, static_cast<cudaStream_t>(stream));
  HC_TRY_CUDA(cudaGetLastError());
  return nullptr;
}

}  // extern "C"
