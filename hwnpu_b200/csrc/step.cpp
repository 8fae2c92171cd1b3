// step.cpp: sessions and the decode step (decode.Session.Step/Speculate, internal/llm/decode/
// decode.go:1221-1260; chat.tokenSession, internal/chat/session.go:26-32), one CUDA graph per
// chunk size replayed with the step's tokens and positions read from device memory.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>

#include "engine.h"

using hc::kMaxChunk;

hc_session::~hc_session() {
  if (!m) return;
  cudaSetDevice(m->ordinal);
  if (st) cudaStreamSynchronize(st);
  for (auto &g : graphs) cudaGraphExecDestroy(g.second);
  if (gen_graph) cudaGraphExecDestroy(gen_graph);
  if (gen_out) cudaFree(gen_out);
  if (gen_count) cudaFree(gen_count);
  for (void *p : {(void *)kp, (void *)vp, (void *)kps, (void *)vps, (void *)btab_dev, (void *)kv_stage})
    if (p) cudaFree(p);
  for (void *p : {(void *)kc, (void *)vc, (void *)rope, (void *)x, (void *)qkv, (void *)q, (void *)h,
                  (void *)act, (void *)part_ml, (void *)part_o, (void *)toks_dev, (void *)logits_dev,
                  (void *)amax, (void *)am_dev, (void *)res_dev})
    if (p) cudaFree(p);
  for (void *p : {(void *)xn, (void *)oatt, (void *)mlog, (void *)mw, (void *)hh, (void *)ey, (void *)midx,
                  (void *)mcnt, (void *)mlist, (void *)act2})
    if (p) cudaFree(p);
  if (toks_host) cudaFreeHost(toks_host);
  if (am_host) cudaFreeHost(am_host);
  if (res_host) cudaFreeHost(res_host);
  if (ev0) cudaEventDestroy(ev0);
  if (ev1) cudaEventDestroy(ev1);
  if (st) cudaStreamDestroy(st);
}

namespace {

constexpr int kMaxSplits = 64;
constexpr int kSplitKeys = 1024;  // keys a split reads, at most, for the chunk's longest context
constexpr int kSplitKeysPaged = 1024;  // the same over the paged int8 cache

// Attention splits of every (token, kv head) of a chunk of n tokens whose longest context is
// max_len positions: enough CTAs to fill the SMs twice (as for one token when n <= 8), and at
// most kSplitKeys keys a split for the longest (rounded up to a power of two, so that few step
// graphs differ by their splits).
int splits_for(const hc_session *s, int n, int max_len) {
  const int kv = int(s->m->d.kv_heads);
  // up to 8 tokens take the one-token count, so that a speculative verify row, or any row of a
  // small batch, is computed exactly as a one-token step (hc_generate) computes it
  const int rows = kv * (n <= 8 ? 1 : n);
  // the paged cache's tensor-core kernel: 4 warps a split, 3 CTAs a SM
  const bool wide = s->paged;
  int sp = ((wide ? 3 : 2) * s->m->sms) / rows;
  int by_len = 1;
  while (by_len < kMaxSplits && by_len * (wide ? kSplitKeysPaged : kSplitKeys) < max_len) by_len *= 2;
  return std::max(1, std::min(kMaxSplits, std::max(sp, by_len)));
}

// The longest context (positions read, its own included) of the chunk's tokens in toks_host.
int chunk_max_len(const hc_session *s, int n) {
  int m = 0;
  for (int i = 0; i < n; ++i) m = std::max(m, s->toks_host[i].pos + 1);
  return m;
}

template <typename T>
char *alloc(T **p, size_t count, const char *what) {
  void *v = nullptr;
  if (char *e = hc::dev_alloc(&v, count * sizeof(T), what)) return e;
  *p = static_cast<T *>(v);
  return nullptr;
}

hc::AttnGeom geom(const hc_session *s, int window) {
  const auto &d = s->m->d;
  return hc::AttnGeom{int(d.heads), int(d.kv_heads), int(d.head_dim), s->cap, window, s->m->score_scale};
}

// The paged int8 cache of layer li.
hc::PagedKV paged_of(const hc_session *s, size_t li) {
  const auto &d = s->m->d;
  const size_t per = size_t(s->n_pages) * d.kv_heads;
  hc::PagedKV pk;
  pk.k = s->kp + li * per * hc::kPage * d.head_dim;
  pk.v = s->vp + li * per * hc::kPage * d.head_dim;
  pk.kscale = s->kps + li * per;
  pk.vscale = s->vps + li * per;
  pk.btab = s->btab_dev;
  pk.max_pages = s->max_pages;
  return pk;
}

// Gives sequence `seq` pages for positions [p0, p1) (paged cache) and copies the changed part of
// its block table to the device, ordered on the session's stream before the step that writes them.
char *ensure_pages(hc_session *s, int seq, int p0, int p1) {
  if (!s->paged || p1 <= p0) return nullptr;
  int32_t *row = s->btab.data() + size_t(seq) * s->max_pages;
  const int g0 = p0 / hc::kPage, g1 = (p1 - 1) / hc::kPage;
  bool changed = false;
  for (int g = g0; g <= g1; ++g) {
    if (row[g] >= 0) continue;
    if (s->free_pages.empty()) return hc::make_error("step: no free KV page");
    row[g] = s->free_pages.back();
    s->free_pages.pop_back();
    changed = true;
  }
  if (changed) {
    HC_TRY_CUDA(cudaMemcpyAsync(s->btab_dev + size_t(seq) * s->max_pages + g0, row + g0,
                                sizeof(int32_t) * (g1 - g0 + 1), cudaMemcpyHostToDevice, s->st));
    HC_TRY_CUDA(cudaStreamSynchronize(s->st));  // the host row may change again at the next call
  }
  return nullptr;
}

// Returns the pages of `seq` past its first `len` positions to the free list.
void release_pages(hc_session *s, int seq, int len) {
  if (!s->paged) return;
  int32_t *row = s->btab.data() + size_t(seq) * s->max_pages;
  for (int g = (len + hc::kPage - 1) / hc::kPage; g < s->max_pages; ++g)
    if (row[g] >= 0) {
      s->free_pages.push_back(row[g]);
      row[g] = -1;
    }
}

// The rows a GEMV reads, normed as nc says (norm_w null: as they are).
hc::ActSrc src_of(const float *x, int ldx, int n, const float *norm_w, const hc::NormCfg &nc) {
  hc::ActSrc a;
  a.x = x;
  a.ldx = ldx;
  a.n = n;
  a.norm_w = norm_w;
  a.scale = norm_w ? nc.scale : 1.f;
  a.eps16 = norm_w ? nc.eps16 : 0.f;
  return a;
}

// Enqueues one chunk of n tokens (already in toks_dev) on the session's stream; returns the
// number of kernels launched. Only `heads` rows go through the final norm and the head: row j is
// chunk token toks[j].head_src (the rows a caller reads; none for the inside of a long prompt).
int enqueue_chunk(hc_session *s, int n, bool accept, int splits, int heads) {
  hc_model *m = s->m;
  const auto &d = m->d;
  const int D = int(d.hidden), F = int(d.inter), H = int(d.heads), KV = int(d.kv_heads);
  const int hd = int(d.head_dim), V = int(d.vocab);
  const int W = (H + 2 * KV) * hd;
  cudaStream_t st = s->st;
  int k = 0;
  hc::embed(s->toks_dev, n, m->embed, m->embed ? nullptr : &m->head->m, D, s->x, s->amax, st);
  ++k;
  for (size_t li = 0; li < m->layers.size(); ++li) {
    const hc::LayerW &w = m->layers[li];
    const hc::NormCfg nc = li == 0 ? m->norm_in0 : m->norm_mid;
    uint16_t *kcl = s->paged ? nullptr : s->kc + li * s->layer_kv;
    uint16_t *vcl = s->paged ? nullptr : s->vc + li * s->layer_kv;
    const hc::PagedKV pk = s->paged ? paged_of(s, li) : hc::PagedKV{};
    const hc::AttnGeom g = geom(s, w.window);
    hc::GemvOut o1;
    o1.mode = hc::kStore; o1.y = s->qkv; o1.ldy = W;
    k += hc::gemv_x(w.qkv->m, src_of(s->x, D, D, w.in_norm, nc), n, s->act, o1, st);
    hc::qkv_post(s->qkv, s->toks_dev, n, g, w.q_norm, w.k_norm, m->norm_mid.scale, m->norm_mid.eps16,
                 s->rope, s->q, kcl, vcl, s->kv_stage, st);
    hc::attn_split(s->q, s->toks_dev, n, g, kcl, vcl, splits, s->part_ml, s->part_o, st, s->paged ? &pk : nullptr,
                   s->kv_stage);
    if (s->paged) {  // the chunk's rows into the pages once its attention has read the earlier ones
      hc::kv_append_int8(s->kv_stage, s->toks_dev, n, KV, hd, pk, st);
      ++k;
    }
    hc::attn_merge_quant(s->part_ml, s->part_o, w.sinks, n, H, hd, splits, s->act, w.o->m.ktiles, nullptr, st,
                         hc::act_layout(w.o->m, n));
    hc::GemvOut o2;
    o2.mode = hc::kAdd; o2.y = s->x; o2.ldy = D;
    hc::gemv(w.o->m, s->act, n, o2, st);
    hc::GemvOut o3;
    o3.mode = hc::kGlu; o3.y = s->h; o3.ldy = F;
    k += hc::gemv_x(w.gu->m, src_of(s->x, D, D, w.post_norm, m->norm_mid), n, s->act, o3, st);
    k += hc::gemv_x(w.down->m, src_of(s->h, F, F, nullptr, hc::NormCfg{}), n, s->act, o2, st);
    k += 4;  // qkv_post, attn_split, attn_merge_quant, the o GEMV
  }
  if (heads > 0) {
    hc::GemvOut oh;
    oh.mode = hc::kLogits; oh.ldy = V; oh.logits = s->logits_dev; oh.amax = s->amax;
    hc::ActSrc hs = src_of(s->x, D, D, m->final_norm, m->norm_head);
    hs.rows = heads == n ? nullptr : s->toks_dev;
    k += hc::gemv_x(m->head->m, hs, heads, s->act, oh, st);
    hc::amax_to_index(s->amax, heads, s->am_dev, st);
    ++k;
  }
  if (accept) { hc::spec_accept(s->am_dev, s->toks_dev, n, s->res_dev, st); ++k; }
  return k;
}

// The gpt-oss step of a chunk (gptoss/build.go's attention part and moeHead, then
// experts.Host.runRow, experts/host.go:478-591, for every row): per layer the RMS norm, the bf16
// q|k|v projection and its biases, RoPE with YaRN's tables, attention over the cache with the
// layer's window and sinks, the bf16 o projection into the residual; then the post-attention norm
// rounded to fp16 (moe_x), the fp16 router's logits (rounded to fp16), the top-k routing, the
// token-grouped MXFP4 experts and their weighted sum, which ends the layer as x = f16(x) + f16(moe).
// Same contract as enqueue_chunk.
int enqueue_chunk_gptoss(hc_session *s, int n, bool accept, int splits, int heads) {
  hc_model *m = s->m;
  const auto &d = m->d;
  const int D = int(d.hidden), I = int(d.inter), H = int(d.heads), KV = int(d.kv_heads);
  const int hd = int(d.head_dim), V = int(d.vocab), E = int(d.experts), K = int(d.top_k);
  const int W = (H + 2 * KV) * hd;
  const int ktD = (D + hc::kTileCols - 1) / hc::kTileCols, ktI = (I + hc::kTileCols - 1) / hc::kTileCols;
  const int ktO = (H * hd + hc::kTileCols - 1) / hc::kTileCols;
  const int maxp = kMaxChunk * K, c8 = (n + 7) / 8;
  const float alpha = float(d.swiglu_alpha), limit = float(d.swiglu_limit), eps = m->norm_in0.eps16;
  cudaStream_t st = s->st;
  int k = 0;
  hc::embed(s->toks_dev, n, m->embed, nullptr, D, s->x, s->amax, st);
  ++k;
  for (size_t li = 0; li < m->layers.size(); ++li) {
    const hc::LayerW &w = m->layers[li];
    uint16_t *kcl = s->paged ? nullptr : s->kc + li * s->layer_kv;
    uint16_t *vcl = s->paged ? nullptr : s->vc + li * s->layer_kv;
    const hc::PagedKV pk = s->paged ? paged_of(s, li) : hc::PagedKV{};
    const hc::AttnGeom g = geom(s, w.window);
    hc::rms_rows(s->x, D, D, n, w.in_norm, eps, s->xn, D, false, st);
    hc::gemv16(w.qkv16, s->xn, D, n, 0, s->qkv, W, nullptr, nullptr, st);
    hc::qkv_post(s->qkv, s->toks_dev, n, g, nullptr, nullptr, 1.f, eps, s->rope, s->q, kcl, vcl, s->kv_stage, st);
    hc::attn_split(s->q, s->toks_dev, n, g, kcl, vcl, splits, s->part_ml, s->part_o, st, s->paged ? &pk : nullptr,
                   s->kv_stage);
    if (s->paged) {
      hc::kv_append_int8(s->kv_stage, s->toks_dev, n, KV, hd, pk, st);
      ++k;
    }
    hc::attn_merge_quant(s->part_ml, s->part_o, w.sinks, n, H, hd, splits, s->act, ktO, s->oatt, st);
    hc::gemv16(w.o16, s->oatt, H * hd, n, 1, s->x, D, nullptr, nullptr, st);
    hc::rms_rows(s->x, D, D, n, w.post_norm, eps, s->xn, D, true, st);
    hc::gemv16(w.router16, s->xn, D, n, 2, s->mlog, E, nullptr, nullptr, st);
    hc::route(s->mlog, n, E, K, s->midx, s->mw, st);
    hc::moe_group(s->midx, n * K, E, s->mcnt, s->mlist, maxp, st);
    hc::act_quant(s->xn, D, D, n, nullptr, 1.f, 0.f, s->act, ktD, st, nullptr, hc::kActTokenMajor);
    hc::moe_gemv(w.egu->m, E, 0, s->mcnt, s->mlist, maxp, K, s->act, w.egb, alpha, limit, s->hh, I, st);
    hc::act_quant(s->hh, I, I, n * K, nullptr, 1.f, 0.f, s->act2, ktI, st, nullptr, hc::kActTokenMajor);
    hc::moe_gemv(w.edown->m, E, 1, s->mcnt, s->mlist, maxp, K, s->act2, nullptr, 0.f, 0.f, s->ey, D, st);
    hc::moe_combine(s->ey, s->midx, s->mw, K, w.edb, D, n, s->x, st);
    k += 11 + 3 * c8;
  }
  if (heads > 0) {
    hc::rms_rows(s->x, D, D, heads, m->final_norm, m->norm_head.eps16, s->xn, D, false, st,
                 heads == n ? nullptr : s->toks_dev);
    hc::gemv16(m->head16, s->xn, D, heads, 3, nullptr, V, s->logits_dev, s->amax, st);
    hc::amax_to_index(s->amax, heads, s->am_dev, st);
    k += 2 + (heads + 7) / 8;
  }
  if (accept) { hc::spec_accept(s->am_dev, s->toks_dev, n, s->res_dev, st); ++k; }
  return k;
}

// The model's kernel sequence for a chunk.
int enqueue_model(hc_session *s, int n, bool accept, int splits, int heads) {
  return s->m->gptoss ? enqueue_chunk_gptoss(s, n, accept, splits, heads) : enqueue_chunk(s, n, accept, splits, heads);
}

// The whole chunk: tokens in, greedy choices (and the accept result) out, as one graph. heads:
// the rows read out (toks_host[j].head_src for j < heads; all n rows for accept).
char *run_chunk(hc_session *s, int n, bool accept, int heads) {
  for (int i = 0; i < n; ++i)
    if (char *e = ensure_pages(s, s->toks_host[i].slot, s->toks_host[i].pos, s->toks_host[i].pos + 1)) return e;
  cudaStream_t st = s->st;
  const bool use_graph = !(s->o.flags & HC_SESSION_NO_GRAPH);
  const int splits = splits_for(s, n, chunk_max_len(s, n));
  const int key = ((splits * 128 + n) * 128 + heads) * 2 + (accept ? 1 : 0);
  auto enqueue_all = [&]() -> int {
    cudaMemcpyAsync(s->toks_dev, s->toks_host, sizeof(hc::StepTok) * n, cudaMemcpyHostToDevice, st);
    const int k = enqueue_model(s, n, accept, splits, heads);
    if (heads > 0) cudaMemcpyAsync(s->am_host, s->am_dev, sizeof(int32_t) * heads, cudaMemcpyDeviceToHost, st);
    if (accept) cudaMemcpyAsync(s->res_host, s->res_dev, sizeof(int32_t) * 2, cudaMemcpyDeviceToHost, st);
    return k;
  };
  if (use_graph && !s->graphs.count(key)) {
    cudaGraph_t graph = nullptr;
    HC_TRY_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    s->launches_per_key[key] = uint64_t(enqueue_all());
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (e != cudaSuccess) return hc::make_error(std::string("graph capture: ") + cudaGetErrorString(e));
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return hc::make_error(std::string("graph instantiate: ") + cudaGetErrorString(e));
    s->graphs[key] = exec;
  }
  HC_TRY_CUDA(cudaEventRecord(s->ev0, st));
  hc::device_stall(hc::take_stall_ms(), st);
  if (use_graph) {
    HC_TRY_CUDA(cudaGraphLaunch(s->graphs[key], st));
  } else {
    s->launches_per_key[key] = uint64_t(enqueue_all());
  }
  HC_TRY_CUDA(cudaGetLastError());
  HC_TRY_CUDA(cudaEventRecord(s->ev1, st));
  s->stats.launches += s->launches_per_key[key];
  return nullptr;
}

// Waits for the last chunk with a deadline (xrtshim.h's xs_run_wait with timeout_ms).
char *wait_done(hc_session *s, uint32_t timeout_ms, int32_t *state) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaEventQuery(s->ev1);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) {
      if (state) *state = HC_STATE_ERROR;
      return hc::make_error(std::string("step: ") + cudaGetErrorString(e));
    }
    if (timeout_ms) {
      auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
      if (ms >= long(timeout_ms)) {
        if (state) *state = HC_STATE_TIMEOUT;
        return nullptr;
      }
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  float ms = 0;
  cudaEventElapsedTime(&ms, s->ev0, s->ev1);
  s->stats.last_step_us = double(ms) * 1000.0;
  if (state) *state = HC_STATE_COMPLETED;
  return nullptr;
}

}  // namespace

extern "C" {

HC_API char *hc_session_new(hc_model *m, const hc_session_opts *opts, hc_session **out) {
  if (!m || !opts || !out) return hc::make_error("hc_session_new: NULL argument");
  *out = nullptr;
  const hc_session_opts &o = *opts;
  if (!o.max_context || !o.max_seqs || !o.max_step) return hc::make_error("hc_session_new: zero size");
  if (o.kv_format != HC_KV_F16 && o.kv_format != HC_KV_INT8_PAGED)
    return hc::make_error("hc_session_new: KV format " + std::to_string(o.kv_format) + " is not supported by this build");
  if (o.kv_format == HC_KV_INT8_PAGED && o.page_size != uint32_t(hc::kPage))
    return hc::make_error("hc_session_new: the paged int8 cache has pages of " + std::to_string(hc::kPage) + " positions");
  HC_TRY_CUDA(cudaSetDevice(m->ordinal));
  if (char *e = hc::gemv_prepare()) return e;
  auto s = std::make_unique<hc_session>();
  s->m = m;
  s->o = o;
  s->cap = int(o.max_context);
  const auto &d = m->d;
  const int D = int(d.hidden), F = int(d.inter), H = int(d.heads), KV = int(d.kv_heads), hd = int(d.head_dim);
  s->paged = o.kv_format == HC_KV_INT8_PAGED;
  if (s->paged) {
    // every slot can hold max_context positions: the pool is slots x pages of max_context
    s->max_pages = (s->cap + hc::kPage - 1) / hc::kPage;
    s->n_pages = int(o.max_seqs) * s->max_pages;
    const size_t rows = size_t(d.layers) * s->n_pages * KV;
    if (char *e = alloc(&s->kp, rows * hc::kPage * hd, "key pages")) return e;
    if (char *e = alloc(&s->vp, rows * hc::kPage * hd, "value pages")) return e;
    if (char *e = alloc(&s->kps, rows, "key page scales")) return e;
    if (char *e = alloc(&s->vps, rows, "value page scales")) return e;
    HC_TRY_CUDA(cudaMemset(s->kps, 0, rows * 2));
    HC_TRY_CUDA(cudaMemset(s->vps, 0, rows * 2));
    if (char *e = alloc(&s->btab_dev, size_t(o.max_seqs) * s->max_pages, "block table")) return e;
    s->btab.assign(size_t(o.max_seqs) * s->max_pages, -1);
    HC_TRY_CUDA(cudaMemcpy(s->btab_dev, s->btab.data(), s->btab.size() * 4, cudaMemcpyHostToDevice));
    for (int p = s->n_pages - 1; p >= 0; --p) s->free_pages.push_back(p);
  } else {
    s->layer_kv = size_t(o.max_seqs) * KV * s->cap * hd;
    const size_t kv_elems = s->layer_kv * d.layers;
    if (char *e = alloc(&s->kc, kv_elems, "key cache")) return e;
    if (char *e = alloc(&s->vc, kv_elems, "value cache")) return e;
    HC_TRY_CUDA(cudaMemset(s->kc, 0, kv_elems * 2));
    HC_TRY_CUDA(cudaMemset(s->vc, 0, kv_elems * 2));
  }
  // blocks.RopeValues (blocks.go:412-427) as fp16 inputs (qwen3 StepInputs, arch.go:117-137)
  std::vector<uint32_t> rope(size_t(s->cap) * (hd / 2));
  for (int p = 0; p < s->cap; ++p)
    for (int j = 0; j < hd / 2; ++j) {
      const double a = double(p) * m->inv_freq[j];
      float c = float(std::cos(a)), sn = float(std::sin(a));
      if (m->rope_factor != 1.f) { c *= m->rope_factor; sn *= m->rope_factor; }
      rope[size_t(p) * (hd / 2) + j] = uint32_t(hc::f16_bits(c)) | (uint32_t(hc::f16_bits(sn)) << 16);
    }
  if (char *e = alloc(&s->rope, rope.size(), "rope tables")) return e;
  if (char *e = hc::copy_h2d(s->rope, rope.data(), rope.size() * 4, nullptr)) return e;
  HC_TRY_CUDA(cudaStreamSynchronize(nullptr));
  int ktiles = 0;
  if (m->gptoss) {
    ktiles = (std::max({D, F, H * hd}) + hc::kTileCols - 1) / hc::kTileCols;
  } else {
    for (auto &w : m->layers)
      ktiles = std::max({ktiles, w.qkv->m.ktiles, w.o->m.ktiles, w.gu->m.ktiles, w.down->m.ktiles});
    ktiles = std::max(ktiles, m->head->m.ktiles);
  }
  const int T = kMaxChunk;
  if (m->gptoss) {
    const int E = int(d.experts), K = int(d.top_k), ktI = (F + hc::kTileCols - 1) / hc::kTileCols;
    if (char *e = alloc(&s->xn, size_t(T) * D, "normed rows")) return e;
    if (char *e = alloc(&s->oatt, size_t(T) * H * hd, "attention output")) return e;
    if (char *e = alloc(&s->mlog, size_t(T) * E, "router logits")) return e;
    if (char *e = alloc(&s->midx, size_t(T) * K, "routing")) return e;
    if (char *e = alloc(&s->mw, size_t(T) * K, "routing weights")) return e;
    if (char *e = alloc(&s->mcnt, size_t(E), "expert counts")) return e;
    if (char *e = alloc(&s->mlist, size_t(E) * T * K, "expert lists")) return e;
    if (char *e = alloc(&s->act2, size_t(T) * K * ktI * hc::kActTile, "expert activation tiles")) return e;
    if (char *e = alloc(&s->hh, size_t(T) * K * F, "expert activations")) return e;
    if (char *e = alloc(&s->ey, size_t(T) * K * D, "expert outputs")) return e;
  }
  if (char *e = alloc(&s->x, size_t(T) * D, "hidden states")) return e;
  if (char *e = alloc(&s->qkv, size_t(T) * (H + 2 * KV) * hd, "qkv")) return e;
  if (char *e = alloc(&s->kv_stage, size_t(T) * 2 * KV * hd, "new key and value rows")) return e;
  if (char *e = alloc(&s->q, size_t(T) * H * hd, "queries")) return e;
  if (char *e = alloc(&s->h, size_t(T) * F, "mlp activations")) return e;
  if (char *e = alloc(&s->act, size_t(T) * ktiles * hc::kActTile, "activation tiles")) return e;
  if (char *e = alloc(&s->part_ml, size_t(T) * H * kMaxSplits * 2, "attention partials")) return e;
  if (char *e = alloc(&s->part_o, size_t(T) * H * kMaxSplits * hd, "attention partials")) return e;
  if (char *e = alloc(&s->toks_dev, T, "step tokens")) return e;
  if (char *e = alloc(&s->logits_dev, size_t(T) * d.vocab, "logits")) return e;
  if (char *e = alloc(&s->amax, size_t(T) * hc::kAmaxSlots, "argmax keys")) return e;
  if (char *e = alloc(&s->am_dev, T, "argmax")) return e;
  if (char *e = alloc(&s->res_dev, 2, "accept result")) return e;
  if (char *e = alloc(&s->gen_out, size_t(s->cap), "generated tokens")) return e;
  if (char *e = alloc(&s->gen_count, 1, "generated count")) return e;
  HC_TRY_CUDA(cudaHostAlloc(&s->toks_host, sizeof(hc::StepTok) * T, cudaHostAllocDefault));
  HC_TRY_CUDA(cudaHostAlloc(&s->am_host, sizeof(int32_t) * T, cudaHostAllocDefault));
  HC_TRY_CUDA(cudaHostAlloc(&s->res_host, sizeof(int32_t) * 2, cudaHostAllocDefault));
  HC_TRY_CUDA(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
  HC_TRY_CUDA(cudaEventCreate(&s->ev0));
  HC_TRY_CUDA(cudaEventCreate(&s->ev1));
  s->pos.assign(o.max_seqs, 0);
  s->poisoned.assign(o.max_seqs, false);
  HC_TRY_CUDA(cudaMemset(s->amax, 0, sizeof(unsigned long long) * T * hc::kAmaxSlots));
  *out = s.release();
  return nullptr;
}

HC_API void hc_session_free(hc_session *s) { delete s; }

HC_API char *hc_step(hc_session *s, const int32_t *seq_ids, const int32_t *n_tokens,
                     const int32_t *tokens, int32_t nseq, int32_t flags, uint16_t *logits,
                     int32_t *argmax, uint32_t timeout_ms, int32_t *state) {
  if (state) *state = HC_STATE_ERROR;
  if (!s || !seq_ids || !n_tokens || !tokens || nseq < 1) return hc::make_error("hc_step: bad argument");
  const int V = int(s->m->d.vocab);
  std::vector<hc::StepTok> all;
  std::vector<int> want;  // indices into `all` whose rows go out
  for (int i = 0; i < nseq; ++i) {
    const int sq = seq_ids[i], n = n_tokens[i];
    if (sq < 0 || sq >= int(s->o.max_seqs)) return hc::make_error("hc_step: sequence " + std::to_string(sq) + " out of range");
    if (n < 1) return hc::make_error("hc_step: a sequence with no tokens");
    if (s->poisoned[sq]) return hc::make_error("hc_step: sequence " + std::to_string(sq) + " failed earlier; reset it");
    for (int j = 0; j < i; ++j)
      if (seq_ids[j] == sq) return hc::make_error("hc_step: sequence listed twice");
    if (s->pos[sq] + n > s->cap) return hc::make_error("hc_step: sequence " + std::to_string(sq) + " would exceed max_context");
  }
  // The chunks of up to kMaxChunk tokens: a sequence's tokens are cut into pieces of kMaxChunk from
  // its first, and a piece never straddles two chunks, so that the keys a token reads in float32
  // (its piece's) do not depend on the other sequences of the call.
  std::vector<std::pair<size_t, size_t>> chunks;  // [begin, end) of `all`
  size_t cb = 0;
  int off = 0;
  for (int i = 0; i < nseq; ++i) {
    for (int j = 0; j < n_tokens[i]; ++j) {
      const int tok = tokens[off + j];
      if (tok < 0 || tok >= V) return hc::make_error("hc_step: token " + std::to_string(tok) + " out of the vocabulary");
    }
    for (int p = 0; p < n_tokens[i]; p += kMaxChunk) {
      const int len = std::min(kMaxChunk, n_tokens[i] - p);
      if (all.size() - cb + len > size_t(kMaxChunk)) {
        chunks.push_back({cb, all.size()});
        cb = all.size();
      }
      const int32_t r0 = int32_t(all.size() - cb);
      for (int j = p; j < p + len; ++j) {
        all.push_back(hc::StepTok{tokens[off + j], seq_ids[i], s->pos[seq_ids[i]] + j, 0, r0});
        if ((flags & HC_STEP_ALL_ROWS) || j == n_tokens[i] - 1) want.push_back(int(all.size()) - 1);
      }
    }
    off += n_tokens[i];
  }
  chunks.push_back({cb, all.size()});
  if (hc::fault_fires(hc::kFaultStep)) return hc::make_error("injected fault: step");
  HC_TRY_CUDA(cudaSetDevice(s->m->ordinal));
  size_t wi = 0;
  int row = 0;
  double step_us = 0;  // the call's device time: the sum over its chunks
  for (const auto &ch : chunks) {
    const size_t c0 = ch.first;
    const int n = int(ch.second - ch.first);
    std::memcpy(s->toks_host, &all[c0], sizeof(hc::StepTok) * n);
    int heads = 0;  // the chunk's rows that are read out, in order
    for (size_t w = wi; w < want.size() && size_t(want[w]) < c0 + n; ++w) s->toks_host[heads++].head_src = int(want[w] - c0);
    if (char *e = run_chunk(s, n, false, heads)) {
      for (int i = 0; i < nseq; ++i) s->poisoned[seq_ids[i]] = true;
      return e;
    }
    int32_t st_ = HC_STATE_ERROR;
    char *e = wait_done(s, timeout_ms, &st_);
    if (e || st_ != HC_STATE_COMPLETED) {
      for (int i = 0; i < nseq; ++i) s->poisoned[seq_ids[i]] = true;
      if (state) *state = e ? HC_STATE_ERROR : st_;
      return e;
    }
    step_us += s->stats.last_step_us;
    for (int j = 0; wi < want.size() && size_t(want[wi]) < c0 + n; ++wi, ++row, ++j) {
      if (argmax) argmax[row] = s->am_host[j];
      if (logits) HC_TRY_CUDA(cudaMemcpy(logits + size_t(row) * V, s->logits_dev + size_t(j) * V, size_t(V) * 2, cudaMemcpyDeviceToHost));
    }
  }
  uint64_t kv = 0;
  const auto &md = s->m->d;
  for (auto &t : all) kv += uint64_t(t.pos + 1) * md.kv_heads * md.head_dim * 4 * md.layers;
  s->stats.kv_bytes = kv;
  s->stats.last_step_us = step_us;
  for (int i = 0; i < nseq; ++i) s->pos[seq_ids[i]] += n_tokens[i];
  s->stats.steps++;
  s->stats.tokens += all.size();
  s->stats.weight_bytes = s->m->weight_bytes;
  if (state) *state = HC_STATE_COMPLETED;
  return nullptr;
}

HC_API char *hc_speculate(hc_session *s, int32_t seq, const int32_t *toks, int32_t n,
                          int32_t *kept, int32_t *next, uint16_t *logits, uint32_t timeout_ms,
                          int32_t *state) {
  if (state) *state = HC_STATE_ERROR;
  if (!s || !toks || !kept || !next) return hc::make_error("hc_speculate: NULL argument");
  if (seq < 0 || seq >= int(s->o.max_seqs)) return hc::make_error("hc_speculate: sequence out of range");
  if (n < 1 || n > kMaxChunk || n > int(s->o.max_step)) return hc::make_error("hc_speculate: " + std::to_string(n) + " tokens");
  if (s->poisoned[seq]) return hc::make_error("hc_speculate: sequence failed earlier; reset it");
  if (s->pos[seq] + n > s->cap) return hc::make_error("hc_speculate: would exceed max_context");
  const int V = int(s->m->d.vocab);
  for (int j = 0; j < n; ++j) {
    if (toks[j] < 0 || toks[j] >= V) return hc::make_error("hc_speculate: token out of the vocabulary");
    s->toks_host[j] = hc::StepTok{toks[j], seq, s->pos[seq] + j, j, 0};
  }
  if (hc::fault_fires(hc::kFaultStep)) return hc::make_error("injected fault: step");
  HC_TRY_CUDA(cudaSetDevice(s->m->ordinal));
  if (char *e = run_chunk(s, n, true, n)) { s->poisoned[seq] = true; return e; }
  int32_t st_ = HC_STATE_ERROR;
  char *e = wait_done(s, timeout_ms, &st_);
  if (e || st_ != HC_STATE_COMPLETED) {
    s->poisoned[seq] = true;
    if (state) *state = e ? HC_STATE_ERROR : st_;
    return e;
  }
  *kept = s->res_host[0];
  *next = s->res_host[1];
  if (logits) HC_TRY_CUDA(cudaMemcpy(logits, s->logits_dev + size_t(*kept - 1) * V, size_t(V) * 2, cudaMemcpyDeviceToHost));
  // decode.Session.keep (decode.go:1685-1705): only the kept rows stay; the others are past pos
  s->pos[seq] += *kept;
  s->stats.steps++;
  s->stats.tokens += n;
  s->stats.weight_bytes = s->m->weight_bytes;
  if (state) *state = HC_STATE_COMPLETED;
  return nullptr;
}

HC_API char *hc_generate(hc_session *s, int32_t seq, int32_t first, int32_t n, int32_t *out_tokens,
                         uint32_t timeout_ms, int32_t *state) {
  if (state) *state = HC_STATE_ERROR;
  if (!s || !out_tokens) return hc::make_error("hc_generate: NULL argument");
  if (seq < 0 || seq >= int(s->o.max_seqs)) return hc::make_error("hc_generate: sequence out of range");
  if (n < 1) return hc::make_error("hc_generate: n must be at least 1");
  if (s->poisoned[seq]) return hc::make_error("hc_generate: sequence failed earlier; reset it");
  if (s->pos[seq] + n > s->cap) return hc::make_error("hc_generate: would exceed max_context");
  if (first < 0 || first >= int(s->m->d.vocab)) return hc::make_error("hc_generate: token out of the vocabulary");
  if (hc::fault_fires(hc::kFaultStep)) return hc::make_error("injected fault: step");
  HC_TRY_CUDA(cudaSetDevice(s->m->ordinal));
  if (char *e = ensure_pages(s, seq, s->pos[seq], s->pos[seq] + n)) return e;
  cudaStream_t st = s->st;
  s->toks_host[0] = hc::StepTok{first, seq, s->pos[seq], 0, 0};
  if (!s->gen_graph) {
    cudaGraph_t graph = nullptr;
    HC_TRY_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    s->launches_per_chunk[0] = uint64_t(enqueue_model(s, 1, false, splits_for(s, 1, 0), 1)) + 1;
    hc::advance(s->toks_dev, s->am_dev, s->gen_out, s->gen_count, st);
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (e != cudaSuccess) return hc::make_error(std::string("graph capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(&s->gen_graph, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return hc::make_error(std::string("graph instantiate: ") + cudaGetErrorString(e));
  }
  HC_TRY_CUDA(cudaMemcpyAsync(s->toks_dev, s->toks_host, sizeof(hc::StepTok), cudaMemcpyHostToDevice, st));
  HC_TRY_CUDA(cudaMemsetAsync(s->gen_count, 0, sizeof(int32_t), st));
  HC_TRY_CUDA(cudaEventRecord(s->ev0, st));
  hc::device_stall(hc::take_stall_ms(), st);
  for (int i = 0; i < n; ++i) HC_TRY_CUDA(cudaGraphLaunch(s->gen_graph, st));
  HC_TRY_CUDA(cudaEventRecord(s->ev1, st));
  s->stats.launches += uint64_t(n) * s->launches_per_chunk[0];
  int32_t st_ = HC_STATE_ERROR;
  char *e = wait_done(s, timeout_ms, &st_);
  if (e || st_ != HC_STATE_COMPLETED) {
    s->poisoned[seq] = true;
    if (state) *state = e ? HC_STATE_ERROR : st_;
    return e;
  }
  HC_TRY_CUDA(cudaMemcpy(out_tokens, s->gen_out, sizeof(int32_t) * n, cudaMemcpyDeviceToHost));
  s->pos[seq] += n;
  s->stats.steps += n;
  s->stats.tokens += n;
  s->stats.weight_bytes = s->m->weight_bytes;
  if (state) *state = HC_STATE_COMPLETED;
  return nullptr;
}

HC_API char *hc_session_stream(hc_session *s, void **stream) {
  if (!s || !stream) return hc::make_error("hc_session_stream: NULL argument");
  *stream = s->st;
  return nullptr;
}

HC_API char *hc_seq_reset(hc_session *s, int32_t seq) {
  if (!s || seq < 0 || seq >= int(s->o.max_seqs)) return hc::make_error("hc_seq_reset: bad sequence");
  s->pos[seq] = 0;
  s->poisoned[seq] = false;
  release_pages(s, seq, 0);
  return nullptr;
}

HC_API char *hc_seq_truncate(hc_session *s, int32_t seq, int32_t len) {
  if (!s || seq < 0 || seq >= int(s->o.max_seqs)) return hc::make_error("hc_seq_truncate: bad sequence");
  if (len < 0 || len > s->pos[seq]) return hc::make_error("hc_seq_truncate: length out of range");
  s->pos[seq] = len;
  release_pages(s, seq, len);
  return nullptr;
}

HC_API char *hc_seq_pos(hc_session *s, int32_t seq, int32_t *pos) {
  if (!s || !pos || seq < 0 || seq >= int(s->o.max_seqs)) return hc::make_error("hc_seq_pos: bad argument");
  *pos = s->pos[seq];
  return nullptr;
}

namespace {
char *rows_copy(hc_session *s, int32_t seq, int32_t start, int32_t n, void *host, bool out) {
  const auto &d = s->m->d;
  const size_t hd = d.head_dim, row = hd * 2;
  char *p = static_cast<char *>(host);
  for (uint32_t li = 0; li < d.layers; ++li)
    for (int kvs = 0; kvs < 2; ++kvs)
      for (uint32_t h = 0; h < d.kv_heads; ++h) {
        uint16_t *base = (kvs ? s->vc : s->kc) + li * s->layer_kv + ((size_t(seq) * d.kv_heads + h) * s->cap + start) * hd;
        const size_t nb = size_t(n) * row;
        cudaError_t e = out ? cudaMemcpy(p, base, nb, cudaMemcpyDeviceToHost) : cudaMemcpy(base, p, nb, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return hc::make_error(std::string("rows copy: ") + cudaGetErrorString(e));
        p += nb;
      }
  return nullptr;
}
}  // namespace

HC_API char *hc_seq_export_rows(hc_session *s, int32_t seq, int32_t start, int32_t n, void *dst,
                                uint64_t cap, uint64_t *need) {
  if (!s || seq < 0 || seq >= int(s->o.max_seqs)) return hc::make_error("hc_seq_export_rows: bad sequence");
  if (start < 0 || n < 0 || start + n > s->pos[seq]) return hc::make_error("hc_seq_export_rows: rows out of range");
  if (s->paged) return hc::make_error("hc_seq_export_rows: not available for the paged int8 cache");
  const auto &d = s->m->d;
  const uint64_t bytes = uint64_t(d.layers) * 2 * d.kv_heads * n * d.head_dim * 2;
  if (need) *need = bytes;
  if (!dst) return nullptr;
  if (cap < bytes) return hc::make_error("hc_seq_export_rows: buffer too small");
  HC_TRY_CUDA(cudaSetDevice(s->m->ordinal));
  HC_TRY_CUDA(cudaStreamSynchronize(s->st));
  return rows_copy(s, seq, start, n, dst, true);
}

HC_API char *hc_seq_import_rows(hc_session *s, int32_t seq, int32_t start, int32_t n,
                                const void *src, uint64_t size) {
  if (!s || !src || seq < 0 || seq >= int(s->o.max_seqs)) return hc::make_error("hc_seq_import_rows: bad argument");
  if (start < 0 || n < 0 || start > s->pos[seq] || start + n > s->cap) return hc::make_error("hc_seq_import_rows: rows out of range");
  if (s->paged) return hc::make_error("hc_seq_import_rows: not available for the paged int8 cache");
  const auto &d = s->m->d;
  const uint64_t bytes = uint64_t(d.layers) * 2 * d.kv_heads * n * d.head_dim * 2;
  if (size != bytes) return hc::make_error("hc_seq_import_rows: size does not match the rows");
  HC_TRY_CUDA(cudaSetDevice(s->m->ordinal));
  HC_TRY_CUDA(cudaStreamSynchronize(s->st));
  if (char *e = rows_copy(s, seq, start, n, const_cast<void *>(src), false)) return e;
  s->pos[seq] = start + n;
  s->poisoned[seq] = false;
  return nullptr;
}

HC_API char *hc_stats_get(hc_session *s, hc_stats *out) {
  if (!s || !out) return hc::make_error("hc_stats_get: NULL argument");
  *out = s->stats;
  return nullptr;
}

}  // extern "C"
