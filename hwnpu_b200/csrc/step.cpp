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
  for (void *p : {(void *)ps_layers, (void *)ps_sync, (void *)ps_status, (void *)ps_trace, (void *)ps_attn,
                  (void *)ps_part_ml, (void *)ps_part_o, (void *)ps_dx})
    if (p) cudaFree(p);
  if (ps_status_host) cudaFreeHost(ps_status_host);
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

// Attention splits of every (token, kv head) of a chunk of n tokens whose longest context is
// max_len positions: enough CTAs to fill the SMs twice (as for one token when n <= 8), and at
// most kSplitKeys keys a split for the longest (rounded up to a power of two, so that few step
// graphs differ by their splits).
int splits_for(const hc_session *s, int n, int max_len) {
  const int kv = int(s->m->d.kv_heads);
  // up to 8 tokens take the one-token count, so that a speculative verify row, or any row of a
  // small batch, is computed exactly as a one-token step (hc_generate) computes it
  int sp = (2 * s->m->sms) / (kv * (n <= 8 ? 1 : n));
  int by_len = 1;
  while (by_len < kMaxSplits && by_len * kSplitKeys < max_len) by_len *= 2;
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
    hc::act_quant(s->x, D, D, n, w.in_norm, nc.scale, nc.eps16, s->act, w.qkv->m.ktiles, st);
    hc::GemvOut o1;
    o1.mode = hc::kStore; o1.y = s->qkv; o1.ldy = W;
    hc::gemv(w.qkv->m, s->act, n, o1, st);
    hc::qkv_post(s->qkv, s->toks_dev, n, g, w.q_norm, w.k_norm, m->norm_mid.scale, m->norm_mid.eps16,
                 s->rope, s->q, kcl, vcl, s->kv_stage, st);
    if (s->paged) {
      hc::kv_append_int8(s->kv_stage, s->toks_dev, n, KV, hd, pk, st);
      ++k;
    }
    hc::attn_split(s->q, s->toks_dev, n, g, kcl, vcl, splits, s->part_ml, s->part_o, st, s->paged ? &pk : nullptr);
    hc::attn_merge_quant(s->part_ml, s->part_o, w.sinks, n, H, hd, splits, s->act, w.o->m.ktiles, nullptr, st, true);
    hc::GemvOut o2;
    o2.mode = hc::kAdd; o2.y = s->x; o2.ldy = D;
    hc::gemv(w.o->m, s->act, n, o2, st);
    hc::act_quant(s->x, D, D, n, w.post_norm, m->norm_mid.scale, m->norm_mid.eps16, s->act, w.gu->m.ktiles, st);
    hc::GemvOut o3;
    o3.mode = hc::kGlu; o3.y = s->h; o3.ldy = F;
    hc::gemv(w.gu->m, s->act, n, o3, st);
    hc::act_quant(s->h, F, F, n, nullptr, 1.f, 0.f, s->act, w.down->m.ktiles, st);
    hc::gemv(w.down->m, s->act, n, o2, st);
    k += 10;
  }
  if (heads > 0) {
    hc::act_quant(s->x, D, D, heads, m->final_norm, m->norm_head.scale, m->norm_head.eps16, s->act,
                  m->head->m.ktiles, st, heads == n ? nullptr : s->toks_dev);
    hc::GemvOut oh;
    oh.mode = hc::kLogits; oh.ldy = V; oh.logits = s->logits_dev; oh.amax = s->amax;
    hc::gemv(m->head->m, s->act, heads, oh, st);
    hc::amax_to_index(s->amax, heads, s->am_dev, st);
    k += 3;
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
    if (s->paged) {
      hc::kv_append_int8(s->kv_stage, s->toks_dev, n, KV, hd, pk, st);
      ++k;
    }
    hc::attn_split(s->q, s->toks_dev, n, g, kcl, vcl, splits, s->part_ml, s->part_o, st, s->paged ? &pk : nullptr);
    hc::attn_merge_quant(s->part_ml, s->part_o, w.sinks, n, H, hd, splits, s->act, ktO, s->oatt, st, false);
    hc::gemv16(w.o16, s->oatt, H * hd, n, 1, s->x, D, nullptr, nullptr, st);
    hc::rms_rows(s->x, D, D, n, w.post_norm, eps, s->xn, D, true, st);
    hc::gemv16(w.router16, s->xn, D, n, 2, s->mlog, E, nullptr, nullptr, st);
    hc::route(s->mlog, n, E, K, s->midx, s->mw, st);
    hc::moe_group(s->midx, n * K, E, s->mcnt, s->mlist, maxp, st);
    hc::act_quant(s->xn, D, D, n, nullptr, 1.f, 0.f, s->act, ktD, st, nullptr, true);
    hc::moe_gemv(w.egu->m, E, 0, s->mcnt, s->mlist, maxp, K, s->act, w.egb, alpha, limit, s->hh, I, st);
    hc::act_quant(s->hh, I, I, n * K, nullptr, 1.f, 0.f, s->act2, ktI, st, nullptr, true);
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

constexpr long long kSpinLimit = 4000000000ll;  // ~2 s of SM clocks: a wait of the persistent step

// The persistent step's parameters for the n tokens in toks_dev; gen: hc_generate's feedback.
hc::PsParams ps_params(hc_session *s, int n, bool gen, long long spin) {
  hc_model *m = s->m;
  const auto &d = m->d;
  hc::PsParams p{};
  p.layers = int(d.layers);
  p.D = int(d.hidden);
  p.F = int(d.inter);
  p.H = int(d.heads);
  p.KV = int(d.kv_heads);
  p.hd = int(d.head_dim);
  p.V = int(d.vocab);
  p.cap = s->cap;
  p.ntok = n;
  p.kt_d = m->layers[0].qkv->m.ktiles;
  p.kt_f = m->layers[0].down->m.ktiles;
  p.kt_o = m->layers[0].o->m.ktiles;
  p.rt_qkv = m->layers[0].qkv->m.rtiles;
  p.rt_o = m->layers[0].o->m.rtiles;
  p.rt_gu = m->layers[0].gu->m.rtiles;
  p.rt_down = m->layers[0].down->m.rtiles;
  p.rt_head = m->head->m.rtiles;
  p.max_splits = s->ps_max_splits;
  p.sc_in0 = m->norm_in0.scale;
  p.eps_in0 = m->norm_in0.eps16;
  p.sc = m->norm_mid.scale;
  p.eps = m->norm_mid.eps16;
  p.sc_head = m->norm_head.scale;
  p.eps_head = m->norm_head.eps16;
  p.score_scale = m->score_scale;
  p.L = s->ps_layers;
  p.head = m->head->m.tiles;
  p.head_scale = m->head->m.row_scale;
  p.embed = m->embed;
  p.final_norm = m->final_norm;
  p.rope = s->rope;
  p.toks = s->toks_dev;
  p.dx_o = s->x;
  p.dx_down = s->ps_dx;
  p.qkv = s->qkv;
  p.attn = s->ps_attn;
  p.h = s->h;
  p.part_ml = s->ps_part_ml;
  p.part_o = s->ps_part_o;
  p.tickets = reinterpret_cast<int *>(s->ps_sync + 4);
  p.logits = gen ? nullptr : s->logits_dev;
  p.amax = s->amax;
  p.am = s->am_dev;
  p.gen_out = gen ? s->gen_out : nullptr;
  p.gen_count = gen ? s->gen_count : nullptr;
  p.bar = s->ps_sync;
  p.status = s->ps_status;
  p.spin_limit = spin;
  p.stall_first_barrier = spin != kSpinLimit ? 1 : 0;
  p.trace = s->ps_trace;
  hc::ps_layout(p, s->ps_kind);
  return p;
}

// Enqueues the persistent step (its barrier and tickets zeroed first); returns its launches.
int enqueue_ps(hc_session *s, int n, bool gen, long long spin) {
  cudaMemsetAsync(s->ps_sync, 0, s->ps_sync_bytes, s->st);
  hc::ps_launch(ps_params(s, n, gen, spin), s->ps_kind, s->ps_ctas, s->st);
  return 1;
}

bool ps_chunk(const hc_session *s, int n) { return s->ps && n <= s->ps_max_tok; }

// The whole chunk: tokens in, greedy choices (and the accept result) out, as one graph. heads:
// the rows read out (toks_host[j].head_src for j < heads; all n rows for accept).
char *run_chunk(hc_session *s, int n, bool accept, int heads) {
  for (int i = 0; i < n; ++i)
    if (char *e = ensure_pages(s, s->toks_host[i].slot, s->toks_host[i].pos, s->toks_host[i].pos + 1)) return e;
  cudaStream_t st = s->st;
  // an armed "spin:N" fault runs this chunk once, outside the graphs, with waits of N cycles
  const long long spin_fault = hc::take_spin_cycles();
  const bool ps = ps_chunk(s, n);
  const bool use_graph = !(s->o.flags & HC_SESSION_NO_GRAPH) && !(ps && spin_fault);
  const int splits = ps ? 0 : splits_for(s, n, chunk_max_len(s, n));
  const int key = ((splits * 128 + n) * 128 + heads) * 4 + (accept ? 1 : 0) + (ps ? 2 : 0);
  s->chunk_ps = ps;
  auto enqueue_all = [&]() -> int {
    cudaMemcpyAsync(s->toks_dev, s->toks_host, sizeof(hc::StepTok) * n, cudaMemcpyHostToDevice, st);
    int k = 0;
    if (ps) {
      // every row's logits and greedy choice (row t: token t); the host picks the rows it reads
      k = enqueue_ps(s, n, false, spin_fault ? spin_fault : kSpinLimit);
      if (accept) { hc::spec_accept(s->am_dev, s->toks_dev, n, s->res_dev, st); ++k; }
      cudaMemcpyAsync(s->ps_status_host, s->ps_status, sizeof(int), cudaMemcpyDeviceToHost, st);
      cudaMemcpyAsync(s->am_host, s->am_dev, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, st);
    } else {
      k = enqueue_model(s, n, accept, splits, heads);
      if (heads > 0) cudaMemcpyAsync(s->am_host, s->am_dev, sizeof(int32_t) * heads, cudaMemcpyDeviceToHost, st);
    }
    if (accept) cudaMemcpyAsync(s->res_host, s->res_dev, sizeof(int32_t) * 2, cudaMemcpyDeviceToHost, st);
    return k;
  };
  if (ps) {
    *s->ps_status_host = 0;
    cudaMemsetAsync(s->ps_status, 0, sizeof(int), st);
  }
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
  s->stats.launches += use_graph ? s->launches_per_key[key] : s->launches_per_key[key];
  return nullptr;
}

// The persistent step's status after a wait: an error string when one of its waits gave up.
char *ps_status_error(hc_session *s) {
  if (!s->ps || !*s->ps_status_host) return nullptr;
  const int c = *s->ps_status_host;
  std::string what = c < 100000 ? "grid barrier " + std::to_string(c) : c < 200000 ? "ring stage release (producer)"
                     : c < 300000 ? "weight stage " + std::to_string(c - 200000) : "key stage " + std::to_string(c - 300000);
  return hc::make_error("step: a device wait timed out (" + what + ")");
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

// Sets up the persistent step when the model and the device allow it (a dense model of one integer
// kind throughout, the fp16 cache, a cooperative launch of one CTA a SM).
char *ps_setup(hc_session *s) {
  hc_model *m = s->m;
  const auto &d = m->d;
  if (!(s->o.flags & HC_SESSION_PERSISTENT) || s->paged || d.arch != HC_ARCH_QWEN3) return nullptr;
  const int kind = m->head->m.kind, rep = int(d.heads / d.kv_heads);
  if (!hc::ps_supported(kind, int(d.head_dim), rep, s->cap)) return nullptr;
  for (auto &w : m->layers)
    if (w.qkv->m.kind != kind || w.o->m.kind != kind || w.gu->m.kind != kind || w.down->m.kind != kind ||
        w.gu->m.bias || w.down->m.bias || w.sinks || w.qkv->m.ktiles != m->layers[0].qkv->m.ktiles)
      return nullptr;
  if (m->head->m.ktiles != m->layers[0].qkv->m.ktiles) return nullptr;
  HC_TRY_CUDA(hc::ps_prepare());
  s->ps_ctas = hc::ps_ctas(m->ordinal);
  if (!s->ps_ctas) return nullptr;
  s->ps_kind = kind;
  s->ps_max_splits = (s->cap + hc::kPsSplitKeys - 1) / hc::kPsSplitKeys;
  // the most tokens a launch takes: its residual rows and activation tiles share the SM's shared
  // memory with a ring of at least 4 stages
  s->ps_max_tok = 0;
  for (int n = 1; n <= hc::kPsMaxTok; ++n) {
    hc::PsParams probe = ps_params(s, n, false, kSpinLimit);
    if (hc::ps_layout(probe, kind)) s->ps_max_tok = n;
  }
  if (!s->ps_max_tok) return nullptr;
  std::vector<hc::PsLayer> L(d.layers);
  for (size_t i = 0; i < L.size(); ++i) {
    const hc::LayerW &w = m->layers[i];
    L[i] = hc::PsLayer{w.qkv->m.tiles, w.o->m.tiles, w.gu->m.tiles, w.down->m.tiles,
                       w.qkv->m.row_scale, w.o->m.row_scale, w.gu->m.row_scale, w.down->m.row_scale,
                       w.qkv->m.bias, w.o->m.bias, w.in_norm, w.post_norm, w.q_norm, w.k_norm, w.sinks,
                       s->kc + i * s->layer_kv, s->vc + i * s->layer_kv, w.window};
  }
  const int T = hc::kPsMaxTok, H = int(d.heads), hd = int(d.head_dim);
  if (char *e = alloc(&s->ps_layers, L.size(), "step layer table")) return e;
  HC_TRY_CUDA(cudaMemcpy(s->ps_layers, L.data(), sizeof(hc::PsLayer) * L.size(), cudaMemcpyHostToDevice));
  s->ps_sync_bytes = sizeof(unsigned) * (4 + size_t(T) * d.kv_heads + 1);
  if (char *e = alloc(&s->ps_sync, s->ps_sync_bytes / sizeof(unsigned), "grid barrier and tickets")) return e;
  HC_TRY_CUDA(cudaMemset(s->ps_sync, 0, s->ps_sync_bytes));
  if (char *e = alloc(&s->ps_status, 1, "step status")) return e;
  HC_TRY_CUDA(cudaMemset(s->ps_status, 0, sizeof(int)));
  HC_TRY_CUDA(cudaHostAlloc(&s->ps_status_host, sizeof(int), cudaHostAllocDefault));
  *s->ps_status_host = 0;
  if (char *e = alloc(&s->ps_attn, size_t(T) * H * hd, "attention output")) return e;
  if (char *e = alloc(&s->ps_dx, size_t(T) * d.hidden, "down projection rows")) return e;
  if (char *e = alloc(&s->ps_part_ml, size_t(T) * H * s->ps_max_splits * 2, "attention partials")) return e;
  if (char *e = alloc(&s->ps_part_o, size_t(T) * H * s->ps_max_splits * hd, "attention partials")) return e;
  if (s->o.flags & HC_SESSION_PROFILE) {
    const size_t n = size_t(4) * hc::ps_phases(int(d.layers)) + size_t(8) * d.layers;
    if (char *e = alloc(&s->ps_trace, n, "phase trace")) return e;
    HC_TRY_CUDA(cudaMemset(s->ps_trace, 0, n * sizeof(unsigned long long)));
  }
  s->ps = true;
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
  if (s->paged)
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
  if (char *e = ps_setup(s.get())) return e;
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
  int off = 0;
  for (int i = 0; i < nseq; ++i) {
    for (int j = 0; j < n_tokens[i]; ++j) {
      const int tok = tokens[off + j];
      if (tok < 0 || tok >= V) return hc::make_error("hc_step: token " + std::to_string(tok) + " out of the vocabulary");
      all.push_back(hc::StepTok{tok, seq_ids[i], s->pos[seq_ids[i]] + j, 0});
      if ((flags & HC_STEP_ALL_ROWS) || j == n_tokens[i] - 1) want.push_back(int(all.size()) - 1);
    }
    off += n_tokens[i];
  }
  if (hc::fault_fires(hc::kFaultStep)) return hc::make_error("injected fault: step");
  HC_TRY_CUDA(cudaSetDevice(s->m->ordinal));
  size_t wi = 0;
  int row = 0;
  double step_us = 0;  // the call's device time: the sum over its chunks
  for (size_t c0 = 0; c0 < all.size(); c0 += kMaxChunk) {
    const int n = int(std::min<size_t>(kMaxChunk, all.size() - c0));
    std::memcpy(s->toks_host, &all[c0], sizeof(hc::StepTok) * n);
    int heads = 0;  // the chunk's rows that are read out, in order
    for (size_t w = wi; w < want.size() && size_t(want[w]) < c0 + n; ++w) s->toks_host[heads++].head_src = int(want[w] - c0);
    if (char *e = run_chunk(s, n, false, heads)) {
      for (int i = 0; i < nseq; ++i) s->poisoned[seq_ids[i]] = true;
      return e;
    }
    int32_t st_ = HC_STATE_ERROR;
    char *e = wait_done(s, timeout_ms, &st_);
    if (!e && st_ == HC_STATE_COMPLETED && s->chunk_ps) e = ps_status_error(s);
    if (e || st_ != HC_STATE_COMPLETED) {
      for (int i = 0; i < nseq; ++i) s->poisoned[seq_ids[i]] = true;
      if (state) *state = e ? HC_STATE_ERROR : st_;
      return e;
    }
    step_us += s->stats.last_step_us;
    for (int j = 0; wi < want.size() && size_t(want[wi]) < c0 + n; ++wi, ++row, ++j) {
      // the kernel sequence writes the read rows in order; the persistent step every token's row
      const int src = s->chunk_ps ? s->toks_host[j].head_src : j;
      if (argmax) argmax[row] = s->am_host[src];
      if (logits) HC_TRY_CUDA(cudaMemcpy(logits + size_t(row) * V, s->logits_dev + size_t(src) * V, size_t(V) * 2, cudaMemcpyDeviceToHost));
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
    s->toks_host[j] = hc::StepTok{toks[j], seq, s->pos[seq] + j, j};
  }
  if (hc::fault_fires(hc::kFaultStep)) return hc::make_error("injected fault: step");
  HC_TRY_CUDA(cudaSetDevice(s->m->ordinal));
  if (char *e = run_chunk(s, n, true, n)) { s->poisoned[seq] = true; return e; }
  int32_t st_ = HC_STATE_ERROR;
  char *e = wait_done(s, timeout_ms, &st_);
  if (!e && st_ == HC_STATE_COMPLETED && s->chunk_ps) e = ps_status_error(s);
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
  s->toks_host[0] = hc::StepTok{first, seq, s->pos[seq], 0};
  const bool ps = ps_chunk(s, 1);
  if (!s->gen_graph) {
    cudaGraph_t graph = nullptr;
    HC_TRY_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    if (ps) {
      // the status word is zeroed once before the loop: after a failed launch the later ones
      // return at once (they see it set)
      s->launches_per_chunk[0] = uint64_t(enqueue_ps(s, 1, true, kSpinLimit));
    } else {
      s->launches_per_chunk[0] = uint64_t(enqueue_model(s, 1, false, splits_for(s, 1, 0), 1)) + 1;
      hc::advance(s->toks_dev, s->am_dev, s->gen_out, s->gen_count, st);
    }
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (e != cudaSuccess) return hc::make_error(std::string("graph capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(&s->gen_graph, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return hc::make_error(std::string("graph instantiate: ") + cudaGetErrorString(e));
  }
  HC_TRY_CUDA(cudaMemcpyAsync(s->toks_dev, s->toks_host, sizeof(hc::StepTok), cudaMemcpyHostToDevice, st));
  HC_TRY_CUDA(cudaMemsetAsync(s->gen_count, 0, sizeof(int32_t), st));
  if (ps) {
    *s->ps_status_host = 0;
    HC_TRY_CUDA(cudaMemsetAsync(s->ps_status, 0, sizeof(int), st));
  }
  HC_TRY_CUDA(cudaEventRecord(s->ev0, st));
  hc::device_stall(hc::take_stall_ms(), st);
  for (int i = 0; i < n; ++i) HC_TRY_CUDA(cudaGraphLaunch(s->gen_graph, st));
  HC_TRY_CUDA(cudaEventRecord(s->ev1, st));
  if (ps) HC_TRY_CUDA(cudaMemcpyAsync(s->ps_status_host, s->ps_status, sizeof(int), cudaMemcpyDeviceToHost, st));
  s->stats.launches += uint64_t(n) * s->launches_per_chunk[0];
  int32_t st_ = HC_STATE_ERROR;
  char *e = wait_done(s, timeout_ms, &st_);
  if (!e && st_ == HC_STATE_COMPLETED && ps) {
    HC_TRY_CUDA(cudaStreamSynchronize(st));
    e = ps_status_error(s);
  }
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

HC_API char *hc_profile_get(hc_session *s, double *us, uint32_t cap, uint32_t *n) {
  if (!s || !n) return hc::make_error("hc_profile_get: NULL argument");
  if (!s->ps_trace)
    return hc::make_error("hc_profile_get: the session was not opened with HC_SESSION_PROFILE and the persistent step");
  const int P = hc::ps_phases(int(s->m->d.layers));
  *n = uint32_t(P);
  if (!us) return nullptr;
  std::vector<unsigned long long> t(size_t(4) * P);
  HC_TRY_CUDA(cudaStreamSynchronize(s->st));
  HC_TRY_CUDA(cudaMemcpy(t.data(), s->ps_trace, t.size() * 8, cudaMemcpyDeviceToHost));
  auto d = [](unsigned long long a, unsigned long long b) { return b > a ? double(b - a) / 1e3 : 0.0; };
  for (int i = 0; i < P; ++i) {
    const unsigned long long start = i ? t[4 * (i - 1) + 2] : t[0];
    const double v[4] = {d(start, t[4 * i]), d(t[4 * i], t[4 * i + 1]), i + 1 < P ? d(t[4 * i + 1], t[4 * i + 2]) : 0.0,
                         double(t[4 * i + 3]) / 1e3};
    for (int k = 0; k < 4; ++k)
      if (uint32_t(4 * i + k) < cap) us[4 * i + k] = v[k];
  }
  // then, per layer, the attention unit that merged (token 0, kv head 0): microseconds from the
  // unit's start to its inputs loaded, its stages in, its partial written, its ticket taken, the
  // merge written; then the CTA and the unit's index in the CTA
  const int L = int(s->m->d.layers);
  if (cap >= uint32_t(4 * P + 8 * L)) {
    std::vector<unsigned long long> u(size_t(8) * L);
    HC_TRY_CUDA(cudaMemcpy(u.data(), s->ps_trace + size_t(4) * P, u.size() * 8, cudaMemcpyDeviceToHost));
    for (int l = 0; l < L; ++l) {
      const unsigned long long *m = &u[size_t(8) * l];
      for (int k = 1; k < 6; ++k) us[4 * P + 8 * l + k - 1] = d(m[0], m[k]);
      us[4 * P + 8 * l + 5] = double(m[6]);
      us[4 * P + 8 * l + 6] = double(m[7]);
      us[4 * P + 8 * l + 7] = 0;
    }
  }
  return nullptr;
}

HC_API char *hc_stats_get(hc_session *s, hc_stats *out) {
  if (!s || !out) return hc::make_error("hc_stats_get: NULL argument");
  *out = s->stats;
  return nullptr;
}

}  // extern "C"
