/*
 * oracle.h — TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A CPU restatement, in C++17, of hwnpu's Go CPU reference path for the decode hot path
 * (internal/milcpu, internal/sgemm, internal/vecops, internal/f32, internal/palette/linear.go,
 * internal/mxfp4, internal/llm/{qwen3,gptoss,experts,paged,decode}, internal/chat/sample.go).
 * Each function cites the reference file:line it follows. The Go reference cannot be built in
 * this environment (no Go toolchain, dependencies not vendored), so parity is pinned by the
 * reference's own known-answer tests, ported in tests/test_oracle.py.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its --impl
 * reference arm) may load this library; the product never does.
 */
#ifndef HWNPU_ORACLE_H
#define HWNPU_ORACLE_H

#include <stdint.h>
#include <stddef.h>
#include "../include/hwnpu_cuda.h"

#define OR_API extern "C" __attribute__((visibility("default")))

/* vecops.F16Bits / F16Value (internal/vecops/vecops.go:297-352) */
OR_API uint16_t or_f16_bits(float f);
OR_API float or_f16_value(uint16_t h);
/* f32.exp, Cephes expf (internal/f32/f32.go:49-70) */
OR_API float or_exp(float x);
/* The reference's synthetic checkpoint values: uniform in [-0.1, 0.1) from the FNV-1a hash of
 * the name (internal/llm/synth.go:17-36). */
OR_API void or_synth_uniform(const char *name, float *out, uint64_t n);

/* The benchmark configurations' seeded inputs (synth.cpp): n values N(0, std^2) for a tensor name,
 * and n token ids uniform on [0, vocab); equal bit for bit to the product's generator. */
OR_API void or_synth_normal(uint64_t seed, const char *name, const float *std_, float *out, uint64_t n);
OR_API void or_synth_tokens(uint64_t seed, int32_t vocab, int32_t *out, uint64_t n);
/* or_f16_bits over n values. */
OR_API void or_f32_to_f16_n(const float *src, uint16_t *dst, uint64_t n);

/* palette.QuantizeLinear / Linear.Dequantize (internal/palette/linear.go:36-169) */
OR_API void or_quantize_linear(const float *w, uint32_t rows, uint32_t cols, uint32_t col_block,
                               int32_t bits, int32_t search, uint8_t *data, uint16_t *scales);
OR_API void or_dequant_linear(const uint8_t *data, const uint16_t *scales, uint32_t rows,
                              uint32_t cols, uint32_t col_block, int32_t bits, float *out);
/* milcpu shiftScale with an fp16 offset (internal/milcpu/ops.go:1589-1610) over unsigned 4-bit
 * codes with 32 columns a block; and the asymmetric quantiser of HC_FMT_INT4_ASYM_G32. */
OR_API void or_dequant_int4_asym(const uint8_t *data, const uint16_t *scales,
                                 const uint16_t *zeros, uint32_t rows, uint32_t cols, float *out);
OR_API void or_quantize_int4_asym(const float *w, uint32_t rows, uint32_t cols, uint8_t *data,
                                  uint16_t *scales, uint16_t *zeros);

/* internal/mxfp4 */
OR_API uint8_t or_mxfp4_nearest(double x);                                    /* encode.go:62-78 */
OR_API void or_mxfp4_encode(const float *row, uint32_t n, uint8_t *w, uint8_t *e); /* encode.go:11-58 */
OR_API void or_mxfp4_dequant(const uint8_t *w, const uint8_t *e, uint32_t n, float *out); /* mxfp4.go:118-128 */
OR_API void or_mxfp4_quantize(const float *x, uint32_t n, int8_t *q, float *s); /* mxfp4.go:33-53 */
OR_API float or_mxfp4_dot(const uint8_t *w, const uint8_t *e, uint32_t n, const int8_t *q,
                          const float *s); /* dotGo, mxfp4.go:80-91 */

/* experts.Routing.Choose, Score softmax (experts/weights.go:33-82) */
OR_API void or_route(const float *logits, int32_t n, int32_t k, int32_t norm, int32_t *idx,
                     float *w);

/* paged.Merge (internal/llm/paged/paged.go:227-310) */
typedef struct or_merge or_merge;
OR_API or_merge *or_merge_new(int32_t rows, int32_t dim);
OR_API void or_merge_free(or_merge *m);
OR_API void or_merge_add(or_merge *m, const float *o, const float *mx, const float *l);
OR_API void or_merge_add_sink(or_merge *m, const float *sinks, int32_t tokens);
OR_API void or_merge_result(or_merge *m, float *out);

/* sgemm.MulAdd's product (internal/sgemm/sgemm.go:127): c[m][n] += sum_k a[m][k] b[n][k] */
OR_API void or_gemm_nt(int32_t m, int32_t n, int32_t k, const float *a, const float *b,
                       float *c, int32_t threads);

/* chat.Sampling.pick at temperature 0 (internal/chat/sample.go:80-88) */
OR_API int32_t or_argmax(const float *logits, int32_t n);
OR_API int32_t or_argmax_f16(const uint16_t *logits, int32_t n);

/* The decode session of one model on the CPU interpreter (decode.Session over milcpu,
 * internal/llm/qwen3/cache_test.go:43-123). */
typedef struct or_model or_model;
typedef struct or_session or_session;
OR_API or_model *or_model_new(const hc_model_desc *desc, int32_t threads);
OR_API void or_model_free(or_model *m);
OR_API or_session *or_session_new(or_model *m, int32_t max_context);
/* A session over a cache of kv_format: HC_KV_F16 as or_session_new, or HC_KV_INT8_PAGED, this
 * library's own paged int8 format restated (16-position pages, an fp16 scale per page and kv head
 * rounded up from max|x| / 127, earlier rows requantised when it grows; the reference has no such
 * cache, so this mode is parity unpinned): the step's own keys and values are used in float32 and
 * go into the pages after the step, as decode.Session.keep does for the fp16 cache. */
OR_API or_session *or_session_new_kv(or_model *m, int32_t max_context, int32_t kv_format);
OR_API void or_session_free(or_session *s);
OR_API int32_t or_session_pos(or_session *s);
/* Session.Step (decode.go:1221): reads n tokens; writes fp16 logits of every row
 * ([n][vocab]) when all_rows, else of the last; keeps all n in the cache. */
OR_API int32_t or_step(or_session *s, const int32_t *tokens, int32_t n, int32_t all_rows,
                       uint16_t *logits);
/* Session.Speculate with the greedy accept of chat/engine.go:1044-1058: returns kept, writes the
 * next token. */
OR_API int32_t or_speculate(or_session *s, const int32_t *toks, int32_t n, int32_t *next,
                            uint16_t *logits_last);
OR_API void or_truncate(or_session *s, int32_t len);
/* One row written into a page of the paged int8 cache, as an int8-paged session writes it (the
 * page's rows [16][hd] and its fp16 scale bits are updated in place; off: the row's slot). */
OR_API void or_page_write(int8_t *page_rows, uint16_t *scale, int32_t off, const float *x, int32_t hd);

#endif
