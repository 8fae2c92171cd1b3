/*
 * hwnpu_cuda.h: the C ABI of libhwnpu_cuda.so, a device-resident decode engine for hwnpu on
 * NVIDIA B200 (sm_100a).
 *
 * hwnpu's host code is Go without cgo; it loads native libraries through purego
 * (internal/dl/dl.go:23-63) and binds a table of symbols with an ABI check
 * (internal/backend/amdxrt/shim.go:110-140). This header follows the conventions of the
 * reference's own C shim, native/xrtshim/xrtshim.h:1-117:
 *   - every function that can fail returns NULL on success, or a heap error string that the
 *     caller frees with hc_free_error (xrtshim.h:6-8, xs_free_error);
 *   - objects are opaque handles freed by their hc_*_free;
 *   - no struct or float is passed by value; descriptors go by pointer; no callbacks;
 *   - the library never keeps a pointer to caller memory past the call that received it:
 *     weights are copied to HBM inside hc_model_load, tokens and logits are copied inside
 *     hc_step (docs/design/architecture.md:135-158 of the reference);
 *   - waits take a timeout in milliseconds and report HC_STATE_TIMEOUT instead of blocking
 *     for ever (xrtshim.h:106-108, xs_run_wait).
 *
 * Threading: a session is used by one thread at a time (graph.go:87 of the reference holds the
 * same rule for requests); distinct sessions of one device may be used from distinct threads.
 */
#ifndef HWNPU_CUDA_H
#define HWNPU_CUDA_H

#include <stddef.h>
#include <stdint.h>

#define HC_API __attribute__((visibility("default")))

#ifdef __cplusplus
extern "C" {
#endif

/* The ABI version. A Go binding refuses a library of another (amdxrt/shim.go:124-128). */
#define HC_ABI 2

typedef struct hc_device hc_device;
typedef struct hc_buf hc_buf;
typedef struct hc_model hc_model;
typedef struct hc_session hc_session;

/* States written by the waiting calls (the subset of xrtshim.h's XS_STATE_* that applies). */
enum {
  HC_STATE_COMPLETED = 4,
  HC_STATE_ERROR = 5,
  HC_STATE_TIMEOUT = 8,
};

/* ---------------------------------------------------------------------------------------- */
/* Version and errors                                                                        */
/* ---------------------------------------------------------------------------------------- */

/* Replaces xs_abi (xrtshim.h:73). */
HC_API int hc_abi(void);
/* Replaces xs_free_error (xrtshim.h:74). NULL is allowed. */
HC_API void hc_free_error(char *err);

/* ---------------------------------------------------------------------------------------- */
/* Devices: backend.Provider.Enumerate/Open (internal/backend/backend.go:13-19)               */
/* ---------------------------------------------------------------------------------------- */

/* Keys of hc_device_info. */
enum {
  HC_INFO_NAME = 0,        /* "NVIDIA B200" */
  HC_INFO_PCI_BUS_ID = 1,  /* "0000:1b:00.0" */
  HC_INFO_ARCH = 2,        /* "sm_100" */
  HC_INFO_MEMORY = 3,      /* total HBM bytes, decimal */
  HC_INFO_SMS = 4,         /* multiprocessor count, decimal */
  HC_INFO_DRIVER = 5,      /* driver version, decimal */
};

/* Replaces xs_device_count (xrtshim.h:76). Honours HWNPU_CUDA_DEVICES=0,2,... as a filter. */
HC_API char *hc_device_count(uint32_t *count);
/* Replaces xs_device_open (xrtshim.h:77). index counts the devices hc_device_count sees. */
HC_API char *hc_device_open(uint32_t index, hc_device **out);
/* Replaces xs_device_free (xrtshim.h:78). */
HC_API void hc_device_free(hc_device *d);
/* Replaces xs_device_info (xrtshim.h:80): writes the value, NUL terminated, into buf of n
 * bytes; *need is its length with the NUL. */
HC_API char *hc_device_info(hc_device *d, int key, char *buf, size_t n, size_t *need);
/* Health of the library's kernels on the device: an error string when a bounded wait inside one of
 * them (the tensor-core GEMV's pipeline waits, about a second each) ran out since the last call --
 * the results of that launch are not to be trusted -- else NULL; clears the record. Waits for the
 * device's queued work first. (The reference's xs_run_wait reports a failed run the same way.) */
HC_API char *hc_device_check(hc_device *d);

/* ---------------------------------------------------------------------------------------- */
/* Buffers: backend.Device.AllocBuffer and backend.Buffer (backend.go:54-67)                  */
/* ---------------------------------------------------------------------------------------- */

enum {
  HC_BUF_DEVICE = 0, /* HBM, with a pinned host mirror that hc_buf_map returns */
  HC_BUF_HOST = 1,   /* pinned host memory only, visible to the device */
};
enum {
  HC_SYNC_TO_DEVICE = 0,
  HC_SYNC_FROM_DEVICE = 1,
};

/* Replaces xs_bo_alloc (xrtshim.h:84). */
HC_API char *hc_buf_alloc(hc_device *d, uint64_t size, int kind, hc_buf **out);
/* Replaces xs_bo_free (xrtshim.h:85). */
HC_API void hc_buf_free(hc_buf *b);
/* Replaces xs_bo_map (xrtshim.h:88): the host view (backend.Buffer.Bytes). */
HC_API char *hc_buf_map(hc_buf *b, void **ptr);
/* The device address of the buffer, for the kernel entry points below (xs_bo_address,
 * xrtshim.h:89). */
HC_API uint64_t hc_buf_address(hc_buf *b);
/* Replaces xs_bo_sync (xrtshim.h:90): SyncToDevice / SyncFromDevice of n bytes from off. */
HC_API char *hc_buf_sync(hc_buf *b, int dir, uint64_t off, uint64_t n);

/* ---------------------------------------------------------------------------------------- */
/* Weight formats (the reference's byte layouts, copied as they are)                        */
/* ---------------------------------------------------------------------------------------- */

enum {
  HC_FMT_NONE = -1,
  HC_FMT_F16 = 0,         /* fp16 [rows][cols] */
  HC_FMT_BF16 = 1,        /* bf16 [rows][cols] (gpt-oss attention, router and head) */
  /* palette.Linear of 8 bits, one fp16 scale a row (internal/palette/linear.go:17-29,
   * mlpackage Int8Scaled program.go:421): data int8 [rows][cols], scales fp16 [rows];
   * w = q * s (Linear.Dequantize, linear.go:152-169). */
  HC_FMT_INT8_ROW = 2,
  /* palette.Linear of 4 bits, one fp16 scale per 32 columns (Int4Scaled, program.go:392-398):
   * two's complement nibbles, low nibble first; w = q * s. */
  HC_FMT_INT4_SYM_G32 = 3,
  /* Unsigned 4-bit codes, low nibble first, with an fp16 scale s and zero point z per
   * (row, 32 columns): w = (float(q) - z) * s in float32, the order of milcpu's shiftScale
   * with an offset (internal/milcpu/ops.go:1589-1610). */
  HC_FMT_INT4_ASYM_G32 = 4,
  /* MXFP4 (internal/mxfp4/mxfp4.go:1-20): e2m1 codes, the even column in the low nibble,
   * 16 bytes a block of 32 columns, and one e8m0 exponent a block: w = e2m1 * 2^(e-127). */
  HC_FMT_MXFP4 = 5,
};

typedef struct hc_linear_desc {
  int32_t format;          /* HC_FMT_* (HC_FMT_NONE: absent) */
  uint32_t rows, cols;     /* the matrix is (rows, cols); y = x W^T (milcpu linear, ops.go:940) */
  const void *data;        /* codes or values in the format's layout */
  const uint16_t *scales;  /* fp16 bits: [rows] for INT8_ROW, [rows][cols/32] for INT4_* */
  const uint16_t *zeros;   /* fp16 bits [rows][cols/32]: INT4_ASYM_G32 only */
  const uint8_t *exps;     /* e8m0 [rows][cols/32]: MXFP4 only */
  const float *bias;       /* [rows], or NULL */
} hc_linear_desc;

/* ---------------------------------------------------------------------------------------- */
/* Models: the weights of llm.Model (internal/llm/arch.go:116-330)                           */
/* ---------------------------------------------------------------------------------------- */

enum {
  /* Qwen3ForCausalLM as internal/llm/qwen3/build.go writes it; a Llama-style decoder is the
   * same without HC_MODEL_QK_NORM. */
  HC_ARCH_QWEN3 = 1,
  /* gpt-oss (internal/llm/gptoss): biases, sinks, alternating sliding/full attention, YaRN,
   * MXFP4 experts behind a softmax top-k router. */
  HC_ARCH_GPTOSS = 2,
};

enum {
  HC_MODEL_QK_NORM = 1 << 0,    /* per-head RMS norms of q and k before RoPE (build.go:283-284) */
  HC_MODEL_TIED = 1 << 1,       /* the head is the embedding table (qwen3/config.go:143-148) */
  HC_MODEL_NORM_SCALE = 1 << 2, /* Qwen3's normScale 64 (build.go:117-151): the norms square x/64
                                 * with epsilon eps/64^2 rounded to fp16; layer 0's input norm x/1 */
  HC_MODEL_ATTN_BIAS = 1 << 3,  /* q/k/v/o projections carry biases (gpt-oss, Qwen2) */
};

typedef struct hc_layer_desc {
  const uint16_t *input_norm;  /* fp16 [hidden] */
  const uint16_t *post_norm;   /* fp16 [hidden] */
  const uint16_t *q_norm;      /* fp16 [head_dim], with HC_MODEL_QK_NORM */
  const uint16_t *k_norm;      /* fp16 [head_dim], with HC_MODEL_QK_NORM */
  hc_linear_desc q, k, v, o;
  hc_linear_desc gate, up, down; /* the SwiGLU MLP (qwen3/build.go:202-229) */
  const float *sinks;          /* [heads]: gpt-oss's sink logits (gptoss/build.go:256-285), or NULL */
  uint32_t sliding_window;     /* 0: full attention; else keys with pos - key < window */
  uint32_t pad_;
  hc_linear_desc router;       /* [experts][hidden] + bias (gptoss/build.go:125-140) */
  hc_linear_desc experts_gate_up; /* MXFP4 [experts*2*inter][hidden], gate rows even, up odd */
  hc_linear_desc experts_down;    /* MXFP4 [experts*hidden][inter] */
} hc_layer_desc;

typedef struct hc_model_desc {
  uint32_t abi;                /* HC_ABI */
  uint32_t arch;               /* HC_ARCH_* */
  uint32_t flags;              /* HC_MODEL_* */
  uint32_t hidden, inter, layers, heads, kv_heads, head_dim, vocab;
  uint32_t experts, top_k;     /* MoE; 0 for a dense model */
  double norm_eps;             /* rms_norm_eps */
  double rope_theta;
  double yarn_factor;          /* <= 1: plain RoPE (gptoss/config.go:136-166) */
  double yarn_beta_fast, yarn_beta_slow;
  uint32_t yarn_original;      /* original_max_position_embeddings */
  uint32_t yarn_truncate;
  double swiglu_alpha, swiglu_limit; /* gpt-oss's gate activation (experts/host.go:515-524) */
  const uint16_t *embed;       /* fp16 [vocab][hidden], or NULL when HC_MODEL_TIED */
  const uint16_t *final_norm;  /* fp16 [hidden] */
  hc_linear_desc head;         /* [vocab][hidden] */
  const hc_layer_desc *layer;  /* [layers] */
} hc_model_desc;

/* Copies the weights to the device's HBM, repacked for the kernels (the repacking keeps every
 * code, so hc_linear_dequant is bit-exact with the format's own dequantisation). The desc and
 * the host bytes it points to are not kept. */
HC_API char *hc_model_load(hc_device *d, const hc_model_desc *desc, hc_model **out);
HC_API void hc_model_free(hc_model *m);
/* Bytes one decode step of one token reads from HBM for the weights (the roofline's numerator
 * less the KV cache). */
HC_API uint64_t hc_model_weight_bytes(hc_model *m);

/* ---------------------------------------------------------------------------------------- */
/* Sessions: chat.session / chat.tokenSession (internal/chat/session.go:9-32) over           */
/* decode.Session (internal/llm/decode/decode.go:102-175)                                    */
/* ---------------------------------------------------------------------------------------- */

enum {
  HC_KV_F16 = 0,        /* fp16 keys and values, (kv_heads, positions, head_dim) per layer */
  /* int8 in pages of page_size (16) positions from a pool with a block table per sequence, one
   * fp16 scale a (page, head) for keys and one for values (BASELINE C5; the reference has no
   * such cache). A page's scale is the fp16 rounding up of max|x| / 127 over its rows; when a new
   * row needs more, the page's rows are requantised to the new scale. Truncating inside a page
   * keeps its scale; truncated pages return to the pool. Export/import of rows is not offered. */
  HC_KV_INT8_PAGED = 1,
};
enum {
  HC_SESSION_NO_GRAPH = 1 << 0,      /* launch the step's kernels one by one (no CUDA graph) */
};

typedef struct hc_session_opts {
  uint32_t max_context;  /* positions a sequence may hold (Session.Cache) */
  uint32_t max_seqs;     /* sequence slots */
  uint32_t max_step;     /* most tokens hc_speculate verifies in one call (1..64); hc_step reads
                          * any number, in passes of up to 64 tokens over the weights */
  uint32_t kv_format;    /* HC_KV_* */
  uint32_t page_size;    /* positions a page (HC_KV_INT8_PAGED), 16 */
  uint32_t flags;        /* HC_SESSION_* */
} hc_session_opts;

HC_API char *hc_session_new(hc_model *m, const hc_session_opts *opts, hc_session **out);
HC_API void hc_session_free(hc_session *s);

enum {
  HC_STEP_ALL_ROWS = 1 << 0, /* logits/argmax for every token read, not only each sequence's last */
};

/* Session.Step / tokenSession.StepTokens (decode.go:1221, session.go:28): sequence seq_ids[i]
 * reads n_tokens[i] tokens (the tokens of all sequences one after another in tokens), their keys
 * and values go into its cache and its position moves past them. For each sequence's last token
 * (every token with HC_STEP_ALL_ROWS) the logits are written as fp16 bits into logits
 * ([rows][vocab]) and the greedy choice (the first largest logit, chat/sample.go:80-88) into
 * argmax ([rows]); either may be NULL. Waits up to timeout_ms (0: for ever) and writes
 * HC_STATE_COMPLETED or HC_STATE_TIMEOUT into *state; a session that timed out or failed is
 * poisoned until hc_seq_reset of its sequences (the cache may be half written, as
 * chat/engine.go:1521-1525 says of the reference's). */
HC_API char *hc_step(hc_session *s, const int32_t *seq_ids, const int32_t *n_tokens,
                     const int32_t *tokens, int32_t nseq, int32_t flags, uint16_t *logits,
                     int32_t *argmax, uint32_t timeout_ms, int32_t *state);

/* tokenSession.SpeculateTokens with greedy acceptance (session.go:30, decode.go:1235-1260,
 * chat/engine.go:1044-1058), on the device: sequence seq reads toks (the token to read next
 * followed by n-1 drafts) in one call; draft i is kept while the greedy choice after token i
 * equals it. *kept (1..n) is how many of toks stay in the cache, *next is the greedy token after
 * the last kept one; logits, if not NULL, gets that row ([vocab] fp16 bits). */
HC_API char *hc_speculate(hc_session *s, int32_t seq, const int32_t *toks, int32_t n,
                          int32_t *kept, int32_t *next, uint16_t *logits, uint32_t timeout_ms,
                          int32_t *state);

/* Greedy generation on the device, the per-token loop of chat.Engine.Generate
 * (internal/chat/engine.go:1509) without a host round trip per token (the device-resident
 * precedent is ironSession, internal/chat/iron.go:22-260): sequence seq reads `first`, then each
 * greedy choice (chat/sample.go:80-88) in turn, n tokens in all; out_tokens ([n]) gets the n
 * choices. The sequence's position moves by n. */
HC_API char *hc_generate(hc_session *s, int32_t seq, int32_t first, int32_t n, int32_t *out_tokens,
                         uint32_t timeout_ms, int32_t *state);

/* The CUDA stream (cudaStream_t) the session's steps run on, for callers that time them with
 * CUDA events or order their own work after them. */
HC_API char *hc_session_stream(hc_session *s, void **stream);

/* Session.Reset (session.go:14). */
HC_API char *hc_seq_reset(hc_session *s, int32_t seq);
/* Session.Truncate (decode.go:1774): keeps the first len positions. */
HC_API char *hc_seq_truncate(hc_session *s, int32_t seq, int32_t len);
/* Session.Pos (session.go:13). */
HC_API char *hc_seq_pos(hc_session *s, int32_t seq, int32_t *pos);
/* Session.ExportRows / ImportRows (decode.go:1859,1883): the keys and values of positions
 * [start, start+n) of every layer, fp16, packed as [layer][k|v][kv_head][n][row bytes]. With dst
 * NULL only *need is written. A session over the paged int8 cache (HC_KV_INT8_PAGED) returns an
 * error from both. */
HC_API char *hc_seq_export_rows(hc_session *s, int32_t seq, int32_t start, int32_t n, void *dst,
                                uint64_t cap, uint64_t *need);
HC_API char *hc_seq_import_rows(hc_session *s, int32_t seq, int32_t start, int32_t n,
                                const void *src, uint64_t size);

typedef struct hc_stats {
  uint64_t steps;          /* calls that ran */
  uint64_t tokens;         /* tokens read */
  uint64_t launches;       /* kernels launched (graph nodes included) */
  uint64_t weight_bytes;   /* weight bytes read by the last step */
  uint64_t kv_bytes;       /* KV bytes read by the last step */
  double last_step_us;     /* device time of the last call (CUDA events; the sum over its chunks) */
} hc_stats;

HC_API char *hc_stats_get(hc_session *s, hc_stats *out);

/* Fault injection for tests (the reference fakes its drivers instead, testdata/zemock):
 * "alloc:N" fails the N-th device allocation from now, "h2d:N" the N-th host-to-device copy,
 * "step:N" the N-th hc_step, each with an error string; "stall:MS" (MS <= 2000) makes the next
 * hc_step, hc_speculate or hc_generate first wait MS milliseconds on the device, so that a shorter
 * timeout_ms runs out (HC_STATE_TIMEOUT, the sequences poisoned until hc_seq_reset); "" clears.
 * Nothing faults or hangs on the GPU: the stall is a bounded wait on the global timer. */
HC_API char *hc_set_fault(const char *spec);

/* ---------------------------------------------------------------------------------------- */
/* Converter side: the reference's quantisers, on the host's cores                            */
/* (the seeded synthetic-weight helpers of tests and benchmarks are in hwnpu_cuda_synth.h)    */
/* ---------------------------------------------------------------------------------------- */

/* palette.QuantizeLinear (internal/palette/linear.go:36-114): bits 4 or 8, one fp16 scale per
 * col_block columns (0: whole rows), with the MSE clip search when search != 0. data gets
 * rows*cols bytes (8 bits) or rows*cols/2 (4 bits), scales rows*(cols/col_block). */
HC_API char *hc_quantize_linear(const float *w, uint32_t rows, uint32_t cols, uint32_t col_block,
                                int32_t bits, int32_t search, uint8_t *data, uint16_t *scales);
/* Asymmetric 4-bit quantiser of HC_FMT_INT4_ASYM_G32 (no counterpart in the reference, whose
 * int4 is symmetric): per (row, 32 columns) s = f16((max - min) / 15) and z = f16(-min / s)
 * (clamped to [0, 15]), q = clamp(round_even(v / s + z), 0, 15); a block whose values are all
 * equal gets s = f16(|v|) or 1 and codes that reproduce it. */
HC_API char *hc_quantize_int4_asym(const float *w, uint32_t rows, uint32_t cols, uint8_t *data,
                                   uint16_t *scales, uint16_t *zeros);
/* mxfp4.Encode of each row (internal/mxfp4/encode.go:11-58): blocks rows*cols/2 bytes, exps
 * rows*cols/32. */
HC_API char *hc_mxfp4_encode(const float *w, uint32_t rows, uint32_t cols, uint8_t *blocks,
                             uint8_t *exps);
/* vecops.F32ToF16 / F16ToF32 (internal/vecops/vecops.go:269-352): RNE, overflow to inf, NaN to
 * sign|0x7e00. */
HC_API void hc_f32_to_f16(const float *src, uint16_t *dst, uint64_t n);
HC_API void hc_f16_to_f32(const uint16_t *src, float *dst, uint64_t n);

/* ---------------------------------------------------------------------------------------- */
/* Kernel entry points on device memory, for parity tests and the bench's kernel timing       */
/* (pointers are device addresses; stream is a cudaStream_t or NULL for the default stream)   */
/* ---------------------------------------------------------------------------------------- */

typedef struct hc_linear hc_linear;

/* One matrix loaded and repacked as hc_model_load does it. */
HC_API char *hc_linear_load(hc_device *d, const hc_linear_desc *desc, hc_linear **out);
HC_API void hc_linear_free(hc_linear *l);
/* The matrix's values in float32, rows [row0, row0+nrows), read back from the repacked device
 * copy with the format's own arithmetic (Linear.Dequantize linear.go:152-169, shiftScale
 * ops.go:1589-1610, mxfp4.Dequantize mxfp4.go:118-128): bit-exact. out is host memory. */
HC_API char *hc_linear_dequant(hc_linear *l, uint32_t row0, uint32_t nrows, float *out);
/* y[t][r] = sum_c x[t][c] W[r][c] (+ bias) for tokens t < ntok (1..8): the decode GEMV. x is
 * float32 [ntok][cols], y float32 [ntok][rows], both device memory. For HC_FMT_MXFP4 the
 * vector is quantised to int8 per 32 as mxfp4.Vec.Quantize does (mxfp4.go:33-53) and the
 * blocks are summed in int32 as dotGo does (mxfp4.go:80-91). */
HC_API char *hc_linear_run(hc_linear *l, const float *x, int32_t ntok, float *y, void *stream);

/* Decode attention of one sequence over an fp16 cache (blocks.SDPAGrouped blocks.go:516-539,
 * gpt-oss's sdpaSink gptoss/build.go:256-285, Flash-Decoding's merge paged.go:227-310):
 * q float32 [ntok][heads][head_dim] (already normed and rotated), kcache/vcache fp16
 * [kv_heads][cap][head_dim] with the key and value of position p at slot p mod cap: a linear cache
 * (pos + ntok <= cap), or a ring of the sliding window (gptoss StepInputs' ring, build.go:291-326)
 * that holds the step's own rows too, which needs window > 0 and cap >= window + ntok - 1;
 * token t at position pos + t sees keys p <= pos + t with pos + t - p < window (window 0: all). sinks float32 [heads] or NULL. o float32
 * [ntok][heads][head_dim]. scale is multiplied into the scores. */
HC_API char *hc_attention_run(const float *q, const uint16_t *kcache, const uint16_t *vcache,
                              const float *sinks, float *o, int32_t ntok, int32_t heads,
                              int32_t kv_heads, int32_t head_dim, int32_t pos, int32_t cap,
                              int32_t window, const float *scale, void *stream);

/* hc_attention_run with the same arguments, results and kernels, but it allocates nothing: no
 * cudaMalloc, no cudaFree, no host-to-device copy. It has no counterpart in the reference (whose
 * CPU attention needs no device scratch); it is for callers that may not allocate device memory
 * per call, such as a serving loop whose device memory is all handed out up front, where a
 * cudaMalloc can fail and a cudaFree stalls every stream of the device until the GPU is idle.
 * Its scratch (step tokens, per-split partials, activation tiles) is one static device array of
 * 8 MiB per device, shared by every call of the process and left holding the last call's
 * contents; nothing in it needs to start at zero, since each call writes all it reads. A call
 * whose scratch (ntok * heads * (16 * 4 * (head_dim + 2)) bytes plus tokens and activation
 * tiles) exceeds 8 MiB is rejected with an error. The work is enqueued on stream and not waited
 * for: errors of the launches are returned, errors of the execution show on the stream. Calls
 * that overlap in time on one device (other streams or threads) share the scratch and race: run
 * them on one stream. A call outside a stream capture looks the array's address up on its device
 * (cudaGetSymbolAddress, with that device current); a call inside a capture uses the address of the
 * last call outside one, so make a first call on each device before any stream capture. */
HC_API char *hc_attention_run_static(const float *q, const uint16_t *kcache, const uint16_t *vcache,
                                     const float *sinks, float *o, int32_t ntok, int32_t heads,
                                     int32_t kv_heads, int32_t head_dim, int32_t pos, int32_t cap,
                                     int32_t window, const float *scale, void *stream);

/* Greedy choice over rows of fp16 logits (chat/sample.go:80-88: the first largest wins):
 * logits [rows][vocab] fp16 bits, out int32 [rows], device memory. */
HC_API char *hc_argmax_run(const uint16_t *logits, int32_t rows, int32_t vocab, int32_t *out,
                           void *stream);

/* MoE routing (experts.Routing.Choose with Score "softmax" and Norm, experts/weights.go:33-82):
 * logits float32 [rows][n], idx int32 [rows][k], w float32 [rows][k], device memory. */
HC_API char *hc_route_run(const float *logits, int32_t rows, int32_t n, int32_t k, int32_t *idx,
                          float *w, void *stream);

#ifdef __cplusplus
}
#endif

#endif
