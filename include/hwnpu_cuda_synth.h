/*
 * hwnpu_cuda_synth.h: seeded synthetic inputs for tests and benchmarks, exported by
 * libhwnpu_cuda.so beside the product ABI of hwnpu_cuda.h but not part of it: a Go binding of the
 * engine (internal/backend/cuda) binds only hwnpu_cuda.h. They stand in for the reference's
 * synthetic checkpoint (llm.NewSynthetic, internal/llm/synth.go:10-36), whose values are uniform,
 * with the normal draws the benchmark configurations ask for. The oracle (oracle/synth.cpp) has
 * its own copy of the same generator, so that CPU runs never map this library.
 *
 * Conventions as in hwnpu_cuda.h: NULL or a heap error string freed by hc_free_error; no float by
 * value.
 */
#ifndef HWNPU_CUDA_SYNTH_H
#define HWNPU_CUDA_SYNTH_H

#include "hwnpu_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* n values drawn N(0, (*std)^2), seeded by (seed, name): PCG32 (XSH RR) streams of 2^20 values
 * each, two 32-bit draws a pair of values by Box-Muller in float64, so the values do not depend
 * on the thread count. */
HC_API char *hc_synth_normal(uint64_t seed, const char *name, const float *std, float *out, uint64_t n);
/* n token ids uniform on [0, vocab) from seed. */
HC_API char *hc_synth_tokens(uint64_t seed, int32_t vocab, int32_t *out, uint64_t n);

#ifdef __cplusplus
}
#endif

#endif
