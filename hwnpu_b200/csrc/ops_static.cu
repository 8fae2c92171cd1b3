// ops_static.cu: hc_attention_run_static, the decode attention entry point that allocates nothing.
//
// Its scratch (the step tokens, the per-split partials and the activation tiles the merge kernel
// also writes) lives in one file-scope __device__ array of kStaticScratchBytes, instead of the
// cudaMalloc'd temporaries of hc_attention_run. The array is one per device for the whole process:
// every call overwrites it and it keeps the last call's contents; nothing in it has to start at
// zero, since each call writes every part it reads (every split writes its partials, empty ones
// included). Two calls in flight at once on one device (other streams, other threads) use the
// same bytes and race.
#include <mutex>
#include <string>

#include "kernels.h"

namespace hc {
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB
constexpr int kStaticSplits = 16;                        // as hc_attention_run
constexpr int kStaticMaxDevices = 64;

__device__ __align__(256) uint8_t g_attn_scratch[kStaticScratchBytes];

// The array's address on each device, looked up once with that device current.
std::mutex g_mu;
void *g_addr[kStaticMaxDevices] = {};

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

__global__ void fill_toks_kernel(StepTok *toks, int ntok, int pos) {
  for (int t = threadIdx.x; t < ntok; t += blockDim.x) toks[t] = StepTok{0, 0, pos + t, 0};
}

}  // namespace
}  // namespace hc

extern "C" {

HC_API char *hc_attention_run_static(const float *q, const uint16_t *kcache, const uint16_t *vcache,
                                     const float *sinks, float *o, int32_t ntok, int32_t heads,
                                     int32_t kv_heads, int32_t head_dim, int32_t pos, int32_t cap,
                                     int32_t window, const float *scale, void *stream) {
  if (!q || !kcache || !vcache || !o || !scale) return hc::make_error("hc_attention_run_static: NULL argument");
  if (ntok < 1 || heads < 1 || kv_heads < 1 || heads % kv_heads)
    return hc::make_error("hc_attention_run_static: bad heads");
  const int rep = heads / kv_heads;
  if (head_dim != 64 && head_dim != 128) return hc::make_error("hc_attention_run_static: head_dim must be 64 or 128");
  if (rep != 1 && rep != 2 && rep != 4 && rep != 8)
    return hc::make_error("hc_attention_run_static: heads per kv head must be 1, 2, 4 or 8");
  if (pos < 0 || cap < 1) return hc::make_error("hc_attention_run_static: bad positions");
  if (pos + ntok > cap && !(window > 0 && cap >= window + ntok - 1))
    return hc::make_error("hc_attention_run_static: positions beyond the cache (a ring needs window > 0 and cap >= window + ntok - 1)");
  // the scratch this call needs, each part on a 256-byte boundary
  const int splits = hc::kStaticSplits;
  const int ktiles = (heads * head_dim + hc::kTileCols - 1) / hc::kTileCols;
  const size_t b_toks = hc::up256(sizeof(hc::StepTok) * size_t(ntok));
  const size_t b_ml = hc::up256(sizeof(float) * size_t(ntok) * heads * splits * 2);
  const size_t b_po = hc::up256(sizeof(float) * size_t(ntok) * heads * splits * head_dim);
  const size_t b_act = hc::up256(size_t(ntok) * ktiles * hc::kActTile);
  const size_t need = b_toks + b_ml + b_po + b_act;
  if (need > hc::kStaticScratchBytes)
    return hc::make_error("hc_attention_run_static: ntok " + std::to_string(ntok) + " x heads " +
                          std::to_string(heads) + " x head_dim " + std::to_string(head_dim) + " needs " +
                          std::to_string(need) + " bytes of scratch, above the static limit of " +
                          std::to_string(hc::kStaticScratchBytes));
  int dev = -1;
  HC_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= hc::kStaticMaxDevices)
    return hc::make_error("hc_attention_run_static: device ordinal " + std::to_string(dev) + " beyond " +
                          std::to_string(hc::kStaticMaxDevices));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Outside a stream capture the address is looked up on every call (a device reset or a new
  // primary context moves the array); inside one, the address of the last call outside it is used.
  cudaStreamCaptureStatus cap_status = cudaStreamCaptureStatusNone;
  HC_TRY_CUDA(cudaStreamIsCapturing(st, &cap_status));
  uint8_t *base = nullptr;
  {
    std::lock_guard<std::mutex> lk(hc::g_mu);
    if (cap_status == cudaStreamCaptureStatusNone) {
      void *a = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&a, hc::g_attn_scratch);
      if (e != cudaSuccess)
        return hc::make_error(std::string("hc_attention_run_static: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      hc::g_addr[dev] = a;
    } else if (!hc::g_addr[dev]) {
      return hc::make_error("hc_attention_run_static: the first call on a device must come before any stream capture");
    }
    base = static_cast<uint8_t *>(hc::g_addr[dev]);
  }
  auto *dt = reinterpret_cast<hc::StepTok *>(base);
  auto *ml = reinterpret_cast<float *>(base + b_toks);
  auto *po = reinterpret_cast<float *>(base + b_toks + b_ml);
  uint8_t *act = base + b_toks + b_ml + b_po;
  hc::fill_toks_kernel<<<1, 32, 0, st>>>(dt, ntok, pos);
  hc::AttnGeom g{heads, kv_heads, head_dim, cap, window, *scale};
  hc::attn_split(q, dt, ntok, g, kcache, vcache, splits, ml, po, st);
  hc::attn_merge_quant(ml, po, sinks, ntok, heads, head_dim, splits, act, ktiles, o, st);
  HC_TRY_CUDA(cudaGetLastError());
  return nullptr;
}

}  // extern "C"
