// api.cpp: errors, fault injection, devices and buffers of the C ABI (include/hwnpu_cuda.h).
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "kernels.h"

namespace hc {

char *make_error(const std::string &msg) {
  char *p = static_cast<char *>(std::malloc(msg.size() + 1));
  if (!p) return nullptr;
  std::memcpy(p, msg.c_str(), msg.size() + 1);
  return p;
}

namespace {
std::mutex g_fault_mu;
int g_fault_point = -1;  // FaultPoint armed, or -1
long g_fault_left = 0;   // calls of that point before the one that fails
}  // namespace

namespace {
std::atomic<long> g_stall_ms{0};  // "stall:MS": the next step first waits MS ms on the device
}  // namespace

long take_stall_ms() { return g_stall_ms.exchange(0); }

namespace {
}  // namespace


bool fault_fires(FaultPoint p) {
  std::lock_guard<std::mutex> g(g_fault_mu);
  if (g_fault_point != int(p)) return false;
  if (g_fault_left > 1) { --g_fault_left; return false; }
  g_fault_point = -1;
  return true;
}

char *dev_alloc(void **p, size_t n, const char *what) {
  *p = nullptr;
  if (fault_fires(kFaultAlloc)) return make_error(std::string("injected fault: device allocation of ") + what);
  if (n == 0) n = 16;
  cudaError_t e = cudaMalloc(p, n);
  if (e != cudaSuccess) {
    *p = nullptr;
    return make_error(std::string("out of device memory: ") + what + " (" + std::to_string(n) +
                      " bytes): " + cudaGetErrorString(e));
  }
  return nullptr;
}

char *copy_h2d(void *dst, const void *src, size_t n, cudaStream_t st) {
  if (fault_fires(kFaultH2D)) return make_error("injected fault: host-to-device copy");
  if (!n) return nullptr;
  HC_TRY_CUDA(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, st));
  return nullptr;
}

}  // namespace hc

struct hc_device {
  int ordinal;
  cudaDeviceProp prop;
};

struct hc_buf {
  hc_device *d;
  int kind;
  uint64_t size;
  void *dev;   // HC_BUF_DEVICE
  void *host;  // pinned
};

namespace {

// The CUDA ordinals hc_device_count lists: all, or those HWNPU_CUDA_DEVICES names.
char *visible(std::vector<int> *out) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e == cudaErrorNoDevice) { cudaGetLastError(); n = 0; }
  else if (e != cudaSuccess) {
    cudaGetLastError();
    return hc::make_error(std::string("cuda: ") + cudaGetErrorString(e));
  }
  out->clear();
  const char *f = std::getenv("HWNPU_CUDA_DEVICES");
  if (!f || !*f) {
    for (int i = 0; i < n; ++i) out->push_back(i);
    return nullptr;
  }
  std::stringstream ss(f);
  std::string item;
  while (std::getline(ss, item, ',')) {
    if (item.empty()) continue;
    char *end = nullptr;
    long v = std::strtol(item.c_str(), &end, 10);
    if (*end || v < 0) return hc::make_error("HWNPU_CUDA_DEVICES: bad entry " + item);
    if (v < n) out->push_back(int(v));
  }
  return nullptr;
}

}  // namespace

extern "C" {

HC_API int hc_abi(void) { return HC_ABI; }

HC_API void hc_free_error(char *err) { std::free(err); }

HC_API char *hc_set_fault(const char *spec) {
  std::lock_guard<std::mutex> g(hc::g_fault_mu);
  hc::g_fault_point = -1;
  if (!spec || !*spec) return nullptr;
  std::string s(spec);
  auto colon = s.find(':');
  if (colon == std::string::npos) return hc::make_error("hc_set_fault: want point:N");
  std::string point = s.substr(0, colon);
  long n = std::strtol(s.c_str() + colon + 1, nullptr, 10);
  if (n < 1) return hc::make_error("hc_set_fault: N must be at least 1");
  if (point == "stall") {
    if (n > 2000) return hc::make_error("hc_set_fault: a stall is at most 2000 ms");
    hc::g_stall_ms = n;
    return nullptr;
  }
  if (point == "alloc") hc::g_fault_point = hc::kFaultAlloc;
  else if (point == "h2d") hc::g_fault_point = hc::kFaultH2D;
  else if (point == "step") hc::g_fault_point = hc::kFaultStep;
  else return hc::make_error("hc_set_fault: unknown point " + point);
  hc::g_fault_left = n;
  return nullptr;
}

HC_API char *hc_device_count(uint32_t *count) {
  if (!count) return hc::make_error("hc_device_count: NULL count");
  std::vector<int> v;
  if (char *e = visible(&v)) return e;
  *count = uint32_t(v.size());
  return nullptr;
}

HC_API char *hc_device_open(uint32_t index, hc_device **out) {
  if (!out) return hc::make_error("hc_device_open: NULL out");
  *out = nullptr;
  std::vector<int> v;
  if (char *e = visible(&v)) return e;
  if (index >= v.size()) return hc::make_error("hc_device_open: no device " + std::to_string(index));
  auto *d = new hc_device{v[index], {}};
  cudaError_t e = cudaGetDeviceProperties(&d->prop, d->ordinal);
  if (e != cudaSuccess) {
    delete d;
    return hc::make_error(std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e));
  }
  if (d->prop.major < 10) {
    std::string name = d->prop.name;
    delete d;
    return hc::make_error("hc_device_open: " + name + " is not sm_100 (this library has sm_100a code only)");
  }
  *out = d;
  return nullptr;
}

HC_API void hc_device_free(hc_device *d) { delete d; }

HC_API char *hc_device_info(hc_device *d, int key, char *buf, size_t n, size_t *need) {
  if (!d) return hc::make_error("hc_device_info: NULL device");
  std::string v;
  switch (key) {
    case HC_INFO_NAME: v = d->prop.name; break;
    case HC_INFO_PCI_BUS_ID: {
      char b[32];
      std::snprintf(b, sizeof b, "%04x:%02x:%02x.0", d->prop.pciDomainID, d->prop.pciBusID, d->prop.pciDeviceID);
      v = b;
      break;
    }
    case HC_INFO_ARCH: v = "sm_" + std::to_string(d->prop.major) + std::to_string(d->prop.minor); break;
    case HC_INFO_MEMORY: v = std::to_string(d->prop.totalGlobalMem); break;
    case HC_INFO_SMS: v = std::to_string(d->prop.multiProcessorCount); break;
    case HC_INFO_DRIVER: {
      int dv = 0;
      cudaDriverGetVersion(&dv);
      v = std::to_string(dv);
      break;
    }
    default: return hc::make_error("hc_device_info: unknown key " + std::to_string(key));
  }
  if (need) *need = v.size() + 1;
  if (buf && n) {
    size_t k = std::min(n - 1, v.size());
    std::memcpy(buf, v.data(), k);
    buf[k] = 0;
  }
  return nullptr;
}

HC_API char *hc_device_check(hc_device *d) {
  if (!d) return hc::make_error("hc_device_check: NULL device");
  HC_TRY_CUDA(cudaSetDevice(d->ordinal));
  HC_TRY_CUDA(cudaDeviceSynchronize());
  const int code = hc::tc_status_take();
  if (code) return hc::make_error("a tensor-core GEMV wait ran out (code " + std::to_string(code) + ")");
  return nullptr;
}

HC_API char *hc_buf_alloc(hc_device *d, uint64_t size, int kind, hc_buf **out) {
  if (!d || !out) return hc::make_error("hc_buf_alloc: NULL argument");
  if (kind != HC_BUF_DEVICE && kind != HC_BUF_HOST) return hc::make_error("hc_buf_alloc: unknown kind");
  *out = nullptr;
  HC_TRY_CUDA(cudaSetDevice(d->ordinal));
  auto *b = new hc_buf{d, kind, size, nullptr, nullptr};
  if (hc::fault_fires(hc::kFaultAlloc)) { delete b; return hc::make_error("injected fault: buffer allocation"); }
  cudaError_t e = cudaHostAlloc(&b->host, size ? size : 1, cudaHostAllocPortable);
  if (e != cudaSuccess) { delete b; return hc::make_error(std::string("cudaHostAlloc: ") + cudaGetErrorString(e)); }
  if (kind == HC_BUF_DEVICE) {
    if (char *err = hc::dev_alloc(&b->dev, size, "buffer")) {
      cudaFreeHost(b->host);
      delete b;
      return err;
    }
  }
  *out = b;
  return nullptr;
}

HC_API void hc_buf_free(hc_buf *b) {
  if (!b) return;
  cudaSetDevice(b->d->ordinal);
  if (b->dev) cudaFree(b->dev);
  if (b->host) cudaFreeHost(b->host);
  delete b;
}

HC_API char *hc_buf_map(hc_buf *b, void **ptr) {
  if (!b || !ptr) return hc::make_error("hc_buf_map: NULL argument");
  *ptr = b->host;
  return nullptr;
}

HC_API uint64_t hc_buf_address(hc_buf *b) {
  if (!b) return 0;
  if (b->dev) return reinterpret_cast<uint64_t>(b->dev);
  void *p = nullptr;
  if (cudaHostGetDevicePointer(&p, b->host, 0) != cudaSuccess) { cudaGetLastError(); return 0; }
  return reinterpret_cast<uint64_t>(p);
}

HC_API char *hc_buf_sync(hc_buf *b, int dir, uint64_t off, uint64_t n) {
  if (!b) return hc::make_error("hc_buf_sync: NULL buffer");
  if (off > b->size || n > b->size - off) return hc::make_error("hc_buf_sync: range out of the buffer");
  if (b->kind == HC_BUF_HOST || n == 0) return nullptr;
  HC_TRY_CUDA(cudaSetDevice(b->d->ordinal));
  char *base = static_cast<char *>(b->dev) + off;
  char *host = static_cast<char *>(b->host) + off;
  if (dir == HC_SYNC_TO_DEVICE) {
    if (char *e = hc::copy_h2d(base, host, n, nullptr)) return e;
    HC_TRY_CUDA(cudaStreamSynchronize(nullptr));
  } else if (dir == HC_SYNC_FROM_DEVICE) {
    HC_TRY_CUDA(cudaMemcpy(host, base, n, cudaMemcpyDeviceToHost));
  } else {
    return hc::make_error("hc_buf_sync: unknown direction");
  }
  return nullptr;
}

}  // extern "C"

// Used by the engine to make a device current.
namespace hc {
int device_ordinal(const hc_device *d) { return d->ordinal; }
int device_sms(const hc_device *d) { return d->prop.multiProcessorCount; }
}  // namespace hc
