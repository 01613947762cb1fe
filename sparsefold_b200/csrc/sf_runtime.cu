// Runtime plumbing of the C ABI: per-thread error messages, launch accounting,
// device check, version.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "sf_common.cuh"

namespace sf {

static thread_local char g_err[1024] = {0};
static std::atomic<uint64_t> g_launches{0};
// One status word per device that loads the library; kernels with bounded
// waits record a timeout here instead of hanging.
static __device__ uint32_t g_device_status;
static uint32_t* g_status_ptr[64] = {nullptr};
static std::mutex g_status_mu;

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("SF_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return SF_ERR_CUDA;
  }
  return SF_OK;
}

uint32_t* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_device_status);
    if (e != cudaSuccess) {
      set_error("cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
      return nullptr;
    }
    g_status_ptr[dev] = static_cast<uint32_t*>(p);
  }
  return g_status_ptr[dev];
}

}  // namespace sf

extern "C" {

const char* sf_version(void) { return "sparsefold_b200 0.1 (sm_100a)"; }

int sf_last_error(char* buf, size_t len) {
  size_t n = strlen(sf::g_err);
  if (buf && len) {
    size_t c = n < len - 1 ? n : len - 1;
    memcpy(buf, sf::g_err, c);
    buf[c] = 0;
  }
  return (int)n;
}

uint64_t sf_launch_count(void) { return sf::g_launches.load(); }

int sf_device_status(uint32_t* out, int clear) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, sf::g_device_status, sizeof(v));
  if (e == cudaSuccess && clear) {
    uint32_t z = 0;
    e = cudaMemcpyToSymbol(sf::g_device_status, &z, sizeof(z));
  }
  if (e != cudaSuccess) {
    sf::set_error("sf_device_status: %s", cudaGetErrorString(e));
    return SF_ERR_CUDA;
  }
  if (out) *out = v;
  return SF_OK;
}

int sf_device_check(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    sf::set_error("cudaGetDevice: %s", cudaGetErrorString(e));
    return SF_ERR_CUDA;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    sf::set_error("device %d is sm_%d%d; this library is built for sm_100a only", dev, major, minor);
    return SF_ERR_DEVICE;
  }
  return SF_OK;
}

}  // extern "C"
