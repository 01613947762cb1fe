// Runtime plumbing of the C ABI: per-thread error messages, launch accounting,
// device check, version.
#include <cstring>

#include "sf_common.cuh"

namespace sf {

static thread_local char g_err[1024] = {0};
static std::atomic<uint64_t> g_launches{0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return SF_ERR_CUDA;
  }
  return SF_OK;
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
