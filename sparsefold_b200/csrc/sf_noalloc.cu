// sf_transition_noalloc: the TransitionBlock entry point for callers that
// cannot allocate device memory.
//
// Some callers of this library have no way to obtain scratch memory: code
// running where cudaMalloc is forbidden (inside a region that must not
// synchronise or change the memory map), embedders with a fixed device memory
// budget and no allocator hook, and bindings that cannot hold a workspace
// across calls.  sf_transition needs a caller-provided workspace; this
// variant uses a fixed scratch array inside the library instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (16 MiB).  Every GPU that loads the library reserves it until the process
// exits.  Its device address is looked up once per device, with that device
// current, on the first call made on that device; make that first call before
// any stream capture.  Calls that would need more scratch than the array holds
// are rejected with SF_ERR_WORKSPACE.  All calls share the one array: two
// calls whose kernels overlap on the GPU (different streams, or different host
// threads) race on it and must be serialised by the caller.  The array keeps
// whatever the previous call left; the transition kernels overwrite every
// scratch element they read, so nothing needs clearing between calls.
#include <mutex>

#include "sf_common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

static __device__ __align__(256) unsigned char g_transition_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {nullptr};

// Device address of g_transition_scratch on the current device.  In host code
// the symbol itself is only a host-side stand-in, never a device address.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    sf::set_error("sf_transition_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return SF_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) {
    sf::set_error("sf_transition_noalloc: device index %d out of range", dev);
    return SF_ERR_ARG;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_transition_scratch);
    if (e != cudaSuccess || !p) {
      sf::set_error("sf_transition_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return SF_OK;
}

}  // namespace

extern "C" {

size_t sf_transition_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

int sf_transition_noalloc(int dtype, const void* x, const float* ln_w, const float* ln_b, const void* w1,
                          const void* w2, void* y, int64_t rows, int64_t c, int64_t inter, sf_stream_t stream) {
  const size_t need = sf_transition_workspace(dtype, rows, inter);
  if (need > kNoAllocScratchBytes) {
    sf::set_error("sf_transition_noalloc: rows=%lld x inter=%lld needs %zu bytes of scratch, above the fixed %zu",
                  (long long)rows, (long long)inter, need, kNoAllocScratchBytes);
    return SF_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  SF_TRY(scratch_address(&scratch));
  return sf_transition(dtype, x, ln_w, ln_b, w1, w2, y, rows, c, inter, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
