// Peer exchanges over NVLink between the ranks of one box (one process per GPU): the
// receive buffers of every rank are mapped into its peers with CUDA IPC, a rank writes
// its blocks straight into the peers' buffers with 16-byte stores from the SMs (or the
// copy engines), and a flag word per (receiver, sender) tells the receiver the data is
// there.  Every wait is bounded.  This is the all-to-all / all-gather of the row-sharded
// path (runtime/dist.py:477-565) without a collective library in between.
//
//  k_scatter_peers  block q of the source (q = 0 .. n-1) -> dsts[q] + dst_offset, 16-byte
//                   chunks, grid-strided over all blocks; dsts are local or peer pointers.
//  k_peer_signal    after everything earlier on the stream: flag = value on a peer
//                   (system-scope release store).
//  k_peer_wait      one warp: lane q waits (bounded) until flags[q] >= value for every
//                   q != self (system-scope acquire loads); on timeout it records
//                   SF_ERR_TIMEOUT in the status word and returns.
#include <cuda.h>
#include <mutex>
#include <string.h>

#include "sf_common.cuh"

namespace sf {
namespace {

// Each thread moves SP_UNROLL chunks per step (their loads issued before any store), so
// enough stores are in flight to keep the NVLink of every peer busy.
constexpr int SP_UNROLL = 4;
__global__ void k_scatter_peers(const uint4* __restrict__ src, uint4* const* __restrict__ dsts, int n, int64_t chunks,
                                int64_t src_stride, int64_t dst_offset) {
  const int64_t total = (int64_t)n * chunks;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e0 < total; e0 += step * SP_UNROLL) {
    uint4 v[SP_UNROLL];
#pragma unroll
    for (int u = 0; u < SP_UNROLL; ++u) {
      const int64_t e = e0 + u * step;
      if (e < total) {
        const int64_t q = e / chunks, c = e - q * chunks;
        v[u] = __ldg(src + q * src_stride + c);
      }
    }
#pragma unroll
    for (int u = 0; u < SP_UNROLL; ++u) {
      const int64_t e = e0 + u * step;
      if (e < total) {
        const int64_t q = e / chunks, c = e - q * chunks;
        dsts[q][dst_offset + c] = v[u];
      }
    }
  }
}

__global__ void k_peer_signal(uint32_t* flag, uint32_t value) {
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
}

__global__ void k_peer_wait(const uint32_t* flags, int n, int self, uint32_t value, uint32_t polls, uint32_t* status) {
  const int q = threadIdx.x;
  if (q >= n || q == self) return;
  for (uint32_t i = 0; i < polls; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + q) : "memory");
    if ((int32_t)(v - value) >= 0) return;
    __nanosleep(256);
  }
  if (status) atomicCAS(status, 0u, (uint32_t)SF_ERR_TIMEOUT);
}

struct Mapping {
  unsigned char handle[CUDA_IPC_HANDLE_SIZE];
  int device;
  void* base;
};
std::mutex g_ipc_mu;
Mapping g_maps[256];
int g_nmaps = 0;

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

int sf_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  SF_REQUIRE(ptr && handle && offset, "sf_ipc_export: null argument");
  CUdeviceptr base = 0;
  size_t size = 0;
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  GetRange get_range = nullptr;
  {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      set_error("sf_ipc_export: cuMemGetAddressRange unavailable");
      return SF_ERR_CUDA;
    }
    get_range = reinterpret_cast<GetRange>(fn);
  }
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("sf_ipc_export: %p is not a device allocation", ptr);
    return SF_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    set_error("cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return SF_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  *offset = (uint64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return SF_OK;
}

int sf_ipc_import(const void* handle, uint64_t offset, void** ptr) {
  SF_REQUIRE(handle && ptr, "sf_ipc_import: null argument");
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  for (int i = 0; i < g_nmaps; ++i)
    if (g_maps[i].device == dev && memcmp(g_maps[i].handle, handle, CUDA_IPC_HANDLE_SIZE) == 0) {
      *ptr = static_cast<char*>(g_maps[i].base) + offset;
      return SF_OK;
    }
  SF_REQUIRE(g_nmaps < 256, "sf_ipc_import: too many mappings");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return SF_ERR_CUDA;
  }
  Mapping& m = g_maps[g_nmaps++];
  memcpy(m.handle, handle, CUDA_IPC_HANDLE_SIZE);
  m.device = dev;
  m.base = base;
  *ptr = static_cast<char*>(base) + offset;
  return SF_OK;
}

int sf_ipc_close_all(void) {
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  int rc = SF_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  for (int i = 0; i < g_nmaps; ++i) {
    cudaSetDevice(g_maps[i].device);
    if (cudaIpcCloseMemHandle(g_maps[i].base) != cudaSuccess) rc = SF_ERR_CUDA;
  }
  cudaSetDevice(dev);
  g_nmaps = 0;
  return rc;
}

int sf_scatter_peers(const void* src, void* const* dsts_dev, int32_t n, int64_t block_bytes, int64_t src_stride_bytes,
                     int64_t dst_offset_bytes, sf_stream_t stream) {
  SF_REQUIRE(src && dsts_dev && n > 0 && block_bytes >= 0, "sf_scatter_peers: bad arguments");
  SF_REQUIRE(((reinterpret_cast<uintptr_t>(src) | (uintptr_t)block_bytes | (uintptr_t)src_stride_bytes |
               (uintptr_t)dst_offset_bytes) & 15) == 0,
             "sf_scatter_peers: pointers, sizes and offsets must be multiples of 16 bytes");
  const int64_t chunks = block_bytes / 16;
  if (chunks == 0) return SF_OK;
  const int64_t want = (n * chunks + 255) / 256, cap = (int64_t)num_sms() * 8;
  k_scatter_peers<<<(unsigned)(want < cap ? want : cap), 256, 0, stream>>>(
      static_cast<const uint4*>(src), reinterpret_cast<uint4* const*>(dsts_dev), n, chunks, src_stride_bytes / 16,
      dst_offset_bytes / 16);
  count_launch();
  return check_launch("sf_scatter_peers");
}

int sf_peer_signal(uint32_t* flag, uint32_t value, sf_stream_t stream) {
  SF_REQUIRE(flag && (reinterpret_cast<uintptr_t>(flag) & 3) == 0, "sf_peer_signal: bad flag pointer");
  k_peer_signal<<<1, 1, 0, stream>>>(flag, value);
  count_launch();
  return check_launch("sf_peer_signal");
}

int sf_peer_wait(const uint32_t* flags, int32_t n, int32_t self, uint32_t value, uint32_t polls, sf_stream_t stream) {
  SF_REQUIRE(flags && n > 0 && n <= 32 && self >= 0 && self < n && polls > 0, "sf_peer_wait: bad arguments");
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  k_peer_wait<<<1, 32, 0, stream>>>(flags, n, self, value, polls, status);
  count_launch();
  return check_launch("sf_peer_wait");
}

}  // extern "C"
