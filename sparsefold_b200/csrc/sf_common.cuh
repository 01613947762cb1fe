// Shared helpers of the sparsefold_b200 kernels: element access, error state,
// launch accounting.  Host-side errors are reported through a thread-local
// message read by sf_last_error(); no C++ exception crosses the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "../../include/sparsefold_b200.h"

namespace sf {

using bf16 = __nv_bfloat16;

// ---- element access (fp32 arithmetic everywhere) ---------------------------
__device__ __forceinline__ float ld(const float* p) { return *p; }
__device__ __forceinline__ float ld(const bf16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st(float* p, float v) { *p = v; }
__device__ __forceinline__ void st(bf16* p, float v) { *p = __float2bfloat16_rn(v); }

// Round a value to the precision of storage type T (identity for fp32).
template <typename T>
__device__ __forceinline__ float ld_round(float v) { return v; }
template <>
__device__ __forceinline__ float ld_round<bf16>(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float swish_f(float x) { return x * sigmoid_f(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- host-side error state --------------------------------------------------
void set_error(const char* fmt, ...);
void count_launch(uint64_t n = 1);
int check_launch(const char* what);  // cudaGetLastError -> status
// Device address of the library's status word on the current device (0 = ok;
// a kernel whose bounded wait gave up stores SF_ERR_TIMEOUT).  nullptr on error.
uint32_t* device_status_ptr();

// Launch with programmatic stream serialisation, so that the kernel's set-up overlaps the tail of
// the kernel before it (the kernel itself waits with tc::griddep_wait() before touching any
// activation); SF_PDL=0 in the environment launches plainly.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// tcgen05 kernels (bf16 track), host launchers defined in sf_*_tc.cu.
int num_sms();
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encoder();
int make_pair_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t n, bool column_tile);
size_t triatt_tc_workspace(int64_t n);
int64_t triatt_query_pitch(int64_t nq);
int triatt_bias_tc(const bf16* z, int64_t rows, int64_t n, const float* ln_w, const bf16* w_bias, bf16* bias,
                   int64_t ldb, cudaStream_t stream);
int triatt_project_tc(const bf16* z, int64_t rows, int64_t cols, int transpose, int compute_bias, const float* ln_w,
                      const bf16* w_qkvg, const bf16* w_bias, bf16* q, bf16* k, bf16* vt, bf16* g, bf16* bias,
                      cudaStream_t stream);
int triatt_core_tc(const bf16* q, const bf16* k, const bf16* vt, const bf16* g, const bf16* bias, const bf16* w_out,
                   const uint8_t* mask, const bf16* z, bf16* z_out, int64_t rows, int64_t cols, int transpose,
                   int64_t batch_offset, cudaStream_t stream);
int contract_chunked_tc(const bf16* a_op, int64_t chunks_a, const bf16* b_op, int64_t chunks_b, bf16* P,
                        int64_t channels, int64_t rows, int64_t cols, int64_t kdim, cudaStream_t stream);
int triatt_tc(const bf16* z, const uint8_t* mask, int64_t n, int transpose, const float* ln_w, const bf16* w_qkvg,
              const bf16* w_bias, const bf16* w_out, bf16* z_out, void* ws_p, size_t ws_bytes, cudaStream_t stream);
int make_2d_tmap(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, uint32_t box_inner,
                 uint32_t box_outer, int swizzle_bytes = 128);
int pair_logits_tc(const bf16* z, const float* ln_w, const float* ln_b, const bf16* w, bf16* logits, int64_t M,
                   int heads, cudaStream_t stream);
int pair_rows_bias_tc(const bf16* z, int64_t rows, int64_t n, const float* ln_w, const bf16* w, int heads, float scale,
                      bf16* bias, int64_t ldb, cudaStream_t stream);
int transition_tc(const bf16* x, const float* ln_w, const float* ln_b, const bf16* w1, const bf16* w2, bf16* y,
                  int64_t M, cudaStream_t stream);
int trimul_output_tc(const bf16* z, const bf16* P, int64_t rows, int64_t n, const float* ln_w, const float* ln_b,
                     const float* center_w, const float* center_b, const bf16* w_gate, const bf16* w_out, bf16* z_out,
                     cudaStream_t stream);
int linear_tc(const bf16* x, const bf16* wt, const float* bias, const bf16* residual, bf16* y, int64_t M, int64_t K,
              int64_t N, int post_op, cudaStream_t stream);
int contract_tc(const bf16* a_op, const bf16* b_op, bf16* P, int64_t channels, int64_t rows, int64_t cols,
                int64_t kdim, cudaStream_t stream);
// Generic pair-biased gated attention on tcgen05 (bf16, head dim <= 64, a multiple of 8);
// SF_ERR_ARG without a message when the call is outside what it takes.
int attention_tc(const sf_attention_args* a, cudaStream_t stream);
int trimul_project_tc(const bf16* z, const uint8_t* mask, int64_t rows, int64_t n, int64_t row_offset, int incoming,
                      const float* ln_w, const float* ln_b, const bf16* w_glu, bf16* a_op, bf16* b_op,
                      cudaStream_t stream);

// Row pitch (elements) of the channel-major triangle-multiplication buffers:
// rows are padded to a multiple of 8 elements so every row starts 16-byte aligned.
__host__ __device__ inline int64_t pair_pitch(int64_t n) { return (n + 7) / 8 * 8; }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Carves aligned sub-buffers out of a caller-provided workspace.
struct Workspace {
  char* base;
  size_t size, used = 0;
  Workspace(void* p, size_t n) : base(static_cast<char*>(p)), size(n) {}
  template <typename T>
  T* take(size_t count) {
    size_t off = align_up(used, 256);
    used = off + count * sizeof(T);
    return used <= size ? reinterpret_cast<T*>(base + off) : nullptr;
  }
  bool ok() const { return used <= size; }
};

// Workspace size accounting that mirrors Workspace::take.
struct WorkspaceSize {
  size_t used = 0;
  template <typename T>
  void take(size_t count) { used = align_up(used, 256) + count * sizeof(T); }
};

}  // namespace sf

#define SF_REQUIRE(cond, ...)           \
  do {                                  \
    if (!(cond)) {                      \
      ::sf::set_error(__VA_ARGS__);     \
      return SF_ERR_ARG;                \
    }                                   \
  } while (0)

#define SF_TRY(expr)                    \
  do {                                  \
    int _st = (expr);                   \
    if (_st != SF_OK) return _st;       \
  } while (0)

// Dispatch on the activation dtype: defines `T` inside the body.
#define SF_DISPATCH(dtype, ...)                                         \
  do {                                                                  \
    if ((dtype) == SF_F32) {                                            \
      using T = float;                                                  \
      __VA_ARGS__                                                       \
    } else if ((dtype) == SF_BF16) {                                    \
      using T = ::sf::bf16;                                             \
      __VA_ARGS__                                                       \
    } else {                                                            \
      ::sf::set_error("unsupported dtype %d", (int)(dtype));            \
      return SF_ERR_ARG;                                                \
    }                                                                   \
  } while (0)
