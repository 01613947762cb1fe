// Embedding-side pair kernels of the trunk (Evoformer, trunk/network.py:195-285):
//
//  k_pair_outer_sum      out[i][j][:] = left[i][:] + right[j][:] (+ addend[i][j][:]),
//                        the sequence pair embedding left_single(t)[:, None] +
//                        right_single(t)[None, :] (network.py:195-212), 16-byte
//                        vectors, one pass over the N x N x C output.
//  k_pair_sparse_linear  out[p][:] = sum_k x[p][k] w[k][:] (+ residual[p][:]) over the
//                        nonzero x[p][k] only: the relative-position encoding (139
//                        one-hot features, network.py:188-193) and the bond contact
//                        map (one 0/1 feature, network.py:214-256) are linear layers
//                        on inputs with a handful of nonzeros per position, so a warp
//                        reads the row once, finds its nonzeros with a ballot and sums
//                        those rows of w from shared memory.  Terms are added in
//                        increasing k in fp32 and rounded once; a zero x skips its term
//                        (0 * w is taken as 0 even where w is infinite).
// Both are HBM-bound: bytes per position = read x (k elements) + write C elements.
#include "sf_pair_tc.cuh"
#include "sf_simt.cuh"

namespace sf {
namespace {

using pt::bf_hi;
using pt::bf_lo;
using pt::pack_bf2;

template <typename T>
struct Vec16;   // 16 bytes of T as fp32 lanes
template <>
struct Vec16<float> {
  static constexpr int n = 4;
  __device__ static void load(const float* p, float (&v)[4]) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
  }
  __device__ static void store(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <>
struct Vec16<bf16> {
  static constexpr int n = 8;
  __device__ static void load(const bf16* p, float (&v)[8]) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = bf_lo(w[i]);
      v[2 * i + 1] = bf_hi(w[i]);
    }
  }
  __device__ static void store(bf16* p, const float (&v)[8]) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf2(v[0], v[1]), pack_bf2(v[2], v[3]), pack_bf2(v[4], v[5]),
                                              pack_bf2(v[6], v[7]));
  }
};

// One 16-byte output vector per thread per step; channels % Vec16<T>::n == 0.
template <typename T>
__global__ void k_pair_outer_sum(const T* __restrict__ left, const T* __restrict__ right, const T* addend,
                                 T* out, int64_t rows, int64_t cols, int64_t channels) {
  constexpr int V = Vec16<T>::n;
  const int64_t cpv = channels / V, total = rows * cols * cpv;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = e / cpv, cv = e - pos * cpv, i = pos / cols, j = pos - i * cols;
    float a[V], b[V];
    Vec16<T>::load(left + i * channels + cv * V, a);
    Vec16<T>::load(right + j * channels + cv * V, b);
#pragma unroll
    for (int t = 0; t < V; ++t) a[t] += b[t];
    if (addend) {
      Vec16<T>::load(addend + pos * channels + cv * V, b);
#pragma unroll
      for (int t = 0; t < V; ++t) a[t] += b[t];
    }
    Vec16<T>::store(out + pos * channels + cv * V, a);
  }
}

// Any channel count and alignment: one element per thread per step.
template <typename T>
__global__ void k_pair_outer_sum_scalar(const T* __restrict__ left, const T* __restrict__ right,
                                        const T* addend, T* out, int64_t rows, int64_t cols,
                                        int64_t channels) {
  const int64_t total = rows * cols * channels;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = e / channels, c = e - pos * channels, i = pos / cols, j = pos - i * cols;
    float v = ld(left + i * channels + c) + ld(right + j * channels + c);
    if (addend) v += ld(addend + e);
    st(out + e, v);
  }
}

constexpr int SL_WARPS = 16;
constexpr int SL_CHUNKS = 4;   // 32-feature chunks of a row requested together
constexpr int SL_ROWS = 2;     // positions per warp and round

// A warp takes SL_ROWS positions at a time; lane l owns channels l*CPL .. l*CPL+CPL-1
// (channels = 32 * CPL).  The features of both rows are requested SL_CHUNKS chunks at a time
// before any is used, so a round costs one memory round trip for up to 2 x 128 features.
// w_g is w [k][channels] fp32 in global memory; it is staged in shared memory when `staged`
// (k * channels * 4 bytes).
template <typename T, int CPL>
__global__ void __launch_bounds__(SL_WARPS * 32) k_pair_sparse_linear(const T* __restrict__ x, const float* __restrict__ w_g,
                                                                      const T* residual, T* out, int64_t positions, int k,
                                                                      bool staged) {
  extern __shared__ float w_s[];
  constexpr int C = 32 * CPL;
  if (staged) {
    for (int e = threadIdx.x; e < k * C; e += blockDim.x) w_s[e] = __ldg(w_g + e);
    __syncthreads();
  }
  const float* w = staged ? w_s : w_g;
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t)blockIdx.x * SL_WARPS + threadIdx.x / 32, nwarps = (int64_t)gridDim.x * SL_WARPS;
  for (int64_t p0 = warp0 * SL_ROWS; p0 < positions; p0 += nwarps * SL_ROWS) {
    float acc[SL_ROWS][CPL], r[SL_ROWS][CPL];
#pragma unroll
    for (int rr = 0; rr < SL_ROWS; ++rr) {
      const int64_t p = p0 + rr;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        acc[rr][c] = 0.f;
        r[rr][c] = residual && p < positions ? ld(residual + p * C + lane * CPL + c) : 0.f;
      }
    }
    for (int k0 = 0; k0 < k; k0 += 32 * SL_CHUNKS) {
      float v[SL_ROWS][SL_CHUNKS];
#pragma unroll
      for (int rr = 0; rr < SL_ROWS; ++rr)
#pragma unroll
        for (int q = 0; q < SL_CHUNKS; ++q) {
          const int kk = k0 + 32 * q + lane;
          v[rr][q] = kk < k && p0 + rr < positions ? ld(x + (p0 + rr) * k + kk) : 0.f;
        }
#pragma unroll
      for (int rr = 0; rr < SL_ROWS; ++rr)
#pragma unroll
        for (int q = 0; q < SL_CHUNKS; ++q) {
          uint32_t nz = __ballot_sync(0xffffffffu, v[rr][q] != 0.f);   // NaN counts as nonzero
          while (nz) {
            const int b = __ffs(nz) - 1;
            nz &= nz - 1;
            const float xv = __shfl_sync(0xffffffffu, v[rr][q], b);
            const float* wr = w + (int64_t)(k0 + 32 * q + b) * C + lane * CPL;
#pragma unroll
            for (int c = 0; c < CPL; ++c) acc[rr][c] = fmaf(xv, wr[c], acc[rr][c]);
          }
        }
    }
#pragma unroll
    for (int rr = 0; rr < SL_ROWS; ++rr) {
      if (p0 + rr >= positions) break;
      T* o = out + (p0 + rr) * C + lane * CPL;
#pragma unroll
      for (int c = 0; c < CPL; ++c) st(o + c, acc[rr][c] + r[rr][c]);
    }
  }
}

template <typename T, int CPL>
int launch_sparse_linear(const T* x, const float* w, const T* residual, T* out, int64_t positions, int k,
                         cudaStream_t stream) {
  static bool attr[64] = {false};
  const size_t wbytes = (size_t)k * 32 * CPL * sizeof(float);
  const bool staged = wbytes <= 200 * 1024;
  int dev = 0;
  cudaGetDevice(&dev);
  if (staged && !attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(k_pair_sparse_linear<T, CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    attr[dev & 63] = true;
  }
  const int64_t want = (positions + SL_WARPS * SL_ROWS - 1) / (SL_WARPS * SL_ROWS);
  const int64_t cap = (int64_t)num_sms() * (staged ? 3 : 4);
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  k_pair_sparse_linear<T, CPL><<<grid, SL_WARPS * 32, staged ? wbytes : 0, stream>>>(x, w, residual, out, positions, k,
                                                                                   staged);
  count_launch();
  return check_launch("sf_pair_sparse_linear");
}

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

int sf_pair_outer_sum(int dtype, const void* left, const void* right, const void* addend, void* out, int64_t rows,
                      int64_t cols, int64_t channels, sf_stream_t stream) {
  SF_REQUIRE(left && right && out && rows >= 0 && cols >= 0 && channels > 0, "sf_pair_outer_sum: bad arguments");
  const int64_t total = rows * cols * channels;
  if (total == 0) return SF_OK;
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(left) | reinterpret_cast<uintptr_t>(right) |
                         reinterpret_cast<uintptr_t>(addend) | reinterpret_cast<uintptr_t>(out);
  SF_DISPATCH(dtype, {
    constexpr int V = Vec16<T>::n;
    const bool vec = (ptrs & 15) == 0 && channels % V == 0;
    const int64_t work = vec ? total / V : total;
    const int64_t want = (work + 255) / 256, cap = (int64_t)num_sms() * 16;
    const unsigned grid = (unsigned)(want < cap ? want : cap);
    if (vec)
      k_pair_outer_sum<T><<<grid, 256, 0, stream>>>((const T*)left, (const T*)right, (const T*)addend, (T*)out, rows,
                                                    cols, channels);
    else
      k_pair_outer_sum_scalar<T><<<grid, 256, 0, stream>>>((const T*)left, (const T*)right, (const T*)addend, (T*)out,
                                                           rows, cols, channels);
    count_launch();
    return check_launch("sf_pair_outer_sum");
  });
}

int sf_pair_sparse_linear(int dtype, const void* x, const float* w, const void* residual, void* out,
                          int64_t positions, int64_t k, int64_t channels, sf_stream_t stream) {
  SF_REQUIRE(x && w && out && positions >= 0 && k > 0 && k <= (1 << 20), "sf_pair_sparse_linear: bad arguments");
  SF_REQUIRE(channels == 32 || channels == 64 || channels == 128 || channels == 256,
             "sf_pair_sparse_linear: channels must be 32, 64, 128 or 256 (got %lld)", (long long)channels);
  if (positions == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    switch (channels) {
      case 32:
        return launch_sparse_linear<T, 1>((const T*)x, w, (const T*)residual, (T*)out, positions, (int)k, stream);
      case 64:
        return launch_sparse_linear<T, 2>((const T*)x, w, (const T*)residual, (T*)out, positions, (int)k, stream);
      case 128:
        return launch_sparse_linear<T, 4>((const T*)x, w, (const T*)residual, (T*)out, positions, (int)k, stream);
      default:
        return launch_sparse_linear<T, 8>((const T*)x, w, (const T*)residual, (T*)out, positions, (int)k, stream);
    }
  });
}

}  // extern "C"
