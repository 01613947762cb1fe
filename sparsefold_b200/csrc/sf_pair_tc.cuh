// Shared pieces of the tcgen05 pair-tile kernels: tensor maps over the pair
// tensor, in-place LayerNorm of a 128-position tile held in the 128B-swizzled
// K-major layout, resident weight loading, bf16 pack/unpack.
#pragma once

#include "sf_tc.cuh"

namespace sf {
namespace pt {

constexpr int C = 128;               // pair channels
constexpr int TILE = 128;            // positions per tile (= UMMA M)
constexpr int ATOM = TILE * 128;     // bytes of one 64-channel atom column of a tile (16 KB)
constexpr int A_BYTES = 2 * ATOM;    // one 128 x 128 bf16 tile (32 KB)

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float fast_sigmoid(float x) { return __frcp_rn(1.0f + __expf(-x)); }
// sigmoid(x) = (1 + tanh(x/2)) / 2 with the single-instruction tanh approximation
// (absolute error ~1e-3 of the hardware tanh, below bf16 resolution of the results).
__device__ __forceinline__ float sigmoid_tanh(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
  return fmaf(0.5f, t, 0.5f);
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// LayerNorm over the 128 channels of row `r` of a tile in place (two-pass
// statistics in fp32; weight/bias fp32, bias may be null).
__device__ __forceinline__ void ln_row_inplace(uint8_t* tile, int r, const float* __restrict__ w,
                                               const float* __restrict__ b, float eps) {
  uint4 v[16];
#pragma unroll
  for (int ka = 0; ka < 2; ++ka)
#pragma unroll
    for (int c = 0; c < 8; ++c)
      v[ka * 8 + c] = *reinterpret_cast<const uint4*>(tile + ka * ATOM + tc::sw128_off(r, c));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) s += bf_lo(u[j]) + bf_hi(u[j]);
  }
  const float mean = s * (1.0f / C);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float d0 = bf_lo(u[j]) - mean, d1 = bf_hi(u[j]) - mean;
      q += d0 * d0 + d1 * d1;
    }
  }
  const float rstd = rsqrtf(q * (1.0f / C) + eps);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t* u = reinterpret_cast<uint32_t*>(&v[i]);
    const int k0 = i * 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + 2 * j;
      float y0 = (bf_lo(u[j]) - mean) * rstd * __ldg(w + k);
      float y1 = (bf_hi(u[j]) - mean) * rstd * __ldg(w + k + 1);
      if (b) {
        y0 += __ldg(b + k);
        y1 += __ldg(b + k + 1);
      }
      u[j] = pack_bf2(y0, y1);
    }
  }
#pragma unroll
  for (int ka = 0; ka < 2; ++ka)
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(tile + ka * ATOM + tc::sw128_off(r, c)) = v[ka * 8 + c];
}

// Same LayerNorm with few registers (for kernels with many warps), from row r
// of tile `src` into row r of tile `dst` (both 128B-swizzled K-major, may be
// the same tile): the row is re-read from shared memory for each statistic
// pass and normalised one 16-byte chunk at a time.  w and b (b may be null)
// must be 16-byte aligned.
__device__ __forceinline__ void ln_row_lr(const uint8_t* src, uint8_t* dst, int r, const float* __restrict__ w,
                                          const float* __restrict__ b, float eps) {
  auto off = [&](int i) -> uint32_t { return (uint32_t)(i >> 3) * ATOM + tc::sw128_off(r, i & 7); };
  float s = 0.f;
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + off(i));
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) s += bf_lo(u[j]) + bf_hi(u[j]);
  }
  const float mean = s * (1.0f / C);
  float q = 0.f;
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + off(i));
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d0 = bf_lo(u[j]) - mean, d1 = bf_hi(u[j]) - mean;
      q += d0 * d0 + d1 * d1;
    }
  }
  const float rstd = rsqrtf(q * (1.0f / C) + eps);
#pragma unroll 2
  for (int i = 0; i < 16; ++i) {
    uint4 v = *reinterpret_cast<const uint4*>(src + off(i));
    uint32_t* u = reinterpret_cast<uint32_t*>(&v);
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + 8 * i));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + 8 * i + 4));
    float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
    if (b) {
      b0 = __ldg(reinterpret_cast<const float4*>(b + 8 * i));
      b1 = __ldg(reinterpret_cast<const float4*>(b + 8 * i + 4));
    }
    u[0] = pack_bf2((bf_lo(u[0]) - mean) * rstd * w0.x + b0.x, (bf_hi(u[0]) - mean) * rstd * w0.y + b0.y);
    u[1] = pack_bf2((bf_lo(u[1]) - mean) * rstd * w0.z + b0.z, (bf_hi(u[1]) - mean) * rstd * w0.w + b0.w);
    u[2] = pack_bf2((bf_lo(u[2]) - mean) * rstd * w1.x + b1.x, (bf_hi(u[2]) - mean) * rstd * w1.y + b1.y);
    u[3] = pack_bf2((bf_lo(u[3]) - mean) * rstd * w1.z + b1.z, (bf_hi(u[3]) - mean) * rstd * w1.w + b1.w);
    *reinterpret_cast<uint4*>(dst + off(i)) = v;
  }
}
__device__ __forceinline__ void ln_row_inplace_lr(uint8_t* tile, int r, const float* __restrict__ w,
                                                  const float* __restrict__ b, float eps) {
  ln_row_lr(tile, tile, r, w, b, eps);
}

// Copies a weight matrix Wt[rows][128] (bf16, k contiguous) into shared memory
// in the 128B-swizzled K-major layout: atom column ka (channels 64ka..) at
// dst + ka * rows * 128.
__device__ __forceinline__ void load_weight_sw128(uint8_t* dst, const bf16* __restrict__ wt, int rows, int tid,
                                                  int nthreads) {
  for (int e = tid; e < rows * 16; e += nthreads) {
    const int r = e >> 4, kc = e & 15;
    const int ka = kc >> 3, c = kc & 7;
    uint4 val = __ldg(reinterpret_cast<const uint4*>(wt + (size_t)r * C + kc * 8));
    *reinterpret_cast<uint4*>(dst + (size_t)ka * rows * 128 + tc::sw128_off(r, c)) = val;
  }
}

}  // namespace pt
}  // namespace sf
