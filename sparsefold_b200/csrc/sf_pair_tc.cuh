// Shared pieces of the tcgen05 pair-tile kernels: tensor maps over the pair
// tensor, in-place LayerNorm of a 128-position tile held in the 128B-swizzled
// K-major layout, resident weight loading, bf16 pack/unpack.
#pragma once

#include <cuda_fp16.h>

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

// Packed fp32 pairs (one instruction for two lanes of arithmetic, each IEEE as its
// scalar form): (a0, a1) - (b0, b1), (a0, a1) * (b0, b1), (a0, a1) * (b0, b1) + (c0, c1).
__device__ __forceinline__ void sub2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "sub.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void mul2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "mul.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1));
}
// (d0, d1) = (a0, a1) * (b0, b1) + (d0, d1)
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tmov.b64 z, {%0, %1};\n\t"
      "fma.rn.f32x2 z, x, y, z;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "+f"(d0), "+f"(d1) : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// The shifted one-pass statistics of 8 bf16 values (one 16-byte chunk) as packed pairs:
// s += (x - k), q += (x - k)^2 over the pairs (even, odd) of the chunk.
__device__ __forceinline__ void ln_accumulate(const uint4 v, float k, float (&s)[2], float (&q)[2]) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float d0 = bf_lo(u[j]), d1 = bf_hi(u[j]);
    sub2(d0, d1, k, k);
    add2(s[0], s[1], d0, d1);
    fma2(q[0], q[1], d0, d1, d0, d1);
  }
}
// One normalised chunk: ((x - mean) * rstd) * w + b for 8 values, packed to bf16.
__device__ __forceinline__ uint4 ln_apply(const uint4 v, float mean, float rstd, const float* w, const float* b) {
  const float4 w0 = *reinterpret_cast<const float4*>(w), w1 = *reinterpret_cast<const float4*>(w + 4);
  const float4 b0 = *reinterpret_cast<const float4*>(b), b1 = *reinterpret_cast<const float4*>(b + 4);
  const float wl[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const float bl[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float x0 = bf_lo(u[j]), x1 = bf_hi(u[j]);
    sub2(x0, x1, mean, mean);
    mul2(x0, x1, rstd, rstd);
    float y0 = bl[2 * j], y1 = bl[2 * j + 1];
    fma2(y0, y1, x0, x1, wl[2 * j], wl[2 * j + 1]);
    o[j] = pack_bf2(y0, y1);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// LayerNorm of tile row r in place, one thread per row (128 channels in two 64-channel
// atoms of the 128B-swizzled K-major layout): statistics in one pass shifted by the row's
// first value k so that E[(x-k)^2] - E[x-k]^2 keeps its precision, then the normalised,
// rounded row written back; arithmetic on packed fp32 pairs, scale and shift (128 floats
// each) from shared memory.
__device__ __forceinline__ void ln_row_shifted(uint8_t* tile, int r, const float* w_s, const float* b_s, float eps) {
  auto off = [&](int i) -> uint32_t { return (uint32_t)(i >> 3) * ATOM + tc::sw128_off(r, i & 7); };
  const float k = bf_lo(*reinterpret_cast<const uint32_t*>(tile + off(0)));
  float s[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, q[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
  for (int i = 0; i < 16; ++i)
    ln_accumulate(*reinterpret_cast<const uint4*>(tile + off(i)), k, s[i & 1], q[i & 1]);
  const float dm = ((s[0][0] + s[0][1]) + (s[1][0] + s[1][1])) * (1.0f / C);
  const float var = fmaxf(((q[0][0] + q[0][1]) + (q[1][0] + q[1][1])) * (1.0f / C) - dm * dm, 0.f);
  const float mean = k + dm, rstd = rsqrtf(var + eps);
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    uint4* p = reinterpret_cast<uint4*>(tile + off(i));
    *p = ln_apply(*p, mean, rstd, w_s + 8 * i, b_s + 8 * i);
  }
}
// The same with two threads per row (thread h takes channels 64h..64h+63, the
// statistics meet through a shuffle with the partner lane); b_s may be null.
__device__ __forceinline__ void ln_half_row_shifted(uint8_t* tile, int r, int h, const float* w_s, const float* b_s,
                                                    float eps) {
  uint8_t* base = tile + h * ATOM;
  auto off = [&](int i) -> uint32_t { return tc::sw128_off(r, (i + 4 * h) & 7); };
  const float k = bf_lo(*reinterpret_cast<const uint32_t*>(tile + tc::sw128_off(r, 0)));
  float s[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, q[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
  for (int i = 0; i < 8; ++i) ln_accumulate(*reinterpret_cast<const uint4*>(base + off(i)), k, s[i & 1], q[i & 1]);
  float ss = (s[0][0] + s[0][1]) + (s[1][0] + s[1][1]), qq = (q[0][0] + q[0][1]) + (q[1][0] + q[1][1]);
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  qq += __shfl_xor_sync(0xffffffffu, qq, 1);
  const float dm = ss * (1.0f / C);
  const float mean = k + dm, rstd = rsqrtf(fmaxf(qq * (1.0f / C) - dm * dm, 0.f) + eps);
  const float zero8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int i = 0; i < 8; ++i) {
    const int c8 = 64 * h + 8 * ((i + 4 * h) & 7);   // first channel of this chunk
    uint4* p = reinterpret_cast<uint4*>(base + off(i));
    *p = ln_apply(*p, mean, rstd, w_s + c8, b_s ? b_s + c8 : zero8);
  }
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

// acc + lo(a) lo(b) + hi(a) hi(b) for packed bf16 pairs a, b, accumulated in fp32
// (the products of two bf16 values are exact in fp32).
__device__ __forceinline__ float fma_bf16x2_f32(uint32_t a, uint32_t b, float acc) {
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %1;\n\t"
      "mov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.bf16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.bf16 %0, ah, bh, %0;\n\t}"
      : "+f"(acc)
      : "r"(a), "r"(b));
  return acc;
}

// Layer norm folded into the GEMM that follows it: with
//   LN(x)[c] = (x[c] - mu) rho w[c] + b[c],
//   LN(x) . W[o] = rho (x . W'[o] - mu s[o]) + b'[o],
//   W'[o][c] = bf16(W[o][c] w[c]),  s[o] = sum_c W'[o][c],  b'[o] = sum_c b[c] W[o][c],
// so the tensor core reads the raw x tile and the epilogue applies rho and mu.
// fold_weight writes W' (128B-swizzled K-major, atom column ka at dst + ka * rows
// * 128) and s, b' for rows [0, rows).  w_s and b_s are the layer-norm scale and
// bias staged in shared memory (b_s all zero for a scale-only norm).  Called by
// every thread of the block (nthreads a multiple of 32): a 16-lane group owns a
// row per pass and reduces s and b' with shuffles.
__device__ __forceinline__ void fold_weight(uint8_t* dst, const bf16* __restrict__ wt, const float* w_s,
                                            const float* b_s, int rows, float* s, float* bp, int tid, int nthreads) {
  const int total = rows * 16;
  for (int e0 = 0; e0 < total; e0 += nthreads) {
    const int e = e0 + tid;
    const bool valid = e < total;
    const int r = e >> 4, kc = e & 15;
    float ps = 0.f, pb = 0.f;
    if (valid) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(wt + (size_t)r * C + kc * 8));
      const float4 w0 = *reinterpret_cast<const float4*>(w_s + kc * 8);
      const float4 w1 = *reinterpret_cast<const float4*>(w_s + kc * 8 + 4);
      const float4 b0 = *reinterpret_cast<const float4*>(b_s + kc * 8);
      const float4 b1 = *reinterpret_cast<const float4*>(b_s + kc * 8 + 4);
      const float wl[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const float bl[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x0 = bf_lo(u[i]), x1 = bf_hi(u[i]);
        o[i] = pack_bf2(x0 * wl[2 * i], x1 * wl[2 * i + 1]);
        ps += bf_lo(o[i]) + bf_hi(o[i]);
        pb = fmaf(bl[2 * i], x0, fmaf(bl[2 * i + 1], x1, pb));
      }
      *reinterpret_cast<uint4*>(dst + (size_t)(kc >> 3) * rows * 128 + tc::sw128_off(r, kc & 7)) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) {
      ps += __shfl_xor_sync(0xffffffffu, ps, m);
      pb += __shfl_xor_sync(0xffffffffu, pb, m);
    }
    if (valid && kc == 0) {
      s[r] = ps;
      bp[r] = pb;
    }
  }
}

// Stages a layer norm's scale and bias (128 floats each; bias may be null) in shared memory.
__device__ __forceinline__ void stage_norm_params(float* w_s, float* b_s, const float* __restrict__ w,
                                                  const float* __restrict__ b, int tid) {
  if (tid < C) {
    w_s[tid] = __ldg(w + tid);
    b_s[tid] = b ? __ldg(b + tid) : 0.f;
  }
}

}  // namespace pt
}  // namespace sf
