// fp32-arithmetic CUDA-core building blocks: LayerNorm, a tiled GEMM with a
// pluggable row accessor / epilogue, and a strided online-softmax attention.
// These carry the fp32 mode (1e-4 tolerance) and the small single-track
// GEMMs; the bf16 pair track uses the tcgen05 kernels.
#pragma once

#include <cfloat>

#include "sf_common.cuh"

namespace sf {

// ---------------------------------------------------------------------------
// LayerNorm over the last axis, one warp per row, exact two-pass statistics.
// ---------------------------------------------------------------------------
template <typename Tin, typename Tout>
__global__ void k_layernorm(const Tin* __restrict__ x, Tout* __restrict__ y,
                            const float* __restrict__ w, const float* __restrict__ b,
                            int64_t rows, int cols, float eps) {
  int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const Tin* xr = x + row * cols;
  float s = 0.f;
  for (int c = lane; c < cols; c += 32) s += ld(xr + c);
  float mean = warp_sum(s) / cols;
  float v = 0.f;
  for (int c = lane; c < cols; c += 32) {
    float d = ld(xr + c) - mean;
    v += d * d;
  }
  float rstd = rsqrtf(warp_sum(v) / cols + eps);
  Tout* yr = y + row * cols;
  for (int c = lane; c < cols; c += 32) {
    float o = (ld(xr + c) - mean) * rstd;
    if (w) o *= w[c];
    if (b) o += b[c];
    st(yr + c, o);
  }
}

// Eight consecutive elements as fp32 (one 16-byte load for bf16, two for fp32).
__device__ __forceinline__ void ld8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void ld8(const bf16* p, float (&v)[8]) {
  const uint4 q = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ void st8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void st8(bf16* p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// The same LayerNorm for rows of G * 8 elements (G = 1 .. 32, a power of two): a group of G
// lanes per row, eight elements per lane held in registers, statistics over the group with
// shuffles (same two passes, mean then the centred squares), one coalesced read and write.
template <typename Tin, typename Tout, int G>
__global__ void k_layernorm_vec(const Tin* __restrict__ x, Tout* __restrict__ y, const float* __restrict__ w,
                                const float* __restrict__ b, int64_t rows, float eps) {
  constexpr int COLS = 8 * G;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / G;
  const int sub = threadIdx.x % G;
  const bool live = row < rows;
  float v[8];
  if (live) ld8(x + row * COLS + sub * 8, v);
  else
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.f;
  float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o, G);
  const float mean = s / COLS;
  float q = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float d = v[e] - mean;
    q = fmaf(d, d, q);
  }
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o, G);
  const float rstd = rsqrtf(q / COLS + eps);
  if (!live) return;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int c = sub * 8 + e;
    float o = (v[e] - mean) * rstd;
    if (w) o *= w[c];
    if (b) o += b[c];
    v[e] = o;
  }
  st8(y + row * COLS + sub * 8, v);
}

template <typename Tin, typename Tout, int G>
inline int launch_layernorm_vec(const Tin* x, Tout* y, const float* w, const float* b, int64_t rows, float eps,
                                cudaStream_t s) {
  const int64_t threads = rows * G;
  k_layernorm_vec<Tin, Tout, G><<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, y, w, b, rows, eps);
  count_launch();
  return check_launch("layernorm");
}

template <typename Tin, typename Tout>
inline int launch_layernorm(const Tin* x, Tout* y, const float* w, const float* b, int64_t rows,
                            int cols, float eps, cudaStream_t s) {
  if (rows == 0) return SF_OK;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (aligned && (rows * cols) / 8 < (int64_t(1) << 31)) {
    switch (cols) {
      case 64: return launch_layernorm_vec<Tin, Tout, 8>(x, y, w, b, rows, eps, s);
      case 128: return launch_layernorm_vec<Tin, Tout, 16>(x, y, w, b, rows, eps, s);
      case 256: return launch_layernorm_vec<Tin, Tout, 32>(x, y, w, b, rows, eps, s);
      default: break;
    }
  }
  int warps = 8;
  k_layernorm<Tin, Tout><<<(unsigned)((rows + warps - 1) / warps), warps * 32, 0, s>>>(x, y, w, b, rows, cols, eps);
  count_launch();
  return check_launch("layernorm");
}

// ---------------------------------------------------------------------------
// Row accessors for the GEMM A operand.
// ---------------------------------------------------------------------------
template <typename T>
struct RowMajor {
  const T* p;
  int64_t ld;
  __device__ float operator()(int64_t m, int k) const { return ld_(p + m * ld + k); }
  __device__ static float ld_(const T* q) { return ::sf::ld(q); }
};

// Pair tensor [n][n][c] read transposed: GEMM row m = i*n + j reads position (j, i).
template <typename T>
struct PairTransposed {
  const T* p;
  int64_t n, c;
  __device__ float operator()(int64_t m, int k) const {
    int64_t i = m / n, j = m % n;
    return ::sf::ld(p + (j * n + i) * c + k);
  }
};

// ---------------------------------------------------------------------------
// C[m, n] = sum_k A(m, k) * Wt[n, k]; epi(m, n, value) stores.
// 64x64 tile, 16-deep k slices, 256 threads each owning a 4x4 block.
// ---------------------------------------------------------------------------
constexpr int GM = 64, GN = 64, GK = 16;

template <typename TW, typename ARow, typename Epi>
__global__ void __launch_bounds__(256) k_gemm(int64_t M, int N, int K, ARow arow,
                                              const TW* __restrict__ wt, Epi epi) {
  __shared__ float As[GK][GM + 4];
  __shared__ float Ws[GK][GN + 4];
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.x * GM;
  const int n0 = blockIdx.y * GN;
  const int tm = tid / 16, tn = tid % 16;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += GK) {
    for (int e = tid; e < GM * GK; e += 256) {
      int r = e / GK, c = e % GK;
      int64_t m = m0 + r;
      int k = k0 + c;
      As[c][r] = (m < M && k < K) ? arow(m, k) : 0.f;
    }
    for (int e = tid; e < GN * GK; e += 256) {
      int r = e / GK, c = e % GK;  // r: output column, c: k
      int n = n0 + r, k = k0 + c;
      Ws[c][r] = (n < N && k < K) ? ld(wt + (int64_t)n * K + k) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < GK; ++kk) {
      float a[4], w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][tm * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = Ws[kk][tn * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t m = m0 + tm * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int n = n0 + tn * 4 + j;
      if (n < N) epi(m, n, acc[i][j]);
    }
  }
}

template <typename TW, typename ARow, typename Epi>
inline int launch_gemm(int64_t M, int N, int K, ARow arow, const TW* wt, Epi epi, cudaStream_t s,
                       const char* what) {
  if (M == 0 || N == 0) return SF_OK;
  dim3 grid((unsigned)((M + GM - 1) / GM), (N + GN - 1) / GN);
  k_gemm<TW, ARow, Epi><<<grid, 256, 0, s>>>(M, N, K, arow, wt, epi);
  count_launch();
  return check_launch(what);
}

// ---- common epilogues -------------------------------------------------------
template <typename T>
struct EpiStore {  // out[m*ld + n] = v
  T* out;
  int64_t ld;
  __device__ void operator()(int64_t m, int n, float v) const { st(out + m * ld + n, v); }
};

template <typename T>
struct EpiLinear {  // y = post(v + bias + residual)
  T* out;
  const float* bias;
  const T* residual;
  int64_t ld;
  int post;
  __device__ void operator()(int64_t m, int n, float v) const {
    if (bias) v += bias[n];
    if (residual) v += ld_res(m, n);
    if (post == SF_POST_RELU) v = fmaxf(v, 0.f);
    else if (post == SF_POST_SILU) v = swish_f(v);
    else if (post == SF_POST_SIGMOID) v = sigmoid_f(v);
    st(out + m * ld + n, v);
  }
  __device__ float ld_res(int64_t m, int n) const { return ::sf::ld(residual + m * ld + n); }
};

// ---------------------------------------------------------------------------
// Strided attention (fp32 online softmax).  Masked logits are -FLT_MAX (not
// -inf), which reproduces the reference's uniform average for a query whose
// keys are all masked (sdpa.py:61-80); keys beyond k_len take no part at all.
// ---------------------------------------------------------------------------
constexpr int ATT_QB = 32, ATT_NS = 8, ATT_KT = 128, ATT_DMAX = 64;
constexpr int ATT_KPS = ATT_KT / ATT_NS;            // keys of a tile handled by one split (warp)

// Block = (batch b, head h, 32 queries); warp w = key split, lane = query.  Each
// 128-key tile of K and V (fp32 rows) and the block's 32 x 128 bias tile are
// staged in shared memory once per block (coalesced), so the eight warps read
// K/V rows as broadcasts (16-byte vectors when the head dim DK is a compile-time
// multiple of 4; DK = 0 is the generic runtime head dim).  Each thread scores its
// split's 16 keys, takes their max, rescales its running state once per tile and
// spends one exp per key; the eight split states of a query are merged through
// shared memory at the end.
// Head dims up to 32 fit in 128 registers, which lets two blocks share an SM (with 256
// blocks for a 512-token, 16-head call, one block per SM left it two latency-bound waves).
template <typename T, typename TB, int DK, int DM>
__global__ void __launch_bounds__(ATT_NS * 32, (DM > 0 && DM <= 32) ? 2 : 1) k_attention(sf_attention_args a) {
  extern __shared__ float4 att_smem4[];
  float* att_smem = reinterpret_cast<float*>(att_smem4);
  const int D = DK > 0 ? DK : (int)a.head_dim;
  // value head dim: the query/key dim unless value_dim says otherwise (runtime-dim kernel only)
  const int DV = DK > 0 ? DK : (a.value_dim > 0 ? (int)a.value_dim : D);
  constexpr bool VEC = DK > 0 && DK % 4 == 0;
  float* ks = att_smem;                               // [KT][D]
  float* vs = ks + ATT_KT * D;                        // [KT][DV]
  float* bs = vs + ATT_KT * DV;                       // [QB][KT + 1]
  uint8_t* kvalid = reinterpret_cast<uint8_t*>(bs + ATT_QB * (ATT_KT + 1));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.z, h = blockIdx.y;
  const int64_t q0 = (int64_t)blockIdx.x * ATT_QB, qi = q0 + lane;
  const bool qin = qi < a.q_len;
  const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + h * a.q_sh + (qin ? qi : 0) * a.q_sq;
  const T* kp = static_cast<const T*>(a.k) + b * a.k_sb + h * a.k_sh;
  const T* vp = static_cast<const T*>(a.v) + b * a.v_sb + h * a.v_sh;
  const TB* bbase = a.bias ? static_cast<const TB*>(a.bias) + b * a.b_sb + h * a.b_sh : nullptr;
  bool row_ok = true;
  if (a.mask_row) row_ok = a.mask_row[b] != 0;
  if (a.mask_q && qin) row_ok = row_ok && a.mask_q[b * a.mq_sb + qi] != 0;

  float q[DM], acc[DM];
#pragma unroll
  for (int d = 0; d < DM; ++d) {
    q[d] = (d < D && qin) ? ld(qp + d) * a.scale : 0.f;
    acc[d] = 0.f;
  }
  auto dot = [&](const float* kr) {
    float s = 0.f;
    if constexpr (VEC) {
#pragma unroll
      for (int d = 0; d < DK; d += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
        s = fmaf(q[d], k4.x, s);
        s = fmaf(q[d + 1], k4.y, s);
        s = fmaf(q[d + 2], k4.z, s);
        s = fmaf(q[d + 3], k4.w, s);
      }
    } else {
#pragma unroll
      for (int d = 0; d < DM; ++d)
        if (d < D) s = fmaf(q[d], kr[d], s);
    }
    return s;
  };
  auto axpy = [&](float pr, const float* vr) {
    if constexpr (VEC) {
#pragma unroll
      for (int d = 0; d < DK; d += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(vr + d);
        acc[d] = fmaf(pr, v4.x, acc[d]);
        acc[d + 1] = fmaf(pr, v4.y, acc[d + 1]);
        acc[d + 2] = fmaf(pr, v4.z, acc[d + 2]);
        acc[d + 3] = fmaf(pr, v4.w, acc[d + 3]);
      }
    } else {
#pragma unroll
      for (int d = 0; d < DM; ++d)
        if (d < DV) acc[d] = fmaf(pr, vr[d], acc[d]);
    }
  };
  float mrun = -INFINITY, lrun = 0.f;
  for (int64_t k0 = 0; k0 < a.k_len; k0 += ATT_KT) {
    const int kn = (a.k_len - k0) < ATT_KT ? (int)(a.k_len - k0) : ATT_KT;
    // With 16-bit K/V (head dim a multiple of 8) and 16-byte aligned rows, every thread first
    // issues all its 16-byte loads of the tile, then converts and stores them.
    constexpr bool CHUNKED = DK > 0 && DK % 8 == 0 && sizeof(T) == 2;
    constexpr int NT = ATT_NS * 32;
    const bool kv_chunked =
        CHUNKED && ((reinterpret_cast<uintptr_t>(kp) | reinterpret_cast<uintptr_t>(vp) | (uintptr_t)(a.k_sk * 2) |
                     (uintptr_t)(a.v_sk * 2)) & 15) == 0;
    if (kv_chunked) {
      constexpr int CPR = DK > 0 ? DK / 8 : 1, KVC = ATT_KT * CPR, PER = (2 * KVC + NT - 1) / NT;
      uint4 buf[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = threadIdx.x + i * NT, w = e / KVC, rem = e - w * KVC, r = rem / CPR, c = rem - r * CPR;
        if (e < 2 * KVC && r < kn)
          buf[i] = __ldg(reinterpret_cast<const uint4*>((w ? vp + (k0 + r) * a.v_sk : kp + (k0 + r) * a.k_sk) + 8 * c));
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = threadIdx.x + i * NT, w = e / KVC, rem = e - w * KVC, r = rem / CPR, c = rem - r * CPR;
        if (e < 2 * KVC && r < kn) {
          float4* dst = reinterpret_cast<float4*>((w ? vs : ks) + r * D + 8 * c);
          dst[0] = make_float4(__uint_as_float(buf[i].x << 16), __uint_as_float(buf[i].x & 0xffff0000u),
                               __uint_as_float(buf[i].y << 16), __uint_as_float(buf[i].y & 0xffff0000u));
          dst[1] = make_float4(__uint_as_float(buf[i].z << 16), __uint_as_float(buf[i].z & 0xffff0000u),
                               __uint_as_float(buf[i].w << 16), __uint_as_float(buf[i].w & 0xffff0000u));
        }
      }
    } else {
      for (int r = warp; r < kn; r += ATT_NS) {         // one key row per warp, lanes along d
        const T* kr = kp + (k0 + r) * a.k_sk;
        const T* vr = vp + (k0 + r) * a.v_sk;
        for (int c = lane; c < D; c += 32) ks[r * D + c] = ld(kr + c);
        for (int c = lane; c < DV; c += 32) vs[r * DV + c] = ld(vr + c);
      }
    }
    if (bbase) {
      const bool b_chunked = sizeof(TB) == 2 && kn % 8 == 0 &&
                             ((reinterpret_cast<uintptr_t>(bbase) | (uintptr_t)(a.b_sq * 2)) & 15) == 0;
      if (b_chunked) {   // the bias tile the same way, 8 keys per 16-byte load
        constexpr int CPQ = ATT_KT / 8, BC = ATT_QB * CPQ, BPER = (BC + NT - 1) / NT;
        uint4 bb[BPER];
#pragma unroll
        for (int i = 0; i < BPER; ++i) {
          const int e = threadIdx.x + i * NT, qq = e / CPQ, k = 8 * (e - qq * CPQ);
          if (e < BC && q0 + qq < a.q_len && k < kn)
            bb[i] = __ldg(reinterpret_cast<const uint4*>(bbase + (q0 + qq) * a.b_sq + k0 + k));
        }
#pragma unroll
        for (int i = 0; i < BPER; ++i) {
          const int e = threadIdx.x + i * NT, qq = e / CPQ, k = 8 * (e - qq * CPQ);
          if (e < BC && q0 + qq < a.q_len && k < kn) {
            float* dst = bs + qq * (ATT_KT + 1) + k;
            const uint32_t u[4] = {bb[i].x, bb[i].y, bb[i].z, bb[i].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              dst[2 * j] = __uint_as_float(u[j] << 16);
              dst[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
            }
          }
        }
      } else {
        for (int qq = warp; qq < ATT_QB; qq += ATT_NS) {
          if (q0 + qq >= a.q_len) continue;
          const TB* br = bbase + (q0 + qq) * a.b_sq + k0;
          for (int k = lane; k < kn; k += 32) bs[qq * (ATT_KT + 1) + k] = ld(br + k);
        }
      }
    }
    for (int r = threadIdx.x; r < kn; r += blockDim.x)
      kvalid[r] = !a.mask_k || a.mask_k[b * a.mk_sb + k0 + r] != 0;
    __syncthreads();
    float sc[ATT_KPS];
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < ATT_KPS; ++j) {
      const int kk = warp * ATT_KPS + j;
      float s = -INFINITY;                            // beyond the last key: excluded
      if (kk < kn) {
        if (row_ok && kvalid[kk]) {
          s = dot(ks + kk * D);
          if (bbase) s += bs[lane * (ATT_KT + 1) + kk];
        } else {
          s = -FLT_MAX;                               // masked: the reference's -finfo.max bias
        }
      }
      sc[j] = s;
      mt = fmaxf(mt, s);
    }
    const float mnew = fmaxf(mrun, mt);
    if (mnew != -INFINITY) {
      const float corr = (mrun == -INFINITY) ? 0.f : expf(mrun - mnew);
      lrun *= corr;
#pragma unroll
      for (int d = 0; d < DM; ++d) acc[d] *= corr;
#pragma unroll
      for (int j = 0; j < ATT_KPS; ++j) {
        const int kk = warp * ATT_KPS + j;
        if (kk < kn) {
          const float pr = expf(sc[j] - mnew);
          lrun += pr;
          axpy(pr, vs + kk * DV);
        }
      }
      mrun = mnew;
    }
    __syncthreads();
  }
  // merge the key splits of each query (the K/V area is free now)
  float* ms = att_smem;                               // [NS][QB]
  float* ls = ms + ATT_NS * ATT_QB;                   // [NS][QB]
  float* as = ls + ATT_NS * ATT_QB;                   // [NS][QB][DV]
  ms[warp * ATT_QB + lane] = mrun;
  ls[warp * ATT_QB + lane] = lrun;
#pragma unroll
  for (int d = 0; d < DM; ++d)
    if (d < DV) as[(warp * ATT_QB + lane) * DV + d] = acc[d];
  __syncthreads();
  const int qq = threadIdx.x % ATT_QB, d0 = threadIdx.x / ATT_QB;
  const int64_t qo = q0 + qq;
  if (qo >= a.q_len) return;
  float m = -INFINITY;
#pragma unroll
  for (int sp = 0; sp < ATT_NS; ++sp) m = fmaxf(m, ms[sp * ATT_QB + qq]);
  float wgt[ATT_NS], l = 0.f;
#pragma unroll
  for (int sp = 0; sp < ATT_NS; ++sp) {
    const float ms_ = ms[sp * ATT_QB + qq];
    wgt[sp] = (ms_ == -INFINITY) ? 0.f : expf(ms_ - m);
    l += ls[sp * ATT_QB + qq] * wgt[sp];
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* op = static_cast<T*>(a.out) + b * a.o_sb + h * a.o_sh + qo * a.o_sq;
  const T* gp = a.gate ? static_cast<const T*>(a.gate) + b * a.g_sb + h * a.g_sh + qo * a.g_sq : nullptr;
  for (int d = d0; d < DV; d += ATT_NS) {
    float o = 0.f;
#pragma unroll
    for (int sp = 0; sp < ATT_NS; ++sp) o += as[(sp * ATT_QB + qq) * DV + d] * wgt[sp];
    o *= inv;
    if (gp) o *= sigmoid_f(ld(gp + d));
    st(op + d, o);
  }
}

inline size_t attention_smem_bytes(int D, int DV) {
  const size_t main = (size_t)(ATT_KT * (D + DV) + ATT_QB * (ATT_KT + 1)) * sizeof(float) + ATT_KT;
  const size_t merge = (size_t)ATT_NS * ATT_QB * (DV + 2) * sizeof(float);
  return main > merge ? main : merge;
}

}  // namespace sf
