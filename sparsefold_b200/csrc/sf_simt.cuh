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

template <typename Tin, typename Tout>
inline int launch_layernorm(const Tin* x, Tout* y, const float* w, const float* b, int64_t rows,
                            int cols, float eps, cudaStream_t s) {
  if (rows == 0) return SF_OK;
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
// Strided attention, one warp per query: the 32 lanes split the keys of each
// shared-memory key tile, keep their own exact online-softmax state (fp32),
// and merge the states by butterfly shuffles at the end.  Masked logits are
// -FLT_MAX (not -inf), which reproduces the reference's uniform average for a
// query whose keys are all masked (sdpa.py:61-80); keys beyond k_len take no
// part at all.
// ---------------------------------------------------------------------------
constexpr int ATT_WARPS = 8, ATT_KT = 128, ATT_DMAX = 64;

template <typename T, typename TB, int DM>
__global__ void __launch_bounds__(ATT_WARPS * 32) k_attention(sf_attention_args a) {
  extern __shared__ float att_smem[];
  float* ks = att_smem;                              // [ATT_KT][D + 1]
  const int D = (int)a.head_dim, DP = D + 1;
  float* vs = ks + ATT_KT * DP;                      // [ATT_KT][D + 1]
  uint8_t* kvalid = reinterpret_cast<uint8_t*>(vs + ATT_KT * DP);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.z, h = blockIdx.y;
  const int64_t qi = (int64_t)blockIdx.x * ATT_WARPS + warp;
  const bool qin = qi < a.q_len;
  const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + h * a.q_sh + (qin ? qi : 0) * a.q_sq;
  const T* kp = static_cast<const T*>(a.k) + b * a.k_sb + h * a.k_sh;
  const T* vp = static_cast<const T*>(a.v) + b * a.v_sb + h * a.v_sh;
  const TB* bp = a.bias ? static_cast<const TB*>(a.bias) + b * a.b_sb + h * a.b_sh + (qin ? qi : 0) * a.b_sq : nullptr;
  bool row_ok = true;
  if (a.mask_row) row_ok = a.mask_row[b] != 0;
  if (a.mask_q && qin) row_ok = row_ok && a.mask_q[b * a.mq_sb + qi] != 0;

  float q[DM], acc[DM];
#pragma unroll
  for (int d = 0; d < DM; ++d) {
    q[d] = (d < D && qin) ? ld(qp + d) * a.scale : 0.f;
    acc[d] = 0.f;
  }
  float mrun = -INFINITY, lrun = 0.f;
  for (int64_t k0 = 0; k0 < a.k_len; k0 += ATT_KT) {
    const int kn = (a.k_len - k0) < ATT_KT ? (int)(a.k_len - k0) : ATT_KT;
    for (int e = threadIdx.x; e < kn * D; e += blockDim.x) {
      const int r = e / D, c = e % D;
      ks[r * DP + c] = ld(kp + (k0 + r) * a.k_sk + c);
      vs[r * DP + c] = ld(vp + (k0 + r) * a.v_sk + c);
    }
    for (int r = threadIdx.x; r < kn; r += blockDim.x)
      kvalid[r] = !a.mask_k || a.mask_k[b * a.mk_sb + k0 + r] != 0;
    __syncthreads();
    for (int r = lane; r < kn; r += 32) {
      float s;
      if (row_ok && kvalid[r]) {
        s = 0.f;
#pragma unroll
        for (int d = 0; d < DM; ++d)
          if (d < D) s = fmaf(q[d], ks[r * DP + d], s);
        if (bp) s += ld(bp + k0 + r);
      } else {
        s = -FLT_MAX;
      }
      const float mnew = fmaxf(mrun, s);
      const float corr = expf(mrun - mnew);
      const float pr = expf(s - mnew);
      lrun = lrun * corr + pr;
#pragma unroll
      for (int d = 0; d < DM; ++d)
        if (d < D) acc[d] = fmaf(acc[d], corr, pr * vs[r * DP + d]);
      mrun = mnew;
    }
    __syncthreads();
  }
  // merge the 32 lane states (lanes that saw no key have m = -inf, l = 0)
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, mrun, off);
    const float lo = __shfl_xor_sync(0xffffffffu, lrun, off);
    const float mnew = fmaxf(mrun, mo);
    const float ca = (mrun == -INFINITY) ? 0.f : expf(mrun - mnew);
    const float cb = (mo == -INFINITY) ? 0.f : expf(mo - mnew);
    lrun = lrun * ca + lo * cb;
#pragma unroll
    for (int d = 0; d < DM; ++d) {
      const float ao = __shfl_xor_sync(0xffffffffu, acc[d], off);
      acc[d] = acc[d] * ca + ao * cb;
    }
    mrun = mnew;
  }
  if (!qin) return;
  T* op = static_cast<T*>(a.out) + b * a.o_sb + h * a.o_sh + qi * a.o_sq;
  const T* gp = a.gate ? static_cast<const T*>(a.gate) + b * a.g_sb + h * a.g_sh + qi * a.g_sq : nullptr;
  const float inv = lrun > 0.f ? 1.f / lrun : 0.f;
#pragma unroll
  for (int d = 0; d < DM; ++d) {
    if (d < D && (d & 31) == lane) {
      float o = acc[d] * inv;
      if (gp) o *= sigmoid_f(ld(gp + d));
      st(op + d, o);
    }
  }
}

inline size_t attention_smem_bytes(int D) {
  return (size_t)2 * ATT_KT * (D + 1) * sizeof(float) + ATT_KT;
}

}  // namespace sf
