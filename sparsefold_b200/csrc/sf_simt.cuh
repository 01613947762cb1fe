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
// Strided attention, one thread per query, keys streamed through shared memory
// in tiles; exact online softmax in fp32.  Masked logits are -FLT_MAX (not
// -inf), which reproduces the reference's uniform average for a query whose
// keys are all masked (sdpa.py:61-80).
// ---------------------------------------------------------------------------
constexpr int ATT_Q = 128, ATT_K = 32, ATT_DMAX = 64;

template <typename T, typename TB>
__global__ void __launch_bounds__(ATT_Q) k_attention(sf_attention_args a) {
  __shared__ float ks[ATT_K][ATT_DMAX + 1];
  __shared__ float vs[ATT_K][ATT_DMAX + 1];
  __shared__ uint8_t kvalid[ATT_K];
  const int D = (int)a.head_dim;
  const int64_t b = blockIdx.z, h = blockIdx.y;
  const int64_t qi = (int64_t)blockIdx.x * ATT_Q + threadIdx.x;
  const bool qin = qi < a.q_len;
  const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + h * a.q_sh + (qin ? qi : 0) * a.q_sq;
  const T* kp = static_cast<const T*>(a.k) + b * a.k_sb + h * a.k_sh;
  const T* vp = static_cast<const T*>(a.v) + b * a.v_sb + h * a.v_sh;
  const TB* bp = a.bias ? static_cast<const TB*>(a.bias) + b * a.b_sb + h * a.b_sh + (qin ? qi : 0) * a.b_sq : nullptr;
  bool row_ok = true;
  if (a.mask_row) row_ok = a.mask_row[b] != 0;
  if (a.mask_q && qin) row_ok = row_ok && a.mask_q[b * a.mq_sb + qi] != 0;

  float q[ATT_DMAX], acc[ATT_DMAX];
#pragma unroll
  for (int d = 0; d < ATT_DMAX; ++d) {
    q[d] = (d < D) ? ld(qp + d) * a.scale : 0.f;
    acc[d] = 0.f;
  }
  float mrun = -INFINITY, lrun = 0.f;
  for (int64_t k0 = 0; k0 < a.k_len; k0 += ATT_K) {
    for (int e = threadIdx.x; e < ATT_K * D; e += ATT_Q) {
      int r = e / D, c = e % D;
      int64_t kk = k0 + r;
      ks[r][c] = kk < a.k_len ? ld(kp + kk * a.k_sk + c) : 0.f;
      vs[r][c] = kk < a.k_len ? ld(vp + kk * a.v_sk + c) : 0.f;
    }
    if (threadIdx.x < ATT_K) {
      int64_t kk = k0 + threadIdx.x;
      kvalid[threadIdx.x] = kk < a.k_len && (!a.mask_k || a.mask_k[b * a.mk_sb + kk] != 0);
    }
    __syncthreads();
    const int kn = (a.k_len - k0) < ATT_K ? (int)(a.k_len - k0) : ATT_K;
    for (int r = 0; r < kn; ++r) {
      float s;
      if (row_ok && kvalid[r]) {
        s = 0.f;
#pragma unroll
        for (int d = 0; d < ATT_DMAX; ++d)
          if (d < D) s = fmaf(q[d], ks[r][d], s);
        if (bp) s += ld(bp + k0 + r);
      } else {
        s = -FLT_MAX;
      }
      float mnew = fmaxf(mrun, s);
      float corr = expf(mrun - mnew);
      float p = expf(s - mnew);
      lrun = lrun * corr + p;
#pragma unroll
      for (int d = 0; d < ATT_DMAX; ++d)
        if (d < D) acc[d] = fmaf(acc[d], corr, p * vs[r][d]);
      mrun = mnew;
    }
    __syncthreads();
  }
  if (!qin) return;
  T* op = static_cast<T*>(a.out) + b * a.o_sb + h * a.o_sh + qi * a.o_sq;
  const T* gp = a.gate ? static_cast<const T*>(a.gate) + b * a.g_sb + h * a.g_sh + qi * a.g_sq : nullptr;
  float inv = lrun > 0.f ? 1.f / lrun : 0.f;
#pragma unroll
  for (int d = 0; d < ATT_DMAX; ++d) {
    if (d < D) {
      float o = acc[d] * inv;
      if (gp) o *= sigmoid_f(ld(gp + d));
      st(op + d, o);
    }
  }
}

}  // namespace sf
