// C-ABI entry points of the generic ops (attention, LayerNorm, Linear) and the
// pair-track ops (triangle multiplication, triangle attention, transition,
// pair logits) composed from the building blocks of sf_simt.cuh.
#include "sf_simt.cuh"

namespace sf {

// ---- epilogues of the pair-track ops ------------------------------------------
template <typename T>
struct EpiColMajor {  // out[n * M + m] = v  (e.g. pair bias [H][q][k])
  T* out;
  int64_t M;
  __device__ void operator()(int64_t m, int n, float v) const { st(out + (int64_t)n * M + m, v); }
};

template <typename T>
struct EpiPairResidual {  // z_out[pos] = z[pos] + v, pos = m or its transpose
  const T* z;
  T* z_out;
  int64_t n, c;
  int transpose;
  __device__ void operator()(int64_t m, int col, float v) const {
    int64_t pos = m;
    if (transpose) pos = (m % n) * n + m / n;
    int64_t off = pos * c + col;
    st(z_out + off, ld(z + off) + v);
  }
};

template <typename T>
struct EpiGatedResidual {  // z_out = z + v * sigmoid(G)
  const T* z;
  const float* g;
  T* z_out;
  int64_t c;
  __device__ void operator()(int64_t m, int col, float v) const {
    int64_t off = m * c + col;
    st(z_out + off, ld(z + off) + v * sigmoid_f(g[off]));
  }
};

template <typename T>
struct EpiResidual {  // y = x + v (row-major, ld = c)
  const T* x;
  T* y;
  int64_t c;
  __device__ void operator()(int64_t m, int col, float v) const {
    int64_t off = m * c + col;
    st(y + off, ld(x + off) + v);
  }
};

// ---- triangle-multiplication helpers -------------------------------------------
// y: [n*n][4C] fp32 = (gate_a, val_a, gate_b, val_b).  Writes the contraction
// operands channel-major through a 32x32 shared-memory transpose.
template <typename T>
__global__ void k_tri_glu_scatter(const float* __restrict__ y, const uint8_t* __restrict__ mask,
                                  int64_t n, int64_t pitch, int C, int incoming, T* __restrict__ a_op,
                                  T* __restrict__ b_op) {
  __shared__ float ta[32][33], tb[32][33];
  const int64_t M = n * n;
  const int64_t m0 = (int64_t)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    int64_t m = m0 + r;
    int c = c0 + tx;
    float va = 0.f, vb = 0.f;
    if (m < M) {
      int64_t i = m / n, k = m % n;
      bool keep = mask[i] && mask[k];
      const float* yr = y + m * 4 * C;
      if (keep) {
        va = sigmoid_f(yr[c]) * yr[C + c];
        vb = sigmoid_f(yr[2 * C + c]) * yr[3 * C + c];
      }
    }
    ta[r][tx] = va;
    tb[r][tx] = vb;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    int c = c0 + r;
    int64_t m = m0 + tx;
    if (m >= M) continue;
    int64_t i = m / n, k = m % n;
    float va = ta[tx][r], vb = tb[tx][r];
    if (!incoming) {
      int64_t t = (i * C + c) * pitch + k;
      st(a_op + t, va);   // A[i][c][k] = a[c,i,k]
      st(b_op + t, vb);   // B[j][c][k] = b[c,j,k]
    } else {
      int64_t t = (k * C + c) * pitch + i;     // transpose of position (i, k)
      st(a_op + t, vb);   // A[i][c][k] = b[c,k,i]
      st(b_op + t, va);   // B[j][c][k] = a[c,k,j]
    }
  }
}

// P[c][i][j] = sum_k A[c][i][k] B[c][j][k] (batched over c through blockIdx.z).
template <typename T>
__global__ void __launch_bounds__(256) k_contract(const T* __restrict__ A, const T* __restrict__ B,
                                                  T* __restrict__ P, int64_t rows, int64_t cols,
                                                  int64_t K) {
  __shared__ float As[GK][GM + 4];
  __shared__ float Bs[GK][GN + 4];
  const int64_t c = blockIdx.z, C = gridDim.z;
  const int64_t kp = pair_pitch(K), cp = pair_pitch(cols);
  // operands [row][channel][pitch]: row r of channel c starts at (r * C + c) * pitch
  const T* Ab = A + c * kp;
  const T* Bb = B + c * kp;
  T* Pb = P + c * cp;
  const int tid = threadIdx.x, tm = tid / 16, tn = tid % 16;
  const int64_t m0 = (int64_t)blockIdx.y * GM, n0 = (int64_t)blockIdx.x * GN;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += GK) {
    for (int e = tid; e < GM * GK; e += 256) {
      int r = e / GK, kk = e % GK;
      As[kk][r] = (m0 + r < rows && k0 + kk < K) ? ld(Ab + (m0 + r) * C * kp + k0 + kk) : 0.f;
      Bs[kk][r] = (n0 + r < cols && k0 + kk < K) ? ld(Bb + (n0 + r) * C * kp + k0 + kk) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < GK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][tm * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tn * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t m = m0 + tm * 4 + i;
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t nn = n0 + tn * 4 + j;
      if (nn < cols) st(Pb + m * C * cp + nn, acc[i][j]);
    }
  }
}

// LayerNorm over the channel axis of a channel-major [C][M] tensor, written
// position-major [M][C] (the reference center_norm with dim=-3).
template <typename T>
__global__ void __launch_bounds__(256) k_center_ln(const T* __restrict__ p, T* __restrict__ y,
                                                   const float* __restrict__ w,
                                                   const float* __restrict__ b, int64_t M, int64_t n, int C,
                                                   float eps) {
  extern __shared__ float tile[];  // [C][33]
  __shared__ float mean_s[32], rstd_s[32];
  const int64_t m0 = (int64_t)blockIdx.x * 32;
  const int64_t pitch = pair_pitch(n);
  for (int e = threadIdx.x; e < C * 32; e += blockDim.x) {
    int c = e / 32, r = e % 32;
    const int64_t m = m0 + r;
    tile[c * 33 + r] = (m < M) ? ld(p + ((m / n) * C + c) * pitch + m % n) : 0.f;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    int r = threadIdx.x;
    float s = 0.f;
    for (int c = 0; c < C; ++c) s += tile[c * 33 + r];
    float mean = s / C, v = 0.f;
    for (int c = 0; c < C; ++c) {
      float d = tile[c * 33 + r] - mean;
      v += d * d;
    }
    mean_s[r] = mean;
    rstd_s[r] = rsqrtf(v / C + eps);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < C * 32; e += blockDim.x) {
    int r = e / C, c = e % C;
    if (m0 + r < M) st(y + (m0 + r) * C + c, (tile[c * 33 + r] - mean_s[r]) * rstd_s[r] * w[c] + b[c]);
  }
}

// 8 outputs per thread from 16-byte loads (I a multiple of 8, rows 16-byte aligned).
__global__ void k_swiglu_bf16x8(const bf16* __restrict__ h, bf16* __restrict__ out, int64_t rows, int64_t I) {
  const int64_t e8 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, per = I / 8;
  if (e8 >= rows * per) return;
  const int64_t r = e8 / per, i0 = (e8 - r * per) * 8;
  const uint4 av = __ldg(reinterpret_cast<const uint4*>(h + r * 2 * I + i0));
  const uint4 bv = __ldg(reinterpret_cast<const uint4*>(h + r * 2 * I + I + i0));
  const uint32_t au[4] = {av.x, av.y, av.z, av.w}, bu[4] = {bv.x, bv.y, bv.z, bv.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float a0 = __uint_as_float(au[j] << 16), a1 = __uint_as_float(au[j] & 0xffff0000u);
    const float b0 = __uint_as_float(bu[j] << 16), b1 = __uint_as_float(bu[j] & 0xffff0000u);
    const __nv_bfloat162 v = __floats2bfloat162_rn(swish_f(a0) * b0, swish_f(a1) * b1);
    o[j] = *reinterpret_cast<const uint32_t*>(&v);
  }
  *reinterpret_cast<uint4*>(out + r * I + i0) = make_uint4(o[0], o[1], o[2], o[3]);
}


template <typename T>
__global__ void k_swiglu(const float* __restrict__ h, T* __restrict__ out, int64_t rows, int64_t I) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= rows * I) return;
  int64_t r = e / I, i = e % I;
  const float* hr = h + r * 2 * I;
  st(out + e, swish_f(hr[i]) * hr[I + i]);
}

// ---- workspace layouts --------------------------------------------------------
template <typename T>
struct TriMultProjectWs {
  T* x;
  float* y;
  template <typename WS>
  void carve(WS& ws, int64_t n, int64_t C) {
    x = ws.template take<T>(n * n * C);
    y = ws.template take<float>(n * n * 4 * C);
  }
};

}  // namespace sf

using namespace sf;

static size_t dsize(int dtype) { return dtype == SF_F32 ? 4 : 2; }


template <typename F>
static size_t ws_of(F f) {
  WorkspaceSize w;
  f(w);
  return w.used;
}

extern "C" {

int64_t sf_pair_pitch(int64_t n) { return pair_pitch(n); }

// ---- phases of the row-sharded path (bf16 only) ---------------------------------
#define SF_REQUIRE_BF16(dtype, what) SF_REQUIRE((dtype) == SF_BF16, what ": the sharded path is bf16 only")

int sf_tri_mult_project_rows(int dtype, const void* z, const uint8_t* mask, int64_t rows, int64_t n,
                             int64_t row_offset, int incoming, const sf_tri_mult_weights* w, void* a_op, void* b_op,
                             sf_stream_t stream) {
  SF_REQUIRE_BF16(dtype, "sf_tri_mult_project_rows");
  SF_REQUIRE(z && mask && w && a_op && b_op && rows >= 0 && n > 0 && row_offset >= 0,
             "sf_tri_mult_project_rows: bad arguments");
  const int64_t pitch = pair_pitch(incoming ? rows : n), nrow = incoming ? n : rows;
  if (pitch != (incoming ? rows : n)) {
    const size_t bytes = (size_t)nrow * 128 * pitch * 2;
    if (cudaMemsetAsync(a_op, 0, bytes, stream) != cudaSuccess || cudaMemsetAsync(b_op, 0, bytes, stream) != cudaSuccess)
      return check_launch("sf_tri_mult_project_rows.memset");
  }
  return trimul_project_tc((const bf16*)z, mask, rows, n, row_offset, incoming, w->ln_w, w->ln_b,
                           (const bf16*)w->w_glu, (bf16*)a_op, (bf16*)b_op, stream);
}

int sf_tri_mult_contract_chunked(int dtype, const void* a_op, int64_t chunks_a, const void* b_op, int64_t chunks_b,
                                 void* p, int64_t channels, int64_t rows, int64_t cols, int64_t kdim,
                                 sf_stream_t stream) {
  SF_REQUIRE_BF16(dtype, "sf_tri_mult_contract_chunked");
  SF_REQUIRE(a_op && b_op && p && channels > 0 && rows >= 0 && cols >= 0 && kdim > 0,
             "sf_tri_mult_contract_chunked: bad arguments");
  return contract_chunked_tc((const bf16*)a_op, chunks_a, (const bf16*)b_op, chunks_b, (bf16*)p, channels, rows, cols,
                             kdim, stream);
}

int64_t sf_tri_attention_query_pitch(int64_t nq) { return triatt_query_pitch(nq); }

int sf_tri_attention_bias(int dtype, const void* z, int64_t rows, int64_t n, const sf_tri_attention_weights* w,
                          void* bias, int64_t ldb, sf_stream_t stream) {
  SF_REQUIRE_BF16(dtype, "sf_tri_attention_bias");
  SF_REQUIRE(z && w && bias && w->heads == 4, "sf_tri_attention_bias: bad arguments");
  return triatt_bias_tc((const bf16*)z, rows, n, w->ln_w, (const bf16*)w->w_bias, (bf16*)bias, ldb, stream);
}

int sf_tri_attention_project(int dtype, const void* z, int64_t rows, int64_t cols, int transpose, int compute_bias,
                             const sf_tri_attention_weights* w, void* q, void* k, void* vt, void* g, void* bias,
                             sf_stream_t stream) {
  SF_REQUIRE_BF16(dtype, "sf_tri_attention_project");
  SF_REQUIRE(z && w && q && k && vt && g && (bias || !compute_bias) && w->heads == 4,
             "sf_tri_attention_project: bad arguments");
  return triatt_project_tc((const bf16*)z, rows, cols, transpose, compute_bias, w->ln_w, (const bf16*)w->w_qkvg,
                           (const bf16*)w->w_bias, (bf16*)q, (bf16*)k, (bf16*)vt, (bf16*)g, (bf16*)bias, stream);
}

int sf_tri_attention_core(int dtype, const void* q, const void* k, const void* vt, const void* g, const void* bias,
                          const uint8_t* mask, const void* z, void* z_out, int64_t rows, int64_t cols, int transpose,
                          int64_t batch_offset, const sf_tri_attention_weights* w, sf_stream_t stream) {
  SF_REQUIRE_BF16(dtype, "sf_tri_attention_core");
  SF_REQUIRE(q && k && vt && g && bias && mask && z && z_out && w && w->heads == 4, "sf_tri_attention_core: bad arguments");
  return triatt_core_tc((const bf16*)q, (const bf16*)k, (const bf16*)vt, (const bf16*)g, (const bf16*)bias,
                        (const bf16*)w->w_out, mask, (const bf16*)z, (bf16*)z_out, rows, cols, transpose, batch_offset,
                        stream);
}

// ---------------------------------------------------------------------------
int sf_layernorm(int dtype, const void* x, void* y, const float* weight, const float* bias,
                 int64_t rows, int64_t cols, float eps, sf_stream_t stream) {
  SF_REQUIRE(x && y && rows >= 0 && cols > 0, "sf_layernorm: bad arguments");
  SF_DISPATCH(dtype, {
    return launch_layernorm((const T*)x, (T*)y, weight, bias, rows, (int)cols, eps, stream);
  });
}

int sf_linear(int dtype, const void* x, const void* wt, const float* bias, const void* residual,
              void* y, int64_t rows, int64_t k, int64_t n, int post_op, sf_stream_t stream) {
  SF_REQUIRE(x && wt && y && rows >= 0 && k > 0 && n > 0, "sf_linear: bad arguments");
  SF_REQUIRE(post_op >= SF_POST_NONE && post_op <= SF_POST_SIGMOID, "sf_linear: bad post_op %d", post_op);
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(wt) |
                         reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(residual)) & 15) == 0;
  if (dtype == SF_BF16 && k % 8 == 0 && n % 8 == 0 && aligned && rows > 0)
    return linear_tc((const bf16*)x, (const bf16*)wt, bias, (const bf16*)residual, (bf16*)y, rows, k, n, post_op,
                     stream);
  SF_DISPATCH(dtype, {
    EpiLinear<T> epi{(T*)y, bias, (const T*)residual, n, post_op};
    return launch_gemm(rows, (int)n, (int)k, RowMajor<T>{(const T*)x, k}, (const T*)wt, epi, stream, "sf_linear");
  });
}

int sf_attention(const sf_attention_args* a, sf_stream_t stream) {
  SF_REQUIRE(a && a->q && a->k && a->v && a->out, "sf_attention: null tensor");
  SF_REQUIRE(a->head_dim > 0 && a->head_dim <= ATT_DMAX, "sf_attention: head_dim %lld outside (0, %d]",
             (long long)a->head_dim, ATT_DMAX);
  SF_REQUIRE(a->value_dim >= 0 && a->value_dim <= ATT_DMAX, "sf_attention: value_dim %lld outside [0, %d]",
             (long long)a->value_dim, ATT_DMAX);
  const int dv = a->value_dim > 0 ? (int)a->value_dim : (int)a->head_dim;
  SF_REQUIRE(a->batch >= 0 && a->heads > 0 && a->q_len >= 0 && a->k_len >= 0, "sf_attention: bad sizes");
  SF_REQUIRE(a->batch <= 65535 && a->heads <= 65535, "sf_attention: batch/heads exceed grid limits");
  if (a->batch == 0 || a->q_len == 0) return SF_OK;
  SF_REQUIRE(a->k_len > 0, "sf_attention: k_len must be positive");
  SF_REQUIRE(!a->bias || a->bias_dtype == SF_F32 || a->bias_dtype == a->dtype, "sf_attention: bias dtype");
  SF_REQUIRE((a->q_len + ATT_QB - 1) / ATT_QB <= 0x7fffffff, "sf_attention: q_len too large");
  {
    const int st = attention_tc(a, stream);   // bf16, head dim <= 64: the tensor-core kernel
    if (st != SF_ERR_ARG) return st;
  }
  dim3 grid((unsigned)((a->q_len + ATT_QB - 1) / ATT_QB), (unsigned)a->heads, (unsigned)a->batch);
  const size_t smem = attention_smem_bytes((int)a->head_dim, dv);
  SF_DISPATCH(a->dtype, {
    const bool f32bias = a->bias && a->bias_dtype == SF_F32;
    using K = void (*)(sf_attention_args);
    // compile-time head dims for the common sizes; the generic kernel takes any D <= 64
    const int hd = (int)a->head_dim;
    const int di = dv != hd ? 5 : hd == 16 ? 0 : hd == 24 ? 1 : hd == 32 ? 2 : hd == 48 ? 3 : hd == 64 ? 4 : 5;
    static const K kerns[2][6] = {
        {k_attention<T, T, 16, 16>, k_attention<T, T, 24, 24>, k_attention<T, T, 32, 32>,
         k_attention<T, T, 48, 48>, k_attention<T, T, 64, 64>, k_attention<T, T, 0, 64>},
        {k_attention<T, float, 16, 16>, k_attention<T, float, 24, 24>, k_attention<T, float, 32, 32>,
         k_attention<T, float, 48, 48>, k_attention<T, float, 64, 64>, k_attention<T, float, 0, 64>}};
    K kern = kerns[f32bias ? 1 : 0][di];
    static bool attr_done[64][2][6] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev & 63][f32bias ? 1 : 0][di]) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attention_smem_bytes(64, 64));
      attr_done[dev & 63][f32bias ? 1 : 0][di] = true;
    }
    kern<<<grid, ATT_NS * 32, smem, stream>>>(*a);
    count_launch();
    return check_launch("sf_attention");
  });
}

// ---------------------------------------------------------------------------
size_t sf_tri_mult_project_workspace(int dtype, int64_t n) {
  const int64_t C = 128;
  WorkspaceSize w;
  w.used = 0;
  size_t ds = dsize(dtype);
  w.used = align_up(0, 256) + n * n * C * ds;
  w.take<float>(n * n * 4 * C);
  return w.used;
}

int sf_tri_mult_project(int dtype, const void* z, const uint8_t* mask, int64_t n, int incoming,
                        const sf_tri_mult_weights* w, void* a_op, void* b_op, void* ws_p,
                        size_t ws_bytes, sf_stream_t stream) {
  const int64_t C = 128;
  SF_REQUIRE(z && mask && w && a_op && b_op && n > 0, "sf_tri_mult_project: bad arguments");
  SF_REQUIRE(w->ln_w && w->ln_b && w->w_glu, "sf_tri_mult_project: missing weights");
  if (ws_bytes < sf_tri_mult_project_workspace(dtype, n)) {
    set_error("sf_tri_mult_project: workspace %zu < %zu", ws_bytes, sf_tri_mult_project_workspace(dtype, n));
    return SF_ERR_WORKSPACE;
  }
  if (pair_pitch(n) != n) {  // zero the row padding the contraction reads as K
    const size_t bytes = (size_t)C * n * pair_pitch(n) * dsize(dtype);
    if (cudaMemsetAsync(a_op, 0, bytes, stream) != cudaSuccess || cudaMemsetAsync(b_op, 0, bytes, stream) != cudaSuccess)
      return check_launch("tri_mult_project.memset");
  }
  if (dtype == SF_BF16)
    return trimul_project_tc((const bf16*)z, mask, n, n, 0, incoming, w->ln_w, w->ln_b, (const bf16*)w->w_glu,
                             (bf16*)a_op, (bf16*)b_op, stream);
  SF_DISPATCH(dtype, {
    Workspace ws(ws_p, ws_bytes);
    T* x = ws.take<T>(n * n * C);
    float* y = ws.take<float>(n * n * 4 * C);
    SF_TRY(launch_layernorm((const T*)z, x, w->ln_w, w->ln_b, n * n, (int)C, 1e-5f, stream));
    SF_TRY(launch_gemm(n * n, (int)(4 * C), (int)C, RowMajor<T>{x, C}, (const T*)w->w_glu,
                       EpiStore<float>{y, 4 * C}, stream, "tri_mult_project.gemm"));
    dim3 grid((unsigned)((n * n + 31) / 32), (unsigned)(C / 32));
    k_tri_glu_scatter<T><<<grid, dim3(32, 8), 0, stream>>>(y, mask, n, pair_pitch(n), (int)C, incoming, (T*)a_op,
                                                           (T*)b_op);
    count_launch();
    return check_launch("tri_mult_project.scatter");
  });
}

int sf_tri_mult_contract(int dtype, const void* a_op, const void* b_op, void* p, int64_t channels,
                         int64_t rows, int64_t cols, int64_t kdim, sf_stream_t stream) {
  SF_REQUIRE(a_op && b_op && p && channels > 0 && rows >= 0 && cols >= 0 && kdim > 0,
             "sf_tri_mult_contract: bad arguments");
  SF_REQUIRE(channels <= 65535, "sf_tri_mult_contract: too many channels");
  if (rows == 0 || cols == 0) return SF_OK;
  if (dtype == SF_BF16)
    return contract_tc((const bf16*)a_op, (const bf16*)b_op, (bf16*)p, channels, rows, cols, kdim, stream);
  SF_DISPATCH(dtype, {
    dim3 grid((unsigned)((cols + GN - 1) / GN), (unsigned)((rows + GM - 1) / GM), (unsigned)channels);
    k_contract<T><<<grid, 256, 0, stream>>>((const T*)a_op, (const T*)b_op, (T*)p, rows, cols, kdim);
    count_launch();
    return check_launch("tri_mult_contract");
  });
}

size_t sf_tri_mult_output_workspace(int dtype, int64_t rows, int64_t n) {
  const int64_t C = 128;
  size_t ds = dsize(dtype);
  size_t used = rows * n * C * ds;                           // x
  used = align_up(used, 256) + rows * n * C * ds;            // yhat
  used = align_up(used, 256) + rows * n * C * sizeof(float); // gate logits
  return used;
}

int sf_tri_mult_output(int dtype, const void* z, const void* p, int64_t rows, int64_t n,
                       const sf_tri_mult_weights* w, void* z_out, void* ws_p, size_t ws_bytes,
                       sf_stream_t stream) {
  const int64_t C = 128;
  SF_REQUIRE(z && p && w && z_out && rows >= 0 && n > 0, "sf_tri_mult_output: bad arguments");
  SF_REQUIRE(w->center_w && w->center_b && w->w_out && w->w_gate && w->ln_w && w->ln_b,
             "sf_tri_mult_output: missing weights");
  if (rows == 0) return SF_OK;
  if (dtype == SF_BF16)   // the tcgen05 path needs no workspace
    return trimul_output_tc((const bf16*)z, (const bf16*)p, rows, n, w->ln_w, w->ln_b, w->center_w, w->center_b,
                            (const bf16*)w->w_gate, (const bf16*)w->w_out, (bf16*)z_out, stream);
  if (ws_bytes < sf_tri_mult_output_workspace(dtype, rows, n)) {
    set_error("sf_tri_mult_output: workspace too small");
    return SF_ERR_WORKSPACE;
  }
  SF_DISPATCH(dtype, {
    Workspace ws(ws_p, ws_bytes);
    const int64_t M = rows * n;
    T* x = ws.take<T>(M * C);
    T* yh = ws.take<T>(M * C);
    float* g = ws.take<float>(M * C);
    SF_TRY(launch_layernorm((const T*)z, x, w->ln_w, w->ln_b, M, (int)C, 1e-5f, stream));
    k_center_ln<T><<<(unsigned)((M + 31) / 32), 256, C * 33 * sizeof(float), stream>>>(
        (const T*)p, yh, w->center_w, w->center_b, M, n, (int)C, 1e-5f);
    count_launch();
    SF_TRY(check_launch("tri_mult_output.center_ln"));
    SF_TRY(launch_gemm(M, (int)C, (int)C, RowMajor<T>{x, C}, (const T*)w->w_gate, EpiStore<float>{g, C},
                       stream, "tri_mult_output.gate"));
    return launch_gemm(M, (int)C, (int)C, RowMajor<T>{yh, C}, (const T*)w->w_out,
                       EpiGatedResidual<T>{(const T*)z, g, (T*)z_out, C}, stream, "tri_mult_output.out");
  });
}

// ---------------------------------------------------------------------------
size_t sf_tri_attention_workspace(int dtype, int64_t n, int64_t heads) {
  const int64_t C = 128;
  if (dtype == SF_BF16 && heads == 4) return triatt_tc_workspace(n);
  size_t ds = dsize(dtype);
  size_t used = n * n * C * ds;                                  // x
  used = align_up(used, 256) + heads * n * n * sizeof(float);    // bias
  used = align_up(used, 256) + n * n * 4 * C * ds;               // q k v g
  used = align_up(used, 256) + n * n * C * ds;                   // gated attention output
  return used;
}

int sf_tri_attention(int dtype, const void* z, const uint8_t* mask, int64_t n, int transpose,
                     const sf_tri_attention_weights* w, void* z_out, void* ws_p, size_t ws_bytes,
                     sf_stream_t stream) {
  const int64_t C = 128;
  SF_REQUIRE(z && mask && w && z_out && n > 0, "sf_tri_attention: bad arguments");
  SF_REQUIRE(w->ln_w && w->w_qkvg && w->w_bias && w->w_out, "sf_tri_attention: missing weights");
  SF_REQUIRE(w->heads > 0 && C % w->heads == 0 && C / w->heads <= ATT_DMAX, "sf_tri_attention: heads");
  SF_REQUIRE(n <= 65535, "sf_tri_attention: n too large for this kernel");
  if (ws_bytes < sf_tri_attention_workspace(dtype, n, w->heads)) {
    set_error("sf_tri_attention: workspace too small");
    return SF_ERR_WORKSPACE;
  }
  const int64_t H = w->heads, D = C / H, M = n * n;
  if (dtype == SF_BF16 && H == 4)
    return triatt_tc((const bf16*)z, mask, n, transpose, w->ln_w, (const bf16*)w->w_qkvg, (const bf16*)w->w_bias,
                     (const bf16*)w->w_out, (bf16*)z_out, ws_p, ws_bytes, stream);
  SF_DISPATCH(dtype, {
    Workspace ws(ws_p, ws_bytes);
    T* x = ws.take<T>(M * C);
    float* bias = ws.take<float>(H * M);
    T* y = ws.take<T>(M * 4 * C);
    T* o = ws.take<T>(M * C);
    SF_TRY(launch_layernorm((const T*)z, x, w->ln_w, (const float*)nullptr, M, (int)C, 1e-5f, stream));
    SF_TRY(launch_gemm(M, (int)H, (int)C, RowMajor<T>{x, C}, (const T*)w->w_bias, EpiColMajor<float>{bias, M},
                       stream, "tri_attention.bias"));
    if (transpose)
      SF_TRY(launch_gemm(M, (int)(4 * C), (int)C, PairTransposed<T>{x, n, C}, (const T*)w->w_qkvg,
                         EpiStore<T>{y, 4 * C}, stream, "tri_attention.qkvg"));
    else
      SF_TRY(launch_gemm(M, (int)(4 * C), (int)C, RowMajor<T>{x, C}, (const T*)w->w_qkvg,
                         EpiStore<T>{y, 4 * C}, stream, "tri_attention.qkvg"));
    sf_attention_args a{};
    a.dtype = dtype;
    a.batch = n; a.heads = H; a.q_len = n; a.k_len = n; a.head_dim = D;
    a.q = y;         a.q_sb = n * 4 * C; a.q_sh = D; a.q_sq = 4 * C;
    a.k = y + C;     a.k_sb = n * 4 * C; a.k_sh = D; a.k_sk = 4 * C;
    a.v = y + 2 * C; a.v_sb = n * 4 * C; a.v_sh = D; a.v_sk = 4 * C;
    a.gate = y + 3 * C; a.g_sb = n * 4 * C; a.g_sh = D; a.g_sq = 4 * C;
    a.out = o;       a.o_sb = n * C; a.o_sh = D; a.o_sq = C;
    a.bias = bias; a.bias_dtype = SF_F32; a.b_sb = 0; a.b_sh = M; a.b_sq = n;
    a.mask_k = mask; a.mk_sb = 0; a.mask_row = mask;
    a.scale = 1.0f / sqrtf((float)D);
    SF_TRY(sf_attention(&a, stream));
    return launch_gemm(M, (int)C, (int)C, RowMajor<T>{o, C}, (const T*)w->w_out,
                       EpiPairResidual<T>{(const T*)z, (T*)z_out, n, C, transpose}, stream,
                       "tri_attention.out");
  });
}

// ---------------------------------------------------------------------------
size_t sf_transition_workspace(int dtype, int64_t rows, int64_t inter) {
  // x is normalised into the workspace (c <= inter always holds for factor >= 1)
  size_t ds = dsize(dtype);
  size_t used = rows * inter * ds;                                   // LN(x) (c <= inter)
  used = align_up(used, 256) + rows * 2 * inter * sizeof(float);     // h1
  used = align_up(used, 256) + rows * inter * ds;                    // swiglu
  return used;
}

int sf_transition(int dtype, const void* x, const float* ln_w, const float* ln_b, const void* w1,
                  const void* w2, void* y, int64_t rows, int64_t c, int64_t inter, void* ws_p,
                  size_t ws_bytes, sf_stream_t stream) {
  SF_REQUIRE(x && ln_w && ln_b && w1 && w2 && y && rows >= 0 && c > 0 && inter >= c,
             "sf_transition: bad arguments");
  if (ws_bytes < sf_transition_workspace(dtype, rows, inter)) {
    set_error("sf_transition: workspace too small");
    return SF_ERR_WORKSPACE;
  }
  if (rows == 0) return SF_OK;
  if (dtype == SF_BF16 && c == 128 && inter == 512)   // the pair transition runs on tcgen05
    return transition_tc((const bf16*)x, ln_w, ln_b, (const bf16*)w1, (const bf16*)w2, (bf16*)y, rows, stream);
  if (dtype == SF_BF16 && c % 8 == 0 && inter % 8 == 0 &&
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(w1) |
        reinterpret_cast<uintptr_t>(w2) | reinterpret_cast<uintptr_t>(ws_p)) & 15) == 0) {
    // other widths (the single transition): LN -> tcgen05 GEMM -> SwiGLU -> tcgen05 GEMM + residual
    Workspace ws(ws_p, ws_bytes);
    bf16* xn = ws.take<bf16>(rows * inter);
    bf16* h1 = ws.take<bf16>(rows * 2 * inter);
    bf16* h = ws.take<bf16>(rows * inter);
    SF_TRY(launch_layernorm((const bf16*)x, xn, ln_w, ln_b, rows, (int)c, 1e-5f, stream));
    SF_TRY(linear_tc(xn, (const bf16*)w1, nullptr, nullptr, h1, rows, c, 2 * inter, SF_POST_NONE, stream));
    const int64_t tot8 = rows * (inter / 8);   // inter % 8 == 0 and 16-byte aligned buffers on this path
    k_swiglu_bf16x8<<<(unsigned)((tot8 + 255) / 256), 256, 0, stream>>>(h1, h, rows, inter);
    count_launch();
    SF_TRY(check_launch("transition.swiglu"));
    return linear_tc(h, (const bf16*)w2, nullptr, (const bf16*)x, (bf16*)y, rows, inter, c, SF_POST_NONE, stream);
  }
  SF_DISPATCH(dtype, {
    Workspace ws(ws_p, ws_bytes);
    T* xn = ws.take<T>(rows * inter);
    float* h1 = ws.take<float>(rows * 2 * inter);
    T* h = ws.take<T>(rows * inter);
    SF_TRY(launch_layernorm((const T*)x, xn, ln_w, ln_b, rows, (int)c, 1e-5f, stream));
    SF_TRY(launch_gemm(rows, (int)(2 * inter), (int)c, RowMajor<T>{xn, c}, (const T*)w1,
                       EpiStore<float>{h1, 2 * inter}, stream, "transition.w1"));
    int64_t tot = rows * inter;
    k_swiglu<T><<<(unsigned)((tot + 255) / 256), 256, 0, stream>>>(h1, h, rows, inter);
    count_launch();
    SF_TRY(check_launch("transition.swiglu"));
    return launch_gemm(rows, (int)c, (int)inter, RowMajor<T>{h, inter}, (const T*)w2,
                       EpiResidual<T>{(const T*)x, (T*)y, c}, stream, "transition.w2");
  });
}

// ---------------------------------------------------------------------------
size_t sf_pair_logits_workspace(int dtype, int64_t rows, int64_t n, int64_t c) {
  return rows * n * c * dsize(dtype);
}

int sf_pair_logits(int dtype, const void* z, const float* ln_w, const float* ln_b, const void* w,
                   void* logits, int64_t rows, int64_t n, int64_t c, int64_t heads, void* ws_p,
                   size_t ws_bytes, sf_stream_t stream) {
  SF_REQUIRE(z && ln_w && ln_b && w && logits && rows >= 0 && n > 0 && c > 0 && heads > 0,
             "sf_pair_logits: bad arguments");
  if (ws_bytes < sf_pair_logits_workspace(dtype, rows, n, c)) {
    set_error("sf_pair_logits: workspace too small");
    return SF_ERR_WORKSPACE;
  }
  if (rows == 0) return SF_OK;
  if (dtype == SF_BF16 && c == 128 && heads <= 16) {
    return pair_logits_tc((const bf16*)z, ln_w, ln_b, (const bf16*)w, (bf16*)logits, rows * n, (int)heads, stream);
  }
  SF_DISPATCH(dtype, {
    T* x = (T*)ws_p;
    const int64_t M = rows * n;
    SF_TRY(launch_layernorm((const T*)z, x, ln_w, ln_b, M, (int)c, 1e-5f, stream));
    return launch_gemm(M, (int)heads, (int)c, RowMajor<T>{x, c}, (const T*)w, EpiColMajor<T>{(T*)logits, M},
                       stream, "pair_logits");
  });
}

}  // extern "C"
