// Auxiliary kernels of the diffusion and MSA ops: adaptive LayerNorm, gated
// residual, masked row gather (atom layout), row masking, masked row softmax,
// batched 2-D transposes, and the outer-product-mean helpers.  All are
// bandwidth-bound CUDA-core kernels; fp32 arithmetic, fp32 or bf16 storage.
#include <cfloat>

#include "sf_simt.cuh"

namespace sf {
namespace {

// y = scale * LayerNorm(x) + bias (no affine in the norm itself): the
// single_cond branch of AdaptiveLayerNorm (diffusion/transformer.py:85-93).
template <typename T>
__global__ void k_adaln(const T* __restrict__ x, const T* __restrict__ scale, const T* __restrict__ bias,
                        T* __restrict__ y, int64_t rows, int cols, int64_t cond_rows, float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * cols;
  float s = 0.f;
  for (int c = lane; c < cols; c += 32) s += ld(xr + c);
  const float mean = warp_sum(s) / cols;
  float v = 0.f;
  for (int c = lane; c < cols; c += 32) {
    const float d = ld(xr + c) - mean;
    v += d * d;
  }
  const float rstd = rsqrtf(warp_sum(v) / cols + eps);
  const int64_t cr = (row % cond_rows) * cols;   // scale and bias repeat every cond_rows rows
  for (int c = lane; c < cols; c += 32) {
    // the reference rounds LN(x) and the scale/bias to the activation dtype first
    const float xn = ld_round<T>((ld(xr + c) - mean) * rstd);
    st(y + row * cols + c, ld(scale + cr + c) * xn + ld(bias + cr + c));
  }
}

// out = base + u * gate (base may be null)
template <typename T>
__global__ void k_gated_residual(const T* __restrict__ base, const T* __restrict__ u, const T* __restrict__ gate,
                                 T* __restrict__ out, int64_t n, int64_t gate_period) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const float v = ld(u + e) * ld(gate + e % gate_period);
  st(out + e, base ? ld(base + e) + v : v);
}

// Strided block copy in 16-byte units: block b, row r, chunk c of dst <- the same of src,
// with independent block and row strides (the row-shard <-> column-shard packing of the pair
// tensor around the all-to-all of the ending-node attention).
__global__ void k_copy_blocks(uint4* __restrict__ dst, const uint4* __restrict__ src, int64_t nblk, int64_t rows,
                              int64_t width, int64_t sbs, int64_t srs, int64_t dbs, int64_t drs) {
  const int64_t per_blk = rows * width, total = nblk * per_blk;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = e / per_blk, rem = e - b * per_blk, r = rem / width, c = rem - r * width;
    dst[b * dbs + r * drs + c] = __ldg(src + b * sbs + r * srs + c);
  }
}

// out[b][i][:] = mask[i] ? src[b][idx[i]][:] : 0   (atom_layout.convert, schema/atom_layout.py:52-83)
template <typename T>
__global__ void k_gather_rows(const T* __restrict__ src, const int32_t* __restrict__ idx,
                              const uint8_t* __restrict__ mask, T* __restrict__ out, int64_t src_rows, int64_t n_out,
                              int cols) {
  const int64_t b = blockIdx.y;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_out * cols; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / cols;
    const int c = (int)(e % cols);
    const int32_t j = idx[i];
    const bool ok = mask[i] && j >= 0 && j < src_rows;
    st(out + (b * n_out + i) * cols + c, ok ? ld(src + (b * src_rows + j) * cols + c) : 0.f);
  }
}

// x[r][:] *= mask[r]
template <typename T>
__global__ void k_mask_rows(T* __restrict__ x, const uint8_t* __restrict__ mask, int64_t rows, int cols) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= rows * cols) return;
  if (!mask[e / cols]) st(x + e, 0.f);
}

}  // namespace
}  // namespace sf

namespace sf {
namespace {

// softmax over the last axis with an optional additive per-key bias:
// the pair-weighted averaging weights of MSAAttention (trunk/blocks.py:163-170).
template <typename T>
__global__ void k_softmax_rows(const T* __restrict__ x, const float* __restrict__ key_bias, T* __restrict__ y,
                               int64_t rows, int K, int64_t ldy) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * K;
  float m = -INFINITY;
  for (int k = lane; k < K; k += 32) m = fmaxf(m, ld_round<T>(ld(xr + k) + (key_bias ? key_bias[k] : 0.f)));
  m = warp_max(m);
  float s = 0.f;
  for (int k = lane; k < K; k += 32) s += expf(ld_round<T>(ld(xr + k) + (key_bias ? key_bias[k] : 0.f)) - m);
  const float inv = 1.0f / warp_sum(s);
  for (int k = lane; k < K; k += 32)
    st(y + row * ldy + k, expf(ld_round<T>(ld(xr + k) + (key_bias ? key_bias[k] : 0.f)) - m) * inv);
}

// Batched strided transpose: out[ob(b) + c*os_c + r] = in[ib(b) + r*is_r + c],
// b = (b1, b2), ib(b) = b1*ib1 + b2*ib2, ob(b) = b1*ob1 + b2*ob2; 32x32 tiles.
template <typename T>
__global__ void k_transpose(const T* __restrict__ in, T* __restrict__ out, int nb2, int64_t R, int64_t Cc,
                            int64_t ib1, int64_t ib2, int64_t is_r, int64_t ob1, int64_t ob2, int64_t os_c) {
  __shared__ float t[32][33];
  const int64_t b1 = blockIdx.z / nb2, b2 = blockIdx.z % nb2;
  const T* ip = in + b1 * ib1 + b2 * ib2;
  T* op = out + b1 * ob1 + b2 * ob2;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    t[i][threadIdx.x] = (r < R && c < Cc) ? ld(ip + r * is_r + c) : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < Cc) st(op + c * os_c + r, t[threadIdx.x][i]);
  }
}

// Column masks bit-packed: bits[i][w] bit e = mask[32w + e][i]  (mask [M][N] uint8).
__global__ void k_pack_mask_columns(const uint8_t* __restrict__ mask, uint32_t* __restrict__ bits, int64_t M,
                                    int64_t N, int64_t words) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= N * words) return;
  const int64_t i = e / words, w = e % words;
  uint32_t v = 0;
  for (int b = 0; b < 32; ++b) {
    const int64_t m = w * 32 + b;
    if (m < M && mask[m * N + i]) v |= 1u << b;
  }
  bits[e] = v;
}

// norm[i][j] = 1 / (1e-3 + count), count = sum_m mask[m,i] mask[m,j].  The
// reference forms it from bf16 masks in bf16 arithmetic whatever the activation
// dtype (trunk/blocks.py:683-686): count, the sum with 1e-3 and the reciprocal
// are each rounded to bf16, and so are they here.
__global__ void k_opm_norm(const uint32_t* __restrict__ bits, float* __restrict__ norm, int64_t N, int64_t words) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= N * N) return;
  const int64_t i = e / N, j = e % N;
  int cnt = 0;
  for (int64_t w = 0; w < words; ++w) cnt += __popc(bits[i * words + w] & bits[j * words + w]);
  const float c = ld_round<bf16>((float)cnt);
  const float s = ld_round<bf16>(1e-3f + c);
  norm[e] = ld_round<bf16>(1.0f / s);
}

// outer-product block repack: out[(i*N + j)][a*D + b] = O[i*D + a][j*D + b]  (O row pitch `pitch`)
template <typename T>
__global__ void k_opm_repack(const T* __restrict__ O, T* __restrict__ out, int64_t N, int D, int64_t pitch) {
  const int64_t total = N * N * D * D;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ij = e / (D * D);
    const int ab = (int)(e % (D * D));
    const int64_t i = ij / N, j = ij % N;
    const int a = ab / D, b = ab % D;
    out[e] = O[(i * D + a) * pitch + j * D + b];
  }
}

// x[r][:] *= s[r]
template <typename T>
__global__ void k_scale_rows(T* __restrict__ x, const float* __restrict__ s, int64_t rows, int cols) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= rows * cols) return;
  st(x + e, ld(x + e) * s[e / cols]);
}

// out[r][i] = swish(h[r][i]) * h[r][I + i]  (GatedLinearUnit with Swish, layers/primitives.py:624-631)
template <typename T>
__global__ void k_swiglu_any(const T* __restrict__ h, T* __restrict__ out, int64_t rows, int64_t I) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= rows * I) return;
  const int64_t r = e / I, i = e % I;
  st(out + e, swish_f(ld(h + r * 2 * I + i)) * ld(h + r * 2 * I + I + i));
}

inline unsigned blocks_for(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

int sf_adaln(int dtype, const void* x, const void* scale, const void* bias, void* y, int64_t rows, int64_t cols,
             int64_t cond_rows, sf_stream_t stream) {
  SF_REQUIRE(x && scale && bias && y && rows >= 0 && cols > 0 && cond_rows > 0 && rows % cond_rows == 0,
             "sf_adaln: bad arguments");
  if (rows == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    k_adaln<T><<<blocks_for(rows, 8), 256, 0, stream>>>((const T*)x, (const T*)scale, (const T*)bias, (T*)y, rows,
                                                        (int)cols, cond_rows, 1e-5f);
    count_launch();
    return check_launch("sf_adaln");
  });
}

int sf_gated_residual(int dtype, const void* base, const void* u, const void* gate, void* out, int64_t n,
                      int64_t gate_period, sf_stream_t stream) {
  SF_REQUIRE(u && gate && out && n >= 0 && gate_period > 0 && n % gate_period == 0,
             "sf_gated_residual: bad arguments");
  if (n == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    k_gated_residual<T><<<blocks_for(n), 256, 0, stream>>>((const T*)base, (const T*)u, (const T*)gate, (T*)out, n,
                                                           gate_period);
    count_launch();
    return check_launch("sf_gated_residual");
  });
}

int sf_gather_rows(int dtype, const void* src, int64_t batch, int64_t src_rows, const int32_t* idx,
                   const uint8_t* mask, int64_t n_out, int64_t cols, void* out, sf_stream_t stream) {
  SF_REQUIRE(src && idx && mask && out && batch >= 0 && src_rows >= 0 && n_out >= 0 && cols > 0,
             "sf_gather_rows: bad arguments");
  SF_REQUIRE(batch <= 65535, "sf_gather_rows: batch too large");
  if (batch == 0 || n_out == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    const int64_t tot = n_out * cols;
    dim3 grid(blocks_for(tot) < 4096u ? blocks_for(tot) : 4096u, (unsigned)batch);
    k_gather_rows<T><<<grid, 256, 0, stream>>>((const T*)src, idx, mask, (T*)out, src_rows, n_out, (int)cols);
    count_launch();
    return check_launch("sf_gather_rows");
  });
}

int sf_mask_rows(int dtype, void* x, const uint8_t* mask, int64_t rows, int64_t cols, sf_stream_t stream) {
  SF_REQUIRE(x && mask && rows >= 0 && cols > 0, "sf_mask_rows: bad arguments");
  if (rows == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    k_mask_rows<T><<<blocks_for(rows * cols), 256, 0, stream>>>((T*)x, mask, rows, (int)cols);
    count_launch();
    return check_launch("sf_mask_rows");
  });
}

int sf_softmax_rows(int dtype, const void* x, const float* key_bias, void* y, int64_t rows, int64_t k, int64_t ldy,
                    sf_stream_t stream) {
  SF_REQUIRE(x && y && rows >= 0 && k > 0 && ldy >= k, "sf_softmax_rows: bad arguments");
  if (rows == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    k_softmax_rows<T><<<blocks_for(rows, 8), 256, 0, stream>>>((const T*)x, key_bias, (T*)y, rows, (int)k, ldy);
    count_launch();
    return check_launch("sf_softmax_rows");
  });
}

int sf_transpose(int dtype, const void* in, void* out, int64_t nb1, int64_t nb2, int64_t rows, int64_t cols,
                 int64_t ib1, int64_t ib2, int64_t is_r, int64_t ob1, int64_t ob2, int64_t os_c, sf_stream_t stream) {
  SF_REQUIRE(in && out && nb1 >= 0 && nb2 > 0 && rows >= 0 && cols >= 0, "sf_transpose: bad arguments");
  SF_REQUIRE(nb1 * nb2 <= 65535, "sf_transpose: too many batches");
  if (nb1 == 0 || rows == 0 || cols == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)(nb1 * nb2));
    SF_REQUIRE((rows + 31) / 32 <= 65535, "sf_transpose: too many rows");
    k_transpose<T><<<grid, dim3(32, 8), 0, stream>>>((const T*)in, (T*)out, (int)nb2, rows, cols, ib1, ib2, is_r,
                                                      ob1, ob2, os_c);
    count_launch();
    return check_launch("sf_transpose");
  });
}

size_t sf_opm_norm_workspace(int64_t n_seq, int64_t n_res) { return (size_t)n_res * ((n_seq + 31) / 32) * 4; }

int sf_opm_norm(int dtype, const uint8_t* mask, int64_t n_seq, int64_t n_res, float* norm, void* ws, size_t ws_bytes,
                sf_stream_t stream) {
  SF_REQUIRE(mask && norm && n_seq >= 0 && n_res >= 0, "sf_opm_norm: bad arguments");
  if (n_res == 0) return SF_OK;
  if (ws_bytes < sf_opm_norm_workspace(n_seq, n_res)) {
    set_error("sf_opm_norm: workspace too small");
    return SF_ERR_WORKSPACE;
  }
  const int64_t words = (n_seq + 31) / 32;
  uint32_t* bits = static_cast<uint32_t*>(ws);
  k_pack_mask_columns<<<blocks_for(n_res * words), 256, 0, stream>>>(mask, bits, n_seq, n_res, words);
  count_launch();
  SF_TRY(check_launch("sf_opm_norm.pack"));
  (void)dtype;
  k_opm_norm<<<blocks_for(n_res * n_res), 256, 0, stream>>>(bits, norm, n_res, words);
  count_launch();
  return check_launch("sf_opm_norm");
}

int sf_opm_repack(int dtype, const void* o, int64_t pitch, int64_t n_res, int64_t d, void* out, sf_stream_t stream) {
  SF_REQUIRE(o && out && n_res >= 0 && d > 0 && pitch >= n_res * d, "sf_opm_repack: bad arguments");
  if (n_res == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    const int64_t tot = n_res * n_res * d * d;
    k_opm_repack<T><<<blocks_for(tot) < 65536u ? blocks_for(tot) : 65536u, 256, 0, stream>>>((const T*)o, (T*)out, n_res,
                                                                                           (int)d, pitch);
    count_launch();
    return check_launch("sf_opm_repack");
  });
}

int sf_swiglu(int dtype, const void* h, void* out, int64_t rows, int64_t inter, sf_stream_t stream) {
  SF_REQUIRE(h && out && rows >= 0 && inter > 0, "sf_swiglu: bad arguments");
  if (rows == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    k_swiglu_any<T><<<blocks_for(rows * inter), 256, 0, stream>>>((const T*)h, (T*)out, rows, inter);
    count_launch();
    return check_launch("sf_swiglu");
  });
}

int sf_copy_blocks(void* dst, const void* src, int64_t nblk, int64_t rows, int64_t width_bytes, int64_t src_blk_stride,
                   int64_t src_row_stride, int64_t dst_blk_stride, int64_t dst_row_stride, sf_stream_t stream) {
  SF_REQUIRE(dst && src && nblk >= 0 && rows >= 0 && width_bytes >= 0, "sf_copy_blocks: bad arguments");
  const int64_t all = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | width_bytes |
                      src_blk_stride | src_row_stride | dst_blk_stride | dst_row_stride;
  SF_REQUIRE((all & 15) == 0, "sf_copy_blocks: pointers, width and strides must be multiples of 16 bytes");
  const int64_t total = nblk * rows * (width_bytes / 16);
  if (total == 0) return SF_OK;
  const int64_t want = (total + 255) / 256;
  const unsigned grid = (unsigned)(want < 148 * 16 ? want : 148 * 16);
  k_copy_blocks<<<grid, 256, 0, stream>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src), nblk, rows,
                                          width_bytes / 16, src_blk_stride / 16, src_row_stride / 16,
                                          dst_blk_stride / 16, dst_row_stride / 16);
  count_launch();
  return check_launch("sf_copy_blocks");
}

int sf_scale_rows(int dtype, void* x, const float* s, int64_t rows, int64_t cols, sf_stream_t stream) {
  SF_REQUIRE(x && s && rows >= 0 && cols > 0, "sf_scale_rows: bad arguments");
  if (rows == 0) return SF_OK;
  SF_DISPATCH(dtype, {
    k_scale_rows<T><<<blocks_for(rows * cols), 256, 0, stream>>>((T*)x, s, rows, (int)cols);
    count_launch();
    return check_launch("sf_scale_rows");
  });
}

}  // extern "C"
