// Triangle attention (GridSelfAttention, blocks.py:270-366), bf16 track, on tcgen05.
//
// Two kernels per call:
//  k_triatt_project_tc  LN(z) (scale only, blocks.py:260-264) -> [q | k | v | gate]
//                       (one tcgen05 GEMM, N = 4 x 128) and the 4-head pair bias
//                       (CUDA-core dot products while the row is in registers).
//                       Tiles run along the query axis of the attention: a row
//                       tile for the starting node, a column tile for the ending
//                       node (transpose=True), so every store is contiguous.
//  k_triatt_core_tc     flash attention + gate + output projection + residual for
//                       one (attention row b, 128-query block): two softmax
//                       warpgroups each own two heads; S = Q K^T (M128 N64 K32)
//                       and O_blk = P V (M128 N32 K64) run on tcgen05 with TMEM
//                       accumulators, the online softmax runs in exp2 with the
//                       reference's -FLT_MAX masking, and the gated outputs of all
//                       four heads feed one more tcgen05 GEMM with the resident
//                       output projection, whose epilogue adds the residual.
//
// Intermediate layouts (qp = n rounded up to 128; padded query rows are zero):
//   Q, K  [b][h][qp][32]    Vt [b][h][32][qp]    G = sigmoid(gate) [b][qp][128]
//   bias  [q][h][qp] (bias[q][h][k] = LN(z)[q,k] . W_b[h], untransposed; rows q all-gathered
//         from the row shards when the pair tensor is distributed)
#include <cfloat>

#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int H = 4, D = 32;
constexpr float kLog2e = 1.4426950408889634f;   // the bias is stored pre-scaled by log2(e)

struct AttProjParams {
  const float* ln_w;      // act_norm scale [128]
  const bf16* w_qkvg;     // [512][128]
  const bf16* w_bias;     // [4][128]
  bf16 *q, *k, *vt, *g, *bias;
  int64_t rows, cols;     // the z block [rows][cols][128]
  int64_t nb, nq, qp;     // attention rows (batches), queries = keys, query pitch
  int transpose;          // attention along columns: batch = column, query = row
  int compute_bias;       // write bias[(r*H + h)*qp + s] for the block's positions (r, s)
  uint32_t* status;
};

constexpr int NOUT = 512;
constexpr int W_BYTES = NOUT * C * 2;
constexpr int VT_STAGE = D * TILE * 2;     // one head's V^T tile [32][128] bf16 (8 KB)
constexpr int SMEM_PROJ = 2 * A_BYTES + W_BYTES + VT_STAGE + 1024 + 1024;

// LayerNorm (scale only) of row r in place, returning the 4 pair-bias logits of
// the normalised (bf16-rounded) row.
__device__ __forceinline__ void ln_row_bias(uint8_t* tile, int r, const float* __restrict__ w,
                                            const bf16* __restrict__ wb, float (&bias)[H]) {
  uint4 v[16];
#pragma unroll
  for (int ka = 0; ka < 2; ++ka)
#pragma unroll
    for (int c = 0; c < 8; ++c) v[ka * 8 + c] = *reinterpret_cast<const uint4*>(tile + ka * ATOM + tc::sw128_off(r, c));
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
      const float d0 = bf_lo(u[j]) - mean, d1 = bf_hi(u[j]) - mean;
      q += d0 * d0 + d1 * d1;
    }
  }
  const float rstd = rsqrtf(q * (1.0f / C) + 1e-5f);
#pragma unroll
  for (int h = 0; h < H; ++h) bias[h] = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t* u = reinterpret_cast<uint32_t*>(&v[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = i * 8 + 2 * j;
      u[j] = pack_bf2((bf_lo(u[j]) - mean) * rstd * __ldg(w + k), (bf_hi(u[j]) - mean) * rstd * __ldg(w + k + 1));
      const float y0 = bf_lo(u[j]), y1 = bf_hi(u[j]);
#pragma unroll
      for (int h = 0; h < H; ++h)
        bias[h] += y0 * __bfloat162float(wb[h * C + k]) + y1 * __bfloat162float(wb[h * C + k + 1]);
    }
  }
#pragma unroll
  for (int ka = 0; ka < 2; ++ka)
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(tile + ka * ATOM + tc::sw128_off(r, c)) = v[ka * 8 + c];
}

__device__ __forceinline__ void store_row32(bf16* dst, const float* v, bool zero) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint4 o;
    o.x = zero ? 0u : pack_bf2(v[8 * g + 0], v[8 * g + 1]);
    o.y = zero ? 0u : pack_bf2(v[8 * g + 2], v[8 * g + 3]);
    o.z = zero ? 0u : pack_bf2(v[8 * g + 4], v[8 * g + 5]);
    o.w = zero ? 0u : pack_bf2(v[8 * g + 6], v[8 * g + 7]);
    reinterpret_cast<uint4*>(dst)[g] = o;
  }
}

__global__ void __launch_bounds__(128, 1) k_triatt_project_tc(const __grid_constant__ CUtensorMap tmap,
                                                              AttProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* A = smem;
  uint8_t* W = smem + 2 * A_BYTES;
  bf16* vst = reinterpret_cast<bf16*>(W + W_BYTES);                 // [32][128] staging of V^T
  uint64_t* bars = reinterpret_cast<uint64_t*>(W + W_BYTES + VT_STAGE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t nqb = p.qp / TILE;
  const int64_t ntiles = p.nb * nqb;

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bars[0], 1);
    tc::mbar_init(&bars[1], 1);
    tc::mbar_init(&bars[2], 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmap);
  }
  load_weight_sw128(W, p.w_qkvg, NOUT, tid, 128);
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  bool aborted = false;

  auto issue = [&](int64_t tile, int stage) {
    const int b = (int)(tile / nqb), q0 = (int)((tile % nqb) * TILE);
    const int c1 = p.transpose ? b : q0;     // column coordinate
    const int c2 = p.transpose ? q0 : b;     // row coordinate
    tc::mbar_expect_tx(&bars[stage], A_BYTES);
    tc::tma_load_3d(A + stage * A_BYTES, &tmap, &bars[stage], 0, c1, c2);
    tc::tma_load_3d(A + stage * A_BYTES + ATOM, &tmap, &bars[stage], 64, c1, c2);
  };

  constexpr uint32_t IDESC = tc::idesc_bf16(128, 256);
  const uint32_t a_base = tc::smem_u32(A), w_base = tc::smem_u32(W);

  int64_t tile = blockIdx.x;
  if (tid == 0 && tile < ntiles) issue(tile, 0);
  for (uint32_t it = 0; tile < ntiles; tile += gridDim.x, ++it) {
    const int stage = it & 1;
    if (tid == 0 && tile + gridDim.x < ntiles) {
      tc::fence_proxy_async();
      issue(tile + gridDim.x, stage ^ 1);
    }
    tc::mbar_wait(&bars[stage], (it >> 1) & 1, p.status, aborted);
    const int64_t b = tile / nqb, qi = (tile % nqb) * TILE + tid;
    const bool valid = qi < p.nq;
    float bias[H];
    ln_row_bias(A + stage * A_BYTES, tid, p.ln_w, p.w_bias, bias);
    if (valid && p.compute_bias) {
      const int64_t r = p.transpose ? qi : b, s = p.transpose ? b : qi;
#pragma unroll
      for (int h = 0; h < H; ++h) p.bias[(r * H + h) * p.qp + s] = __float2bfloat16_rn(bias[h] * kLog2e);
    }
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int ka = k >> 2, kk = k & 3;
        const uint64_t ad = tc::smem_desc(a_base + stage * A_BYTES + ka * ATOM + kk * 32, 1024, tc::kSW128);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint64_t bd = tc::smem_desc(w_base + ka * (NOUT * 128) + hh * (256 * 128) + kk * 32, 1024, tc::kSW128);
          tc::mma_bf16(tbase + hh * 256, ad, bd, IDESC, k > 0);
        }
      }
      tc::mma_commit(&bars[2]);
    }
    tc::mbar_wait(&bars[2], it & 1, p.status, aborted);
    tc::tc_fence_after();

    // ---- epilogue: query qi of attention row b ----
    const uint32_t lane_addr = tbase + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int h = 0; h < H; ++h) {
      float v0[16], v1[16], row[32];
      tc::tmem_ld16(lane_addr + h * D, v0);                 // q
      tc::tmem_ld16(lane_addr + h * D + 16, v1);
#pragma unroll
      for (int e = 0; e < 16; ++e) { row[e] = v0[e]; row[16 + e] = v1[e]; }
      store_row32(p.q + ((b * H + h) * p.qp + qi) * D, row, !valid);
      tc::tmem_ld16(lane_addr + 128 + h * D, v0);           // k
      tc::tmem_ld16(lane_addr + 128 + h * D + 16, v1);
#pragma unroll
      for (int e = 0; e < 16; ++e) { row[e] = v0[e]; row[16 + e] = v1[e]; }
      store_row32(p.k + ((b * H + h) * p.qp + qi) * D, row, !valid);
      tc::tmem_ld16(lane_addr + 256 + h * D, v0);           // v, stored transposed (keys contiguous)
      tc::tmem_ld16(lane_addr + 256 + h * D + 16, v1);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        vst[e * TILE + tid] = __float2bfloat16_rn(valid ? v0[e] : 0.f);
        vst[(16 + e) * TILE + tid] = __float2bfloat16_rn(valid ? v1[e] : 0.f);
      }
      __syncthreads();
      {
        // 32 rows (d) x 256 bytes: V^T[b][h][d][q0 .. q0+127]
        bf16* vt = p.vt + ((b * H + h) * D) * p.qp + (tile % nqb) * TILE;
#pragma unroll
        for (int i = 0; i < (D * 16) / 128; ++i) {
          const int e = tid + 128 * i, d = e >> 4, part = e & 15;
          *reinterpret_cast<uint4*>(vt + (int64_t)d * p.qp + part * 8) =
              *reinterpret_cast<const uint4*>(vst + d * TILE + part * 8);
        }
      }
      __syncthreads();
      tc::tmem_ld16(lane_addr + 384 + h * D, v0);           // gate -> sigmoid
      tc::tmem_ld16(lane_addr + 384 + h * D + 16, v1);
#pragma unroll
      for (int e = 0; e < 16; ++e) { row[e] = fast_sigmoid(v0[e]); row[16 + e] = fast_sigmoid(v1[e]); }
      store_row32(p.g + (b * p.qp + qi) * C + h * D, row, false);
    }
    tc::tc_fence_before();
    __syncthreads();
  }
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------
// attention core
// ---------------------------------------------------------------------------
struct AttCoreParams {
  const bf16 *q, *k, *vt, *g, *bias;
  const bf16* w_out;      // output_projection^T [128 out][128 in]
  const uint8_t* mask;    // [N] token mask (keys/queries are all N tokens)
  const bf16* z;          // the z block [rows][cols][128] (residual)
  bf16* z_out;
  int64_t cols;           // columns of the z block
  int64_t nq, qp;         // queries = keys, pitch
  int64_t batch_offset;   // global token index of attention row 0 (row mask)
  int transpose;
  float scale_log2;       // (1/sqrt(D)) * log2(e)
  uint32_t* status;
};

constexpr int KB = 64;                     // keys per block
constexpr int OFF_Q = 0;                   // 4 heads x 128 x 64 B (64B swizzle)
constexpr int OFF_KV = 32 * 1024;          // [wg][stage] x (K 4 KB | Vt 4 KB)
constexpr int OFF_P = 64 * 1024;           // [wg] x 128 x 128 B (128B swizzle)
constexpr int OFF_O = 96 * 1024;           // 128 x 256 B gated outputs of all heads
constexpr int OFF_W = 128 * 1024;          // 128 x 256 B output projection
constexpr int OFF_BAR = 160 * 1024;
constexpr int OFF_KBITS = OFF_BAR + 1024;       // key-valid bits, qp/32 words (qp <= 65536)
constexpr int SMEM_CORE = OFF_KBITS + 8192 + 1024;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void wg_sync(int g) { asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory"); }
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// K block (64 keys x 32) into 64B-swizzled K-major rows and Vt block (32 x 64 keys)
// into 128B-swizzled K-major rows, by the 128 threads of one warpgroup.
__device__ __forceinline__ void load_kv(uint8_t* dst, const AttCoreParams& p, int64_t b, int h, int kb, int t) {
  const bf16* ksrc = p.k + ((b * H + h) * p.qp + (int64_t)kb * KB) * D;
  const bf16* vsrc = p.vt + ((b * H + h) * D) * p.qp + (int64_t)kb * KB;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int e = t + 128 * i;
    const int key = e >> 2, c = e & 3;
    cp_async16(dst + tc::sw64_off(key, c), ksrc + key * D + c * 8);
    const int d = e >> 3, c8 = e & 7;
    cp_async16(dst + 4096 + tc::sw128_off(d, c8), vsrc + (int64_t)d * p.qp + c8 * 8);
  }
}

__global__ void __launch_bounds__(256, 1) k_triatt_core_tc(AttCoreParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* sdone = reinterpret_cast<uint64_t*>(smem + OFF_BAR);   // [2]
  uint64_t* odone = sdone + 2;                                     // [2]
  uint64_t* outdone = sdone + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sdone + 6);
  const int tid = threadIdx.x, warp = tid >> 5, g = tid >> 7, t = tid & 127;
  const int64_t q0 = (int64_t)blockIdx.x * TILE, b = blockIdx.y;
  const int nkb = (int)(p.qp / KB);

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 5; ++i) tc::mbar_init(&sdone[i], 1);
    tc::fence_mbar_init();
  }
  // key k is attended iff mask[b] && mask[k] (pair mask, blocks.py:314)
  uint32_t* kbits = reinterpret_cast<uint32_t*>(smem + OFF_KBITS);
  {
    const bool rok = p.mask[b + p.batch_offset] != 0;
    for (int w = tid; w < (int)(p.qp / 32); w += 256) {
      uint32_t bits = 0;
      for (int e = 0; e < 32; ++e) {
        const int64_t key = (int64_t)w * 32 + e;
        if (rok && key < p.nq && p.mask[key]) bits |= 1u << e;
      }
      kbits[w] = bits;
    }
  }
  // Q of all four heads and the output projection, by all 256 threads.
  for (int e = tid; e < H * TILE * 4; e += 256) {
    const int h = e >> 9, q = (e >> 2) & 127, c = e & 3;
    cp_async16(smem + OFF_Q + h * 8192 + tc::sw64_off(q, c), p.q + ((b * H + h) * p.qp + q0 + q) * D + c * 8);
  }
  for (int e = tid; e < C * 16; e += 256) {
    const int r = e >> 4, kc = e & 15;
    cp_async16(smem + OFF_W + (kc >> 3) * 16384 + tc::sw128_off(r, kc & 7), p.w_out + r * C + kc * 8);
  }
  cp_async_commit();
  uint8_t* kv = smem + OFF_KV + g * 16384;
  load_kv(kv, p, b, g, 0, t);   // first step of this warpgroup: head g, key block 0
  cp_async_commit();
  cp_async_wait<1>();           // Q and W_o landed (loaded by both warpgroups)
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t lane_addr = tbase + ((uint32_t)(32 * (warp & 3)) << 16);
  const uint32_t s_col = g * KB, o_col = 128 + g * D;
  bool aborted = false;

  const int64_t q = q0 + t;
  const uint32_t sb = tc::smem_u32(smem);
  constexpr uint32_t IDESC_S = tc::idesc_bf16(128, KB), IDESC_O = tc::idesc_bf16(128, D);
  float m = -INFINITY, l = 0.f, o[D];
  const int nsteps = 2 * nkb;
  // bias row (query q, head h) of the key block of a step; prefetched one step ahead
  uint4 bias_raw[KB / 8];
  auto load_bias = [&](int step) {
    const int hh_ = step / nkb, kb_ = step % nkb, h_ = g + 2 * hh_;
    const uint4* brow = reinterpret_cast<const uint4*>(p.bias + (q * H + h_) * p.qp + (int64_t)kb_ * KB);
#pragma unroll
    for (int c = 0; c < KB / 8; ++c) bias_raw[c] = __ldg(brow + c);
  };
  load_bias(0);
  for (int j = 0; j < nsteps; ++j) {
    const int hh = j / nkb, kb = j % nkb, h = g + 2 * hh, s = j & 1;
    if (j + 1 < nsteps) {
      const int j1 = j + 1;
      load_kv(kv + (s ^ 1) * 8192, p, b, g + 2 * (j1 / nkb), j1 % nkb, t);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    tc::fence_proxy_async();
    tc::tc_fence_before();
    wg_sync(g);
    const uint32_t kvs = sb + OFF_KV + g * 16384 + s * 8192;
    if (t == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        tc::mma_bf16(tbase + s_col, tc::smem_desc(sb + OFF_Q + h * 8192 + kk * 32, 512, tc::kSW64),
                     tc::smem_desc(kvs + kk * 32, 512, tc::kSW64), IDESC_S, kk > 0);
      tc::mma_commit(&sdone[g]);
    }
    const uint64_t vbits = (uint64_t)kbits[kb * 2] | ((uint64_t)kbits[kb * 2 + 1] << 32);
    tc::mbar_wait(&sdone[g], j & 1, p.status, aborted);
    tc::tc_fence_after();
    if (kb == 0) {
      m = -INFINITY;
      l = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) o[d] = 0.f;
    }
    // ---- online softmax over this key block (log2 domain) ----
    float sv[KB];
#pragma unroll
    for (int i = 0; i < KB / 16; ++i) {
      float v[16];
      tc::tmem_ld16(lane_addr + s_col + 16 * i, v);
#pragma unroll
      for (int e = 0; e < 16; ++e) sv[16 * i + e] = v[e];
    }
    float mx = -INFINITY;
    const bool full = (vbits == ~0ull) && ((int64_t)kb * KB + KB <= p.nq);
#pragma unroll
    for (int c = 0; c < KB / 8; ++c) {
      const uint32_t* bu = reinterpret_cast<const uint32_t*>(&bias_raw[c]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int kidx = c * 8 + e;
        const float bv = (e & 1) ? bf_hi(bu[e >> 1]) : bf_lo(bu[e >> 1]);
        float x = fmaf(sv[kidx], p.scale_log2, bv);      // log2 domain (bias pre-scaled by log2 e)
        if (!full) {
          const int64_t key = (int64_t)kb * KB + kidx;
          if (key >= p.nq) x = -INFINITY;                 // padding beyond the N keys: excluded
          else if (!((vbits >> kidx) & 1)) x = -FLT_MAX;  // masked key: the reference's -finfo.max bias
        }
        sv[kidx] = x;
        mx = fmaxf(mx, x);
      }
    }
    const float m_new = fmaxf(m, mx);
    const float corr = ex2(m - m_new);
    float psum = 0.f;
    uint8_t* prow = smem + OFF_P + g * 16384;
#pragma unroll
    for (int c = 0; c < KB / 8; ++c) {
      float pv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        pv[e] = ex2(sv[c * 8 + e] - m_new);
        psum += pv[e];
      }
      uint4 pk;
      pk.x = pack_bf2(pv[0], pv[1]);
      pk.y = pack_bf2(pv[2], pv[3]);
      pk.z = pack_bf2(pv[4], pv[5]);
      pk.w = pack_bf2(pv[6], pv[7]);
      *reinterpret_cast<uint4*>(prow + tc::sw128_off(t, c)) = pk;
    }
    l = l * corr + psum;
    m = m_new;
    if (j + 1 < nsteps) load_bias(j + 1);   // in flight during the P.V MMA and the next S MMA
    tc::fence_proxy_async();
    tc::tc_fence_before();
    wg_sync(g);
    if (t == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < KB / 16; ++kk)
        tc::mma_bf16(tbase + o_col, tc::smem_desc(sb + OFF_P + g * 16384 + kk * 32, 1024, tc::kSW128),
                     tc::smem_desc(kvs + 4096 + kk * 32, 1024, tc::kSW128), IDESC_O, kk > 0);
      tc::mma_commit(&odone[g]);
    }
    tc::mbar_wait(&odone[g], j & 1, p.status, aborted);
    tc::tc_fence_after();
    {
      float v0[16], v1[16];
      tc::tmem_ld16(lane_addr + o_col, v0);
      tc::tmem_ld16(lane_addr + o_col + 16, v1);
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        o[d] = o[d] * corr + v0[d];
        o[16 + d] = o[16 + d] * corr + v1[d];
      }
    }
    if (kb == nkb - 1) {
      // normalise, gate with sigmoid(gate), stage as the A operand of the output projection
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      const uint4* grow = reinterpret_cast<const uint4*>(p.g + (b * p.qp + q) * C + h * D);
      uint8_t* orow = smem + OFF_O + (h >> 1) * 16384;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const uint4 gg = __ldg(grow + cc);
        const uint32_t* gu = reinterpret_cast<const uint32_t*>(&gg);
        uint4 ok;
        uint32_t* ou = reinterpret_cast<uint32_t*>(&ok);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          ou[e] = pack_bf2(o[cc * 8 + 2 * e] * inv * bf_lo(gu[e]), o[cc * 8 + 2 * e + 1] * inv * bf_hi(gu[e]));
        *reinterpret_cast<uint4*>(orow + tc::sw128_off(t, (h & 1) * 4 + cc)) = ok;
      }
    }
  }

  // ---- output projection of the gated heads + residual ----
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    tc::tc_fence_after();
    constexpr uint32_t IDESC = tc::idesc_bf16(128, 128);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int ka = k >> 2, kk = k & 3;
      tc::mma_bf16(tbase + 256, tc::smem_desc(sb + OFF_O + ka * 16384 + kk * 32, 1024, tc::kSW128),
                   tc::smem_desc(sb + OFF_W + ka * 16384 + kk * 32, 1024, tc::kSW128), IDESC, k > 0);
    }
    tc::mma_commit(outdone);
  }
  tc::mbar_wait(outdone, 0, p.status, aborted);
  tc::tc_fence_after();
  {
    const bool live = q < p.nq;
    const int64_t pos = live ? (p.transpose ? q * p.cols + b : b * p.cols + q) : 0;
    const uint4* zin = reinterpret_cast<const uint4*>(p.z + pos * C + g * 64);
    uint4* zo = reinterpret_cast<uint4*>(p.z_out + pos * C + g * 64);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v[16];
      tc::tmem_ld16(lane_addr + 256 + g * 64 + 16 * i, v);   // warp-collective: every lane loads
#pragma unroll
      for (int hlf = 0; hlf < 2 && live; ++hlf) {
        const uint4 zz = zin[2 * i + hlf];
        const uint32_t* zu = reinterpret_cast<const uint32_t*>(&zz);
        uint4 r;
        uint32_t* ru = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          ru[e] = pack_bf2(bf_lo(zu[e]) + v[hlf * 8 + 2 * e], bf_hi(zu[e]) + v[hlf * 8 + 2 * e + 1]);
        zo[2 * i + hlf] = r;
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

template <typename K>
int set_smem(K kernel, int bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (!done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    done[dev & 63] = true;
  }
  return SF_OK;
}

// Pair bias of the local pair rows only: bias[(r*H + h)*ldb + s] = LN(z[r,s]) . W_b[h]
// (blocks.py:317-320), one warp per position.  Used when the attention runs on a
// transposed block whose own positions are not the rows the bias needs.
__global__ void k_triatt_bias(const bf16* __restrict__ z, const float* __restrict__ ln_w, const bf16* __restrict__ wb,
                              bf16* __restrict__ bias, int64_t rows, int64_t n, int64_t ldb) {
  const int64_t pos = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (pos >= rows * n) return;
  const bf16* zr = z + pos * C;
  float x[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) x[e] = __bfloat162float(zr[lane * 4 + e]);
  const float mean = warp_sum(x[0] + x[1] + x[2] + x[3]) * (1.0f / C);
  float v = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) v += (x[e] - mean) * (x[e] - mean);
  const float rstd = rsqrtf(warp_sum(v) * (1.0f / C) + 1e-5f);
  float acc[H] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int c = lane * 4 + e;
    const float y = __bfloat162float(__float2bfloat16_rn((x[e] - mean) * rstd * ln_w[c]));
#pragma unroll
    for (int h = 0; h < H; ++h) acc[h] += y * __bfloat162float(wb[h * C + c]);
  }
#pragma unroll
  for (int h = 0; h < H; ++h) acc[h] = warp_sum(acc[h]);
  if (lane == 0) {
    const int64_t r = pos / n, sc = pos % n;
#pragma unroll
    for (int h = 0; h < H; ++h) bias[(r * H + h) * ldb + sc] = __float2bfloat16_rn(acc[h] * kLog2e);
  }
}

}  // namespace

int64_t triatt_query_pitch(int64_t nq) { return (nq + 127) / 128 * 128; }

int triatt_bias_tc(const bf16* z, int64_t rows, int64_t n, const float* ln_w, const bf16* w_bias, bf16* bias,
                   int64_t ldb, cudaStream_t stream) {
  if (rows == 0 || n == 0) return SF_OK;
  SF_REQUIRE(ldb >= n, "triatt_bias: ldb %lld < n %lld", (long long)ldb, (long long)n);
  const int64_t total = rows * n;
  k_triatt_bias<<<(unsigned)((total + 7) / 8), 256, 0, stream>>>(z, ln_w, w_bias, bias, rows, n, ldb);
  count_launch();
  return check_launch("triatt_bias");
}

int triatt_project_tc(const bf16* z, int64_t rows, int64_t cols, int transpose, int compute_bias, const float* ln_w,
                      const bf16* w_qkvg, const bf16* w_bias, bf16* q, bf16* k, bf16* vt, bf16* g, bf16* bias,
                      cudaStream_t stream) {
  if (rows == 0 || cols == 0) return SF_OK;
  const int64_t nb = transpose ? cols : rows, nq = transpose ? rows : cols;
  SF_REQUIRE(nb <= 65535 && nq <= 65535, "triatt_project: block [%lld][%lld] too large", (long long)rows,
             (long long)cols);
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  static bool attr[64] = {false};
  SF_TRY(set_smem(k_triatt_project_tc, SMEM_PROJ, attr));
  CUtensorMap map;
  SF_TRY(make_pair_tmap(&map, z, rows, cols, transpose != 0));
  const int64_t qp = triatt_query_pitch(nq);
  AttProjParams pp{ln_w, w_qkvg, w_bias, q, k, vt, g, bias, rows, cols, nb, nq, qp, transpose, compute_bias, status};
  const int64_t ntiles = nb * (qp / TILE);
  const int grid = (int)(ntiles < num_sms() ? ntiles : num_sms());
  k_triatt_project_tc<<<grid, 128, SMEM_PROJ, stream>>>(map, pp);
  count_launch();
  return check_launch("triatt_project_tc");
}

int triatt_core_tc(const bf16* q, const bf16* k, const bf16* vt, const bf16* g, const bf16* bias, const bf16* w_out,
                   const uint8_t* mask, const bf16* z, bf16* z_out, int64_t rows, int64_t cols, int transpose,
                   int64_t batch_offset, cudaStream_t stream) {
  if (rows == 0 || cols == 0) return SF_OK;
  const int64_t nb = transpose ? cols : rows, nq = transpose ? rows : cols;
  SF_REQUIRE(nb <= 65535 && nq <= 65535, "triatt_core: block too large");
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  static bool attr[64] = {false};
  SF_TRY(set_smem(k_triatt_core_tc, SMEM_CORE, attr));
  const int64_t qp = triatt_query_pitch(nq);
  AttCoreParams cp{q, k, vt, g, bias, w_out, mask, z, z_out, cols, nq, qp, batch_offset, transpose,
                   (1.0f / sqrtf((float)D)) * kLog2e, status};
  dim3 cgrid((unsigned)(qp / TILE), (unsigned)nb);
  k_triatt_core_tc<<<cgrid, 256, SMEM_CORE, stream>>>(cp);
  count_launch();
  return check_launch("triatt_core_tc");
}

// Buffer sizes of one attention call: Q, K, Vt [nb][H][qp][32], G [nb][qp][128], bias [qp][H][qp].
size_t triatt_tc_workspace(int64_t n) {
  const int64_t qp = triatt_query_pitch(n);
  const size_t per = (size_t)n * H * qp * D * 2;
  size_t used = 0;
  for (int i = 0; i < 3; ++i) used = align_up(used, 256) + per;
  used = align_up(used, 256) + (size_t)n * qp * C * 2;
  used = align_up(used, 256) + (size_t)qp * H * qp * 2;
  return used;
}

// The whole op on one device (the z block is the full [n][n] pair tensor).
int triatt_tc(const bf16* z, const uint8_t* mask, int64_t n, int transpose, const float* ln_w, const bf16* w_qkvg,
              const bf16* w_bias, const bf16* w_out, bf16* z_out, void* ws_p, size_t ws_bytes, cudaStream_t stream) {
  if (n == 0) return SF_OK;
  if (ws_bytes < triatt_tc_workspace(n)) {
    set_error("sf_tri_attention: workspace %zu < %zu", ws_bytes, triatt_tc_workspace(n));
    return SF_ERR_WORKSPACE;
  }
  const int64_t qp = triatt_query_pitch(n);
  Workspace ws(ws_p, ws_bytes);
  bf16* q = ws.take<bf16>((size_t)n * H * qp * D);
  bf16* k = ws.take<bf16>((size_t)n * H * qp * D);
  bf16* vt = ws.take<bf16>((size_t)n * H * qp * D);
  bf16* g = ws.take<bf16>((size_t)n * qp * C);
  bf16* bias = ws.take<bf16>((size_t)qp * H * qp);
  SF_TRY(triatt_project_tc(z, n, n, transpose, 1, ln_w, w_qkvg, w_bias, q, k, vt, g, bias, stream));
  return triatt_core_tc(q, k, vt, g, bias, w_out, mask, z, z_out, n, n, transpose, 0, stream);
}

}  // namespace sf
