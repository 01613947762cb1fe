// Pair transition (TransitionBlock, blocks.py:79-96) on tcgen05, bf16 track:
//   y = x + (swish(LN(x) W1a) * (LN(x) W1b)) W2,   C = 128, I = 512.
//
// One CTA (8 epilogue warps + 1 weight-producer warp) handles 256 positions per
// iteration as two 128-row tiles that share every weight chunk.  The hidden
// layer is walked in 8 chunks of 64 units: GEMM1 (M128 N128 K128 per tile,
// a- and b-halves of the chunk side by side) lands in TMEM columns [0,256);
// the epilogue warps turn it into swish(a)*b (bf16) in shared memory; GEMM2
// (M128 N128 K64 per tile) accumulates the down projection in TMEM columns
// [256,512).  W1/W2 chunks (32 + 16 KB) stream through a 2-stage TMA ring, so
// the full 384 KB of weights is read once per 256 positions from L2.
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int I = 512, HC = 64, NCHUNK = I / HC;
constexpr int X_BYTES = 2 * A_BYTES;           // two 128x128 input tiles
constexpr int H_BYTES = 2 * TILE * 128;        // two 128x64 hidden tiles (one 128B atom each)
constexpr int W1C_BYTES = 128 * 256;           // 128 rows (64 a + 64 b) x 128 k
constexpr int W2C_BYTES = 128 * 128;           // 128 out rows x 64 k
constexpr int WST_BYTES = W1C_BYTES + W2C_BYTES;
constexpr int OFF_X = 0, OFF_H = X_BYTES, OFF_W = OFF_H + H_BYTES, OFF_BAR = OFF_W + 2 * WST_BYTES;
constexpr int SMEM_TR = OFF_BAR + 1024 + 1024;

struct TrParams {
  const bf16* x;
  bf16* y;
  const float* ln_w;
  const float* ln_b;
  int64_t M;
  uint32_t* status;
};

__global__ void __launch_bounds__(288, 1) k_transition_tc(const __grid_constant__ CUtensorMap tmX,
                                                          const __grid_constant__ CUtensorMap tmW1,
                                                          const __grid_constant__ CUtensorMap tmW2, TrParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + OFF_BAR);   // [2]
  uint64_t* wempty = wfull + 2;                                     // [2]
  uint64_t* xbar = wfull + 4;
  uint64_t* g1bar = wfull + 5;
  uint64_t* g2bar = wfull + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wfull + 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t npairs = (p.M + 2 * TILE - 1) / (2 * TILE);

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 7; ++i) tc::mbar_init(&wfull[i], 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmX);
    tc::prefetch_tmap(&tmW1);
    tc::prefetch_tmap(&tmW2);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  bool aborted = false;

  if (warp == 8) {
    // ---- weight producer: W1/W2 chunks for every (pair, chunk), 2-stage ring ----
    if (lane == 0) {
      uint32_t q = 0;
      for (int64_t pr = blockIdx.x; pr < npairs; pr += gridDim.x) {
        for (int hc = 0; hc < NCHUNK; ++hc, ++q) {
          const int s = q & 1;
          tc::mbar_wait(&wempty[s], ((q >> 1) & 1) ^ 1, p.status, aborted);
          uint8_t* w = smem + OFF_W + s * WST_BYTES;
          tc::mbar_expect_tx(&wfull[s], WST_BYTES);
          for (int ka = 0; ka < 2; ++ka) {
            tc::tma_load_2d(w + ka * (128 * 128), &tmW1, &wfull[s], ka * 64, hc * HC);             // a rows
            tc::tma_load_2d(w + ka * (128 * 128) + 64 * 128, &tmW1, &wfull[s], ka * 64, I + hc * HC);  // b rows
          }
          tc::tma_load_2d(w + W1C_BYTES, &tmW2, &wfull[s], hc * HC, 0);
        }
      }
    }
  } else {
    // ---- 8 epilogue warps: warps 0-3 own tile 0, warps 4-7 tile 1; thread = row ----
    const int tt = warp >> 2, r = tid & 127;
    const uint32_t lane_addr = tbase + ((uint32_t)(32 * (warp & 3)) << 16);
    const uint32_t sb = tc::smem_u32(smem);
    uint32_t q = 0, it = 0;
    for (int64_t pr = blockIdx.x; pr < npairs; pr += gridDim.x, ++it) {
      const int64_t m0 = pr * 2 * TILE;
      if (tid == 0) {
        tc::mbar_expect_tx(xbar, X_BYTES);
        for (int t2 = 0; t2 < 2; ++t2)
          for (int ka = 0; ka < 2; ++ka)
            tc::tma_load_2d(smem + OFF_X + t2 * A_BYTES + ka * ATOM, &tmX, xbar, ka * 64, (int)(m0 + t2 * TILE));
      }
      tc::mbar_wait(xbar, it & 1, p.status, aborted);
      ln_row_inplace(smem + OFF_X + tt * A_BYTES, r, p.ln_w, p.ln_b, 1e-5f);
      tc::fence_proxy_async();
      tc::tc_fence_before();
      asm volatile("bar.sync 1, 256;" ::: "memory");
      for (int hc = 0; hc < NCHUNK; ++hc, ++q) {
        const int s = q & 1;
        if (tid == 0) {
          // GEMM1 for both tiles: acc1[t2] = LN(x)[t2] (128 x 128) . W1 chunk (128 x 128)
          tc::mbar_wait(&wfull[s], (q >> 1) & 1, p.status, aborted);
          tc::tc_fence_after();
          constexpr uint32_t ID1 = tc::idesc_bf16(128, 128);
          const uint32_t wb = sb + OFF_W + s * WST_BYTES;
          for (int t2 = 0; t2 < 2; ++t2)
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int ka = k >> 2, kk = k & 3;
              tc::mma_bf16(tbase + t2 * 128,
                           tc::smem_desc(sb + OFF_X + t2 * A_BYTES + ka * ATOM + kk * 32, 1024, tc::kSW128),
                           tc::smem_desc(wb + ka * (128 * 128) + kk * 32, 1024, tc::kSW128), ID1, k > 0);
            }
          tc::mma_commit(g1bar);
        }
        // the hidden tile H is reused: GEMM2 of the previous chunk must have finished with it
        if (q > 0) tc::mbar_wait(g2bar, (q - 1) & 1, p.status, aborted);
        tc::mbar_wait(g1bar, q & 1, p.status, aborted);
        tc::tc_fence_after();
        uint8_t* hrow = smem + OFF_H + tt * (TILE * 128);
#pragma unroll 1
        for (int cg = 0; cg < 4; ++cg) {   // 16 hidden units at a time
          float a[16], bv[16];
          tc::tmem_ld16(lane_addr + tt * 128 + cg * 16, a);
          tc::tmem_ld16(lane_addr + tt * 128 + 64 + cg * 16, bv);
          uint4 o0, o1;
          uint32_t* u0 = reinterpret_cast<uint32_t*>(&o0);
          uint32_t* u1 = reinterpret_cast<uint32_t*>(&o1);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            u0[e] = pack_bf2(a[2 * e] * fast_sigmoid(a[2 * e]) * bv[2 * e],
                             a[2 * e + 1] * fast_sigmoid(a[2 * e + 1]) * bv[2 * e + 1]);
            u1[e] = pack_bf2(a[8 + 2 * e] * fast_sigmoid(a[8 + 2 * e]) * bv[8 + 2 * e],
                             a[9 + 2 * e] * fast_sigmoid(a[9 + 2 * e]) * bv[9 + 2 * e]);
          }
          *reinterpret_cast<uint4*>(hrow + tc::sw128_off(r, 2 * cg)) = o0;
          *reinterpret_cast<uint4*>(hrow + tc::sw128_off(r, 2 * cg + 1)) = o1;
        }
        tc::fence_proxy_async();
        tc::tc_fence_before();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (tid == 0) {
          // GEMM2 for both tiles: acc2[t2] += H[t2] (128 x 64) . W2 chunk (128 x 64)
          tc::tc_fence_after();
          constexpr uint32_t ID2 = tc::idesc_bf16(128, 128);
          const uint32_t wb = sb + OFF_W + s * WST_BYTES + W1C_BYTES;
          for (int t2 = 0; t2 < 2; ++t2)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc::mma_bf16(tbase + 256 + t2 * 128,
                           tc::smem_desc(sb + OFF_H + t2 * (TILE * 128) + kk * 32, 1024, tc::kSW128),
                           tc::smem_desc(wb + kk * 32, 1024, tc::kSW128), ID2, (hc | kk) != 0);
          tc::mma_commit(&wempty[s]);   // weight stage free once both GEMMs of this chunk are done
          tc::mma_commit(g2bar);
        }
      }
      // ---- residual epilogue: y = x + acc2 ----
      tc::mbar_wait(g2bar, (q - 1) & 1, p.status, aborted);
      tc::tc_fence_after();
      const int64_t m = m0 + tt * TILE + r;
      const bool live = m < p.M;
      const uint4* xr = reinterpret_cast<const uint4*>(p.x + (live ? m : 0) * C);
      uint4* yr = reinterpret_cast<uint4*>(p.y + (live ? m : 0) * C);
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        float v[16];
        tc::tmem_ld16(lane_addr + 256 + tt * 128 + 16 * i, v);
        if (live) {
#pragma unroll
          for (int hlf = 0; hlf < 2; ++hlf) {
            const uint4 xx = xr[2 * i + hlf];
            const uint32_t* xu = reinterpret_cast<const uint32_t*>(&xx);
            uint4 o;
            uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              ou[e] = pack_bf2(bf_lo(xu[e]) + v[hlf * 8 + 2 * e], bf_hi(xu[e]) + v[hlf * 8 + 2 * e + 1]);
            yr[2 * i + hlf] = o;
          }
        }
      }
      tc::tc_fence_before();
      asm volatile("bar.sync 1, 256;" ::: "memory");   // x tile and TMEM free for the next pair
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

}  // namespace

// 2-D bf16 tensor map [outer][inner] (inner contiguous), 128B (default) or 64B swizzle.
int make_2d_tmap(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, uint32_t box_inner,
                 uint32_t box_outer, int swizzle_bytes) {
  auto encode = tensor_map_encoder();
  if (!encode) return SF_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (inner * 2) % 16 != 0) {
    set_error("2-d tensor map: base %p / row bytes %lld not 16-byte aligned", base, (long long)(inner * 2));
    return SF_ERR_ARG;
  }
  if (swizzle_bytes != 128 && swizzle_bytes != 64) {
    set_error("2-d tensor map: unsupported swizzle %d", swizzle_bytes);
    return SF_ERR_ARG;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for [%lld][%lld]", (int)r, (long long)outer, (long long)inner);
    return SF_ERR_CUDA;
  }
  return SF_OK;
}

// Pair transition (C = 128, I = 512) on tcgen05; y may alias x.
int transition_tc(const bf16* x, const float* ln_w, const float* ln_b, const bf16* w1, const bf16* w2, bf16* y,
                  int64_t M, cudaStream_t stream) {
  if (M == 0) return SF_OK;
  SF_REQUIRE(M < (int64_t(1) << 31), "transition_tc: too many rows");
  CUtensorMap mx, mw1, mw2;
  SF_TRY(make_2d_tmap(&mx, x, C, M, 64, TILE));
  SF_TRY(make_2d_tmap(&mw1, w1, C, 2 * I, 64, HC));
  SF_TRY(make_2d_tmap(&mw2, w2, I, C, 64, C));
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(k_transition_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TR);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(transition): %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    attr[dev & 63] = true;
  }
  TrParams p{x, y, ln_w, ln_b, M, status};
  const int64_t npairs = (M + 2 * TILE - 1) / (2 * TILE);
  const int grid = (int)(npairs < num_sms() ? npairs : num_sms());
  k_transition_tc<<<grid, 288, SMEM_TR, stream>>>(mx, mw1, mw2, p);
  count_launch();
  return check_launch("transition_tc");
}

}  // namespace sf
