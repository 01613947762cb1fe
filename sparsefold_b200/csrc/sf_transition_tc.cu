// Pair transition (TransitionBlock, blocks.py:79-96) on tcgen05, bf16 track:
//   y = x + (swish(LN(x) W1a) * (LN(x) W1b)) W2,   C = 128, I = 512.
//
// Persistent, one warp-specialised CTA per SM; 256 positions (two 128-row
// tiles sharing every weight chunk) per pass.  The hidden layer is walked in 16
// chunks of 32 units:
//   warp 8      TMA producer: the x tiles of a pass, and per chunk the 64 rows of
//               W1 (32 a + 32 b, 16 KB) in a 4-stage ring
//   warps 9, 11 GEMM1 issuers, one per tile (an issuing warp gets one MMA per
//               ~126 cycles, so a single issuer of both tiles bounds the kernel):
//               chunk c (M128 N64 K128) into one of two TMEM buffers as soon as
//               the tile's half of the buffer and the weight chunk are free
//   warp 10     GEMM2 issuer: chunk c (M128 N128 K32 per tile) from the hidden
//               tile, accumulating the down projection in TMEM columns [256,512);
//               it also refills the 4-stage ring of W2 columns (8 KB per chunk), so
//               W1 refills never wait for GEMM2, which runs a chunk or more behind
//   warps 0-7   thread = position (warps 0-3 tile 0, 4-7 tile 1): LayerNorm of
//               the pass in place (statistics in one shifted pass, scale and
//               shift from shared memory), then per chunk swish(a) * b from TMEM
//               into the 64B-swizzled hidden tile; then straight on to the next
//               pass's LayerNorm
//   warps 12-15 residual epilogue (warp 12+q reads TMEM lanes 32q..): y = x + acc in
//               eight units of [128 rows][32 channels], the x rows of each brought
//               by TMA into one of two 8 KB staging buffers, the sum written over
//               them and TMA-stored; this runs while warps 0-7 normalise the next
//               pass and the GEMMs start on it (GEMM2 waits only for the
//               accumulators to have been read)
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int I = 512, HC = 32, NCHUNK = I / HC;
constexpr int W1_STAGES = 4;
constexpr int W2_STAGES = 4;
constexpr int X_BYTES = 2 * A_BYTES;           // two 128x128 input tiles
constexpr int H_BYTES = TILE * HC * 2;         // one 128 x 32 hidden tile (8 KB)
constexpr int W1C_BYTES = 2 * 64 * 128;        // 64 rows (32 a + 32 b) x 128 k, two 64-channel atoms
constexpr int W2C_BYTES = C * HC * 2;          // 128 out rows x 32 k (64B swizzle)
constexpr int OFF_X = 0;
constexpr int HBUF = 3;                                      // hidden tiles in flight
constexpr int OFF_H = OFF_X + X_BYTES;                       // [HBUF buffers][2 tiles]
constexpr int OFF_W1 = OFF_H + HBUF * 2 * H_BYTES;           // [stage]
constexpr int OFF_W2 = OFF_W1 + W1_STAGES * W1C_BYTES;       // [stage]
constexpr int Y_BYTES = TILE * 32 * 2;                       // one epilogue unit: 128 rows x 32 channels (64B swizzle)
constexpr int OFF_Y = OFF_W2 + W2_STAGES * W2C_BYTES;        // [2] residual / output staging
constexpr int OFF_LNP = OFF_Y + 2 * Y_BYTES;                 // LayerNorm scale [128] and shift [128], fp32
constexpr int OFF_BAR = OFF_LNP + 2 * C * 4;
constexpr int SMEM_TR = OFF_BAR + 512 + 1024;
static_assert(SMEM_TR <= 232448, "transition shared memory");

// the four epilogue warps (named barrier 1)
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
constexpr int TR_THREADS = 16 * 32;

struct TrParams {
  const bf16* x;
  bf16* y;
  const float* ln_w;
  const float* ln_b;
  int64_t M;
  uint32_t* status;
};

__global__ void __launch_bounds__(TR_THREADS, 1) k_transition_tc(const __grid_constant__ CUtensorMap tmX,
                                                                 const __grid_constant__ CUtensorMap tmW1,
                                                                 const __grid_constant__ CUtensorMap tmW2,
                                                                 const __grid_constant__ CUtensorMap tmY,
                                                                 const __grid_constant__ CUtensorMap tmR, TrParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* xfull = bars;                        // x tiles landed
  uint64_t* xready = bars + 1;                   // LN done (256)
  uint64_t* xfree = bars + 2;                    // last GEMM1 of the pass done (both issuers)
  uint64_t* accfull = bars + 3;                  // last GEMM2 of the pass done
  uint64_t* accfree = bars + 4;                  // accumulators read (4 epilogue warps)
  uint64_t* w1full = bars + 5;                   // [W1_STAGES]
  uint64_t* w1free = w1full + W1_STAGES;         // both GEMM1 issuers done with the chunk
  uint64_t* w2full = w1free + W1_STAGES;
  uint64_t* w2free = w2full + W2_STAGES;
  uint64_t* s1full = w2free + W2_STAGES;         // [2 buffers][2 tiles]
  uint64_t* s1free = s1full + 4;                 // [2 buffers][2 tiles] (4 warps)
  uint64_t* hfull = s1free + 4;                  // [HBUF] (8 warps)
  uint64_t* hfree = hfull + HBUF;                // [HBUF]
  uint64_t* drain = hfree + HBUF;                // [3] drain barriers of the MMA issuers, warps 9-11 (abort path)
  uint64_t* ybar = drain + 3;                    // [2] residual rows of an epilogue unit landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ybar + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t npasses = (p.M + 2 * TILE - 1) / (2 * TILE);
  float* lnp = reinterpret_cast<float*>(smem + OFF_LNP);
  if (tid < 2 * C) lnp[tid] = tid < C ? p.ln_w[tid] : (p.ln_b ? p.ln_b[tid - C] : 0.f);

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(xfull, 1);
    tc::mbar_init(xready, 256);
    tc::mbar_init(xfree, 2);
    tc::mbar_init(accfull, 1);
    tc::mbar_init(accfree, 4);
    for (int s = 0; s < W1_STAGES; ++s) {
      tc::mbar_init(&w1full[s], 1);
      tc::mbar_init(&w1free[s], 2);
    }
    for (int s = 0; s < W2_STAGES; ++s) {
      tc::mbar_init(&w2full[s], 1);
      tc::mbar_init(&w2free[s], 1);
    }
    for (int s = 0; s < 4; ++s) {
      tc::mbar_init(&s1full[s], 1);
      tc::mbar_init(&s1free[s], 4);
    }
    for (int s = 0; s < HBUF; ++s) {
      tc::mbar_init(&hfull[s], 8);
      tc::mbar_init(&hfree[s], 1);
    }
    for (int s = 0; s < 3; ++s) tc::mbar_init(&drain[s], 1);
    for (int s = 0; s < 2; ++s) tc::mbar_init(&ybar[s], 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmX);
    tc::prefetch_tmap(&tmW1);
    tc::prefetch_tmap(&tmW2);
    tc::prefetch_tmap(&tmY);
    tc::prefetch_tmap(&tmR);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  tc::griddep_wait();     // the previous kernel's outputs are complete and visible from here on
  tc::griddep_launch();
  const uint32_t tbase = *tmem_slot;
  const uint32_t sb = tc::smem_u32(smem);
  bool aborted = false;
  uint32_t xloads = 0, w1loads = 0, w2loads = 0, yloads = 0;   // TMA loads issued per ring (abort-path drain)

  if (warp == 8) {
    // ---- TMA producer (stops at its first failed wait) ----
    if (lane == 0) {
      uint32_t& q = w1loads;
      uint32_t pi = 0;
      for (int64_t ps = blockIdx.x; ps < npasses && !aborted; ps += gridDim.x, ++pi) {
        const int64_t m0 = ps * 2 * TILE;
        if (pi >= 1 && !tc::mbar_wait(xfree, (pi - 1) & 1, p.status, aborted)) break;
        tc::mbar_expect_tx(xfull, X_BYTES);
        for (int t2 = 0; t2 < 2; ++t2)
          for (int ka = 0; ka < 2; ++ka)
            tc::tma_load_2d(smem + OFF_X + t2 * A_BYTES + ka * ATOM, &tmX, xfull, ka * 64, (int)(m0 + t2 * TILE));
        ++xloads;
        for (int hc = 0; hc < NCHUNK; ++hc, ++q) {
          const int st = q % W1_STAGES;
          const uint32_t ph = ((q / W1_STAGES) + 1) & 1;
          if (q >= W1_STAGES && !tc::mbar_wait(&w1free[st], ph, p.status, aborted)) break;
          uint8_t* w1 = smem + OFF_W1 + st * W1C_BYTES;
          tc::mbar_expect_tx(&w1full[st], W1C_BYTES);
          for (int ka = 0; ka < 2; ++ka) {
            tc::tma_load_2d(w1 + ka * 8192, &tmW1, &w1full[st], ka * 64, hc * HC);              // a rows
            tc::tma_load_2d(w1 + ka * 8192 + 4096, &tmW1, &w1full[st], ka * 64, I + hc * HC);   // b rows
          }
        }
      }
    }
  } else if (warp == 9 || warp == 11) {
    // ---- GEMM1 issuer of tile t2 (stops at its first failed wait) ----
    if (lane == 0) {
      const int t2 = warp == 9 ? 0 : 1;
      constexpr uint32_t ID1 = tc::idesc_bf16(128, 2 * HC);
      uint32_t q = 0, pi = 0;
      for (int64_t ps = blockIdx.x; ps < npasses && !aborted; ps += gridDim.x, ++pi) {
        if (!tc::mbar_wait(xready, pi & 1, p.status, aborted)) break;
        for (int hc = 0; hc < NCHUNK; ++hc, ++q) {
          const int st = q % W1_STAGES, sbuf = q & 1;
          if (!tc::mbar_wait(&w1full[st], (q / W1_STAGES) & 1, p.status, aborted)) break;
          if (q >= 2 && !tc::mbar_wait(&s1free[sbuf * 2 + t2], ((q >> 1) + 1) & 1, p.status, aborted)) break;
          tc::tc_fence_after();
          const uint32_t w1 = sb + OFF_W1 + st * W1C_BYTES;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int ka = k >> 2, kk = k & 3;
            tc::mma_bf16(tbase + sbuf * 128 + t2 * 64,
                         tc::smem_desc(sb + OFF_X + t2 * A_BYTES + ka * ATOM + kk * 32, 1024, tc::kSW128),
                         tc::smem_desc(w1 + ka * 8192 + kk * 32, 1024, tc::kSW128), ID1, k > 0);
          }
          tc::mma_commit(&s1full[sbuf * 2 + t2]);
          tc::mma_commit(&w1free[st]);
          if (hc == NCHUNK - 1) tc::mma_commit(xfree);
        }
      }
    }
  } else if (warp == 10) {
    // ---- GEMM2 issuer: acc[t2] += H[t2] . W2 chunk^T; it also keeps the W2 ring filled (GEMM2
    // runs a chunk or more behind GEMM1, and one producer for both rings held W1 to its pace) ----
    if (lane == 0) {
      constexpr uint32_t ID2 = tc::idesc_bf16(128, 128);
      const uint32_t total = (uint32_t)((npasses - blockIdx.x + gridDim.x - 1) / gridDim.x) * NCHUNK;
      auto load_w2 = [&](uint32_t c) {   // chunk c of this CTA into stage c % W2_STAGES (c == w2loads)
        const int st = c % W2_STAGES;
        tc::mbar_expect_tx(&w2full[st], W2C_BYTES);
        tc::tma_load_2d(smem + OFF_W2 + st * W2C_BYTES, &tmW2, &w2full[st], (int)(c % NCHUNK) * HC, 0);
        ++w2loads;
      };
      for (uint32_t c = 0; c < W2_STAGES && c < total; ++c) load_w2(c);
      uint32_t q = 0, pi = 0;
      for (int64_t ps = blockIdx.x; ps < npasses && !aborted; ps += gridDim.x, ++pi) {
        for (int hc = 0; hc < NCHUNK; ++hc, ++q) {
          const int st = q % W2_STAGES, hb = q % HBUF;
          // chunk q-1+W2_STAGES into the stage of chunk q-1 once its GEMM2 is done (it usually is)
          if (q >= 1 && q - 1 + W2_STAGES < total) {
            if (!tc::mbar_wait(&w2free[(q - 1) % W2_STAGES], ((q - 1) / W2_STAGES) & 1, p.status, aborted)) break;
            load_w2(q - 1 + W2_STAGES);
          }
          if (hc == 0 && pi >= 1 && !tc::mbar_wait(accfree, (pi - 1) & 1, p.status, aborted)) break;
          if (!tc::mbar_wait(&hfull[hb], (q / HBUF) & 1, p.status, aborted)) break;
          if (!tc::mbar_wait(&w2full[st], (q / W2_STAGES) & 1, p.status, aborted)) break;
          tc::tc_fence_after();
          const uint32_t w2 = sb + OFF_W2 + st * W2C_BYTES;
          for (int t2 = 0; t2 < 2; ++t2)
#pragma unroll
            for (int kk = 0; kk < HC / 16; ++kk)
              tc::mma_bf16(tbase + 256 + t2 * 128,
                           tc::smem_desc(sb + OFF_H + (hb * 2 + t2) * H_BYTES + kk * 32, 512, tc::kSW64),
                           tc::smem_desc(w2 + kk * 32, 512, tc::kSW64), ID2, !(hc == 0 && kk == 0));
          tc::mma_commit(&hfree[hb]);
          tc::mma_commit(&w2free[st]);
        }
        if (aborted) break;
        tc::mma_commit(accfull);
      }
    }
  } else if (warp >= 12) {
    // ---- residual epilogue: y = x + acc in units u = 4 t2 + cq (tile t2, channels 32 cq ..) ----
    const int quad = warp & 3, r = tid - 12 * 32;   // r: row of the tile = TMEM lane
    const bool leader = r == 0;                     // issues the unit loads and stores
    const uint32_t lane_addr = tbase + ((uint32_t)(32 * quad) << 16);
    // x[m0 + 128 t2 ..][32 cq ..] of unit u into staging buffer u & 1 (by the leader)
    auto load_unit = [&](int64_t m0, int u) {
      tc::mbar_expect_tx(&ybar[u & 1], Y_BYTES);
      tc::tma_load_2d(smem + OFF_Y + (u & 1) * Y_BYTES, &tmR, &ybar[u & 1], (u & 3) * 32, (int)(m0 + (u >> 2) * TILE));
      ++yloads;
    };
    uint32_t pi = 0;
    for (int64_t ps = blockIdx.x; ps < npasses; ps += gridDim.x, ++pi) {
      const int64_t m0 = ps * 2 * TILE;
      // the staging buffers are free: the leader waited for the last pass's stores to read them
      if (leader && !aborted) {
        load_unit(m0, 0);
        load_unit(m0, 1);
      }
      tc::mbar_wait(accfull, pi & 1, p.status, aborted);
      tc::tc_fence_after();
      for (int u = 0; u < 8; ++u) {
        const int t2 = u >> 2, cq = u & 3;
        uint8_t* ys = smem + OFF_Y + (u & 1) * Y_BYTES;
        float v[32];
        tc::tmem_ld32(lane_addr + 256 + t2 * 128 + 32 * cq, v);
        if (u == 7) {   // every accumulator column has been read: the next pass's GEMM2 may start
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(accfree);
        }
        // unit u's x rows are in buffer u & 1 (its use (u >> 1) of this pass, four per pass)
        tc::mbar_wait(&ybar[u & 1], (u >> 1) & 1, p.status, aborted);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4* yp = reinterpret_cast<uint4*>(ys + tc::sw64_off(r, c));
          const uint4 xx = *yp;
          const uint32_t xu[4] = {xx.x, xx.y, xx.z, xx.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) o[e] = pack_bf2(bf_lo(xu[e]) + v[8 * c + 2 * e], bf_hi(xu[e]) + v[8 * c + 2 * e + 1]);
          *yp = make_uint4(o[0], o[1], o[2], o[3]);
        }
        tc::fence_proxy_async();
        epi_sync();
        if (leader) {
          tc::tma_store_2d(&tmY, ys, cq * 32, (int)(m0 + t2 * TILE));   // rows past M are clipped
          tc::bulk_commit();
          tc::bulk_wait_read0();   // buffer u & 1 may take unit u + 2 (or the next pass's units)
          if (u + 2 < 8 && !aborted) load_unit(m0, u + 2);
        }
      }
    }
    if (leader) tc::bulk_wait0();
  } else {
    // ---- 8 warps, thread = position: warps 0-3 tile 0, 4-7 tile 1 ----
    const int t2 = warp >> 2, r = tid & 127;
    const uint32_t lane_addr = tbase + ((uint32_t)(32 * (warp & 3)) << 16);
    uint32_t q = 0, pi = 0;
    for (int64_t ps = blockIdx.x; ps < npasses; ps += gridDim.x, ++pi) {
      tc::mbar_wait(xfull, pi & 1, p.status, aborted);
      ln_row_shifted(smem + OFF_X + t2 * A_BYTES, r, lnp, lnp + C, 1e-5f);
      tc::fence_proxy_async();
      tc::mbar_arrive(xready);
      for (int hc = 0; hc < NCHUNK; ++hc, ++q) {
        const int sbuf = q & 1;
        tc::mbar_wait(&s1full[sbuf * 2 + t2], (q >> 1) & 1, p.status, aborted);
        tc::tc_fence_after();
        float ab[2 * HC];   // a (swish input) then b, adjacent columns: one load, one wait
        tc::tmem_ld64(lane_addr + sbuf * 128 + t2 * 64, ab);
        const float* a = ab;
        const float* bv = ab + HC;
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s1free[sbuf * 2 + t2]);
        uint32_t hv[HC / 2];
#pragma unroll
        for (int e = 0; e < HC / 2; ++e)
          hv[e] = pack_bf2(a[2 * e] * sigmoid_tanh(a[2 * e]) * bv[2 * e],
                           a[2 * e + 1] * sigmoid_tanh(a[2 * e + 1]) * bv[2 * e + 1]);
        const int hbuf = q % HBUF;
        if (q >= HBUF) tc::mbar_wait(&hfree[hbuf], ((q / HBUF) + 1) & 1, p.status, aborted);
        uint8_t* hrow = smem + OFF_H + (hbuf * 2 + t2) * H_BYTES;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(hrow + tc::sw64_off(r, c)) =
              make_uint4(hv[4 * c], hv[4 * c + 1], hv[4 * c + 2], hv[4 * c + 3]);
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&hfull[hbuf]);
      }
    }
  }
  tc::tc_fence_before();
  if (__syncthreads_or(aborted)) {   // abort path: drain every ring's loads and every issuer's MMAs
    if (lane == 0) {
      if (warp == 8) {
        tc::drain_ring(xfull, 1, xloads, p.status);
        tc::drain_ring(w1full, W1_STAGES, w1loads, p.status);
      }
      if (warp == 12) tc::drain_ring(ybar, 2, yloads, p.status);
      if (warp >= 9 && warp <= 11) {
        if (warp == 10) tc::drain_ring(w2full, W2_STAGES, w2loads, p.status);
        tc::drain_mma(&drain[warp - 9], p.status);
      }
    }
    __syncthreads();
  }
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
  if (swizzle_bytes != 128 && swizzle_bytes != 64 && swizzle_bytes != 0) {
    set_error("2-d tensor map: unsupported swizzle %d", swizzle_bytes);
    return SF_ERR_ARG;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
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
  SF_REQUIRE((reinterpret_cast<uintptr_t>(ln_w) & 15) == 0 && (reinterpret_cast<uintptr_t>(ln_b) & 15) == 0,
             "transition_tc: layer-norm parameters must be 16-byte aligned");
  CUtensorMap mx, mw1, mw2, my;
  SF_TRY(make_2d_tmap(&mx, x, C, M, 64, TILE));
  SF_TRY(make_2d_tmap(&my, y, C, M, 32, TILE, 64));          // residual epilogue units: 32 channels x 128 rows
  CUtensorMap mr;
  SF_TRY(make_2d_tmap(&mr, x, C, M, 32, TILE, 64));
  SF_TRY(make_2d_tmap(&mw1, w1, C, 2 * I, 64, HC));         // W1 [1024][128]: 64 k x 32 rows
  SF_TRY(make_2d_tmap(&mw2, w2, I, C, HC, C, 64));          // W2 [128][512]: 32 k x 128 rows, 64B swizzle
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
  launch_pdl(k_transition_tc, dim3(grid), dim3(TR_THREADS), SMEM_TR, stream, mx, mw1, mw2, my, mr, p);
  count_launch();
  return check_launch("transition_tc");
}

}  // namespace sf
