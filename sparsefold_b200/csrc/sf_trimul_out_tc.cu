// Output phase of triangle multiplication on tcgen05 (blocks.py:559-566), bf16 track:
//   z_out = z + (centerLN(P) W_out) * sigmoid(LN(z) W_gate)
//
// Persistent, one warp-specialised CTA per SM, one 128-position tile (pair row
// r, columns s0..s0+127) at a time, two tiles in flight:
//   warp 12     TMA producer: raw z tile (128B swizzle, two stages) and P tile
//               ([128 channels][128 positions] of one pair row, no swizzle)
//   warps 8-11  thread = position: LN(z) into the A1 tile; center LayerNorm of the
//               position's 128 channels of P (center_norm, dim=-3) into the K-major
//               A2 tile
//   warp 13     MMA issuer: gate = A1 W_gate^T and update = A2 W_out^T (M=N=K=128,
//               weights resident) into one of two TMEM buffers of 256 columns
//   warps 0-7   epilogue: warp w takes positions 32(w%4).. and channels 64(w/4)..,
//               adds update * sigmoid(gate) to the raw z still in shared memory, in
//               place, and TMA-stores that 32 x 64 block of z_out.
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int OUT_EPI_WARPS = 8;
constexpr int OUT_THREADS = (OUT_EPI_WARPS + 4 + 2) * 32;
constexpr int OFF_WG = 0, OFF_WO = A_BYTES;
constexpr int OFF_Z = 2 * A_BYTES;              // [2] raw z tiles, then z_out staging
constexpr int OFF_P = OFF_Z + 2 * A_BYTES;      // P tile [channel][position]
constexpr int OFF_A1 = OFF_P + A_BYTES;         // LN(z)
constexpr int OFF_A2 = OFF_A1 + A_BYTES;        // centerLN(P), K-major
constexpr int OFF_BAR = OFF_A2 + A_BYTES;
constexpr int OFF_CW = OFF_BAR + 256;           // center-norm scale and offset, 128 floats each
constexpr int OFF_CB = OFF_CW + C * 4;
constexpr int SMEM_OUT = OFF_CB + C * 4 + 1024;

struct OutParams {
  const float *ln_w, *ln_b, *center_w, *center_b;
  int64_t rows, n;
  uint32_t* status;
};

__global__ void __launch_bounds__(OUT_THREADS, 1) k_trimul_output_tc(const __grid_constant__ CUtensorMap tmZ,
                                                                     const __grid_constant__ CUtensorMap tmP,
                                                                     const __grid_constant__ CUtensorMap tmO,
                                                                     const bf16* __restrict__ w_gate,
                                                                     const bf16* __restrict__ w_out, OutParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* zfull = reinterpret_cast<uint64_t*>(smem + OFF_BAR);  // [2] z tile landed
  uint64_t* zfree = zfull + 2;                                      // [2] z_out stored (8 warps)
  uint64_t* tfull = zfree + 2;                                      // [2] TMEM buffer written
  uint64_t* tfree = tfull + 2;                                      // [2] TMEM buffer read (8 warps)
  uint64_t* pfull = tfree + 2;                                      // P tile landed
  uint64_t* pfree = pfull + 1;                                      // P tile read (128)
  uint64_t* normed = pfree + 1;                                     // A1 and A2 written (128)
  uint64_t* afree = normed + 1;                                     // MMAs done with A1 and A2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(afree + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t nb = (p.n + TILE - 1) / TILE, ntiles = p.rows * nb;

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(&zfull[s], 1);
      tc::mbar_init(&zfree[s], OUT_EPI_WARPS);
      tc::mbar_init(&tfull[s], 1);
      tc::mbar_init(&tfree[s], OUT_EPI_WARPS);
    }
    tc::mbar_init(pfull, 1);
    tc::mbar_init(pfree, 128);
    tc::mbar_init(normed, 128);
    tc::mbar_init(afree, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmZ);
    tc::prefetch_tmap(&tmP);
    tc::prefetch_tmap(&tmO);
  }
  if (tid < C) {
    reinterpret_cast<float*>(smem + OFF_CW)[tid] = p.center_w[tid];
    reinterpret_cast<float*>(smem + OFF_CB)[tid] = p.center_b[tid];
  }
  load_weight_sw128(smem + OFF_WG, w_gate, C, tid, OUT_THREADS);
  load_weight_sw128(smem + OFF_WO, w_out, C, tid, OUT_THREADS);
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t sb = tc::smem_u32(smem);
  bool aborted = false;

  if (warp == 12) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const int st = it & 1;
        if (it >= 2) tc::mbar_wait(&zfree[st], ((it >> 1) + 1) & 1, p.status, aborted);
        const int64_t r = tile / nb, s0 = (tile % nb) * TILE;
        uint8_t* zs = smem + OFF_Z + st * A_BYTES;
        tc::mbar_expect_tx(&zfull[st], A_BYTES);
        tc::tma_load_3d(zs, &tmZ, &zfull[st], 0, (int)s0, (int)r);
        tc::tma_load_3d(zs + ATOM, &tmZ, &zfull[st], 64, (int)s0, (int)r);
        if (it >= 1) tc::mbar_wait(pfree, (it - 1) & 1, p.status, aborted);
        tc::mbar_expect_tx(pfull, A_BYTES);
        tc::tma_load_3d(smem + OFF_P, &tmP, pfull, (int)s0, 0, (int)r);
      }
    }
  } else if (warp == 13) {
    if (lane == 0) {
      constexpr uint32_t IDESC = tc::idesc_bf16(128, 128);
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        tc::mbar_wait(normed, it & 1, p.status, aborted);
        if (it >= 2) tc::mbar_wait(&tfree[buf], ((it >> 1) + 1) & 1, p.status, aborted);
        tc::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int ka = k >> 2, kk = k & 3;
          tc::mma_bf16(tbase + buf * 256, tc::smem_desc(sb + OFF_A1 + ka * ATOM + kk * 32, 1024, tc::kSW128),
                       tc::smem_desc(sb + OFF_WG + ka * ATOM + kk * 32, 1024, tc::kSW128), IDESC, k > 0);
          tc::mma_bf16(tbase + buf * 256 + 128, tc::smem_desc(sb + OFF_A2 + ka * ATOM + kk * 32, 1024, tc::kSW128),
                       tc::smem_desc(sb + OFF_WO + ka * ATOM + kk * 32, 1024, tc::kSW128), IDESC, k > 0);
        }
        tc::mma_commit(&tfull[buf]);
        tc::mma_commit(afree);
      }
    }
  } else if (warp >= OUT_EPI_WARPS) {
    // ---- layer norms, thread = position ----
    const int pos = tid - OUT_EPI_WARPS * 32;
    const float* cw = reinterpret_cast<const float*>(smem + OFF_CW);
    const float* cb = reinterpret_cast<const float*>(smem + OFF_CB);
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int st = it & 1;
      tc::mbar_wait(&zfull[st], (it >> 1) & 1, p.status, aborted);
      if (it >= 1) tc::mbar_wait(afree, (it - 1) & 1, p.status, aborted);
      ln_row_lr(smem + OFF_Z + st * A_BYTES, smem + OFF_A1, pos, p.ln_w, p.ln_b, 1e-5f);
      // center LayerNorm of this position across the 128 channels of P (column `pos`)
      tc::mbar_wait(pfull, it & 1, p.status, aborted);
      const bf16* pc = reinterpret_cast<const bf16*>(smem + OFF_P) + pos;
      float s = 0.f;
#pragma unroll 16
      for (int c = 0; c < C; ++c) s += __bfloat162float(pc[c * TILE]);
      const float mean = s * (1.0f / C);
      float q = 0.f;
#pragma unroll 16
      for (int c = 0; c < C; ++c) {
        const float d = __bfloat162float(pc[c * TILE]) - mean;
        q += d * d;
      }
      const float rstd = rsqrtf(q * (1.0f / C) + 1e-5f);
#pragma unroll 2
      for (int kc = 0; kc < 16; ++kc) {
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 8 * kc + 2 * e;
          o[e] = pack_bf2((__bfloat162float(pc[c * TILE]) - mean) * rstd * cw[c] + cb[c],
                          (__bfloat162float(pc[(c + 1) * TILE]) - mean) * rstd * cw[c + 1] + cb[c + 1]);
        }
        *reinterpret_cast<uint4*>(smem + OFF_A2 + (kc >> 3) * ATOM + tc::sw128_off(pos, kc & 7)) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
      tc::mbar_arrive(pfree);
      tc::fence_proxy_async();
      tc::mbar_arrive(normed);
    }
  } else {
    // ---- epilogue: positions 32*quad.., channels 64*hf.. ----
    const int quad = warp & 3, hf = warp >> 2, pos = 32 * quad + lane;
    const uint32_t lane_addr = tbase + ((uint32_t)(32 * quad) << 16);
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int st = it & 1, buf = it & 1;
      const int64_t r = tile / nb, s0 = (tile % nb) * TILE;
      tc::mbar_wait(&tfull[buf], (it >> 1) & 1, p.status, aborted);
      tc::tc_fence_after();
      uint8_t* zrow = smem + OFF_Z + st * A_BYTES + hf * ATOM;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float g[16], u[16];
        tc::tmem_ld16(lane_addr + buf * 256 + 64 * hf + 16 * k, g);
        tc::tmem_ld16(lane_addr + buf * 256 + 128 + 64 * hf + 16 * k, u);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint4* zp = reinterpret_cast<uint4*>(zrow + tc::sw128_off(pos, 2 * k + h2));
          uint4 zz = *zp;
          uint32_t* zu = reinterpret_cast<uint32_t*>(&zz);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 8 * h2 + 2 * e;
            zu[e] = pack_bf2(bf_lo(zu[e]) + u[j] * sigmoid_tanh(g[j]), bf_hi(zu[e]) + u[j + 1] * sigmoid_tanh(g[j + 1]));
          }
          *zp = zz;
        }
      }
      tc::tc_fence_before();
      tc::fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&tfree[buf]);
        if (s0 + 32 * quad < p.n) {
          tc::tma_store_3d(&tmO, zrow + 32 * quad * 128, 64 * hf, (int)(s0 + 32 * quad), (int)r);
          tc::bulk_commit();
          tc::bulk_wait_read0();
        }
        tc::mbar_arrive(&zfree[st]);
      }
    }
    if (lane == 0) tc::bulk_wait0();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

}  // namespace

// Output phase on tcgen05; z_out may alias z (each tile is read before it is written).
int trimul_output_tc(const bf16* z, const bf16* P, int64_t rows, int64_t n, const float* ln_w, const float* ln_b,
                     const float* center_w, const float* center_b, const bf16* w_gate, const bf16* w_out, bf16* z_out,
                     cudaStream_t stream) {
  if (rows == 0 || n == 0) return SF_OK;
  SF_REQUIRE(n <= (1 << 24) && rows <= (1 << 24), "trimul_output_tc: size too large");
  SF_REQUIRE((reinterpret_cast<uintptr_t>(ln_w) & 15) == 0 && (reinterpret_cast<uintptr_t>(ln_b) & 15) == 0,
             "trimul_output_tc: layer-norm parameters must be 16-byte aligned");
  CUtensorMap mz, mp, mo;
  SF_TRY(make_pair_tmap(&mz, z, rows, n, false));
  {
    auto encode = tensor_map_encoder();
    if (!encode) return SF_ERR_CUDA;
    if ((reinterpret_cast<uintptr_t>(P) & 15) != 0 || (reinterpret_cast<uintptr_t>(z_out) & 15) != 0) {
      set_error("trimul_output_tc: P %p / z_out %p not 16-byte aligned", (const void*)P, (void*)z_out);
      return SF_ERR_ARG;
    }
    const int64_t pitch = pair_pitch(n);
    // P is [rows][C][pitch]: box = 128 positions x all 128 channels of one pair row
    cuuint64_t dims[3] = {(cuuint64_t)pitch, (cuuint64_t)C, (cuuint64_t)rows};
    cuuint64_t strides[2] = {(cuuint64_t)pitch * 2, (cuuint64_t)(C * pitch * 2)};
    cuuint32_t box[3] = {(cuuint32_t)TILE, (cuuint32_t)C, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(&mp, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16*>(P), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled failed (%d) for P", (int)r);
      return SF_ERR_CUDA;
    }
    // z_out [rows][n][128]: store box = 64 channels x 32 positions x 1 row (128B swizzle)
    cuuint64_t odims[3] = {(cuuint64_t)C, (cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t ostr[2] = {(cuuint64_t)C * 2, (cuuint64_t)(n * C * 2)};
    cuuint32_t obox[3] = {64, 32, 1};
    r = encode(&mo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, z_out, odims, ostr, obox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled failed (%d) for z_out", (int)r);
      return SF_ERR_CUDA;
    }
  }
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(k_trimul_output_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_OUT);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(trimul_output): %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    attr[dev & 63] = true;
  }
  OutParams p{ln_w, ln_b, center_w, center_b, rows, n, status};
  const int64_t ntiles = rows * ((n + TILE - 1) / TILE);
  const int grid = (int)(ntiles < num_sms() ? ntiles : num_sms());
  k_trimul_output_tc<<<grid, OUT_THREADS, SMEM_OUT, stream>>>(mz, mp, mo, w_gate, w_out, p);
  count_launch();
  return check_launch("trimul_output_tc");
}

}  // namespace sf
