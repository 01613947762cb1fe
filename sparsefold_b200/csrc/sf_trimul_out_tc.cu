// Output phase of triangle multiplication on tcgen05 (blocks.py:559-566), bf16 track:
//   z_out = z + (centerLN(P) W_out) * sigmoid(LN(z) W_gate)
//
// Persistent, one CTA (4 warps) per SM, one 128-position tile (pair row r,
// columns s0..s0+127) per iteration.  TMA brings the raw z tile (128B swizzle)
// and the P tile ([128 channels][128 positions] of one pair row, no swizzle).
// Each thread layer-norms its z row in place (A1) and normalises its
// position's 128 channels of P across the channel axis (center_norm, dim=-3)
// into the K-major A2 tile.  Two tcgen05 GEMMs against the resident gating and
// output weights fill TMEM columns [0,128) and [128,256); the epilogue adds
// the gated update to z.
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int OFF_A1 = 0, OFF_A2 = A_BYTES, OFF_P = 2 * A_BYTES, OFF_WG = 3 * A_BYTES, OFF_WO = 4 * A_BYTES;
constexpr int OFF_BAR = 5 * A_BYTES;
constexpr int SMEM_OUT = OFF_BAR + 1024 + 1024;

struct OutParams {
  const bf16* z;
  bf16* z_out;
  const float *ln_w, *ln_b, *center_w, *center_b;
  const bf16 *w_gate, *w_out;
  int64_t rows, n;
  uint32_t* status;
};

__global__ void __launch_bounds__(128, 1) k_trimul_output_tc(const __grid_constant__ CUtensorMap tmZ,
                                                             const __grid_constant__ CUtensorMap tmP,
                                                             OutParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* ldbar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* mmabar = ldbar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ldbar + 2);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t nb = (p.n + TILE - 1) / TILE, ntiles = p.rows * nb;

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(ldbar, 1);
    tc::mbar_init(mmabar, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmZ);
    tc::prefetch_tmap(&tmP);
  }
  load_weight_sw128(smem + OFF_WG, p.w_gate, C, tid, 128);
  load_weight_sw128(smem + OFF_WO, p.w_out, C, tid, 128);
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t sb = tc::smem_u32(smem);
  const uint32_t lane_addr = tbase + ((uint32_t)(warp * 32) << 16);
  bool aborted = false;
  constexpr uint32_t IDESC = tc::idesc_bf16(128, 128);

  uint32_t it = 0;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
    const int64_t r = tile / nb, s0 = (tile % nb) * TILE;
    if (tid == 0) {
      tc::mbar_expect_tx(ldbar, 2 * A_BYTES);
      tc::tma_load_3d(smem + OFF_A1, &tmZ, ldbar, 0, (int)s0, (int)r);
      tc::tma_load_3d(smem + OFF_A1 + ATOM, &tmZ, ldbar, 64, (int)s0, (int)r);
      tc::tma_load_3d(smem + OFF_P, &tmP, ldbar, (int)s0, 0, (int)r);
    }
    tc::mbar_wait(ldbar, it & 1, p.status, aborted);
    ln_row_inplace(smem + OFF_A1, tid, p.ln_w, p.ln_b, 1e-5f);
    {
      // center LayerNorm of position tid across the 128 channels of P
      const bf16* pc = reinterpret_cast<const bf16*>(smem + OFF_P) + tid;
      float s = 0.f;
#pragma unroll 8
      for (int c = 0; c < C; ++c) s += __bfloat162float(pc[c * TILE]);
      const float mean = s * (1.0f / C);
      float q = 0.f;
#pragma unroll 8
      for (int c = 0; c < C; ++c) {
        const float d = __bfloat162float(pc[c * TILE]) - mean;
        q += d * d;
      }
      const float rstd = rsqrtf(q * (1.0f / C) + 1e-5f);
#pragma unroll 2
      for (int kc = 0; kc < 16; ++kc) {
        uint4 o;
        uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = kc * 8 + 2 * e;
          ou[e] = pack_bf2((__bfloat162float(pc[c * TILE]) - mean) * rstd * __ldg(p.center_w + c) + __ldg(p.center_b + c),
                           (__bfloat162float(pc[(c + 1) * TILE]) - mean) * rstd * __ldg(p.center_w + c + 1) +
                               __ldg(p.center_b + c + 1));
        }
        *reinterpret_cast<uint4*>(smem + OFF_A2 + (kc >> 3) * ATOM + tc::sw128_off(tid, kc & 7)) = o;
      }
    }
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int ka = k >> 2, kk = k & 3;
        tc::mma_bf16(tbase, tc::smem_desc(sb + OFF_A1 + ka * ATOM + kk * 32, 1024, tc::kSW128),
                     tc::smem_desc(sb + OFF_WG + ka * ATOM + kk * 32, 1024, tc::kSW128), IDESC, k > 0);
        tc::mma_bf16(tbase + 128, tc::smem_desc(sb + OFF_A2 + ka * ATOM + kk * 32, 1024, tc::kSW128),
                     tc::smem_desc(sb + OFF_WO + ka * ATOM + kk * 32, 1024, tc::kSW128), IDESC, k > 0);
      }
      tc::mma_commit(mmabar);
    }
    tc::mbar_wait(mmabar, it & 1, p.status, aborted);
    tc::tc_fence_after();
    const int64_t s = s0 + tid;
    const bool live = s < p.n;
    const int64_t pos = live ? r * p.n + s : 0;
    const uint4* zin = reinterpret_cast<const uint4*>(p.z + pos * C);
    uint4* zo = reinterpret_cast<uint4*>(p.z_out + pos * C);
#pragma unroll 1
    for (int i = 0; i < 8; ++i) {
      float g[16], u[16];
      tc::tmem_ld16(lane_addr + 16 * i, g);
      tc::tmem_ld16(lane_addr + 128 + 16 * i, u);
      if (live) {
#pragma unroll
        for (int hlf = 0; hlf < 2; ++hlf) {
          const uint4 zz = zin[2 * i + hlf];
          const uint32_t* zu = reinterpret_cast<const uint32_t*>(&zz);
          uint4 o;
          uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = hlf * 8 + 2 * e;
            ou[e] = pack_bf2(bf_lo(zu[e]) + u[j] * fast_sigmoid(g[j]), bf_hi(zu[e]) + u[j + 1] * fast_sigmoid(g[j + 1]));
          }
          zo[2 * i + hlf] = o;
        }
      }
    }
    tc::tc_fence_before();
    __syncthreads();   // smem tiles and TMEM free for the next tile
  }
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 256);
  }
}

}  // namespace

// Output phase on tcgen05; z_out may alias z (each position is read and written by one thread).
int trimul_output_tc(const bf16* z, const bf16* P, int64_t rows, int64_t n, const float* ln_w, const float* ln_b,
                     const float* center_w, const float* center_b, const bf16* w_gate, const bf16* w_out, bf16* z_out,
                     cudaStream_t stream) {
  if (rows == 0 || n == 0) return SF_OK;
  CUtensorMap mz, mp;
  SF_TRY(make_pair_tmap(&mz, z, rows, n, false));
  {
    auto encode = tensor_map_encoder();
    if (!encode) return SF_ERR_CUDA;
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
  OutParams p{z, z_out, ln_w, ln_b, center_w, center_b, w_gate, w_out, rows, n, status};
  const int64_t ntiles = rows * ((n + TILE - 1) / TILE);
  const int grid = (int)(ntiles < num_sms() ? ntiles : num_sms());
  k_trimul_output_tc<<<grid, 128, SMEM_OUT, stream>>>(mz, mp, p);
  count_launch();
  return check_launch("trimul_output_tc");
}

}  // namespace sf
