// Output phase of triangle multiplication on tcgen05 (blocks.py:559-566), bf16 track:
//   z_out = z + (centerLN(P) W_out) * sigmoid(LN(z) W_gate)
//
// Both layer norms are folded into the GEMMs, so the tensor core reads the raw
// tiles as they arrive: with LN(x)[c] = (x[c] - mu) rho w[c] + b[c],
//   LN(x) . W[o] = rho (x . W'[o] - mu s[o]) + b'[o],
//   W'[o][c] = W[o][c] w[c] (bf16),  s[o] = sum_c W'[o][c],  b'[o] = sum_c b[c] W[o][c],
// and the epilogue applies rho, mu of each position.  Persistent, one
// warp-specialised CTA per SM, one 128-position tile (pair row r, columns
// s0..s0+127) at a time, two tiles in flight:
//   warp 12     TMA producer: raw z tile (K-major, 128B swizzle) and P tile
//               ([128 channels][128 positions] as two 64-position boxes, 128B
//               swizzle: the M-major A operand of the update GEMM), two stages each
//   warp 13     MMA issuer: gate = z W_gate'^T and update = P^T W_out'^T (M=N=K=128,
//               folded weights resident) into one of two TMEM buffers of 256 columns
//   warps 8-11  per-position statistics, all as one pass of sums shifted by a
//               value of the row or column: thread = position for its z row; for
//               the P columns each thread sums a 16-byte chunk (8 positions) over 16
//               channel rows and thread = position adds the 8 groups' partials
//   warps 0-7   epilogue: warp w takes positions 32(w%4).. and channels 64(w/4)..,
//               applies the folded norms, adds update * sigmoid(gate) to the raw z
//               still in shared memory, in place, and TMA-stores that 32 x 64 block.
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int OUT_EPI_WARPS = 8;
constexpr int OUT_THREADS = (OUT_EPI_WARPS + 4 + 2) * 32;
constexpr int OFF_WG = 0, OFF_WO = A_BYTES;     // folded weights (K-major, 128B swizzle)
constexpr int OFF_Z = 2 * A_BYTES;              // [2] raw z tiles, then z_out staging
constexpr int OFF_P = OFF_Z + 2 * A_BYTES;      // [2] P tiles: two 64-position boxes of [128 ch][64 pos]
constexpr int OFF_ST = OFF_P + 2 * A_BYTES;     // [2][4][128] floats: mean z, rstd z, mean P, rstd P
constexpr int OFF_VEC = OFF_ST + 2 * 4 * C * 4; // [4][128] floats: s_gate, b_gate, s_out, b_out
constexpr int OFF_PART = OFF_VEC + 4 * C * 4;   // [2][8 channel groups][2][128] floats: P column partial sums
constexpr int OFF_BAR = OFF_PART + 2 * 8 * 2 * C * 4;
constexpr int SMEM_OUT = OFF_BAR + 256 + 1024;
static_assert(SMEM_OUT <= 232448, "trimul output shared memory");

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
  uint64_t* pfull = zfree + 2;                                      // [2] P tile landed
  uint64_t* pfree = pfull + 2;                                      // [2] P read by the MMA (commit) and the stats (128)
  uint64_t* sfull = pfree + 2;                                      // [2] stats written (128)
  uint64_t* tfull = sfull + 2;                                      // [2] TMEM buffer written
  uint64_t* tfree = tfull + 2;                                      // [2] TMEM buffer read (8 warps)
  uint64_t* drain = tfree + 2;                                      // MMA drain barrier (abort path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t nb = (p.n + TILE - 1) / TILE, ntiles = p.rows * nb;
  float* vec = reinterpret_cast<float*>(smem + OFF_VEC);

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(&zfull[s], 1);
      tc::mbar_init(&zfree[s], OUT_EPI_WARPS);
      tc::mbar_init(&pfull[s], 1);
      tc::mbar_init(&pfree[s], 1 + 128);
      tc::mbar_init(&sfull[s], 128);
      tc::mbar_init(&tfull[s], 1);
      tc::mbar_init(&tfree[s], OUT_EPI_WARPS);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmZ);
    tc::prefetch_tmap(&tmP);
    tc::prefetch_tmap(&tmO);
  }
  {
    // both norms folded into their weights; their parameters go through the (still unused) stats area
    float* prm = reinterpret_cast<float*>(smem + OFF_ST);
    stage_norm_params(prm, prm + C, p.ln_w, p.ln_b, tid);
    stage_norm_params(prm + 2 * C, prm + 3 * C, p.center_w, p.center_b, tid);
    __syncthreads();
    fold_weight(smem + OFF_WG, w_gate, prm, prm + C, C, vec, vec + C, tid, OUT_THREADS);
    fold_weight(smem + OFF_WO, w_out, prm + 2 * C, prm + 3 * C, C, vec + 2 * C, vec + 3 * C, tid, OUT_THREADS);
  }
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  tc::griddep_wait();     // the previous kernel's outputs are complete and visible from here on
  tc::griddep_launch();
  const uint32_t tbase = *tmem_slot;
  const uint32_t sb = tc::smem_u32(smem);
  bool aborted = false;
  uint32_t zloads = 0, ploads = 0;   // z and P tiles requested by the producer (abort-path drain)

  if (warp == 12) {
    // ---- TMA producer (stops at its first failed wait) ----
    if (lane == 0) {
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const int st = it & 1;
        const int64_t r = tile / nb, s0 = (tile % nb) * TILE;
        if (it >= 2 && !tc::mbar_wait(&zfree[st], ((it >> 1) + 1) & 1, p.status, aborted)) break;
        uint8_t* zs = smem + OFF_Z + st * A_BYTES;
        tc::mbar_expect_tx(&zfull[st], A_BYTES);
        tc::tma_load_3d(zs, &tmZ, &zfull[st], 0, (int)s0, (int)r);
        tc::tma_load_3d(zs + ATOM, &tmZ, &zfull[st], 64, (int)s0, (int)r);
        ++zloads;
        if (it >= 2 && !tc::mbar_wait(&pfree[st], ((it >> 1) + 1) & 1, p.status, aborted)) break;
        uint8_t* ps = smem + OFF_P + st * A_BYTES;
        tc::mbar_expect_tx(&pfull[st], A_BYTES);
        tc::tma_load_3d(ps, &tmP, &pfull[st], (int)s0, 0, (int)r);
        tc::tma_load_3d(ps + ATOM, &tmP, &pfull[st], (int)s0 + 64, 0, (int)r);
        ++ploads;
      }
    }
  } else if (warp == 13) {
    // ---- MMA issuer (stops at its first failed wait) ----
    if (lane == 0) {
      constexpr uint32_t IDESC_G = tc::idesc_bf16(128, 128);
      constexpr uint32_t IDESC_U = tc::idesc_bf16(128, 128) | (1u << 15);   // A (P) M-major
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const int st = it & 1, buf = it & 1;
        if (!tc::mbar_wait(&zfull[st], (it >> 1) & 1, p.status, aborted)) break;
        if (!tc::mbar_wait(&pfull[st], (it >> 1) & 1, p.status, aborted)) break;
        if (it >= 2 && !tc::mbar_wait(&tfree[buf], ((it >> 1) + 1) & 1, p.status, aborted)) break;
        tc::tc_fence_after();
        const uint32_t zb = sb + OFF_Z + st * A_BYTES, pb = sb + OFF_P + st * A_BYTES;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int ka = k >> 2, kk = k & 3;
          tc::mma_bf16(tbase + buf * 256, tc::smem_desc(zb + ka * ATOM + kk * 32, 1024, tc::kSW128),
                       tc::smem_desc(sb + OFF_WG + ka * ATOM + kk * 32, 1024, tc::kSW128), IDESC_G, k > 0);
          // P: channels 16k .. 16k+15 are rows 16k.. of both 64-position boxes (atoms 16 KB apart)
          tc::mma_bf16(tbase + buf * 256 + 128, tc::smem_desc_mn(pb + k * 2048, ATOM, 1024, tc::kSW128),
                       tc::smem_desc(sb + OFF_WO + ka * ATOM + kk * 32, 1024, tc::kSW128), IDESC_U, k > 0);
        }
        tc::mma_commit(&tfull[buf]);
        tc::mma_commit(&pfree[st]);
      }
    }
  } else if (warp >= OUT_EPI_WARPS) {
    // ---- per-position statistics ----
    const int pos = tid - OUT_EPI_WARPS * 32;
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int st = it & 1;
      float* stats = reinterpret_cast<float*>(smem + OFF_ST) + st * 4 * C;
      tc::mbar_wait(&zfull[st], (it >> 1) & 1, p.status, aborted);
      {
        // z row: one pass of sums shifted by its first value (E[(x-k)^2] - E[x-k]^2 keeps its
        // precision), four independent accumulator pairs
        const uint8_t* zs = smem + OFF_Z + st * A_BYTES;
        const float k0 = bf_lo(*reinterpret_cast<const uint32_t*>(zs + tc::sw128_off(pos, 0)));
        float s[4] = {0.f, 0.f, 0.f, 0.f}, q[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const uint4 v = *reinterpret_cast<const uint4*>(zs + (i >> 3) * ATOM + tc::sw128_off(pos, i & 7));
          const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float d0 = bf_lo(u[e]) - k0, d1 = bf_hi(u[e]) - k0;
            s[e] += d0 + d1;
            q[e] = fmaf(d0, d0, fmaf(d1, d1, q[e]));
          }
        }
        const float md = ((s[0] + s[1]) + (s[2] + s[3])) * (1.0f / C);
        stats[pos] = k0 + md;
        stats[C + pos] = rsqrtf(fmaxf(((q[0] + q[1]) + (q[2] + q[3])) * (1.0f / C) - md * md, 0.f) + 1e-5f);
      }
      tc::mbar_wait(&pfull[st], (it >> 1) & 1, p.status, aborted);
      {
        // P column sums shifted by the column's channel-0 value: thread t takes the 8 positions
        // of one 16-byte chunk (group t % 16) over 16 channel rows (group t / 16), then thread
        // pos adds the 8 groups' partials for its column
        const int pg = pos & 15, cg = pos >> 4;
        const uint8_t* pbox = smem + OFF_P + st * A_BYTES + (pg >> 3) * ATOM;
        const int chunk = pg & 7;
        auto prow = [&](int c) { return *reinterpret_cast<const uint4*>(pbox + c * 128 + ((chunk ^ (c & 7)) << 4)); };
        float x0[8];
        {
          const uint4 v = prow(0);
          const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            x0[2 * e] = bf_lo(u[e]);
            x0[2 * e + 1] = bf_hi(u[e]);
          }
        }
        float s8[8], q8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) s8[e] = q8[e] = 0.f;
#pragma unroll 4
        for (int c = 16 * cg; c < 16 * cg + 16; ++c) {
          const uint4 v = prow(c);
          const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float d0 = bf_lo(u[e]) - x0[2 * e], d1 = bf_hi(u[e]) - x0[2 * e + 1];
            s8[2 * e] += d0;
            s8[2 * e + 1] += d1;
            q8[2 * e] = fmaf(d0, d0, q8[2 * e]);
            q8[2 * e + 1] = fmaf(d1, d1, q8[2 * e + 1]);
          }
        }
        float* part = reinterpret_cast<float*>(smem + OFF_PART) + st * 8 * 2 * C + cg * 2 * C;
        *reinterpret_cast<float4*>(part + 8 * pg) = make_float4(s8[0], s8[1], s8[2], s8[3]);
        *reinterpret_cast<float4*>(part + 8 * pg + 4) = make_float4(s8[4], s8[5], s8[6], s8[7]);
        *reinterpret_cast<float4*>(part + C + 8 * pg) = make_float4(q8[0], q8[1], q8[2], q8[3]);
        *reinterpret_cast<float4*>(part + C + 8 * pg + 4) = make_float4(q8[4], q8[5], q8[6], q8[7]);
        asm volatile("bar.sync 1, 128;" ::: "memory");   // the four statistics warps
        const float* pall = reinterpret_cast<const float*>(smem + OFF_PART) + st * 8 * 2 * C;
        float ss = 0.f, qq = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          ss += pall[g * 2 * C + pos];
          qq += pall[g * 2 * C + C + pos];
        }
        // the shift of column pos is its own channel-0 value
        const float x0p = __bfloat162float(*reinterpret_cast<const bf16*>(
            smem + OFF_P + st * A_BYTES + (pos >> 6) * ATOM + ((((pos & 63) >> 3) ^ 0) << 4) + (pos & 7) * 2));
        const float md = ss * (1.0f / C);
        stats[2 * C + pos] = x0p + md;
        stats[3 * C + pos] = rsqrtf(fmaxf(qq * (1.0f / C) - md * md, 0.f) + 1e-5f);
      }
      tc::mbar_arrive(&pfree[st]);
      tc::mbar_arrive(&sfull[st]);
    }
  } else {
    // ---- epilogue: positions 32*quad.., channels 64*hf.. ----
    const int quad = warp & 3, hf = warp >> 2, pos = 32 * quad + lane;
    const uint32_t lane_addr = tbase + ((uint32_t)(32 * quad) << 16);
    const float* sg = vec + 64 * hf;
    const float* bg = vec + C + 64 * hf;
    const float* so = vec + 2 * C + 64 * hf;
    const float* bo = vec + 3 * C + 64 * hf;
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int st = it & 1, buf = it & 1;
      const int64_t r = tile / nb, s0 = (tile % nb) * TILE;
      const float* stats = reinterpret_cast<const float*>(smem + OFF_ST) + st * 4 * C;
      tc::mbar_wait(&sfull[st], (it >> 1) & 1, p.status, aborted);
      const float mz = stats[pos], rz = stats[C + pos], mp = stats[2 * C + pos], rp = stats[3 * C + pos];
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
          const uint4 zz = *zp;
          const uint32_t zu[4] = {zz.x, zz.y, zz.z, zz.w};
          // the folded-norm vectors of these 8 channels, 16-byte loads (the same for every lane)
          const int c0 = 16 * k + 8 * h2;
          float vs[4][8];
          const float* srcv[4] = {sg, bg, so, bo};
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            const float4 a = *reinterpret_cast<const float4*>(srcv[v4] + c0);
            const float4 b = *reinterpret_cast<const float4*>(srcv[v4] + c0 + 4);
            vs[v4][0] = a.x; vs[v4][1] = a.y; vs[v4][2] = a.z; vs[v4][3] = a.w;
            vs[v4][4] = b.x; vs[v4][5] = b.y; vs[v4][6] = b.z; vs[v4][7] = b.w;
          }
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 8 * h2 + 2 * e, c = 2 * e;
            const float g0 = fmaf(rz, fmaf(-mz, vs[0][c], g[j]), vs[1][c]);
            const float g1 = fmaf(rz, fmaf(-mz, vs[0][c + 1], g[j + 1]), vs[1][c + 1]);
            const float u0 = fmaf(rp, fmaf(-mp, vs[2][c], u[j]), vs[3][c]);
            const float u1 = fmaf(rp, fmaf(-mp, vs[2][c + 1], u[j + 1]), vs[3][c + 1]);
            o[e] = pack_bf2(fmaf(u0, sigmoid_tanh(g0), bf_lo(zu[e])), fmaf(u1, sigmoid_tanh(g1), bf_hi(zu[e])));
          }
          *zp = make_uint4(o[0], o[1], o[2], o[3]);
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
  if (__syncthreads_or(aborted)) {   // abort path: drain the producer's loads and the issuer's MMAs
    if (warp == 12 && lane == 0) {
      tc::drain_ring(zfull, 2, zloads, p.status);
      tc::drain_ring(pfull, 2, ploads, p.status);
    }
    if (warp == 13 && lane == 0) tc::drain_mma(drain, p.status);
    __syncthreads();
  }
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
  SF_REQUIRE(((reinterpret_cast<uintptr_t>(ln_w) | reinterpret_cast<uintptr_t>(center_w) |
               reinterpret_cast<uintptr_t>(w_gate) | reinterpret_cast<uintptr_t>(w_out)) & 15) == 0,
             "trimul_output_tc: layer-norm scales and weights must be 16-byte aligned");
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
    // P is [rows][C][pitch]: box = 64 positions x all 128 channels of one pair row (128B swizzle)
    cuuint64_t dims[3] = {(cuuint64_t)pitch, (cuuint64_t)C, (cuuint64_t)rows};
    cuuint64_t strides[2] = {(cuuint64_t)pitch * 2, (cuuint64_t)(C * pitch * 2)};
    cuuint32_t box[3] = {64, (cuuint32_t)C, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(&mp, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16*>(P), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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
  launch_pdl(k_trimul_output_tc, dim3(grid), dim3(OUT_THREADS), SMEM_OUT, stream, mz, mp, mo, w_gate, w_out, p);
  count_launch();
  return check_launch("trimul_output_tc");
}

}  // namespace sf
