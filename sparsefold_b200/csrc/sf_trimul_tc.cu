// Triangle multiplication, bf16 track, on tcgen05 (blocks.py:484-566).
//
// k_trimul_project_tc: persistent, one warp-specialised CTA per SM.  Per
// 128-position tile: TMA brings the raw z tile into shared memory (128B
// swizzle, the UMMA K-major layout, two stages), eight warps layer-norm its
// rows in place (two threads per row), one thread issues the GLU GEMMs transposed,
// D[out channel][position] = W . LN(z)^T (M=128, N=128, K=128, four weight
// matrices kept resident), into two TMEM halves so the epilogue of one operand
// overlaps the GEMM of the other, and sixteen epilogue warps apply
// sigmoid(gate) * value * mask and TMA-store the contraction operands as
// [row][channel][pitch] (each TMEM lane is one channel row of the output).  The
// next tile's GEMM of a half waits for every epilogue warp to have read it, so the
// epilogue is split thin (a clock64 trace with eight warps: a tile every ~7.1k
// cycles against ~5.2k of LayerNorm, each half's hand-off waiting 1-3k cycles on
// the slowest epilogue warp).
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

struct ProjParams {
  const uint8_t* mask;      // [n] token mask
  const float* ln_w;
  const float* ln_b;
  int64_t rows, n, row_offset, pitch;
  int incoming;
  uint32_t* status;
};

// Warp roles (832 threads):
//   warps 0-15  epilogue: warp w reads TMEM lanes 32(w%4).. (output channels) and
//               positions 32(w/4)..+31 of the tile; stages sigmoid(gate) * value *
//               mask as [32 channels][32 positions] (64B swizzle) and TMA-stores it
//   warps 16-23 layer norm of the tile rows in place (two threads per position)
//   warp 24     TMA producer of z tiles (two stages)
//   warp 25     MMA issuer: D[out channel][position] = W_x . LN(z)^T for the four
//               GLU matrices, two at a time (TMEM halves a = cols 0-255, b = 256-511)
constexpr int NOUT = 512;
constexpr int W_BYTES = NOUT * C * 2;                       // 128 KB, rows = gate_a, val_a, gate_b, val_b
constexpr int EPI_WARPS = 16;
constexpr int LN_WARPS = 8;
constexpr int PROJ_THREADS = (EPI_WARPS + LN_WARPS + 2) * 32;
constexpr int ST_BYTES = 32 * 64;                           // one epilogue warp's staging: 32 channels x 32 positions
constexpr int OFF_PW = 0;
constexpr int OFF_PZ = W_BYTES;                             // two z stages
constexpr int OFF_PST = OFF_PZ + 2 * A_BYTES;               // EPI_WARPS staging tiles
constexpr int OFF_PLN = OFF_PST + EPI_WARPS * ST_BYTES;    // LayerNorm scale and shift, 2 x 128 fp32
constexpr int OFF_PBAR = OFF_PLN + 2 * C * 4;
constexpr int SMEM_PROJ = OFF_PBAR + 256 + 1024;
static_assert(SMEM_PROJ <= 232448, "trimul projection shared memory");

__global__ void __launch_bounds__(PROJ_THREADS, 1) k_trimul_project_tc(const __grid_constant__ CUtensorMap tmZ,
                                                                       const __grid_constant__ CUtensorMap tmA,
                                                                       const __grid_constant__ CUtensorMap tmB,
                                                                       const bf16* __restrict__ w_glu, ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_PBAR);   // [2] z tile landed
  uint64_t* normed = full + 2;                                      // [2] z tile normalised (128 arrivals)
  uint64_t* zfree = normed + 2;                                     // [2] MMAs of the stage done
  uint64_t* tfull = zfree + 2;                                      // [2] TMEM half written
  uint64_t* tfree = tfull + 2;                                      // [2] TMEM half read (16 warps)
  uint64_t* drain = tfree + 2;                                      // MMA drain barrier (abort path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int64_t span = p.incoming ? p.rows : p.n;              // positions along a tile's axis
  const int64_t nb = (span + TILE - 1) / TILE;
  const int64_t ntiles = (p.incoming ? p.n : p.rows) * nb;

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&normed[s], LN_WARPS * 32);
      tc::mbar_init(&zfree[s], 1);
      tc::mbar_init(&tfull[s], 1);
      tc::mbar_init(&tfree[s], EPI_WARPS);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmZ);
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  load_weight_sw128(smem + OFF_PW, w_glu, NOUT, tid, PROJ_THREADS);
  float* lnp = reinterpret_cast<float*>(smem + OFF_PLN);
  if (tid < 2 * C) lnp[tid] = tid < C ? p.ln_w[tid] : (p.ln_b ? p.ln_b[tid - C] : 0.f);
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  tc::griddep_wait();     // the previous kernel's outputs are complete and visible from here on
  tc::griddep_launch();
  const uint32_t tbase = *tmem_slot;
  const uint32_t sb = tc::smem_u32(smem);
  bool aborted = false;
  uint32_t loads = 0;   // z tiles requested by the producer (abort-path drain)

  if (warp == EPI_WARPS + LN_WARPS) {
    // ---- TMA producer (stops at its first failed wait) ----
    if (lane == 0) {
      uint32_t& it = loads;
      for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const int st = it & 1;
        if (it >= 2 && !tc::mbar_wait(&zfree[st], ((it >> 1) + 1) & 1, p.status, aborted)) break;
        const int64_t major = tile / nb, minor = (tile % nb) * TILE;
        const int c1 = (int)(p.incoming ? major : minor);    // tensor coordinates (channel, column, row)
        const int c2 = (int)(p.incoming ? minor : major);
        uint8_t* dst = smem + OFF_PZ + st * A_BYTES;
        tc::mbar_expect_tx(&full[st], A_BYTES);
        tc::tma_load_3d(dst, &tmZ, &full[st], 0, c1, c2);
        tc::tma_load_3d(dst + ATOM, &tmZ, &full[st], 64, c1, c2);
      }
    }
  } else if (warp == EPI_WARPS + LN_WARPS + 1) {
    // ---- MMA issuer (stops at its first failed wait) ----
    if (lane == 0) {
      constexpr uint32_t IDESC = tc::idesc_bf16(128, 128);
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles && !aborted; tile += gridDim.x, ++it) {
        const int st = it & 1;
        if (!tc::mbar_wait(&normed[st], (it >> 1) & 1, p.status, aborted)) break;
        tc::tc_fence_after();
        const uint32_t zb = sb + OFF_PZ + st * A_BYTES;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (it >= 1 && !tc::mbar_wait(&tfree[hh], (it - 1) & 1, p.status, aborted)) break;
          tc::tc_fence_after();
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {          // gate, value of operand hh
            const int mtx = 2 * hh + mt;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int ka = k >> 2, kk = k & 3;
              tc::mma_bf16(tbase + hh * 256 + mt * 128,
                           tc::smem_desc(sb + OFF_PW + ka * (NOUT * 128) + mtx * (128 * 128) + kk * 32, 1024, tc::kSW128),
                           tc::smem_desc(zb + ka * ATOM + kk * 32, 1024, tc::kSW128), IDESC, k > 0);
            }
          }
          tc::mma_commit(&tfull[hh]);
        }
        if (aborted) break;
        tc::mma_commit(&zfree[st]);
      }
    }
  } else if (warp >= EPI_WARPS) {
    // ---- layer norm (two threads per tile row) ----
    const int u = tid - EPI_WARPS * 32, r = u >> 1, half = u & 1;
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int st = it & 1;
      tc::mbar_wait(&full[st], (it >> 1) & 1, p.status, aborted);
      ln_half_row_shifted(smem + OFF_PZ + st * A_BYTES, r, half, lnp, lnp + C, 1e-5f);
      tc::fence_proxy_async();
      tc::mbar_arrive(&normed[st]);
    }
  } else {
    // ---- epilogue ----
    const int quad = warp & 3, pg = warp >> 2;   // channels 32 quad .., positions 32 pg ..
    const uint32_t lane_addr = tbase + ((uint32_t)(32 * quad) << 16);
    uint8_t* stg = smem + OFF_PST + warp * ST_BYTES;
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int64_t major = tile / nb, minor0 = (tile % nb) * TILE + 32 * pg;
      // keep[pos] = valid && mask[row] && mask[col] for the warp's 32 positions
      uint32_t keep;
      {
        const int64_t minor = minor0 + lane;
        bool k = minor < span;
        if (k) {
          const int64_t rr = p.incoming ? minor : major, ss = p.incoming ? major : minor;
          k = p.mask[p.row_offset + rr] != 0 && p.mask[ss] != 0;
        }
        keep = __ballot_sync(0xffffffffu, k);
      }
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        tc::mbar_wait(&tfull[hh], it & 1, p.status, aborted);
        tc::tc_fence_after();
        if (lane == 0) tc::bulk_wait_read0();   // previous store from this staging tile has read it
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          float gt[16], vl[16];
          tc::tmem_ld16(lane_addr + hh * 256 + 32 * pg + 16 * k, gt);
          tc::tmem_ld16(lane_addr + hh * 256 + 128 + 32 * pg + 16 * k, vl);
          uint32_t pk[8];
          // a column is one position, the same for every lane: the mask test is warp-uniform
          const uint32_t kw = (keep >> (16 * k)) & 0xFFFFu;
          if (kw == 0xFFFFu) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              pk[e] = pack_bf2(sigmoid_tanh(gt[2 * e]) * vl[2 * e], sigmoid_tanh(gt[2 * e + 1]) * vl[2 * e + 1]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float o0 = ((kw >> (2 * e)) & 1) ? sigmoid_tanh(gt[2 * e]) * vl[2 * e] : 0.f;
              const float o1 = ((kw >> (2 * e + 1)) & 1) ? sigmoid_tanh(gt[2 * e + 1]) * vl[2 * e + 1] : 0.f;
              pk[e] = pack_bf2(o0, o1);
            }
          }
          *reinterpret_cast<uint4*>(stg + tc::sw64_off(lane, 2 * k)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(stg + tc::sw64_off(lane, 2 * k + 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
        tc::tc_fence_before();
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(&tfree[hh]);
          // tmA receives the gate_a/val_a product, tmB the gate_b/val_b one (the host swaps
          // the operands for the incoming direction)
          if (minor0 < p.pitch) {
            tc::tma_store_3d(hh == 0 ? &tmA : &tmB, stg, (int)minor0, 32 * quad, (int)major);
            tc::bulk_commit();
          }
        }
      }
    }
    if (lane == 0) tc::bulk_wait0();
  }
  tc::tc_fence_before();
  if (__syncthreads_or(aborted)) {   // abort path: drain the producer's loads and the issuer's MMAs
    if (warp == EPI_WARPS + LN_WARPS && lane == 0) tc::drain_ring(full, 2, loads, p.status);
    if (warp == EPI_WARPS + LN_WARPS + 1 && lane == 0) tc::drain_mma(drain, p.status);
    __syncthreads();
  }
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

// cuTensorMapEncodeTiled resolved through the runtime, so the library does not
// link libcuda directly (it loads on machines without a driver).
EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) {
      set_error("cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(e));
      return nullptr;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Tensor map over a bf16 pair tensor [rows][n][128]; box = 64 channels x
// (128 columns x 1 row) for row tiles or (1 column x 128 rows) for column tiles.
int make_pair_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t n, bool column_tile) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) {
    set_error("pair tensor base %p is not 16-byte aligned", base);
    return SF_ERR_ARG;
  }
  cuuint64_t dims[3] = {(cuuint64_t)pt::C, (cuuint64_t)n, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)pt::C * 2, (cuuint64_t)(n * pt::C * 2)};
  cuuint32_t box[3] = {64, column_tile ? 1u : 128u, column_tile ? 128u : 1u};
  cuuint32_t estr[3] = {1, 1, 1};
  auto encode = tensor_map_encoder();
  if (!encode) return SF_ERR_CUDA;
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for pair [%lld][%lld][128]", (int)r, (long long)rows, (long long)n);
    return SF_ERR_CUDA;
  }
  return SF_OK;
}

// Projection phase of triangle multiplication on tcgen05 (bf16 only).
int trimul_project_tc(const bf16* z, const uint8_t* mask, int64_t rows, int64_t n, int64_t row_offset, int incoming,
                      const float* ln_w, const float* ln_b, const bf16* w_glu, bf16* a_op, bf16* b_op,
                      cudaStream_t stream) {
  if (rows == 0 || n == 0) return SF_OK;
  SF_REQUIRE(n <= (1 << 24) && rows <= (1 << 24), "trimul_project_tc: size too large");
  SF_REQUIRE((reinterpret_cast<uintptr_t>(ln_w) & 15) == 0 && (reinterpret_cast<uintptr_t>(ln_b) & 15) == 0,
             "trimul_project_tc: layer-norm parameters must be 16-byte aligned");
  CUtensorMap mz, ma, mb;
  SF_TRY(make_pair_tmap(&mz, z, rows, n, incoming != 0));
  // operands [majors][C][pitch]: outgoing majors = local rows (positions = columns),
  // incoming majors = columns (positions = local rows) with A <- b and B <- a
  const int64_t majors = incoming ? n : rows;
  const int64_t pitch = pair_pitch(incoming ? rows : n);
  {
    auto encode = tensor_map_encoder();
    if (!encode) return SF_ERR_CUDA;
    bf16* dst[2] = {incoming ? b_op : a_op, incoming ? a_op : b_op};
    CUtensorMap* maps[2] = {&ma, &mb};
    for (int i = 0; i < 2; ++i) {
      if ((reinterpret_cast<uintptr_t>(dst[i]) & 15) != 0) {
        set_error("trimul_project_tc: operand %p is not 16-byte aligned", (void*)dst[i]);
        return SF_ERR_ARG;
      }
      cuuint64_t dims[3] = {(cuuint64_t)pitch, (cuuint64_t)pt::C, (cuuint64_t)majors};
      cuuint64_t strides[2] = {(cuuint64_t)pitch * 2, (cuuint64_t)(pt::C * pitch * 2)};
      cuuint32_t box[3] = {32, 32, 1};   // one epilogue warp's [32 channels][32 positions]
      cuuint32_t estr[3] = {1, 1, 1};
      CUresult r = encode(maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dst[i], dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) for operand [%lld][128][%lld]", (int)r, (long long)majors,
                  (long long)pitch);
        return SF_ERR_CUDA;
      }
    }
  }
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(k_trimul_project_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_PROJ);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(trimul_project): %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    attr_set[dev & 63] = true;
  }
  ProjParams p{mask, ln_w, ln_b, rows, n, row_offset, pitch, incoming, status};
  const int64_t span = incoming ? rows : n;
  const int64_t ntiles = majors * ((span + pt::TILE - 1) / pt::TILE);
  const int grid = (int)(ntiles < num_sms() ? ntiles : num_sms());
  launch_pdl(k_trimul_project_tc, dim3(grid), dim3(PROJ_THREADS), SMEM_PROJ, stream, mz, ma, mb, w_glu, p);
  count_launch();
  return check_launch("trimul_project_tc");
}

}  // namespace sf
