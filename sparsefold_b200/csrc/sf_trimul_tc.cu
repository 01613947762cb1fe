// Triangle multiplication, bf16 track, on tcgen05 (blocks.py:484-566).
//
// k_trimul_project_tc: persistent, one CTA (4 warps) per SM.  Per 128-position
// tile: TMA brings the raw z tile into shared memory (128B swizzle, the UMMA
// K-major layout), every thread layer-norms its row in place, one thread
// issues 16 tcgen05.mma (M=128, N=2x256, K=128) against the GLU weight kept
// resident in shared memory, and the epilogue reads the 512 fp32 TMEM columns
// per row, applies sigmoid(gate) * value * mask and writes the contraction
// operands as [row][channel][pitch].  The next tile's TMA is issued before the current
// tile is processed (two A stages).
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

struct ProjParams {
  const uint8_t* mask;      // [n] token mask
  const float* ln_w;
  const float* ln_b;
  const bf16* w_glu;        // [512][128]
  bf16* a_op;
  bf16* b_op;
  int64_t rows, n, row_offset;
  int incoming;
  uint32_t* status;
};

constexpr int NOUT = 512;
constexpr int W_BYTES = NOUT * C * 2;                       // 128 KB
constexpr int CH_CHUNK = 32;                                // channels staged per epilogue step
constexpr int STAGE_OUT = CH_CHUNK * TILE * 2;              // one [32][128] bf16 staging tile (8 KB)
constexpr int SMEM_PROJ = 2 * A_BYTES + W_BYTES + 2 * STAGE_OUT + 1024 + 1024;

__global__ void __launch_bounds__(128, 1) k_trimul_project_tc(const __grid_constant__ CUtensorMap tmap,
                                                              ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* A = smem;
  uint8_t* W = smem + 2 * A_BYTES;
  bf16* stA = reinterpret_cast<bf16*>(W + W_BYTES);             // [32 channels][128 positions]
  bf16* stB = stA + CH_CHUNK * TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(W + W_BYTES + 2 * STAGE_OUT);   // [0,1] tma stages, [2] mma
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  const int tid = threadIdx.x, warp = tid >> 5;

  const int64_t span = p.incoming ? p.rows : p.n;              // positions along a tile's axis
  const int64_t nb = (span + TILE - 1) / TILE;
  const int64_t ntiles = (p.incoming ? p.n : p.rows) * nb;

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
  load_weight_sw128(W, p.w_glu, NOUT, tid, 128);
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  bool aborted = false;

  auto issue = [&](int64_t tile, int stage) {
    const int64_t major = tile / nb, minor = (tile % nb) * TILE;
    // tensor coordinates (channel, column, row)
    const int c1 = (int)(p.incoming ? major : minor);
    const int c2 = (int)(p.incoming ? minor : major);
    tc::mbar_expect_tx(&bars[stage], A_BYTES);
    tc::tma_load_3d(A + stage * A_BYTES, &tmap, &bars[stage], 0, c1, c2);
    tc::tma_load_3d(A + stage * A_BYTES + ATOM, &tmap, &bars[stage], 64, c1, c2);
  };

  constexpr uint32_t IDESC = tc::idesc_bf16(128, 256);
  const uint32_t a_base = tc::smem_u32(A), w_base = tc::smem_u32(W);
  // operands are [row][channel][pitch]: outgoing rows = pair rows r, columns s;
  // incoming (transposed) rows = pair columns s, columns = local pair rows r
  const int64_t pitch = pair_pitch(p.incoming ? p.rows : p.n);

  int64_t tile = blockIdx.x;
  if (tid == 0 && tile < ntiles) issue(tile, 0);
  for (uint32_t it = 0; tile < ntiles; tile += gridDim.x, ++it) {
    const int stage = it & 1;
    if (tid == 0 && tile + gridDim.x < ntiles) {
      tc::fence_proxy_async();
      issue(tile + gridDim.x, stage ^ 1);
    }
    tc::mbar_wait(&bars[stage], (it >> 1) & 1, p.status, aborted);
    uint8_t* At = A + stage * A_BYTES;
    ln_row_inplace(At, tid, p.ln_w, p.ln_b, 1e-5f);
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
        for (int h = 0; h < 2; ++h) {
          const uint64_t bd = tc::smem_desc(w_base + ka * (NOUT * 128) + h * (256 * 128) + kk * 32, 1024, tc::kSW128);
          tc::mma_bf16(tbase + h * 256, ad, bd, IDESC, k > 0);
        }
      }
      tc::mma_commit(&bars[2]);
    }
    tc::mbar_wait(&bars[2], it & 1, p.status, aborted);
    tc::tc_fence_after();

    // ---- epilogue: position tid of the tile; 32 channels at a time are staged as
    // [channel][position] and written as contiguous 256-byte rows of the operands ----
    const int64_t major = tile / nb, minor0 = (tile % nb) * TILE, minor = minor0 + tid;
    const bool valid = minor < span;
    const int64_t r = p.incoming ? minor : major;     // local pair row
    const int64_t s = p.incoming ? major : minor;     // pair column
    const bool keep = valid && p.mask[p.row_offset + r] && p.mask[s];
    bf16* ao = p.incoming ? p.b_op : p.a_op;          // incoming: A <- b, B <- a (transposed)
    bf16* bo = p.incoming ? p.a_op : p.b_op;
    const uint32_t lane_addr = tbase + ((uint32_t)(warp * 32) << 16);
    const int64_t row_base = major * C * pitch + minor0;   // operand row `major`, first position of the tile
#pragma unroll 1
    for (int cc = 0; cc < C / CH_CHUNK; ++cc) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int c0 = cc * CH_CHUNK + hf * 16;
        float ga[16], va[16], gb[16], vb[16];
        tc::tmem_ld16(lane_addr + c0, ga);
        tc::tmem_ld16(lane_addr + 128 + c0, va);
        tc::tmem_ld16(lane_addr + 256 + c0, gb);
        tc::tmem_ld16(lane_addr + 384 + c0, vb);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          stA[(hf * 16 + e) * TILE + tid] = __float2bfloat16_rn(keep ? fast_sigmoid(ga[e]) * va[e] : 0.f);
          stB[(hf * 16 + e) * TILE + tid] = __float2bfloat16_rn(keep ? fast_sigmoid(gb[e]) * vb[e] : 0.f);
        }
      }
      __syncthreads();
      // 32 channel rows x 16 chunks of 16 bytes per operand
#pragma unroll
      for (int i = 0; i < (CH_CHUNK * 16) / 128; ++i) {
        const int e = tid + 128 * i;
        const int c = e >> 4, part = e & 15;
        if (minor0 + part * 8 + 8 <= pitch) {
          const int64_t off = row_base + (int64_t)(cc * CH_CHUNK + c) * pitch + part * 8;
          *reinterpret_cast<uint4*>(ao + off) = *reinterpret_cast<const uint4*>(stA + c * TILE + part * 8);
          *reinterpret_cast<uint4*>(bo + off) = *reinterpret_cast<const uint4*>(stB + c * TILE + part * 8);
        }
      }
      __syncthreads();
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
  CUtensorMap map;
  SF_TRY(make_pair_tmap(&map, z, rows, n, incoming != 0));
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
  ProjParams p{mask, ln_w, ln_b, w_glu, a_op, b_op, rows, n, row_offset, incoming, status};
  const int64_t span = incoming ? rows : n;
  const int64_t ntiles = (incoming ? n : rows) * ((span + pt::TILE - 1) / pt::TILE);
  const int grid = (int)(ntiles < num_sms() ? ntiles : num_sms());
  k_trimul_project_tc<<<grid, 128, SMEM_PROJ, stream>>>(map, p);
  count_launch();
  return check_launch("trimul_project_tc");
}

}  // namespace sf
