// Triangle-multiplication contraction on tcgen05 (blocks.py:558):
//   P[i][c][j] = sum_k A[i][c][k] * B[j][c][k]   (bf16 in, fp32 accumulate, bf16 out)
// for each of the 128 channels c.  Both operands are K-major ([row][channel][k]),
// which is how the projection phase writes them for either equation; after a
// collective an operand may arrive as [rank][row][channel][k-chunk], which the
// 4-D tensor maps read in place.
//
// Persistent, warp-specialised: warp 8 streams 128x64 A and 256x64 B tiles by
// TMA through a 4-stage shared-memory ring; one thread of warp 9 issues
// tcgen05.mma (M=128, N=256, K=16) into one of two TMEM accumulators
// (2 x 256 fp32 columns); warps 0-7 drain the other accumulator (tcgen05.ld of
// 32 columns at a time, one row per thread, each warp half of the columns) and
// store bf16 rows of P while the next tile computes.
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

constexpr int BM = 128, BK = 64, STAGES = 4;
// warps 0-7 epilogue (warp w: TMEM lanes 32 (w % 4).., columns (w / 4) BN/2 ..), warp 8 TMA
// producer, warp 9 MMA issuer
constexpr int CT_EPI_WARPS = 8;
constexpr int CT_THREADS = (CT_EPI_WARPS + 2) * 32;
constexpr int SA_BYTES = BM * BK * 2;              // 16 KB
template <int BN>
struct Tile {
  static constexpr int SB_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = SA_BYTES + SB_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 1024;
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
};

struct ContractParams {
  bf16* P;
  int64_t channels, rows, cols, kdim;
  int64_t kl_a, kl_b;       // K chunk length of each operand (kdim when unchunked)
  const float* bias;        // [cols] or null
  const bf16* residual;     // laid out like P, or null
  int post_op;              // SF_POST_*
  uint32_t* status;
};

__device__ __forceinline__ float post(float v, int op) {
  if (op == SF_POST_RELU) return fmaxf(v, 0.f);
  if (op == SF_POST_SILU) return v * pt::fast_sigmoid(v);
  if (op == SF_POST_SIGMOID) return pt::fast_sigmoid(v);
  return v;
}

template <int BN>
__global__ void __launch_bounds__(CT_THREADS, 1) k_contract_tc(const __grid_constant__ CUtensorMap tmA,
                                                        const __grid_constant__ CUtensorMap tmB,
                                                        ContractParams p) {
  constexpr int STAGE_BYTES = Tile<BN>::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = pt::align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;                    // MMA issuer's drain barrier (abort path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int64_t mt = (p.rows + BM - 1) / BM, nt = (p.cols + BN - 1) / BN;
  const int64_t ntiles = p.channels * mt * nt;
  const int nk = (int)((p.kdim + BK - 1) / BK);

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, Tile<BN>::TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&accf[a], 1);
      tc::mbar_init(&acce[a], CT_EPI_WARPS * 32);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  tc::griddep_wait();     // the previous kernel's outputs are complete and visible from here on
  tc::griddep_launch();
  const uint32_t tbase = *tmem_slot;
  bool aborted = false;
  uint32_t loads = 0;   // TMA loads issued by the producer (abort-path drain)

  if (warp == CT_EPI_WARPS && lane == 0) {
    // ---- TMA producer (stops at its first failed wait) ----
    uint32_t& q = loads;
    for (int64_t t = blockIdx.x; t < ntiles && !aborted; t += gridDim.x) {
      const int64_t c = t / (mt * nt), rem = t % (mt * nt);
      const int i0 = (int)((rem / nt) * BM), j0 = (int)((rem % nt) * BN);
      for (int kb = 0; kb < nk; ++kb, ++q) {
        const int s = q % STAGES;
        if (!tc::mbar_wait(&empty[s], ((q / STAGES) & 1) ^ 1, p.status, aborted)) break;
        uint8_t* st = smem + s * STAGE_BYTES;
        tc::mbar_expect_tx(&full[s], STAGE_BYTES);
        // K index -> (chunk, offset in chunk); chunks hold whole 64-wide K blocks
        const int64_t k = (int64_t)kb * BK;
        tc::tma_load_4d(st, &tmA, &full[s], (int)(k % p.kl_a), (int)c, i0, (int)(k / p.kl_a));
        tc::tma_load_4d(st + SA_BYTES, &tmB, &full[s], (int)(k % p.kl_b), (int)c, j0, (int)(k / p.kl_b));
      }
    }
  } else if (warp == CT_EPI_WARPS + 1 && lane == 0) {
    // ---- MMA issuer (stops at its first failed wait) ----
    constexpr uint32_t IDESC = tc::idesc_bf16(BM, BN);
    const uint32_t sbase = tc::smem_u32(smem);
    uint32_t q = 0, u = 0;
    for (int64_t t = blockIdx.x; t < ntiles && !aborted; t += gridDim.x, ++u) {
      const uint32_t acc = u & 1;
      if (!tc::mbar_wait(&acce[acc], ((u >> 1) & 1) ^ 1, p.status, aborted)) break;
      tc::tc_fence_after();
      for (int kb = 0; kb < nk; ++kb, ++q) {
        const int s = q % STAGES;
        if (!tc::mbar_wait(&full[s], (q / STAGES) & 1, p.status, aborted)) break;
        tc::tc_fence_after();
        const uint32_t sa = sbase + s * STAGE_BYTES, sb = sa + SA_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = tc::smem_desc(sa + kk * 32, 1024, tc::kSW128);
          const uint64_t bd = tc::smem_desc(sb + kk * 32, 1024, tc::kSW128);
          tc::mma_bf16(tbase + acc * BN, ad, bd, IDESC, (kb | kk) != 0);
        }
        tc::mma_commit(&empty[s]);
      }
      if (aborted) break;
      tc::mma_commit(&accf[acc]);
    }
  } else if (warp < CT_EPI_WARPS) {
    // ---- epilogue: 32 columns per TMEM load, one wait each ----
    constexpr int HALF = BN / 2, CW = HALF < 32 ? HALF : 32;
    const int64_t cp = pair_pitch(p.cols);
    const int quad = warp & 3, half = warp >> 2;
    const uint32_t lane_addr = tbase + ((uint32_t)(quad * 32) << 16);
    uint32_t u = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++u) {
      const uint32_t acc = u & 1;
      const int64_t c = t / (mt * nt), rem = t % (mt * nt);
      const int64_t i = (rem / nt) * BM + quad * 32 + lane, j0 = (rem % nt) * BN + half * HALF;
      tc::mbar_wait(&accf[acc], (u >> 1) & 1, p.status, aborted);
      tc::tc_fence_after();
      bf16* prow = p.P + (i * p.channels + c) * cp;
#pragma unroll 1
      for (int ch = 0; ch < HALF / CW; ++ch) {
        float v[CW];
        if constexpr (CW == 32) tc::tmem_ld32(lane_addr + acc * BN + half * HALF + ch * CW, v);
        else tc::tmem_ld16(lane_addr + acc * BN + half * HALF + ch * CW, v);
        if (i < p.rows) {
#pragma unroll
          for (int g = 0; g < CW / 8; ++g) {
            const int64_t j = j0 + ch * CW + g * 8;
            if (j + 8 <= cp) {
              if (p.bias || p.residual || p.post_op) {
                float bv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (p.bias) {
                  if (j + 8 <= p.cols) {   // bias is [cols] fp32, 16-byte aligned (checked on the host)
                    const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.bias + j));
                    const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.bias + j + 4));
                    bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
                    bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
                  } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) bv[e] = j + e < p.cols ? __ldg(p.bias + j + e) : 0.f;
                  }
                }
                uint32_t ru[4] = {0u, 0u, 0u, 0u};
                if (p.residual) {
                  const uint4 rr = *reinterpret_cast<const uint4*>(p.residual + (i * p.channels + c) * cp + j);
                  ru[0] = rr.x; ru[1] = rr.y; ru[2] = rr.z; ru[3] = rr.w;
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float r = (e & 1) ? pt::bf_hi(ru[e >> 1]) : pt::bf_lo(ru[e >> 1]);
                  v[g * 8 + e] = post(v[g * 8 + e] + bv[e] + r, p.post_op);
                }
              }
              uint4 o;
              o.x = pt::pack_bf2(v[g * 8 + 0], v[g * 8 + 1]);
              o.y = pt::pack_bf2(v[g * 8 + 2], v[g * 8 + 3]);
              o.z = pt::pack_bf2(v[g * 8 + 4], v[g * 8 + 5]);
              o.w = pt::pack_bf2(v[g * 8 + 6], v[g * 8 + 7]);
              *reinterpret_cast<uint4*>(prow + j) = o;
            }
          }
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&acce[acc]);
    }
  }
  tc::tc_fence_before();
  if (__syncthreads_or(aborted)) {   // abort path: drain the producer's loads and the issuer's MMAs
    if (warp == CT_EPI_WARPS && lane == 0) tc::drain_ring(full, STAGES, loads, p.status);
    if (warp == CT_EPI_WARPS + 1 && lane == 0) tc::drain_mma(drain, p.status);
    __syncthreads();
  }
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, Tile<BN>::TMEM_COLS);
  }
}

// Tensor map over an operand [chunks][rows][channels][pitch(kl)] bf16 (K split into
// `chunks` pieces of kl, one per source rank after a collective), box 64 (k) x box_rows.
int make_operand_tmap(CUtensorMap* map, const void* base, int64_t chunks, int64_t rows, int64_t channels,
                      int64_t kl, uint32_t box_rows) {
  auto encode = tensor_map_encoder();
  if (!encode) return SF_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) {
    set_error("contraction operand %p is not 16-byte aligned", base);
    return SF_ERR_ARG;
  }
  const int64_t kp = pair_pitch(kl);
  cuuint64_t dims[4] = {(cuuint64_t)kp, (cuuint64_t)channels, (cuuint64_t)rows, (cuuint64_t)chunks};
  cuuint64_t strides[3] = {(cuuint64_t)kp * 2, (cuuint64_t)(channels * kp * 2), (cuuint64_t)(rows * channels * kp * 2)};
  cuuint32_t box[4] = {(cuuint32_t)BK, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for operand [%lld][%lld][%lld][%lld]", (int)r, (long long)chunks,
              (long long)rows, (long long)channels, (long long)kp);
    return SF_ERR_CUDA;
  }
  return SF_OK;
}

}  // namespace

static int gemm_tc_impl(const bf16* a_op, const bf16* b_op, bf16* P, int64_t channels, int64_t rows, int64_t cols,
                        int64_t chunks_a, int64_t kl_a, int64_t chunks_b, int64_t kl_b, const float* bias,
                        const bf16* residual, int post_op, cudaStream_t stream);

int contract_tc(const bf16* a_op, const bf16* b_op, bf16* P, int64_t channels, int64_t rows, int64_t cols,
                int64_t kdim, cudaStream_t stream) {
  return gemm_tc_impl(a_op, b_op, P, channels, rows, cols, 1, kdim, 1, kdim, nullptr, nullptr, SF_POST_NONE, stream);
}

int contract_chunked_tc(const bf16* a_op, int64_t chunks_a, const bf16* b_op, int64_t chunks_b, bf16* P,
                        int64_t channels, int64_t rows, int64_t cols, int64_t kdim, cudaStream_t stream) {
  SF_REQUIRE(chunks_a > 0 && chunks_b > 0 && kdim % chunks_a == 0 && kdim % chunks_b == 0,
             "contract: K=%lld does not split into %lld / %lld chunks", (long long)kdim, (long long)chunks_a,
             (long long)chunks_b);
  const int64_t kl_a = kdim / chunks_a, kl_b = kdim / chunks_b;
  SF_REQUIRE((chunks_a == 1 || kl_a % BK == 0) && (chunks_b == 1 || kl_b % BK == 0),
             "contract: chunked K needs chunk lengths that are multiples of %d (got %lld / %lld)", BK,
             (long long)kl_a, (long long)kl_b);
  return gemm_tc_impl(a_op, b_op, P, channels, rows, cols, chunks_a, kl_a, chunks_b, kl_b, nullptr, nullptr,
                      SF_POST_NONE, stream);
}

// y[M][N] = post(x[M][K] . wt[N][K]^T + bias + residual); K and N multiples of 8.
int linear_tc(const bf16* x, const bf16* wt, const float* bias, const bf16* residual, bf16* y, int64_t M, int64_t K,
              int64_t N, int post_op, cudaStream_t stream) {
  return gemm_tc_impl(x, wt, y, 1, M, N, 1, K, 1, K, bias, residual, post_op, stream);
}

template <int BN>
static int launch_gemm_tc(const CUtensorMap& ma, const bf16* b_op, int64_t chunks_b, int64_t kl_b, int64_t channels,
                          int64_t cols, const ContractParams& p, int64_t ntiles, cudaStream_t stream) {
  CUtensorMap mb;
  SF_TRY(make_operand_tmap(&mb, b_op, chunks_b, cols, channels, kl_b, BN));
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(k_contract_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Tile<BN>::SMEM);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(contract): %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    attr_set[dev & 63] = true;
  }
  const int grid = (int)(ntiles < num_sms() ? ntiles : num_sms());
  launch_pdl(k_contract_tc<BN>, dim3(grid), dim3(CT_THREADS), Tile<BN>::SMEM, stream, ma, mb, p);
  count_launch();
  return check_launch("contract_tc");
}

static int gemm_tc_impl(const bf16* a_op, const bf16* b_op, bf16* P, int64_t channels, int64_t rows, int64_t cols,
                        int64_t chunks_a, int64_t kl_a, int64_t chunks_b, int64_t kl_b, const float* bias,
                        const bf16* residual, int post_op, cudaStream_t stream) {
  const int64_t kdim = chunks_a * kl_a;
  if (channels == 0 || rows == 0 || cols == 0) return SF_OK;
  SF_REQUIRE(rows < (1 << 30) && cols < (1 << 30) && kdim < (1 << 30) && channels < (1 << 30),
             "contract_tc: size too large");
  SF_REQUIRE((reinterpret_cast<uintptr_t>(bias) & 15) == 0 && (reinterpret_cast<uintptr_t>(residual) & 15) == 0,
             "contract_tc: bias and residual must be 16-byte aligned");
  CUtensorMap ma;
  SF_TRY(make_operand_tmap(&ma, a_op, chunks_a, rows, channels, kl_a, BM));
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  ContractParams p{P, channels, rows, cols, kdim, kl_a, kl_b, bias, residual, post_op, status};
  const int64_t mt = (rows + BM - 1) / BM;
  auto tiles = [&](int64_t bn) { return channels * mt * ((cols + bn - 1) / bn); };
  // the widest N tile that still gives every SM a tile (or that covers N exactly)
  if (cols > 128 && tiles(256) >= num_sms()) return launch_gemm_tc<256>(ma, b_op, chunks_b, kl_b, channels, cols, p, tiles(256), stream);
  if (cols > 64 && tiles(128) >= num_sms() / 2) return launch_gemm_tc<128>(ma, b_op, chunks_b, kl_b, channels, cols, p, tiles(128), stream);
  return launch_gemm_tc<64>(ma, b_op, chunks_b, kl_b, channels, cols, p, tiles(64), stream);
}

}  // namespace sf
