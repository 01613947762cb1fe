// Pair-logit projection of SingleActUpdate (blocks.py:745-749), bf16 track, on tcgen05:
//   logits[h][m] = LN(z[m]) . W[h],   z [M][128], W [heads <= 16][128], logits [heads][M].
//
// One CTA (4 warps) per 128-position tile, several CTAs per SM: TMA brings the z
// tile (128B swizzle), each thread layer-norms its row in place (rounded to
// bf16 as the reference does before the projection), one thread issues 8
// tcgen05.mma (M128 N16 K16) against the 16-row weight tile, and each thread
// reads its 16 logits from TMEM and writes them head-major (coalesced per head).
#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int PL_HEADS = 16;                       // N of the MMA; weight rows beyond `heads` are zero
constexpr int PL_W_BYTES = PL_HEADS * C * 2;       // two 64-channel atoms of 16 x 128 B
constexpr int OFF_PLZ = 0, OFF_PLW = A_BYTES, OFF_PLLN = OFF_PLW + PL_W_BYTES, OFF_PLBAR = OFF_PLLN + 2 * C * 4;
constexpr int SMEM_PL = OFF_PLBAR + 64 + 1024;

struct PlParams {
  const float *ln_w, *ln_b;
  const bf16* w;
  bf16* logits;
  int64_t M;
  int heads;
  uint32_t* status;
  int64_t ncols, ldb;   // ldb > 0: position m = r * ncols + s goes to logits[(r * heads + h) * ldb + s]
  float scale;          // ... times scale
};

__global__ void __launch_bounds__(128) k_pair_logits_tc(const __grid_constant__ CUtensorMap tmZ, PlParams p) {
  extern __shared__ uint8_t smem_raw[];
  tc::griddep_wait();     // the previous kernel's outputs are complete and visible from here on
  tc::griddep_launch();
  uint8_t* smem = align1024(smem_raw);
  uint64_t* ldbar = reinterpret_cast<uint64_t*>(smem + OFF_PLBAR);
  uint64_t* mmabar = ldbar + 1;
  uint64_t* drain = ldbar + 2;                   // MMA drain barrier (abort path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ldbar + 3);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t m0 = (int64_t)blockIdx.x * TILE;

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 32);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(ldbar, 1);
    tc::mbar_init(mmabar, 1);
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
    tc::mbar_expect_tx(ldbar, A_BYTES);
    tc::tma_load_2d(smem + OFF_PLZ, &tmZ, ldbar, 0, (int)m0);
    tc::tma_load_2d(smem + OFF_PLZ + ATOM, &tmZ, ldbar, 64, (int)m0);
  }
  // weight rows h < heads, zero rows after: K-major, 128B swizzle, atom ka at ka * 16 rows * 128 B
  for (int e = tid; e < PL_HEADS * 16; e += 128) {
    const int r = e >> 4, kc = e & 15;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < p.heads) v = __ldg(reinterpret_cast<const uint4*>(p.w + (size_t)r * C + kc * 8));
    *reinterpret_cast<uint4*>(smem + OFF_PLW + (kc >> 3) * (PL_HEADS * 128) + tc::sw128_off(r, kc & 7)) = v;
  }
  float* lnp = reinterpret_cast<float*>(smem + OFF_PLLN);   // LayerNorm scale and shift
  lnp[tid] = p.ln_w[tid];
  lnp[C + tid] = p.ln_b ? p.ln_b[tid] : 0.f;
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  bool aborted = false;
  tc::mbar_wait(ldbar, 0, p.status, aborted);
  ln_row_shifted(smem + OFF_PLZ, tid, lnp, lnp + C, 1e-5f);
  tc::fence_proxy_async();
  tc::tc_fence_before();
  // the tile is only used by the tensor core if every thread saw it land (abort path)
  const bool loaded = !__syncthreads_or(aborted);
  if (tid == 0 && loaded) {
    tc::tc_fence_after();
    const uint32_t sb = tc::smem_u32(smem);
    constexpr uint32_t IDESC = tc::idesc_bf16(128, PL_HEADS);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int ka = k >> 2, kk = k & 3;
      tc::mma_bf16(tbase, tc::smem_desc(sb + OFF_PLZ + ka * ATOM + kk * 32, 1024, tc::kSW128),
                   tc::smem_desc(sb + OFF_PLW + ka * (PL_HEADS * 128) + kk * 32, 1024, tc::kSW128), IDESC, k > 0);
    }
    tc::mma_commit(mmabar);
  }
  if (loaded) tc::mbar_wait(mmabar, 0, p.status, aborted);
  tc::tc_fence_after();
  float v[16];
  tc::tmem_ld16(tbase + ((uint32_t)(32 * warp) << 16), v);
  const int64_t m = m0 + tid;
  if (m < p.M) {
    if (p.ldb > 0) {
      const int64_t r = m / p.ncols, sc = m - r * p.ncols;
#pragma unroll
      for (int h = 0; h < PL_HEADS; ++h)
        if (h < p.heads) p.logits[(r * p.heads + h) * p.ldb + sc] = __float2bfloat16_rn(v[h] * p.scale);
    } else {
#pragma unroll
      for (int h = 0; h < PL_HEADS; ++h)
        if (h < p.heads) p.logits[(int64_t)h * p.M + m] = __float2bfloat16_rn(v[h]);
    }
  }
  tc::tc_fence_before();
  if (__syncthreads_or(aborted)) {   // abort path: the tile load and the MMAs must be done before exit
    if (tid == 0) {
      tc::mbar_wait_drain(ldbar, 0, p.status);
      if (loaded) tc::drain_mma(drain, p.status);
    }
    __syncthreads();
  }
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 32);
  }
}

}  // namespace

// LN(z) W^T for z [M][128] bf16 and heads <= 16: logits [heads][M] (ldb = 0), or, with the
// positions as rows of ncols, rows [M / ncols][heads][ldb] times scale.
static int pair_logits_launch(const bf16* z, const float* ln_w, const float* ln_b, const bf16* w, bf16* logits,
                              int64_t M, int heads, int64_t ncols, int64_t ldb, float scale, cudaStream_t stream) {
  if (M == 0) return SF_OK;
  SF_REQUIRE(heads >= 1 && heads <= PL_HEADS, "pair_logits_tc: %d heads (1..16)", heads);
  SF_REQUIRE(M < (int64_t(1) << 31), "pair_logits_tc: too many positions");
  SF_REQUIRE((reinterpret_cast<uintptr_t>(ln_w) & 15) == 0 && (reinterpret_cast<uintptr_t>(ln_b) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(w) & 15) == 0,
             "pair_logits_tc: weights must be 16-byte aligned");
  CUtensorMap mz;
  SF_TRY(make_2d_tmap(&mz, z, C, M, 64, TILE));
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(k_pair_logits_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_PL);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(pair_logits): %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    attr[dev & 63] = true;
  }
  PlParams pp{ln_w, ln_b, w, logits, M, heads, status, ncols, ldb, scale};
  launch_pdl(k_pair_logits_tc, dim3((unsigned)((M + TILE - 1) / TILE)), dim3(128), SMEM_PL, stream, mz, pp);
  count_launch();
  return check_launch("pair_logits_tc");
}

// logits [heads][M] = LN(z) W^T for z [M][128] bf16, heads <= 16.
int pair_logits_tc(const bf16* z, const float* ln_w, const float* ln_b, const bf16* w, bf16* logits, int64_t M,
                   int heads, cudaStream_t stream) {
  return pair_logits_launch(z, ln_w, ln_b, w, logits, M, heads, 1, 0, 1.0f, stream);
}

// bias [rows][heads][ldb] = scale * LN(z[r][s]) . W[h] for the pair rows z [rows][n][128]: the same
// kernel with row-major output (the pair bias of a row block for triangle attention).
int pair_rows_bias_tc(const bf16* z, int64_t rows, int64_t n, const float* ln_w, const bf16* w, int heads, float scale,
                      bf16* bias, int64_t ldb, cudaStream_t stream) {
  if (rows == 0 || n == 0) return SF_OK;
  SF_REQUIRE(ldb >= n, "pair_rows_bias_tc: ldb %lld < n %lld", (long long)ldb, (long long)n);
  return pair_logits_launch(z, ln_w, nullptr, w, bias, rows * n, heads, n, ldb, scale, stream);
}

}  // namespace sf
