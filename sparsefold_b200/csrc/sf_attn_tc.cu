// Pair-biased gated attention on tcgen05 (bf16, fp32 accumulation): the
// dot_product_attention of the single, token and atom attentions
// (backends/torch/attention/sdpa.py:22-121 with the gate of
// diffusion/transformer.py:306-345 and :549-585):
//   out[b,q,h,:] = sigmoid(gate[b,q,h,:]) * softmax_k(scale q.k + bias[b,h,q,k] + maskbias) v
// with maskbias = -FLT_MAX for a masked query row or key (the reference's
// -finfo.max bias: a fully masked row averages v uniformly over every key).
//
// One CTA per (128 queries, head h, batch b); head dims D <= 64 (a multiple of 8).
//   one thread  TMA producer: per 64-key block the K tile [64 keys][32 or 64 dims]
//               (64B or 128B swizzle), the V tile [64 keys][64 dims] (128B swizzle)
//               and the bf16 bias tile [128 queries][64 keys] (128B swizzle) into a
//               3-slot ring; dims beyond D and keys beyond k_len arrive as zeros
//               (the tensor maps' bounds), so nothing is staged by hand.
//   warps 0-3   softmax / epilogue, thread = query row: Q (pre-scaled by
//               scale * log2 e) into TMEM, then per block the S row from TMEM plus
//               the bias row from shared memory times log2 e, exp2 against a running
//               max that moves only when a block exceeds it by 2^8 (then O is
//               rescaled in TMEM), P as bf16 written over S; finally O / l, times
//               the gate, stored with 16-byte stores.
//   warp 5      one thread issues S_j = Q K_j^T (A from TMEM) and O += P_j V_j (A =
//               P_j from TMEM, V as an MN-major B operand, so V needs no transpose),
//               S_{j+2} right after P_j V_j into the same TMEM buffer (MMAs of one
//               thread complete in issue order).
// TMEM: S/P double buffer [0,128), O [128,192), Q [192,224) of 256 columns.
#include <cfloat>

#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int MH_KB = 64;                          // keys per block
constexpr int MH_DP = 64;                          // padded head dim of V, O (and of K when D > 32)
constexpr int MH_RING = 3;                         // key blocks staged ahead
constexpr int MH_K_BYTES = MH_KB * 128;            // K tile (64 rows of up to 128 B)
constexpr int MH_V_BYTES = MH_KB * 128;            // V tile [64 keys][64 dims]
constexpr int MH_B_BYTES = TILE * MH_KB * 2;       // bias tile [128 queries][64 keys]
constexpr int MH_SLOT_BYTES = MH_K_BYTES + MH_V_BYTES + MH_B_BYTES;   // 32 KB
constexpr int MH_MAX_KEYS = 65536;                 // key-valid bits kept in shared memory
constexpr int MH_OFF_RING = 0;
constexpr int MH_OFF_KBITS = MH_OFF_RING + MH_RING * MH_SLOT_BYTES;
constexpr int MH_OFF_BAR = MH_OFF_KBITS + MH_MAX_KEYS / 8;
constexpr int MH_SMEM = MH_OFF_BAR + 256 + 1024;
static_assert(MH_SMEM <= 232448 / 2, "two attention CTAs per SM");
constexpr int MH_THREADS = 6 * 32;
constexpr float MH_RESCALE = 8.0f;

struct MhaParams {
  sf_attention_args a;
  int bias_batched;   // the bias map has a batch dimension (else one bias for every batch entry)
  uint32_t* status;
};

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// KSW: swizzle of the K tile, 64 (rows of 32 dims, D <= 32) or 128 (rows of 64 dims).
// G: batch entries per CTA.  G = 1: 128 query rows of one entry, 64-key blocks.  G = 4
// (entries of at most 32 queries, the atom windows): warp w holds the 32 query rows of
// entry 4 * blockIdx.z + w, and each 64-key block is 16 keys of each of the four entries
// (their own key windows); a warp reads only its entry's 16 columns of S and writes zeros
// over the other entries' columns of P, so one M128 N64 MMA for S and one K=64 P V serve
// all four entries.
template <int KSW, int G>
__global__ void __launch_bounds__(MH_THREADS, 1) k_mha_tc(const __grid_constant__ CUtensorMap tmK,
                                                          const __grid_constant__ CUtensorMap tmV,
                                                          const __grid_constant__ CUtensorMap tmB, MhaParams P) {
  tc::griddep_wait();     // the previous kernel's outputs are complete and visible from here on
  tc::griddep_launch();
  constexpr int DK = KSW / 2;                     // padded head dim of K (32 or 64)
  constexpr int KBG = MH_KB / G;                  // keys of one entry in a 64-key block
  constexpr int QG = TILE / G;                    // query rows of one entry
  constexpr int BIAS_BOX = KBG * QG * 2;          // bytes of one entry's bias box
  const sf_attention_args& a = P.a;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* kvfull = reinterpret_cast<uint64_t*>(smem + MH_OFF_BAR);   // [RING] K, V and bias of a block landed
  uint64_t* kvfree = kvfull + MH_RING;                                  // [RING] P V of the slot's block done
  uint64_t* sbar = kvfree + MH_RING;                                    // [2] S_j written and block j landed (2)
  uint64_t* pready = sbar + 2;                                          // [2] P_j written (4 warps)
  uint64_t* pvbar = pready + 2;                                         // [2] P_j V_j done
  uint64_t* drain = pvbar + 2;                                          // issuer's drain barrier (abort path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint32_t* kbits = reinterpret_cast<uint32_t*>(smem + MH_OFF_KBITS);   // [G][nkw]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t h = blockIdx.y;
  const int64_t bz = (int64_t)blockIdx.z * G;                           // first batch entry of the CTA
  const int64_t q0 = G == 1 ? (int64_t)blockIdx.x * TILE : 0;
  const int D = (int)a.head_dim;
  const int nkb = (int)((a.k_len + KBG - 1) / KBG);
  const int nkw = (int)((a.k_len + 31) / 32);
  const bool has_bias = a.bias != nullptr;
  bool aborted = false;
  uint32_t loads = 0;   // key blocks requested by the producer (abort-path drain)
  auto slot_of = [&](int jj) { return smem + MH_OFF_RING + (jj % MH_RING) * MH_SLOT_BYTES; };
  auto issue_load = [&](int jj) {   // block jj into slot jj % RING (jj == loads)
    ++loads;
    uint8_t* sl = slot_of(jj);
    uint64_t* bar = &kvfull[jj % MH_RING];
    tc::mbar_expect_tx(bar, MH_KB * KSW + MH_V_BYTES + (has_bias ? G * BIAS_BOX : 0));
#pragma unroll
    for (int g = 0; g < G; ++g) {   // entry g's keys: rows g * KBG .. of the K and V tiles
      const int be = (int)(bz + g);
      tc::tma_load_4d(sl + g * KBG * KSW, &tmK, bar, 0, jj * KBG, (int)h, be);
      tc::tma_load_4d(sl + MH_K_BYTES + g * KBG * 128, &tmV, bar, 0, jj * KBG, (int)h, be);
      if (has_bias) {   // G = 1: one [128 q][64 k] tile; G = 4: four [32 q][16 k] tiles
        uint8_t* bt = sl + MH_K_BYTES + MH_V_BYTES + g * (MH_B_BYTES / G);
        if (P.bias_batched)
          tc::tma_load_4d(bt, &tmB, bar, jj * KBG, (int)q0, (int)h, be);
        else
          tc::tma_load_3d(bt, &tmB, bar, jj * KBG, (int)q0, (int)h);
      }
    }
  };

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 256);
    tc::tmem_relinquish();
  }
  if (tid == 4 * 32) {
    for (int s = 0; s < MH_RING; ++s) {
      tc::mbar_init(&kvfull[s], 1);
      tc::mbar_init(&kvfree[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(&sbar[s], 2);
      tc::mbar_init(&pready[s], 4);
      tc::mbar_init(&pvbar[s], 1);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmK);
    tc::prefetch_tmap(&tmV);
    if (has_bias) tc::prefetch_tmap(&tmB);
    // the ring's first blocks at once, under the Q and mask loads
    for (int jj = 0; jj < MH_RING && jj < nkb; ++jj) issue_load(jj);
  }
  // key k of entry g counts iff k < k_len and mask_k[g, k] (sdpa.py:61-80); one bit per key
  for (int w = warp; w < G * nkw; w += MH_THREADS / 32) {
    const int g = w / nkw;
    const int64_t key = (int64_t)(w - g * nkw) * 32 + lane, be = bz + g;
    const bool ok = be < a.batch && key < a.k_len && (!a.mask_k || a.mask_k[be * a.mk_sb + key] != 0);
    const uint32_t bits = __ballot_sync(0xffffffffu, ok);
    if (lane == 0) kbits[w] = bits;
  }
  // the query row of this thread (softmax warps): entry bz + ge, query q
  const int ge = G == 1 ? 0 : warp;
  const int64_t be = bz + ge;
  const int64_t q = q0 + (G == 1 ? tid : lane);
  const bool qin = warp < 4 && be < a.batch && q < a.q_len && (G == 1 || lane < QG);
  bool row_ok = qin;
  if (qin && a.mask_row) row_ok = a.mask_row[be] != 0;
  if (qin && a.mask_q) row_ok = row_ok && a.mask_q[be * a.mq_sb + q] != 0;
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  constexpr uint32_t S_COL = 0, O_COL = 128, Q_COL = 192;

  if (warp < 4) {
    const uint32_t lane_addr = tbase + ((uint32_t)(32 * warp) << 16);
    {   // Q row, scaled by scale * log2 e, into TMEM (zero beyond D)
      uint32_t qw[32];
      const float qs = a.scale * 1.4426950408889634f;
      const bf16* qp = static_cast<const bf16*>(a.q) + (qin ? be * a.q_sb + h * a.q_sh + q * a.q_sq : 0);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (qin && 8 * c < D) v = __ldg(reinterpret_cast<const uint4*>(qp + 8 * c));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) qw[4 * c + e] = pack_bf2(bf_lo(u[e]) * qs, bf_hi(u[e]) * qs);
      }
      tc::tmem_st32(lane_addr + Q_COL, qw);
      tc::tmem_wait_st();
    }
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&pready[1]);   // "Q is in TMEM": phase 0 of pready[1] (4 warps)

    const bool use_bias = has_bias && row_ok;
    const uint32_t* kb = kbits + ge * nkw;
    float m_run = -INFINITY, l = 0.f;
    for (int j = 0; j < nkb; ++j) {
      const int64_t k0 = (int64_t)j * KBG;
      // S_j is written and block j (its bias tile) has landed
      tc::mbar_wait(&sbar[j & 1], (j >> 1) & 1, P.status, aborted);
      tc::tc_fence_after();
      float sv[KBG];
      if constexpr (G == 1) {
        tc::tmem_ld64(lane_addr + S_COL + (j & 1) * MH_KB, sv);
      } else {
        tc::tmem_ld16(lane_addr + S_COL + (j & 1) * MH_KB + ge * KBG, sv);   // warp-uniform column
      }
      if (use_bias) {
        const uint8_t* bt = slot_of(j) + MH_K_BYTES + MH_V_BYTES;
#pragma unroll
        for (int c = 0; c < KBG / 8; ++c) {
          const uint4 v = G == 1 ? *reinterpret_cast<const uint4*>(bt + tc::sw128_off(tid, c))
                                 : *reinterpret_cast<const uint4*>(bt + ge * (MH_B_BYTES / G) + lane * (KBG * 2) + 16 * c);
          const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            sv[8 * c + 2 * e] = fmaf(bf_lo(u[e]), 1.4426950408889634f, sv[8 * c + 2 * e]);
            sv[8 * c + 2 * e + 1] = fmaf(bf_hi(u[e]), 1.4426950408889634f, sv[8 * c + 2 * e + 1]);
          }
        }
      }
      uint32_t vb = kb[(k0 >> 5)];                // KBG divides 32: one word covers the block
      if constexpr (G == 1) (void)vb;
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < KBG; ++e) {
        const int64_t key = k0 + e;
        const bool inb = key < a.k_len;
        bool valid;
        if constexpr (G == 1) {
          valid = ((kb[2 * j + (e >> 5)] >> (e & 31)) & 1u) != 0;
        } else {
          valid = ((vb >> ((int)(k0 & 31) + e)) & 1u) != 0;
        }
        const float sc = !inb ? -INFINITY : (row_ok && valid) ? sv[e] : -FLT_MAX;   // beyond k_len: no part at all
        sv[e] = sc;
        mx = fmaxf(mx, sc);
      }
      // the running max moves only when the block exceeds it by 2^8 (values stay <= 2^8)
      const bool moves = m_run == -INFINITY ? mx != -INFINITY : mx > m_run + MH_RESCALE;
      float corr = 1.f;
      if (moves) {
        corr = m_run == -INFINITY ? 0.f : ex2f(m_run - mx);
        m_run = mx;
      }
      const float mref = m_run == -INFINITY ? 0.f : m_run;
      uint32_t pk[MH_KB / 2];
#pragma unroll
      for (int e = 0; e < MH_KB / 2; ++e) pk[e] = 0u;   // G > 1: the other entries' columns stay zero
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int e = 0; e < KBG; e += 2) {
        const float p0 = ex2f(sv[e] - mref), p1 = ex2f(sv[e + 1] - mref);
        ps0 += p0;
        ps1 += p1;
        const uint32_t pp = pack_bf2(p0, p1);
        if constexpr (G == 1) {
          pk[e >> 1] = pp;
        } else {
#pragma unroll
          for (int g = 0; g < G; ++g)
            if (g == ge) pk[g * (KBG / 2) + (e >> 1)] = pp;   // static indices, warp-uniform choice
        }
      }
      l = l * corr + (ps0 + ps1);
      // O holds P V up to block j-1: rescale it once P_{j-1} V_{j-1} is done (warp-uniform branch)
      if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
        tc::mbar_wait(&pvbar[(j - 1) & 1], ((j - 1) >> 1) & 1, P.status, aborted);
        tc::tc_fence_after();
        float ov[MH_DP];
        tc::tmem_ld64(lane_addr + O_COL, ov);
        uint32_t r0[32], r1[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          r0[e] = __float_as_uint(ov[e] * corr);
          r1[e] = __float_as_uint(ov[32 + e] * corr);
        }
        tc::tmem_st32(lane_addr + O_COL, r0);
        tc::tmem_st32(lane_addr + O_COL + 32, r1);
      }
      tc::tmem_st32(lane_addr + S_COL + (j & 1) * MH_KB, pk);   // P_j over S_j
      tc::tmem_wait_st();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&pready[j & 1]);
    }
    // ---- O / l, gate, store ----
    if (nkb >= 2) tc::mbar_wait(&pvbar[(nkb - 2) & 1], ((nkb - 2) >> 1) & 1, P.status, aborted);
    tc::mbar_wait(&pvbar[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1, P.status, aborted);
    tc::tc_fence_after();
    float ov[MH_DP];
    tc::tmem_ld64(lane_addr + O_COL, ov);
    if (qin) {
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      bf16* op = static_cast<bf16*>(a.out) + be * a.o_sb + h * a.o_sh + q * a.o_sq;
      const bf16* gp = a.gate ? static_cast<const bf16*>(a.gate) + be * a.g_sb + h * a.g_sh + q * a.g_sq : nullptr;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (8 * c < D) {
          float o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = ov[8 * c + e] * inv;
          if (gp) {
            const uint4 g = __ldg(reinterpret_cast<const uint4*>(gp + 8 * c));
            const uint32_t gu[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              o[2 * e] *= fast_sigmoid(bf_lo(gu[e]));
              o[2 * e + 1] *= fast_sigmoid(bf_hi(gu[e]));
            }
          }
          *reinterpret_cast<uint4*>(op + 8 * c) =
              make_uint4(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]), pack_bf2(o[4], o[5]), pack_bf2(o[6], o[7]));
        }
      }
    }
  } else if (warp == 4) {
    // ---- TMA producer: block j + RING into the slot of block j once P_j V_j is done ----
    if (lane == 0) {
      for (int jj = MH_RING; jj < nkb; ++jj) {
        if (!tc::mbar_wait(&kvfree[jj % MH_RING], ((jj / MH_RING) + 1) & 1, P.status, aborted)) break;
        issue_load(jj);
      }
    }
  } else if (lane == 0) {
    // ---- warp 5: MMA issuer (stops at its first failed wait) ----
    constexpr uint32_t ID_S = tc::idesc_bf16(128, MH_KB);
    constexpr uint32_t ID_PV = tc::idesc_bf16(128, MH_DP) | (1u << 16);   // B (V) MN-major
    constexpr tc::Swizzle KSWZ = KSW == 128 ? tc::kSW128 : tc::kSW64;
    const uint32_t sb = tc::smem_u32(smem);
    auto issue_s = [&](int jj) {   // S_jj = Q K_jj^T into buffer jj & 1, once block jj has landed
      if (!tc::mbar_wait(&kvfull[jj % MH_RING], (jj / MH_RING) & 1, P.status, aborted)) return;
      tc::mbar_arrive(&sbar[jj & 1]);   // the softmax reads the bias tile once S_jj is signalled
      tc::tc_fence_after();
      const uint32_t kt = sb + MH_OFF_RING + (jj % MH_RING) * MH_SLOT_BYTES;
#pragma unroll
      for (int kk = 0; kk < DK / 16; ++kk)
        tc::mma_bf16_ts(tbase + S_COL + (jj & 1) * MH_KB, tbase + Q_COL + kk * 8,
                        tc::smem_desc(kt + kk * 32, 8 * KSW, KSWZ), ID_S, kk > 0);
      tc::mma_commit(&sbar[jj & 1]);
    };
    // Q must be in TMEM before the first S
    if (tc::mbar_wait(&pready[1], 0, P.status, aborted)) {
      tc::tc_fence_after();
      issue_s(0);
      if (!aborted && nkb > 1) issue_s(1);
    }
    for (int j = 0; j < nkb && !aborted; ++j) {
      // pready[1] completed one extra phase for Q: block j's phase is (j >> 1) + (j & 1)
      const uint32_t ph = ((j >> 1) + (j & 1)) & 1;
      if (!tc::mbar_wait(&pready[j & 1], ph, P.status, aborted)) break;
      tc::tc_fence_after();
      const uint32_t vt = sb + MH_OFF_RING + (j % MH_RING) * MH_SLOT_BYTES + MH_K_BYTES;
#pragma unroll
      for (int kk = 0; kk < MH_KB / 16; ++kk)
        tc::mma_bf16_ts(tbase + O_COL, tbase + S_COL + (j & 1) * MH_KB + kk * 8,
                        tc::smem_desc_mn(vt + kk * 2048, MH_V_BYTES, 1024, tc::kSW128), ID_PV, j > 0 || kk > 0);
      tc::mma_commit(&pvbar[j & 1]);
      tc::mma_commit(&kvfree[j % MH_RING]);
      if (j + 2 < nkb) issue_s(j + 2);
    }
  }
  tc::tc_fence_before();
  if (__syncthreads_or(aborted)) {   // abort path: the producer's loads and the issuer's MMAs done before exit
    if (warp == 4 && lane == 0) tc::drain_ring(kvfull, MH_RING, loads, P.status);
    if (warp == 5 && lane == 0) tc::drain_mma(drain, P.status);
    __syncthreads();
  }
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 256);
  }
}

// Tensor map over a strided bf16 tensor of up to 4 dims (dim 0 contiguous); dims of extent 1
// get a placeholder stride.  False (no message) when TMA cannot address it.
bool strided_tmap(CUtensorMap* map, const void* base, int rank, const int64_t* dims, const int64_t* strides,
                  const uint32_t* box, CUtensorMapSwizzle sw) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  cuuint64_t gd[4], gs[3];
  cuuint32_t bx[4], es[4] = {1, 1, 1, 1};
  int64_t prev = dims[0] * 2;
  for (int i = 0; i < rank; ++i) {
    if (dims[i] < 1 || dims[i] > (int64_t(1) << 32)) return false;
    gd[i] = (cuuint64_t)dims[i];
    bx[i] = box[i];
    if (i > 0) {
      int64_t st = strides[i - 1] * 2;   // bytes
      if (dims[i] == 1) st = (prev + 15) / 16 * 16;
      if (st <= 0 || st % 16 != 0 || st >= (int64_t(1) << 40)) return false;
      gs[i - 1] = (cuuint64_t)st;
      prev = st * dims[i];
    }
  }
  auto encode = tensor_map_encoder();
  if (!encode) return false;
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), gd, gs, bx, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Returns SF_OK after launching, or SF_ERR_ARG (with no message) when the call is outside what
// this kernel takes, so that the caller uses the CUDA-core kernel instead.
int attention_tc(const sf_attention_args* a, cudaStream_t stream) {
  const int64_t D = a->head_dim;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  bool ok = a->dtype == SF_BF16 && D % 8 == 0 && D <= MH_DP && (a->value_dim == 0 || a->value_dim == D) &&
            a->k_len > 0 && a->k_len <= MH_MAX_KEYS && al16(a->q) && al16(a->out) && (!a->gate || al16(a->gate)) &&
            (a->q_sb | a->q_sh | a->q_sq | a->o_sb | a->o_sh | a->o_sq) % 8 == 0 &&
            (!a->gate || (a->g_sb | a->g_sh | a->g_sq) % 8 == 0) && a->q_len <= (int64_t(1) << 31) - TILE &&
            (!a->bias || a->bias_dtype == SF_BF16);
  if (!ok) return SF_ERR_ARG;
  const int ksw = D <= 32 ? 64 : 128;
  // entries of at most 32 queries (the atom windows) go four to a CTA
  const int G = (a->q_len <= TILE / 4 && a->batch > 1 && ksw == 64 && a->k_len <= MH_MAX_KEYS / 4) ? 4 : 1;
  const uint32_t kbg = (uint32_t)(MH_KB / G);
  CUtensorMap mk, mv, mb;
  {
    const int64_t dk[4] = {D, a->k_len, a->heads, a->batch}, sk[3] = {a->k_sk, a->k_sh, a->k_sb};
    const int64_t sv[3] = {a->v_sk, a->v_sh, a->v_sb};
    const uint32_t bk[4] = {(uint32_t)(ksw / 2), kbg, 1, 1}, bv[4] = {64, kbg, 1, 1};
    if (!strided_tmap(&mk, a->k, 4, dk, sk, bk, ksw == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B) ||
        !strided_tmap(&mv, a->v, 4, dk, sv, bv, CU_TENSOR_MAP_SWIZZLE_128B))
      return SF_ERR_ARG;
  }
  int batched = 0;
  if (a->bias) {
    // G = 1: [128 queries][64 keys] boxes, 128B swizzle; G = 4: [32 queries][16 keys], unswizzled
    const uint32_t bb[4] = {kbg, (uint32_t)(TILE / G), 1, 1};
    batched = a->b_sb != 0 && a->batch > 1;
    const int64_t db[4] = {a->k_len, a->q_len, a->heads, a->batch}, sbs[3] = {a->b_sq, a->b_sh, a->b_sb};
    if (!strided_tmap(&mb, a->bias, batched ? 4 : 3, db, sbs, bb,
                      G == 1 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE))
      return SF_ERR_ARG;
  } else {
    mb = mk;   // unused
  }
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  static bool attr[64][3] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int ki = G == 4 ? 2 : ksw == 64 ? 1 : 0;
  auto kern = G == 4 ? k_mha_tc<64, 4> : ksw == 64 ? k_mha_tc<64, 1> : k_mha_tc<128, 1>;
  if (!attr[dev & 63][ki]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MH_SMEM);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(attention): %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    attr[dev & 63][ki] = true;
  }
  MhaParams p{*a, batched, status};
  dim3 grid(G == 1 ? (unsigned)((a->q_len + TILE - 1) / TILE) : 1u, (unsigned)a->heads,
            (unsigned)((a->batch + G - 1) / G));
  launch_pdl(kern, grid, dim3(MH_THREADS), MH_SMEM, stream, mk, mv, mb, p);
  count_launch();
  return check_launch("attention_tc");
}

}  // namespace sf
