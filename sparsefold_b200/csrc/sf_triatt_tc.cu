// Triangle attention (GridSelfAttention, blocks.py:270-366), bf16 track, on tcgen05.
//
// Two kernels per call:
//  k_triatt_project_tc  persistent and warp-specialised: TMA brings 128-query z
//                       tiles (row tiles for the starting node, column tiles for
//                       the ending node, transpose=True), four warps apply the
//                       scale-only LN (blocks.py:260-264) in place and form the
//                       4-head pair bias on CUDA cores, one thread issues
//                       D[query][channel] = LN(z) . W^T for q|k (one N=256 GEMM)
//                       and the gate, and D[channel][query] for v (so v^T rows
//                       come out of TMEM directly), into two TMEM halves, and
//                       eight epilogue warps stage the outputs in shared memory
//                       and TMA-store them.
//  k_triatt_core_tc     flash attention + gate + output projection + residual for
//                       one (attention row b, 128-query block): four softmax
//                       warpgroups, one per head.  S = Q K^T and O += P V
//                       (M128 N32 K32, Q and P from TMEM) run on tcgen05 with
//                       TMEM accumulators; K/V^T blocks and bias tiles arrive
//                       by TMA; the softmax adds the bias and runs in exp2 with
//                       the reference's -FLT_MAX masking; the gated outputs of
//                       all four heads feed one more tcgen05 GEMM with the
//                       output projection, whose epilogue adds the residual.
//
// Intermediate layouts (qp = n rounded up to 128; padded query rows are zero):
//   K [b][h][qp][32]    Vt [b][h][32][qp]
//   Q (times log2(e)/sqrt(32)) and G = sigmoid(gate) [b][h][qp / 32][4][32][8]: per group of 32
//         queries, four chunks of 8 channels, each [32 queries][8 channels] (2 KB per group), so
//         that a warp holding one query per lane reads each chunk as 512 contiguous bytes
//   bias  [q][h][qp] (bias[q][h][k] = log2(e) LN(z)[q,k] . W_b[h] in bf16, untransposed;
//         rows q all-gathered from the row shards when the pair tensor is distributed)
#include <cfloat>

#include "sf_pair_tc.cuh"

namespace sf {
namespace {

using namespace pt;

constexpr int H = 4, D = 32;
constexpr float kLog2e = 1.4426950408889634f;
// The core works in base 2: Q is stored multiplied by log2(e) / sqrt(D) and the
// pair bias by log2(e), so logit * log2(e) = q'.k + b' takes one add per key.
constexpr float kBiasScale = kLog2e;
constexpr float kQScale = 0.25503486f;   // log2(e) / sqrt(32)

struct AttProjParams {
  bf16* q;                // Q and G in 32-query groups (see the layouts above)
  bf16* g;
  const float* ln_w;      // act_norm scale [128]
  const bf16* w_bias;     // [4][128]
  bf16* bias;             // [.][H][qp]
  int64_t nb, nq, qp;     // attention rows (batches), queries = keys, query pitch
  int transpose;          // attention along columns: batch = column, query = row
  int compute_bias;       // write bias[(r*H + h)*qp + s] for the block's positions (r, s)
  uint32_t* status;
};

// Warp roles (448 threads), one 128-query tile of one attention row at a time:
//   warps 0-7   epilogue: warp w owns TMEM lanes 32(w%4)..: queries 32(w%4)..+31 of
//               q, k and gate (D[query][channel]; heads 2(w/4), 2(w/4)+1) and
//               channels of head w%4 of v (D[channel][query]; queries 64(w/4)..+63);
//               it stages each output in its shared-memory tile (two 2 KB halves, so
//               one TMA store drains while the next is written) and TMA-stores it
//   warps 8-11  thread = query: scale-only LayerNorm of its row in place and the
//               four pair-bias logits LN(z) . W_b[h]
//   warp 12     TMA producer of z tiles (row tiles, or column tiles for the
//               ending node), two stages
//   warp 13     MMA issuer: half 0 (TMEM columns 0-255) = LN(z) . [W_q | W_k]^T
//               (M128 N256); half 1 = LN(z) . W_g^T (columns 256-383) and
//               W_v . LN(z)^T (columns 384-511)
constexpr int NOUT = 512;                   // w_qkvg rows: q, k, v, gate
constexpr int W_BYTES = NOUT * C * 2;
constexpr int PJ_EPI_WARPS = 8;
constexpr int PJ_THREADS = (PJ_EPI_WARPS + 4 + 2) * 32;
constexpr int PJ_ST_BYTES = 64 * D * 2;     // one epilogue warp's staging tile (64 queries x 32 channels)
constexpr int OFF_JW = 0;
constexpr int OFF_JZ = W_BYTES;                            // [2] z tiles
constexpr int OFF_JST = OFF_JZ + 2 * A_BYTES;              // [8] staging tiles
constexpr int OFF_JWB = OFF_JST + PJ_EPI_WARPS * PJ_ST_BYTES;   // W_b [4][128] bf16
constexpr int OFF_JLN = OFF_JWB + H * C * 2;                  // LayerNorm scale [128] fp32
constexpr int OFF_JBAR = OFF_JLN + C * 4;
constexpr int SMEM_PROJ = OFF_JBAR + 256 + 1024;
static_assert(SMEM_PROJ <= 232448, "projection shared memory");

// Scale-only LayerNorm of tile row r in place (one thread per row) and the row's
// pair bias LN(z) . W_b[h] (bf16 operands, fp32 sums): statistics in one pass,
// shifted by the row's first value so E[(x-k)^2] - E[x-k]^2 keeps its precision,
// packed fp32 pair arithmetic; the scale and W_b come from shared memory.
__device__ __forceinline__ void ln_row_bias(uint8_t* tile, int r, const float* w_s, const bf16* wb_s, float (&bias)[H]) {
  auto off = [&](int i) -> uint32_t { return (uint32_t)(i >> 3) * ATOM + tc::sw128_off(r, i & 7); };
  const float k = bf_lo(*reinterpret_cast<const uint32_t*>(tile + off(0)));
  float s[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, q[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
  for (int i = 0; i < 16; ++i)
    ln_accumulate(*reinterpret_cast<const uint4*>(tile + off(i)), k, s[i & 1], q[i & 1]);
  const float dm = ((s[0][0] + s[0][1]) + (s[1][0] + s[1][1])) * (1.0f / C);
  const float mean = k + dm;
  const float rstd =
      rsqrtf(fmaxf(((q[0][0] + q[0][1]) + (q[1][0] + q[1][1])) * (1.0f / C) - dm * dm, 0.f) + 1e-5f);
  float b2[2][H];
#pragma unroll
  for (int h = 0; h < H; ++h) b2[0][h] = b2[1][h] = 0.f;
#pragma unroll 2
  for (int i = 0; i < 16; ++i) {
    uint4 v = *reinterpret_cast<const uint4*>(tile + off(i));
    uint32_t* u = reinterpret_cast<uint32_t*>(&v);
    const float4 w0 = *reinterpret_cast<const float4*>(w_s + 8 * i);
    const float4 w1 = *reinterpret_cast<const float4*>(w_s + 8 * i + 4);
    const float wl[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    uint4 wv[H];
#pragma unroll
    for (int h = 0; h < H; ++h) wv[h] = *reinterpret_cast<const uint4*>(wb_s + h * C + 8 * i);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x0 = bf_lo(u[j]), x1 = bf_hi(u[j]);
      sub2(x0, x1, mean, mean);
      mul2(x0, x1, rstd, rstd);
      mul2(x0, x1, wl[2 * j], wl[2 * j + 1]);
      u[j] = pack_bf2(x0, x1);
      // the bias uses the bf16-rounded normalised row: bf16 x bf16 products accumulated in fp32
#pragma unroll
      for (int h = 0; h < H; ++h)
        b2[j & 1][h] = fma_bf16x2_f32(u[j], reinterpret_cast<const uint32_t*>(&wv[h])[j], b2[j & 1][h]);
    }
    *reinterpret_cast<uint4*>(tile + off(i)) = v;
  }
#pragma unroll
  for (int h = 0; h < H; ++h) bias[h] = b2[0][h] + b2[1][h];
}

__global__ void __launch_bounds__(PJ_THREADS, 1) k_triatt_project_tc(const __grid_constant__ CUtensorMap tmZ,
                                                                     const __grid_constant__ CUtensorMap tmK,
                                                                     const __grid_constant__ CUtensorMap tmV,
                                                                     const bf16* __restrict__ w_qkvg, AttProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_JBAR);   // [2] z tile landed
  uint64_t* normed = full + 2;                                      // [2] z tile normalised (128 arrivals)
  uint64_t* zfree = normed + 2;                                     // [2] MMAs of the stage done
  uint64_t* tfull = zfree + 2;                                      // [2] TMEM half written
  uint64_t* tfree = tfull + 2;                                      // [2] TMEM half read (8 warps)
  uint64_t* drain = tfree + 2;                                      // MMA drain barrier (abort path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t nqb = p.qp / TILE, ntiles = p.nb * nqb;

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&normed[s], 128);
      tc::mbar_init(&zfree[s], 1);
      tc::mbar_init(&tfull[s], 1);
      tc::mbar_init(&tfree[s], PJ_EPI_WARPS);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmZ);
    tc::prefetch_tmap(&tmK);
    tc::prefetch_tmap(&tmV);
  }
  for (int e = tid; e < H * C / 8; e += PJ_THREADS)
    reinterpret_cast<uint4*>(smem + OFF_JWB)[e] = __ldg(reinterpret_cast<const uint4*>(p.w_bias) + e);
  if (tid < C) reinterpret_cast<float*>(smem + OFF_JLN)[tid] = p.ln_w[tid];
  load_weight_sw128(smem + OFF_JW, w_qkvg, NOUT, tid, PJ_THREADS);
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

  if (warp == 12) {
    // ---- TMA producer (stops at its first failed wait) ----
    if (lane == 0) {
      uint32_t& it = loads;
      for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const int st = it & 1;
        if (it >= 2 && !tc::mbar_wait(&zfree[st], ((it >> 1) + 1) & 1, p.status, aborted)) break;
        const int b = (int)(tile / nqb), q0 = (int)((tile % nqb) * TILE);   // (projection tile coordinates)
        const int c1 = p.transpose ? b : q0;     // column coordinate
        const int c2 = p.transpose ? q0 : b;     // row coordinate
        uint8_t* dst = smem + OFF_JZ + st * A_BYTES;
        tc::mbar_expect_tx(&full[st], A_BYTES);
        tc::tma_load_3d(dst, &tmZ, &full[st], 0, c1, c2);
        tc::tma_load_3d(dst + ATOM, &tmZ, &full[st], 64, c1, c2);
      }
    }
  } else if (warp == 13) {
    // ---- MMA issuer (stops at its first failed wait) ----
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = tc::idesc_bf16(128, 256), IDESC = tc::idesc_bf16(128, 128);
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const int st = it & 1;
        if (!tc::mbar_wait(&normed[st], (it >> 1) & 1, p.status, aborted)) break;
        tc::tc_fence_after();
        const uint32_t zb = sb + OFF_JZ + st * A_BYTES;
        auto wdesc = [&](int mtx, int ka, int kk) {   // rows 128 mtx.. of W (q, k, v, gate), K step (ka, kk)
          return tc::smem_desc(sb + OFF_JW + ka * (NOUT * 128) + mtx * (128 * 128) + kk * 32, 1024, tc::kSW128);
        };
        // half 0: [q | k][query] = LN(z) . W_qk^T
        if (it >= 1 && !tc::mbar_wait(&tfree[0], (it - 1) & 1, p.status, aborted)) break;
        tc::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int ka = k >> 2, kk = k & 3;
          tc::mma_bf16(tbase, tc::smem_desc(zb + ka * ATOM + kk * 32, 1024, tc::kSW128), wdesc(0, ka, kk), IDESC_QK, k > 0);
        }
        tc::mma_commit(&tfull[0]);
        // half 1: gate[query][channel] and v[channel][query]
        if (it >= 1 && !tc::mbar_wait(&tfree[1], (it - 1) & 1, p.status, aborted)) break;
        tc::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int ka = k >> 2, kk = k & 3;
          const uint64_t zd = tc::smem_desc(zb + ka * ATOM + kk * 32, 1024, tc::kSW128);
          tc::mma_bf16(tbase + 256, zd, wdesc(3, ka, kk), IDESC, k > 0);
          tc::mma_bf16(tbase + 384, wdesc(2, ka, kk), zd, IDESC, k > 0);
        }
        tc::mma_commit(&tfull[1]);
        tc::mma_commit(&zfree[st]);
      }
    }
  } else if (warp >= PJ_EPI_WARPS) {
    // ---- LayerNorm in place + pair bias (thread = query of the tile) ----
    const int r = tid - PJ_EPI_WARPS * 32;
    const bf16* wb_s = reinterpret_cast<const bf16*>(smem + OFF_JWB);
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int st = it & 1;
      tc::mbar_wait(&full[st], (it >> 1) & 1, p.status, aborted);
      float bias[H];
      ln_row_bias(smem + OFF_JZ + st * A_BYTES, r, reinterpret_cast<const float*>(smem + OFF_JLN), wb_s, bias);
      tc::fence_proxy_async();
      tc::mbar_arrive(&normed[st]);
      const int64_t b = tile / nqb, qi = (tile % nqb) * TILE + r;
      if (p.compute_bias && qi < p.nq) {
        const int64_t rr = p.transpose ? qi : b, ss = p.transpose ? b : qi;
#pragma unroll
        for (int h = 0; h < H; ++h) p.bias[(rr * H + h) * p.qp + ss] = __float2bfloat16_rn(bias[h] * kBiasScale);
      }
    }
  } else {
    // ---- epilogue ----
    const int quad = warp & 3, hf = warp >> 2;
    const uint32_t lane_addr = tbase + ((uint32_t)(32 * quad) << 16);
    uint8_t* stg = smem + OFF_JST + warp * PJ_ST_BYTES;
    int sh = 0;              // staging half for the next [32 queries][32 channels] store
    bool full_used = false;  // the last store read the whole staging tile (v^T)
    // one [32 queries][32 channels] tile (this lane = query row) into the next half, then stored:
    // K by TMA as rows (64B swizzle), Q and G as one 2 KB group of four [32 queries][8 channels]
    // chunks by a plain bulk copy (map == nullptr, dst the group)
    auto store_rows = [&](const float* v, const CUtensorMap* map, int c0, int c1, bf16* dst) {
      if (lane == 0) {
        if (full_used) tc::bulk_wait_read0();
        else tc::bulk_wait_read1();   // the store that used this half (two stores ago) has read it
      }
      __syncwarp();
      uint8_t* half = stg + sh * 2048;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(half + (map ? tc::sw64_off(lane, c) : (uint32_t)(c * 512 + lane * 16))) =
            make_uint4(pack_bf2(v[8 * c], v[8 * c + 1]), pack_bf2(v[8 * c + 2], v[8 * c + 3]),
                       pack_bf2(v[8 * c + 4], v[8 * c + 5]), pack_bf2(v[8 * c + 6], v[8 * c + 7]));
      tc::fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        if (map) tc::tma_store_2d(map, half, c0, c1);
        else tc::bulk_store(dst, half, 2048);
        tc::bulk_commit();
      }
      sh ^= 1;
      full_used = false;
    };
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int b = (int)(tile / nqb), qt0 = (int)((tile % nqb) * TILE);
      const int qrow = qt0 + 32 * quad;   // first query of this warp's TMEM lanes
      // ---- half 0: q and k, heads 2 hf, 2 hf + 1 ----
      tc::mbar_wait(&tfull[0], it & 1, p.status, aborted);
      tc::tc_fence_after();
#pragma unroll 1
      for (int i = 0; i < 4; ++i) {
        const int t = i >> 1, hd = 2 * hf + (i & 1);   // t: 0 q, 1 k
        float v[32];
        tc::tmem_ld32(lane_addr + t * 128 + hd * D, v);
        if (i == 3) {
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&tfree[0]);
        }
        if (t == 0) {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= kQScale;   // q stored pre-scaled for the base-2 softmax
        }
        const int64_t grow0 = ((int64_t)b * H + hd) * p.qp + qrow;   // first row of the 32-query group
        store_rows(v, t == 0 ? nullptr : &tmK, 0, (int)grow0, p.q + grow0 * D);
      }
      // ---- half 1: gate (heads 2 hf, 2 hf + 1) and v^T (head quad, queries 64 hf ..) ----
      tc::mbar_wait(&tfull[1], it & 1, p.status, aborted);
      tc::tc_fence_after();
#pragma unroll 1
      for (int i = 0; i < 2; ++i) {
        const int hd = 2 * hf + i;
        float v[32];
        tc::tmem_ld32(lane_addr + 256 + hd * D, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = sigmoid_tanh(v[e]);
        store_rows(v, nullptr, 0, 0, p.g + (((int64_t)b * H + hd) * p.qp + qrow) * D);
      }
      {
        float v[64];
        tc::tmem_ld64(lane_addr + 384 + 64 * hf, v);   // channel 32 quad + lane, 64 queries
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(&tfree[1]);
          tc::bulk_wait_read0();   // v^T takes the whole staging tile
        }
        __syncwarp();
        // [32 channels][64 queries], 128B swizzle; this lane's row is its channel
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(stg + tc::sw128_off(lane, c)) =
              make_uint4(pack_bf2(v[8 * c], v[8 * c + 1]), pack_bf2(v[8 * c + 2], v[8 * c + 3]),
                         pack_bf2(v[8 * c + 4], v[8 * c + 5]), pack_bf2(v[8 * c + 6], v[8 * c + 7]));
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          tc::tma_store_2d(&tmV, stg, qt0 + 64 * hf, (b * H + quad) * D);
          tc::bulk_commit();
        }
        full_used = true;
        sh = 0;
      }
    }
    if (lane == 0) tc::bulk_wait0();
  }
  tc::tc_fence_before();
  if (__syncthreads_or(aborted)) {   // abort path: drain the producer's loads and the issuer's MMAs
    if (warp == 12 && lane == 0) tc::drain_ring(full, 2, loads, p.status);
    if (warp == 13 && lane == 0) tc::drain_mma(drain, p.status);
    __syncthreads();
  }
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------
// attention core
// ---------------------------------------------------------------------------
struct AttCoreParams {
  const bf16 *q, *g, *bias;
  const bf16* w_out;      // output_projection^T [128 out][128 in]
  const uint8_t* mask;    // [N] token mask (keys/queries are all N tokens)
  const bf16* z;          // the z block [rows][cols][128] (residual)
  bf16* z_out;
  int64_t cols;           // columns of the z block
  int64_t nq, qp;         // queries = keys, pitch
  int64_t batch_offset;   // global token index of attention row 0 (row mask)
  int transpose;
  float scale_log2;       // (1/sqrt(D)) * log2(e), already applied to the stored Q
  uint32_t* status;
};

constexpr int KB = 32;                 // keys per block
constexpr int RING = 4;                // key blocks in flight: K and bias tile of each
constexpr int VRING = 6;               // V^T blocks: two more, so block j+4 lands where block j-2 was
constexpr int K_BYTES = KB * D * 2;    // K block 32 keys x 64 B (64B swizzle)
constexpr int V_BYTES = D * KB * 2;    // V^T block 32 dims x 64 B (64B swizzle)
constexpr int BT_BYTES = TILE * KB * 2;  // bias tile of one head: 128 queries x 32 keys (64B swizzle)
constexpr int HEAD_BYTES = RING * (K_BYTES + BT_BYTES) + VRING * V_BYTES;   // one head's rings
constexpr int MAX_QP = 32768;
constexpr int OFF_RING = 0;                                   // [h]: K [RING] | bias [RING] (residual, W_o, gated O at the end) | V^T [VRING]
constexpr int OFF_KBITS = OFF_RING + H * HEAD_BYTES;          // key-valid bits, qp/32 words
constexpr int OFF_BAR = OFF_KBITS + MAX_QP / 8;
constexpr int SMEM_CORE = OFF_BAR + 1024 + 1024;
static_assert(SMEM_CORE <= 232448, "attention core shared memory");
constexpr float kRescale = 8.0f;       // the running max moves only when a block exceeds it by 2^8
constexpr float kSumLimit = 256.0f;    // a block sum up to 2^8 leaves the running max where it is
constexpr int CORE_THREADS = (16 + 4) * 32;   // four softmax warpgroups + one issue warp per head

// (a0, a1) += (b0, b1) as one packed fp32x2 add.
__device__ __forceinline__ void add_f32x2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\t"
      "mov.b64 x, {%0, %1};\n\t"
      "mov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 x, x, y;\n\t"
      "mov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}
// a0 += lo(w), a1 += hi(w) for a packed bf16 pair w (bf16 * 1.0 + fp32 in one instruction each).
__device__ __forceinline__ void add_bf16x2(uint32_t w, float& a0, float& a1) {
  asm("{\n\t.reg .b16 l, h, one;\n\t"
      "mov.b32 {l, h}, %2;\n\t"
      "mov.b16 one, 0x3F80;\n\t"
      "fma.rn.f32.bf16 %0, l, one, %0;\n\t"
      "fma.rn.f32.bf16 %1, h, one, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(w));
}
__device__ __forceinline__ void wg_sync(int g) { asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory"); }
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One CTA = one (attention row b, 128-query tile); warpgroup h owns head h and
// TMEM columns [128h, 128h+128): two S buffers (32 fp32 columns each; P_j, 16
// columns of bf16 pairs, is written over S_j once it has been read), O (32) and
// Q (16 columns of bf16 pairs).  Keys go in blocks of 32.  The tensor core only
// runs TMEM-operand MMAs: S_j = Q K_j^T (A = Q) and O += P_j V_j (A = P).  The
// pair bias, stored as log2(e) * bias, arrives by TMA as a [128 queries][32
// keys] tile and each thread adds its query's row on the CUDA cores: logit2 =
// S scale + bias'.  Per block j a warpgroup reads S_j and its bias row, sets
// masked and padding keys to -inf and forms 2^(logit2 - m) against the running
// max m, summing and packing them in the same pass; no value exceeds the block's
// sum, so while that sum stays <= 2^8 the running max stands, and otherwise the
// block max is taken from S and the bias (the max moves when the block max
// exceeds m by more than 2^8, the values are redone and O is rescaled in TMEM
// once P_{j-1} V_{j-1} is done).  It writes P_j as bf16 and signals it at the
// start of the next block, once that block's S wait has covered the store.
// One issue warp per head (warps 16-19; an issuing warp gets one tcgen05.mma
// per ~130 cycles, which must not sit on the softmax warps) then issues
// O += P_j V_j and S_{j+2} into the same buffer (MMAs of one thread run in issue
// order, so S_{j+2} writes after P_j V_j reads P_j; S_j complete thus also means
// P_{j-2} V_{j-2} complete), and only then refills the TMA rings, so the next S
// never waits behind a TMA issue.  The K block, V^T block and bias tile of a key
// block arrive by TMA on one barrier, requested four blocks ahead (two blocks
// before its S is issued; V^T in a ring of six, so a refill never waits for the
// P V that read the slot), which the issue warp folds into the S barrier: a
// softmax warp waits once per block.  Each issue warp requests its head's first
// two blocks right after setting up its barriers, under the Q and mask loads, and
// the heads start a few hundred cycles apart.
// A row whose token is masked attends uniformly to all N keys (every logit of
// the reference is -FLT_MAX there).  Freed ring slots receive, near the end, the
// residual tile z[queries][32h .. 32h+31] and the W_o columns of head h; the
// gated, normalised O_h is staged in the last one and head h's issue warp forms
// its share of the output projection, O_h W_o[:, 32h .. 32h+31]^T, in the head's
// own TMEM columns; each warpgroup sums the four heads' shares of its 32 output
// channels, adds them to the residual tile in place and TMA-stores it.
__global__ void __launch_bounds__(CORE_THREADS, 1) k_triatt_core_tc(const __grid_constant__ CUtensorMap tmK,
                                                           const __grid_constant__ CUtensorMap tmV,
                                                           const __grid_constant__ CUtensorMap tmB,
                                                           const __grid_constant__ CUtensorMap tmW,
                                                           const __grid_constant__ CUtensorMap tmR,
                                                           const __grid_constant__ CUtensorMap tmO, AttCoreParams p) {
  extern __shared__ uint8_t smem_raw[];
  tc::griddep_wait();     // the previous kernel's outputs are complete and visible from here on
  tc::griddep_launch();
  uint8_t* smem = align1024(smem_raw);
  // Block-indexed barriers come in pairs (block j uses [j & 1], phase j >> 1): a parity
  // wait only tells phases apart within one phase of the barrier, and the softmax warps,
  // the issue warp and the tensor core may each run up to a block ahead of one another.
  uint64_t* sbar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);   // [H][2] S_j written and block j landed (2 arrivals)
  uint64_t* pvbar = sbar + 2 * H;                                  // [H][2] P_j V_j done
  uint64_t* pready = pvbar + 2 * H;                                // [H][2] P_j written (4 softmax warps)
  uint64_t* lbar = pready + 2 * H;                                 // [H][RING] K, V^T and bias of a block landed
  uint64_t* rbar = lbar + RING * H;                                // [H] residual tile landed
  uint64_t* wbar = rbar + H;                                       // [H] W_o columns landed
  uint64_t* ostaged = wbar + H;                                    // [H] gated O_h staged (4 softmax warps)
  uint64_t* outbar = ostaged + H;                                  // [H] O_h W_o^T done
  uint64_t* drainb = outbar + H;                                   // [H] issue warps' MMA drain (abort path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drainb + H);
  uint32_t* kbits = reinterpret_cast<uint32_t*>(smem + OFF_KBITS);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool issuer = warp >= 16;
  const int g = issuer ? warp - 16 : tid >> 7, t = tid & 127;
  const int64_t q0 = (int64_t)blockIdx.x * TILE, b = blockIdx.y;
  const int nkb = (int)(p.qp / KB);   // >= 4
  const int64_t bh = b * H + g;
  uint8_t* ring = smem + OFF_RING + g * HEAD_BYTES;
  auto k_of = [&](int jj) { return ring + (jj % RING) * K_BYTES; };
  auto bt_of = [&](int jj) { return ring + RING * K_BYTES + (jj % RING) * BT_BYTES; };
  auto v_of = [&](int jj) { return ring + RING * (K_BYTES + BT_BYTES) + (jj % VRING) * V_BYTES; };
  bool aborted = false;
  uint32_t loads = 0;                    // key blocks requested by this head's issue thread (abort-path drain)
  bool rload = false, wload = false;     // residual tile / W_o columns requested

  // this thread's query row of Q (64 B), for TMEM: requested first, it is the longest wait
  uint4 qrow[4];
  if (!issuer) {
    const uint4* qsrc = reinterpret_cast<const uint4*>(p.q + (bh * p.qp + q0 + (t & ~31)) * D) + (t & 31);
#pragma unroll
    for (int c = 0; c < 4; ++c) qrow[c] = __ldg(qsrc + 32 * c);
  }
  auto issue_load = [&](int jj) {   // K, V^T and bias[q0..q0+127][g][32 jj .. 32 jj + 31] of block jj (jj == loads)
    ++loads;
    uint64_t* bar = &lbar[g * RING + jj % RING];
    tc::mbar_expect_tx(bar, K_BYTES + V_BYTES + BT_BYTES);
    tc::tma_load_2d(k_of(jj), &tmK, bar, 0, (int)(bh * p.qp + (int64_t)jj * KB));
    tc::tma_load_2d(v_of(jj), &tmV, bar, jj * KB, (int)(bh * D));
    tc::tma_load_3d(bt_of(jj), &tmB, bar, jj * KB, g, (int)q0);
  };
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (issuer && lane == 0) {
    // each issue warp sets up its head's barriers and starts the first four blocks' loads at once
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&sbar[g * 2 + i], 2);
      tc::mbar_init(&pvbar[g * 2 + i], 1);
      tc::mbar_init(&pready[g * 2 + i], 4);
    }
    for (int i = 0; i < RING; ++i) tc::mbar_init(&lbar[g * RING + i], 1);
    tc::mbar_init(&rbar[g], 1);
    tc::mbar_init(&wbar[g], 1);
    tc::mbar_init(&ostaged[g], 4);
    tc::mbar_init(&outbar[g], 1);
    tc::mbar_init(&drainb[g], 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmK);
    tc::prefetch_tmap(&tmV);
    tc::prefetch_tmap(&tmB);
    // the first two blocks at once, under the Q and mask loads (blocks 2 and 3 follow S_0 and S_1)
    issue_load(0);
    issue_load(1);
  }
  // key k is attended iff mask[row] && mask[k] (pair mask, blocks.py:314); bits hold mask[k] && k < N
  for (int w = warp; w < (int)(p.qp / 32); w += CORE_THREADS / 32) {
    const int64_t key = (int64_t)w * 32 + lane;
    const uint32_t bits = __ballot_sync(0xffffffffu, key < p.nq && p.mask[key] != 0);
    if (lane == 0) kbits[w] = bits;
  }
  const bool uniform = p.mask[b + p.batch_offset] == 0;
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t lane_addr = tbase + ((uint32_t)(32 * (warp & 3)) << 16);
  // S buffers [0,32) and [32,64) (P_j written over the first 16 columns of S_j), O [64,96), Q [96,112)
  const uint32_t s_col = (uint32_t)g * 128, o_col = s_col + 64, qt_col = s_col + 96;
  constexpr uint32_t IDESC = tc::idesc_bf16(128, 32);   // S (N = 32 keys) and O (N = 32 dims)
  if (!issuer) {
    uint32_t qw[16];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      qw[4 * c] = qrow[c].x;
      qw[4 * c + 1] = qrow[c].y;
      qw[4 * c + 2] = qrow[c].z;
      qw[4 * c + 3] = qrow[c].w;
    }
    tc::tmem_st16(lane_addr + qt_col, qw);
    tc::tmem_wait_st();
  }

  auto issue_s = [&](int jj) {   // S_jj = Q K_jj^T into S buffer jj % 2, once block jj has landed
    if (!tc::mbar_wait(&lbar[g * RING + jj % RING], (jj / RING) & 1, p.status, aborted)) return;
    tc::mbar_arrive(&sbar[g * 2 + (jj & 1)]);   // the softmax reads the bias tile once S_jj is signalled
    tc::tc_fence_after();
    const uint32_t ks = tc::smem_u32(k_of(jj));
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      tc::mma_bf16_ts(tbase + s_col + (jj & 1) * KB, tbase + qt_col + kk * 8, tc::smem_desc(ks + kk * 32, 512, tc::kSW64),
                      IDESC, kk > 0);
    tc::mma_commit(&sbar[g * 2 + (jj & 1)]);
  };

  // residual tile z[b][q0..q0+127][32g..] (or z[q0..][b][32g..] for the ending node): 128 rows of 64 B
  const int rc1 = p.transpose ? (int)b : (int)q0, rc2 = p.transpose ? (int)q0 : (int)b;
  uint8_t* resid = bt_of(nkb);        // bias part of the slot of block nkb-4
  uint8_t* wstage = bt_of(nkb + 1);   // ... of block nkb-3
  uint8_t* ostage = bt_of(nkb + 3);   // ... of block nkb-1
  constexpr uint32_t IDESC_OUT = tc::idesc_bf16(128, 128);

  tc::tc_fence_before();
  __syncthreads();   // Q is in TMEM
  float m_run = -INFINITY, l = 0.f;
  if (issuer) {
    if (lane == 0) {
      tc::tc_fence_after();
      // Heads start ~450 cycles apart: the four softmax warps of an SM sub-partition (one per
      // head) then reach their barrier waits at different times and the exponentials of one
      // fill the others' waits (measured: 6 us less per call at N=512 than a common start).
      if (g > 0) {
        const long long until = clock64() + (long long)g * 450;
        while (clock64() < until) {
        }
      }
      // (the issue thread stops issuing at its first failed wait)
      issue_s(0);
      if (!aborted) issue_load(2);
      if (!aborted) issue_s(1);
      if (!aborted) issue_load(3);
      for (int j = 0; j < nkb && !aborted; ++j) {
        // P_j is in TMEM: S_j and bias_j have been read, P_{j-1} V_{j-1} awaited by the softmax
        if (!tc::mbar_wait(&pready[g * 2 + (j & 1)], (j >> 1) & 1, p.status, aborted)) break;
        tc::tc_fence_after();
        // O += P_j V_j (P_j over S_j; V^T of block j landed before S_j was signalled)
        const uint32_t vs = tc::smem_u32(v_of(j));
#pragma unroll
        for (int kk = 0; kk < KB / 16; ++kk)
          tc::mma_bf16_ts(tbase + o_col, tbase + s_col + (j & 1) * KB + kk * 8, tc::smem_desc(vs + kk * 32, 512, tc::kSW64),
                          IDESC, j > 0 || kk > 0);
        tc::mma_commit(&pvbar[g * 2 + (j & 1)]);
        // S_{j+2} over P_j: MMAs issued by one thread run in issue order, so its accumulator
        // writes follow P_j V_j's read of P_j
        if (j + 2 < nkb) issue_s(j + 2);
        if (aborted) break;
        // then block j+4 (two blocks before its S), or an epilogue tile: K and bias into the slots
        // of block j (S_j and the softmax of block j are done), V^T into the slot of block j-2
        // (S_j complete means P_{j-2} V_{j-2}, issued before it, is done)
        if (j + RING < nkb) {
          issue_load(j + RING);
        } else if (j + RING == nkb) {
          tc::prefetch_tmap(&tmR);
          tc::prefetch_tmap(&tmW);
          tc::prefetch_tmap(&tmO);
          tc::mbar_expect_tx(&rbar[g], TILE * D * 2);
          tc::tma_load_3d(resid, &tmR, &rbar[g], g * D, rc1, rc2);
          rload = true;
        } else if (j + RING == nkb + 1) {
          // W_o[:, 32g .. 32g+31] (K-major 128 x 32, 64B swizzle)
          tc::mbar_expect_tx(&wbar[g], 8192);
          tc::tma_load_2d(wstage, &tmW, &wbar[g], g * D, 0);
          wload = true;
        }
      }
      // this head's share of the output projection, D_g = O_g W_o[:, 32g .. 32g+31]^T, into the
      // head's own columns (its S, O, Q and P are dead once O_g is staged)
      if (!aborted && tc::mbar_wait(&ostaged[g], 0, p.status, aborted) &&
          tc::mbar_wait(&wbar[g], 0, p.status, aborted)) {
        tc::tc_fence_after();
        const uint32_t os = tc::smem_u32(ostage), ws = tc::smem_u32(wstage);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::mma_bf16(tbase + s_col, tc::smem_desc(os + kk * 32, 512, tc::kSW64),
                       tc::smem_desc(ws + kk * 32, 512, tc::kSW64), IDESC_OUT, kk > 0);
        tc::mma_commit(&outbar[g]);
      }
    }
  } else {
    const uint4* grow = reinterpret_cast<const uint4*>(p.g + (bh * p.qp + q0 + (t & ~31)) * D) + (t & 31);
    for (int j = 0; j < nkb; ++j) {
      // S_j is written and block j (its bias tile) has landed
      tc::mbar_wait(&sbar[g * 2 + (j & 1)], (j >> 1) & 1, p.status, aborted);
      tc::tc_fence_after();
      // P_{j-1}, stored at the end of the previous block, is signalled only now: its store
      // latency overlaps the wait above
      if (j >= 1) {
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&pready[g * 2 + ((j - 1) & 1)]);
      }
      if (j == nkb - 2) asm volatile("prefetch.global.L2 [%0];" ::"l"(grow));   // the gate row for the epilogue
      float sv[KB];
      float corr = 1.f;
      uint32_t pk[KB / 2];
      float ps0 = 0.f, ps1 = 0.f, ps2 = 0.f, ps3 = 0.f;
      bool packed = false;   // pk and the sums already hold this block's values
      const uint8_t* brow = bt_of(j);
      const uint32_t vb = kbits[j];
      // logit2 of key e: S scale + bias' (bias' = log2(e) bias), -inf where the key is excluded
      auto load_logits = [&]() {
        tc::tmem_ld32(lane_addr + s_col + (j & 1) * KB, sv);
#pragma unroll
        for (int c = 0; c < KB / 8; ++c) {
          const uint4 bb = *reinterpret_cast<const uint4*>(brow + tc::sw64_off(t, c));
          const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const int e = 8 * c + 2 * e2;
            add_bf16x2(bw[e2], sv[e], sv[e + 1]);   // S (already in log2 units) + bias'
          }
        }
        if (vb != ~0u) {   // masked or padding keys in this block
#pragma unroll
          for (int e = 0; e < KB; ++e)
            if (!((vb >> e) & 1)) sv[e] = -INFINITY;
        }
      };
      if (!uniform) {
        load_logits();
        // tcgen05.ld is warp-collective: every branch that reloads S below is warp-uniform
        float ma = -INFINITY, mb = -INFINITY;
        if (j == 0) {
          // first block: its max first
#pragma unroll
          for (int e = 0; e < KB; e += 4) {
            ma = tc::fmax3(ma, sv[e], sv[e + 1]);
            mb = tc::fmax3(mb, sv[e + 2], sv[e + 3]);
          }
          const float mx = fmaxf(ma, mb);
          const float mu = mx == -INFINITY ? 0.f : mx;
#pragma unroll
          for (int e = 0; e < KB; ++e) sv[e] = ex2(sv[e] - mu);
          m_run = mx;
        } else {
          // exponentials against the running max (+inf while no key has counted: all 0)
          const float m_spec = m_run == -INFINITY ? INFINITY : m_run;
#pragma unroll
          for (int e = 0; e < KB; e += 4) {
            float d0 = sv[e], d1 = sv[e + 1], d2 = sv[e + 2], d3 = sv[e + 3];
            add_f32x2(d0, d1, -m_spec, -m_spec);
            add_f32x2(d2, d3, -m_spec, -m_spec);
            sv[e] = ex2(d0);
            sv[e + 1] = ex2(d1);
            sv[e + 2] = ex2(d2);
            sv[e + 3] = ex2(d3);
            // packed and summed in the same pass (redone below in the rare case the max moves)
            add_f32x2(ps0, ps1, sv[e], sv[e + 1]);
            add_f32x2(ps2, ps3, sv[e + 2], sv[e + 3]);
            pk[e >> 1] = pack_bf2(sv[e], sv[e + 1]);
            pk[(e >> 1) + 1] = pack_bf2(sv[e + 2], sv[e + 3]);
          }
          packed = true;
          // No exponential exceeds the block's sum: while that sum stays <= 2^8 the running max
          // stands, and no per-key max is needed.  A larger (or infinite, or NaN) sum, or a row
          // with no key counted yet, takes the exact path: the block max from S and the bias,
          // the running max moved when the block max exceeds it by more than 2^8, values redone.
          const float tot = (ps0 + ps1) + (ps2 + ps3);
          const bool exact = !(tot <= kSumLimit) || m_run == -INFINITY;
          if (__any_sync(0xffffffffu, exact)) {   // warp-uniform: tcgen05.ld is warp-collective
            load_logits();
#pragma unroll
            for (int e = 0; e < KB; e += 4) {
              ma = tc::fmax3(ma, sv[e], sv[e + 1]);
              mb = tc::fmax3(mb, sv[e + 2], sv[e + 3]);
            }
            const float mx = fmaxf(ma, mb);
            const bool moves = mx > m_run + kRescale;   // also the first finite block after -inf
            const float mr = moves ? mx : (m_run == -INFINITY ? 0.f : m_run);
#pragma unroll
            for (int e = 0; e < KB; ++e) sv[e] = ex2(sv[e] - mr);
            if (moves) {
              corr = ex2(m_run - mx);
              m_run = mx;
            }
            packed = false;
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < KB; ++e) sv[e] = ((int64_t)j * KB + e < p.nq) ? 1.f : 0.f;
      }
      // ---- P as bf16 pairs; the row sum (unless the exponential pass made them) ----
      if (!packed) {
        ps0 = ps1 = ps2 = ps3 = 0.f;
#pragma unroll
        for (int e = 0; e < KB; e += 4) {
          add_f32x2(ps0, ps1, sv[e], sv[e + 1]);
          add_f32x2(ps2, ps3, sv[e + 2], sv[e + 3]);
          pk[e >> 1] = pack_bf2(sv[e], sv[e + 1]);
          pk[(e >> 1) + 1] = pack_bf2(sv[e + 2], sv[e + 3]);
        }
      }
      l = l * corr + ((ps0 + ps1) + (ps2 + ps3));
      // P_j over S_j (S_j complete means P_{j-2} V_{j-2}, the last reader of this buffer, is done);
      // O is rescaled only after P_{j-1} V_{j-1}
      if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
        tc::mbar_wait(&pvbar[g * 2 + ((j - 1) & 1)], ((j - 1) >> 1) & 1, p.status, aborted);
        tc::tc_fence_after();
        float ov[D];
        tc::tmem_ld32(lane_addr + o_col, ov);
        uint32_t r[D];
#pragma unroll
        for (int e = 0; e < D; ++e) r[e] = __float_as_uint(ov[e] * corr);
        tc::tmem_st32(lane_addr + o_col, r);
      }
      tc::tmem_st16(lane_addr + s_col + (j & 1) * KB, pk);
    }
    tc::tmem_wait_st();
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&pready[g * 2 + ((nkb - 1) & 1)]);

    // ---- normalise, gate, stage O_h (K-major 128 x 32, 64B swizzle) in the last bias slot ----
    uint4 graw[D / 8];
#pragma unroll
    for (int c = 0; c < D / 8; ++c) graw[c] = __ldg(grow + 32 * c);
    // the last two P V (S_{nkb-1} complete only means P V up to block nkb-3 is)
    tc::mbar_wait(&pvbar[g * 2 + ((nkb - 2) & 1)], ((nkb - 2) >> 1) & 1, p.status, aborted);
    tc::mbar_wait(&pvbar[g * 2 + ((nkb - 1) & 1)], ((nkb - 1) >> 1) & 1, p.status, aborted);
    tc::tc_fence_after();
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    {
      float ov[D];
      tc::tmem_ld32(lane_addr + o_col, ov);
#pragma unroll
      for (int cc = 0; cc < D / 8; ++cc) {
        const uint4 gg = graw[cc];
        const int d = cc * 8;
        *reinterpret_cast<uint4*>(ostage + tc::sw64_off(t, cc)) =
            make_uint4(pack_bf2(ov[d] * inv * bf_lo(gg.x), ov[d + 1] * inv * bf_hi(gg.x)),
                       pack_bf2(ov[d + 2] * inv * bf_lo(gg.y), ov[d + 3] * inv * bf_hi(gg.y)),
                       pack_bf2(ov[d + 4] * inv * bf_lo(gg.z), ov[d + 5] * inv * bf_hi(gg.z)),
                       pack_bf2(ov[d + 6] * inv * bf_lo(gg.w), ov[d + 7] * inv * bf_hi(gg.w)));
      }
    }
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&ostaged[g]);

    // ---- query q, output channels 32g .. 32g+31: the four heads' shares + residual, in place ----
    for (int h = 0; h < H; ++h) tc::mbar_wait(&outbar[h], 0, p.status, aborted);
    tc::tc_fence_after();
    tc::mbar_wait(&rbar[g], 0, p.status, aborted);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {   // 16 channels at a time
      float ov[16];
      tc::tmem_ld16(lane_addr + g * D + hf * 16, ov);
#pragma unroll
      for (int h = 1; h < H; ++h) {
        float oh[16];
        tc::tmem_ld16(lane_addr + h * 128 + g * D + hf * 16, oh);
#pragma unroll
        for (int e = 0; e < 16; e += 2) add_f32x2(ov[e], ov[e + 1], oh[e], oh[e + 1]);
      }
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint4* zp = reinterpret_cast<uint4*>(resid + tc::sw64_off(t, 2 * hf + c2));
        const uint4 zz = *zp;
        const int d = c2 * 8;
        *zp = make_uint4(pack_bf2(bf_lo(zz.x) + ov[d], bf_hi(zz.x) + ov[d + 1]),
                         pack_bf2(bf_lo(zz.y) + ov[d + 2], bf_hi(zz.y) + ov[d + 3]),
                         pack_bf2(bf_lo(zz.z) + ov[d + 4], bf_hi(zz.z) + ov[d + 5]),
                         pack_bf2(bf_lo(zz.w) + ov[d + 6], bf_hi(zz.w) + ov[d + 7]));
      }
    }
    tc::fence_proxy_async();
    wg_sync(g);
    if (t == 0) {
      tc::tma_store_3d(&tmO, resid, g * D, rc1, rc2);   // rows beyond N are clipped
      tc::bulk_commit();
      tc::bulk_wait_read0();   // the tile must stay until the store has read it
    }
  }
  tc::tc_fence_before();
  if (__syncthreads_or(aborted)) {   // abort path: drain each head's loads and MMAs
    if (issuer && lane == 0) {
      tc::drain_ring(&lbar[g * RING], RING, loads, p.status);
      if (rload) tc::mbar_wait_drain(&rbar[g], 0, p.status);
      if (wload) tc::mbar_wait_drain(&wbar[g], 0, p.status);
      tc::drain_mma(&drainb[g], p.status);
    }
    __syncthreads();
  }
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

template <typename K>
int set_smem(K kernel, int bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (!done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return SF_ERR_CUDA;
    }
    done[dev & 63] = true;
  }
  return SF_OK;
}


}  // namespace

int64_t triatt_query_pitch(int64_t nq) { return (nq + 127) / 128 * 128; }

int triatt_bias_tc(const bf16* z, int64_t rows, int64_t n, const float* ln_w, const bf16* w_bias, bf16* bias,
                   int64_t ldb, cudaStream_t stream) {
  // the pair-logit kernel: scale-only LN in place (rounded to bf16), M128 N16 K128 MMA, row-major stores
  return pair_rows_bias_tc(z, rows, n, ln_w, w_bias, H, kBiasScale, bias, ldb, stream);
}

int triatt_project_tc(const bf16* z, int64_t rows, int64_t cols, int transpose, int compute_bias, const float* ln_w,
                      const bf16* w_qkvg, const bf16* w_bias, bf16* q, bf16* k, bf16* vt, bf16* g, bf16* bias,
                      cudaStream_t stream) {
  if (rows == 0 || cols == 0) return SF_OK;
  const int64_t nb = transpose ? cols : rows, nq = transpose ? rows : cols;
  SF_REQUIRE(nb <= 65535 && nq <= 65535, "triatt_project: block [%lld][%lld] too large", (long long)rows,
             (long long)cols);
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  SF_REQUIRE(((reinterpret_cast<uintptr_t>(ln_w) | reinterpret_cast<uintptr_t>(w_qkvg) |
               reinterpret_cast<uintptr_t>(w_bias)) & 15) == 0,
             "triatt_project: weights must be 16-byte aligned");
  const int64_t qp = triatt_query_pitch(nq);
  SF_REQUIRE(nb * H * qp < (int64_t(1) << 31), "triatt_project: %lld attention rows x %lld queries exceed the TMA range",
             (long long)nb, (long long)qp);
  static bool attr[64] = {false};
  SF_TRY(set_smem(k_triatt_project_tc, SMEM_PROJ, attr));
  CUtensorMap mz, mk, mv;
  SF_TRY(make_pair_tmap(&mz, z, rows, cols, transpose != 0));
  // epilogue stores: K [nb*H*qp][32] as 32 queries x 32 channels (64B swizzle), V^T [nb*H*32][qp] as
  // 32 channels x 64 queries (128B swizzle); Q and G as 2 KB groups by plain bulk copies
  SF_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(g)) & 15) == 0,
             "triatt_project: q and g must be 16-byte aligned");
  SF_TRY(make_2d_tmap(&mk, k, D, nb * H * qp, D, 32, 64));
  SF_TRY(make_2d_tmap(&mv, vt, qp, nb * H * D, 64, D, 128));
  AttProjParams pp{q, g, ln_w, w_bias, bias, nb, nq, qp, transpose, compute_bias, status};
  const int64_t ntiles = nb * (qp / TILE);
  const int grid = (int)(ntiles < num_sms() ? ntiles : num_sms());
  launch_pdl(k_triatt_project_tc, dim3(grid), dim3(PJ_THREADS), SMEM_PROJ, stream, mz, mk, mv, w_qkvg, pp);
  count_launch();
  return check_launch("triatt_project_tc");
}

// z block [rows][cols][128] seen as tiles of 32 channels x 128 positions along a row
// (starting node) or along a column (ending node), 64B swizzle.
static int make_resid_tmap(CUtensorMap* map, const bf16* base, int64_t rows, int64_t cols, bool column_tile) {
  auto encode = tensor_map_encoder();
  if (!encode) return SF_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) {
    set_error("triatt_core: z %p is not 16-byte aligned", (const void*)base);
    return SF_ERR_ARG;
  }
  cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)(cols * C * 2)};
  cuuint32_t box[3] = {(cuuint32_t)D, column_tile ? 1u : (cuuint32_t)TILE, column_tile ? (cuuint32_t)TILE : 1u};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for the attention residual", (int)r);
    return SF_ERR_CUDA;
  }
  return SF_OK;
}

int triatt_core_tc(const bf16* q, const bf16* k, const bf16* vt, const bf16* g, const bf16* bias, const bf16* w_out,
                   const uint8_t* mask, const bf16* z, bf16* z_out, int64_t rows, int64_t cols, int transpose,
                   int64_t batch_offset, cudaStream_t stream) {
  if (rows == 0 || cols == 0) return SF_OK;
  const int64_t nb = transpose ? cols : rows, nq = transpose ? rows : cols;
  const int64_t qp = triatt_query_pitch(nq);
  SF_REQUIRE(nb <= 65535 && qp <= MAX_QP, "triatt_core: block [%lld][%lld] too large", (long long)rows,
             (long long)cols);
  SF_REQUIRE(nb * H * qp < (int64_t(1) << 31), "triatt_core: %lld attention rows x %lld keys exceed the TMA range",
             (long long)nb, (long long)qp);
  uint32_t* status = device_status_ptr();
  if (!status) return SF_ERR_CUDA;
  static bool attr[64] = {false};
  SF_TRY(set_smem(k_triatt_core_tc, SMEM_CORE, attr));
  // K [nb*H*qp][32] (32-row boxes); V^T [nb*H*32][qp] (32 keys x 32); 64B swizzle
  SF_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0, "triatt_core: q must be 16-byte aligned");
  CUtensorMap mk, mv;
  SF_TRY(make_2d_tmap(&mk, k, D, nb * H * qp, D, KB, 64));
  SF_TRY(make_2d_tmap(&mv, vt, qp, nb * H * D, KB, D, 64));
  // bias [qp][H][qp]: tiles of 32 keys x 1 head x 128 queries (64B swizzle); keys >= N read as zero
  CUtensorMap mb;
  {
    auto encode = tensor_map_encoder();
    if (!encode) return SF_ERR_CUDA;
    if ((reinterpret_cast<uintptr_t>(bias) & 15) != 0) {
      set_error("triatt_core: bias %p is not 16-byte aligned", (const void*)bias);
      return SF_ERR_ARG;
    }
    cuuint64_t dims[3] = {(cuuint64_t)nq, (cuuint64_t)H, (cuuint64_t)qp};
    cuuint64_t strides[2] = {(cuuint64_t)qp * 2, (cuuint64_t)(H * qp * 2)};
    cuuint32_t box[3] = {(cuuint32_t)KB, 1, (cuuint32_t)TILE};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16*>(bias), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled failed (%d) for the attention bias", (int)r);
      return SF_ERR_CUDA;
    }
  }
  // W_o [128 out][128 in]: 32 input channels x 128 rows per head (64B swizzle)
  CUtensorMap mw, mr, mo;
  SF_TRY(make_2d_tmap(&mw, w_out, C, C, D, C, 64));
  // residual in / out: 32 channels x 128 queries of the z block (64B swizzle)
  SF_TRY(make_resid_tmap(&mr, z, rows, cols, transpose != 0));
  SF_TRY(make_resid_tmap(&mo, z_out, rows, cols, transpose != 0));
  AttCoreParams cp{q, g, bias, w_out, mask, z, z_out, cols, nq, qp, batch_offset, transpose,
                   (1.0f / sqrtf((float)D)) * kLog2e, status};
  dim3 cgrid((unsigned)(qp / TILE), (unsigned)nb);
  launch_pdl(k_triatt_core_tc, cgrid, dim3(CORE_THREADS), SMEM_CORE, stream, mk, mv, mb, mw, mr, mo, cp);
  count_launch();
  return check_launch("triatt_core_tc");
}

// Buffer sizes of one attention call: Q, K, Vt, G [nb][H][qp][32] (Q and G in 32-query groups),
// bias [qp][H][qp].
size_t triatt_tc_workspace(int64_t n) {
  const int64_t qp = triatt_query_pitch(n);
  const size_t per = (size_t)n * H * qp * D * 2;
  size_t used = 0;
  for (int i = 0; i < 3; ++i) used = align_up(used, 256) + per;
  used = align_up(used, 256) + (size_t)n * qp * C * 2;
  used = align_up(used, 256) + (size_t)qp * H * qp * 2;
  return used;
}

// The whole op on one device (the z block is the full [n][n] pair tensor).
int triatt_tc(const bf16* z, const uint8_t* mask, int64_t n, int transpose, const float* ln_w, const bf16* w_qkvg,
              const bf16* w_bias, const bf16* w_out, bf16* z_out, void* ws_p, size_t ws_bytes, cudaStream_t stream) {
  if (n == 0) return SF_OK;
  if (ws_bytes < triatt_tc_workspace(n)) {
    set_error("sf_tri_attention: workspace %zu < %zu", ws_bytes, triatt_tc_workspace(n));
    return SF_ERR_WORKSPACE;
  }
  const int64_t qp = triatt_query_pitch(n);
  Workspace ws(ws_p, ws_bytes);
  bf16* q = ws.take<bf16>((size_t)n * H * qp * D);
  bf16* k = ws.take<bf16>((size_t)n * H * qp * D);
  bf16* vt = ws.take<bf16>((size_t)n * H * qp * D);
  bf16* g = ws.take<bf16>((size_t)n * qp * C);
  bf16* bias = ws.take<bf16>((size_t)qp * H * qp);
  SF_TRY(triatt_project_tc(z, n, n, transpose, 1, ln_w, w_qkvg, w_bias, q, k, vt, g, bias, stream));
  return triatt_core_tc(q, k, vt, g, bias, w_out, mask, z, z_out, n, n, transpose, 0, stream);
}

}  // namespace sf
