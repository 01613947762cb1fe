// Blackwell (sm_100a) primitives written as inline PTX: mbarriers with bounded
// waits, TMA tile loads (no multicast), tcgen05 TMEM allocation, UMMA shared
// memory / instruction descriptors, tcgen05.mma issue and commit, tcgen05.ld.
//
// Descriptor bit layouts (PTX ISA, tcgen05 matrix descriptors):
//   smem descriptor: [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4,
//                    [46,48) version = 1, [49,52) base offset, [61,64) layout
//                    (2 = 128B swizzle, 4 = 64B swizzle, 6 = 32B swizzle).
//   instr descriptor (kind::f16): [4,6) D format (1 = f32), [7,10) A format
//                    (1 = bf16), [10,13) B format, [15] A MN-major, [16] B
//                    MN-major, [17,23) N>>3, [24,29) M>>4.
// K-major operands use the canonical swizzled layout: rows of one swizzle
// atom width (128 B or 64 B), 8-row groups SBO bytes apart, and the 16-byte
// chunk c of row r stored at chunk (c ^ f(r)), f(r) = r & 7 for 128B swizzle
// and (r >> 1) & 3 for 64B swizzle.  Atoms start on 1024-byte boundaries.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "sf_common.cuh"

namespace sf {
namespace tc {

// Every wait gives up after this many try_wait polls (each poll may suspend
// the thread for a hardware-defined interval), records SF_ERR_TIMEOUT in the
// caller's status word and lets the kernel run to its end.
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ----------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// A zero suspend-time hint: on this part a try_wait on an already completed phase
// returns in about 115 cycles with it and about 290 without it (measured), and the
// producer/consumer handshakes here poll phases that are usually complete.
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(0u)
      : "memory");
  return ok != 0;
}
// Bounded wait.  On timeout sets *status (first error wins) and returns false;
// once this thread has timed out (`aborted`), later waits poll only once so the
// kernel still reaches its end in bounded time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status, bool& aborted,
                                          uint32_t wait_limit = kWaitLimit) {
  const uint32_t limit = aborted ? 1u : wait_limit;
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try(bar, parity)) return true;
  aborted = true;
  if (status) atomicCAS(status, 0u, (uint32_t)SF_ERR_TIMEOUT);
  return false;
}

// ---- the abort path -------------------------------------------------------------
// Once a wait has given up, the data or the buffer it waited for may never arrive,
// so a thread that issues asynchronous work (TMA loads, tcgen05.mma) stops issuing
// at its first failed wait.  Work it issued before that may still be in flight, and
// other threads may have given up without waiting for it; so before TMEM is freed
// and the CTA exits, every issuing thread drains what it issued whenever any thread
// of the CTA gave up (the kernels test that with __syncthreads_or over `aborted`):
//  * tcgen05.mma: one more tcgen05.commit, on the thread's own drain barrier (count
//    1, otherwise unused), and a wait for it: a commit tracks every earlier MMA of
//    the thread;
//  * TMA loads into a ring of `stages` slots: a wait for the last phase issued into
//    each slot (one load per slot can be outstanding, as each refill waited for the
//    slot to be freed first).
// The drain waits have their own bound and do not depend on earlier timeouts; if
// one gives up as well, the kernel still ends (its status word says so).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, uint32_t* status) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try(bar, parity)) return true;
  if (status) atomicCAS(status, 0u, (uint32_t)SF_ERR_TIMEOUT);
  return false;
}

// ---- programmatic dependent launch ------------------------------------------------
// A kernel launched with launch_pdl may start while the kernel before it on the stream is
// still running: it sets up (TMEM, barriers, weights in shared memory) and then waits here
// until the previous grid has completed and its memory is visible, before it reads any
// activation or writes any global memory.  (Without the launch attribute this is a no-op.)
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel on the stream launch once every CTA of this grid has passed here.
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- fences --------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- TMA tiled loads (never multicast) -------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// TMA tiled store shared -> global (bulk async group of the issuing thread).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
// Plain (untiled) bulk copy of `bytes` from shared memory to global memory, in the current bulk
// group; both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the issuing thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until at most the issuing thread's most recent bulk store group is still reading.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// Waits until the issuing thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- TMEM allocation (one full warp executes these) ---------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- descriptors -----------------------------------------------------------------
enum Swizzle : uint64_t { kSW128 = 2, kSW64 = 4, kSW32 = 6 };

// K-major operand in the canonical swizzled layout: `sbo_bytes` apart per 8-row
// group; LBO is unused for swizzled K-major layouts and set to 16 bytes.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t sbo_bytes, Swizzle sw) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(1u) << 16;                          // LBO = 16 B
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;  // SBO
  d |= (uint64_t)1 << 46;                             // version
  d |= (uint64_t)sw << 61;
  return d;
}

// Descriptor of an M/N-major operand (M or N contiguous): 128-byte rows of one
// swizzle atom hold consecutive M/N elements, 8 K-rows per atom; lbo_bytes =
// stride between atoms along M/N, sbo_bytes = stride between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, Swizzle sw) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;  // LBO
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;  // SBO
  d |= (uint64_t)1 << 46;                             // version
  d |= (uint64_t)sw << 61;
  return d;
}

// bf16 x bf16 -> fp32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4)                       // D = f32
         | (1u << 7)                     // A = bf16
         | (1u << 10)                    // B = bf16
         | ((uint32_t)(n >> 3) << 17)    // N
         | ((uint32_t)(m >> 4) << 24);   // M
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T: A (M=128 rows on the 128 lanes, K packed two
// bf16 per 32-bit column, the lower half holding the even K index) read from TMEM.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}
// Arrive on `bar` once all tcgen05.mma previously issued by this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Abort path: waits until every tcgen05.mma this thread issued has completed.
// `drain_bar` is the thread's own barrier (count 1), used once.
__device__ __forceinline__ void drain_mma(uint64_t* drain_bar, uint32_t* status) {
  mma_commit(drain_bar);
  mbar_wait_drain(drain_bar, 0, status);
}
// Abort path: waits for the last of `issued` TMA loads made in order q = 0, 1, ...
// into slot q % stages of a ring whose landing barriers are full[0..stages) (load q
// completes phase q / stages of its slot's barrier).
__device__ __forceinline__ void drain_ring(uint64_t* full, uint32_t stages, uint32_t issued, uint32_t* status) {
  const uint32_t first = issued > stages ? issued - stages : 0u;
  for (uint32_t q = first; q < issued; ++q) mbar_wait_drain(&full[q % stages], (q / stages) & 1u, status);
}

// ---- TMEM -> registers: lane = row (warp w reads lanes 32*(w%4)..+31) -----------------
// The wait is in the same asm statement so no instruction can read the
// destination registers before the load has landed.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  __syncwarp();   // .sync.aligned: the whole warp must arrive converged
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 consecutive columns, one round trip.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 64 consecutive columns, one round trip.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- registers -> TMEM: lane = row, 16 consecutive 32-bit columns -----------------------
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  __syncwarp();
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
               : "memory");
}
// Waits until this thread's tcgen05.st have been performed.
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Three-input maximum (sm_100 max.f32 form).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// ---- swizzled shared-memory addressing of a K-major bf16 tile -----------------------
// Byte offset of 16-byte chunk `c` (8 bf16 along K) of row `r` inside one
// 128B-swizzle atom column (rows of 128 bytes).
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }
// Same for a 64B-swizzle atom column (rows of 64 bytes, 4 chunks).
__device__ __forceinline__ uint32_t sw64_off(uint32_t r, uint32_t c) {
  return r * 64u + ((c ^ ((r >> 1) & 3u)) << 4);
}

}  // namespace tc
}  // namespace sf
