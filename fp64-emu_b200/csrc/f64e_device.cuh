// Device-side building blocks shared by the fp64-emu B200 kernels: sizing
// arithmetic, residue helpers, bounded mbarrier waits, TMA and tcgen05 PTX.
// Target: sm_100a only.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "f64e_params.h"

namespace f64e {

// ----------------------------------------------------------------- status --
// Every spin-wait in these kernels is bounded.  A wait that runs out records
// its site in the status word (first writer wins) and the kernel unwinds; the
// host reads the word with f64e_status().
enum : int {
  kWaitFull = 1,      // GEMM consumer waiting for a TMA stage
  kWaitEmpty = 2,     // GEMM producer waiting for a free stage
  kWaitAccFull = 3,   // epilogue waiting for an accumulator
  kWaitAccEmpty = 4,  // MMA issuer waiting for the epilogue to drain TMEM
  kWaitDrain = 5,     // teardown waiting for in-flight copies / MMAs
  kWaitSelfTest = 9,  // f64e_wait_selftest: a barrier nothing arrives at
  // Bounds sites, recorded only by a library built with F64E_DEBUG_BOUNDS:
  // the access lay outside the range its launcher gave, and was skipped.
  kBoundsExtractLoad = 16,   // extraction: operand read
  kBoundsExtractStore = 17,  // extraction: plane write
  kBoundsGemmStore = 18,     // GEMM epilogue: residue or correction write
  kBoundsReconLoad = 19,     // reconstruction: residue or correction read
  kBoundsReconStore = 20,    // reconstruction: output write
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Debug bounds check: true when [p, p + bytes) lies inside s.  A library built
// with F64E_DEBUG_BOUNDS records `site` in the status word on a miss (first
// writer wins) and the caller skips the access; no trap, so the context stays
// usable.  In the release build the check compiles away.
__device__ __forceinline__ bool in_span(const void* p, size_t bytes, const Span& s, int* status, int site) {
#ifdef F64E_DEBUG_BOUNDS
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if (a >= s.lo && a + bytes <= s.hi && a + bytes >= a) return true;
  record_status(status, site);
  return false;
#else
  (void)p; (void)bytes; (void)s; (void)status; (void)site;
  return true;
#endif
}

// ----------------------------------------------------------------- sizing --
// Cauchy-Schwarz widening from the two operand maxima of lg = log2 of the
// scaled row/column 2-norms (reference: fp64_emu.cu:212-223).  Every thread
// that needs the gain recomputes it from the same two floats, so the shifts
// never have to be rewritten in place.
struct Gain {
  int g;         // extra shift folded into every row / column shift
  int bits_eff;  // operand width actually used
};

__device__ __forceinline__ Gain pick_gain(float maxA, float maxB, float log2M, int bits) {
  const float need = maxA + maxB + 0.5f;
  int g = 0;
  if (isfinite(need)) g = (int)floorf((log2M - 1.0f - need) * 0.5f);
  g = min(g, 53 - bits);
  int be = bits + g;
  if (be < 16) be = 16;
  Gain r;
  r.g = be - bits;
  r.bits_eff = be;
  return r;
}

// --------------------------------------------------------------- residues --
// Residue of v in [0, p) for 0 <= v < 2^30 with m = floor(2^32 / p): the
// quotient estimate umulhi(v, m) falls short by at most one, since
// v * (2^32/p - m) / 2^32 < v / 2^32 < 1.
__device__ __forceinline__ uint32_t mod_small(uint32_t v, uint32_t p, uint32_t m) {
  const uint32_t q = __umulhi(v, m);
  uint32_t r = v - q * p;
  if (r >= p) r -= p;
  return r;
}

// Balanced form of a residue r in [0, p]: the representative in
// [-floor(p/2), floor((p-1)/2)] (r == p maps to 0).
__device__ __forceinline__ int balance(uint32_t r, uint32_t p) {
  int rb = (int)r;
  if (rb > (int)(p - 1) / 2) rb -= (int)p;
  return rb;
}

// Balanced residue of a signed 32-bit integer v (|v| < 2^31): v + off is
// non-negative and below 2^32 with off the largest multiple of p not above
// 2^31, so the quotient estimate umulhi(xu, m) is short by at most one.
__device__ __forceinline__ int bal_mod_s32(int v, uint32_t p, uint32_t m, uint32_t off) {
  const uint32_t xu = (uint32_t)v + off;
  const uint32_t q = __umulhi(xu, m);
  uint32_t r = xu - q * p;
  if (r >= p) r -= p;
  return balance(r, p);
}

// ----------------------------------------------------------------- mbarrier --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, "
      "p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `parity` to complete.  Returns false (and
// records `site`) once `limit_ns` of wall time has passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns, int* status,
                                          int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    // Back off between polls: a warp spinning here would otherwise take issue
    // slots from the kernels (extraction, reconstruction) that run beside the
    // persistent GEMM on the same SM.
    __nanosleep(128);
    if (globaltimer_ns() - t0 > limit_ns) {
      record_status(status, site);
      return false;
    }
  }
}

// Limit of the teardown waits (copies and MMAs a CTA issued, before it frees
// TMEM or exits).  Never shorter than kDrainFloorNs, whatever the caller's
// wait limit: a short limit may end a main-loop wait on a device that is only
// slow (time-sliced with another context), and the in-flight work must still
// land before its shared memory and TMEM are released.  Only a device that has
// stopped making progress runs this out.
constexpr uint64_t kDrainFloorNs = 4000000000ull;  // 4 s

__device__ __forceinline__ uint64_t drain_limit(uint64_t limit_ns) {
  return limit_ns > kDrainFloorNs ? limit_ns : kDrainFloorNs;
}

// -------------------------------------------------------------------- TMA --
// Tiled 3-D load, no multicast: box lands in this CTA's shared memory and
// completes `bytes` on the CTA's own mbarrier.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05 --
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
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed (non-multicast form).
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, s8 x s8 -> s32, both K-major.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row core groups 1024 bytes apart
// (stride byte offset), leading byte offset unused (1), descriptor version 1,
// layout type 2 = SWIZZLE_128B.  The tile base must be 1024-byte aligned;
// stepping K inside the 128-byte row adds the byte offset to the start
// address field.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::i8: D = S32 (bits 4-5 = 2), A and B signed
// (bits 7-9 and 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at
// bits 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 32 lanes x 32 columns of 32-bit TMEM words: thread i of the warp receives
// lane (base lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------- CTA-pair (2-SM) --
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of this CTA's shared variable at `smem_addr` in CTA `rank` of the
// cluster (shared::cluster window).
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Arrive + expect_tx on a barrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr),
               "r"(bytes)
               : "memory");
}
// complete-tx of `bytes` on this CTA's mbarrier without a copy: stands in for
// bytes a copy that was never issued would have delivered (teardown only).
__device__ __forceinline__ void mbar_complete_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Store to a 32-bit shared variable of another CTA of the cluster (its
// shared::cluster address); ordered for the reader by a cluster barrier.
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
// Tiled 3-D load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar_cluster_addr)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrive once on the barrier at this shared offset in every CTA of `mask`
// when all prior MMAs of the pair issued by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both]^T, M = 256.
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .b32 rx;\n .reg .pred px;\n elect.sync rx|px, %1;\n selp.u32 %0, 1, 0, px;\n}"
      : "=r"(pred)
      : "r"(0xFFFFFFFFu));
  return pred != 0;
}

}  // namespace f64e
