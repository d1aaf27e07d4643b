// Modular INT8 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// For every plane-batch slot s the kernel computes C_s = A_s * B_s^T exactly
// (s8 x s8 -> s32 in TMEM) and finishes each tile in the epilogue:
//   residue slots:    balanced residue mod p_t (one Barrett step) -> int8
//   correction slot:  raw int32; with corr_mode 1 the two correction products
//                     Ahi.Bq^T + Aq.Bhi^T are accumulated into one tile by
//                     running the K loop over both plane pairs (exact while
//                     2 K 127^2 < 2^31).
// Replaces residue_gemm_kernel / residue_gemm_tma_kernel / the cuBLAS engine
// of the reference (fp64_emu.cu:399-813, 1276-1342) with one engine; the
// epilogue is the reference's (fp64_emu.cu:604-656): balanced int8 residues
// plane-major, raw int32 correction products.
//
// Structure: persistent CTAs (one per SM), 192 threads.
//   warp 0      TMA producer: 128x128 (A) and 256x128 (B) boxes, 128-byte
//               swizzle, 4-stage ring, no multicast.
//   warp 1      TMEM owner; one elected thread issues tcgen05.mma
//               (M=128, N=256, K=32 per instruction) into one of two
//               256-column accumulators and commits stages / tiles.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, Barrett, store.
// Every mbarrier wait is bounded; a timeout records its site in the status
// word and the CTA unwinds: it drains its copies and MMAs (teardown waits of
// at least kDrainFloorNs, whatever the caller's limit), then frees TMEM.
// In the CTA pair, the leader's drain covers both CTAs' copies (its full
// barriers count the bytes of both) and every MMA (only the leader issues
// them); the final cluster barrier keeps the peer from freeing its TMEM
// columns or exiting before the leader's drain has ended.
#include <map>
#include <mutex>
#include <set>

#include "f64e_device.cuh"
#include "f64e_kernels.h"

namespace f64e {

namespace {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr uint32_t A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;  // two 256-column int32 accumulators
constexpr int GROUP_M = 16;          // m-tiles per raster group (L2 reuse of B panels)
constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
constexpr uint32_t IDESC = idesc_i8(BM, BN);

struct Tile {
  int m0, n0;
  int z0, z1;   // plane-batch coordinates of the first / second K half
  int nk;       // K blocks of this tile (2 * nkb for the fused correction slot)
  int kind;     // 0 residue, 1 correction (int32)
  int t;        // modulus index (residue tiles)
  int64_t out;  // element offset of the output slot
};

template <int TBM = BM, int TGM = GROUP_M>
__device__ __forceinline__ Tile decode_tile(int tile, const GemmArgs& g) {
  constexpr int GROUP_M_ = TGM;
  const int ntm = (g.M + TBM - 1) / TBM, ntn = (g.N + BN - 1) / BN;
  const int tps = ntm * ntn;
  const int ncs = g.corr_mode == 1 ? g.batch : (g.corr_mode == 2 ? 2 * g.batch : 0);
  const int slot = tile / tps, r = tile - slot * tps;
  const int gsz = GROUP_M_ * ntn;
  const int gi = r / gsz, o = r - gi * gsz;
  const int mf = gi * GROUP_M_, mh = min(GROUP_M_, ntm - mf);
  Tile T;
  T.m0 = (mf + o % mh) * TBM;
  T.n0 = (o / mh) * BN;
  const int64_t slot_elems = (int64_t)g.M * g.ldn;
  if (slot < ncs) {
    T.kind = 1;
    T.t = 0;
    if (g.corr_mode == 1) {
      const int b = slot;
      T.z0 = g.P * g.batch + b;
      T.z1 = (g.P + 1) * g.batch + b;
      T.nk = 2 * g.nkb;
      T.out = (int64_t)b * slot_elems;
    } else {
      const int h = slot / g.batch, b = slot - h * g.batch;
      T.z0 = T.z1 = (g.P + h) * g.batch + b;
      T.nk = g.nkb;
      T.out = (int64_t)(h * g.batch + b) * slot_elems;
    }
  } else {
    const int s = slot - ncs;  // s = t * batch + b
    T.kind = 0;
    T.t = s / g.batch;
    T.z0 = T.z1 = s;
    T.nk = g.nkb;
    T.out = (int64_t)s * slot_elems;
  }
  return T;
}

template <int TBM = BM>
__device__ __host__ __forceinline__ int total_tiles(const GemmArgs& g) {
  const int ntm = (g.M + TBM - 1) / TBM, ntn = (g.N + BN - 1) / BN;
  const int ncs = g.corr_mode == 1 ? g.batch : (g.corr_mode == 2 ? 2 * g.batch : 0);
  return ntm * ntn * (g.P * g.batch + ncs);
}

}  // namespace

__global__ void __launch_bounds__(NUM_THREADS, 1)
    residue_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmapA, const __grid_constant__ CUtensorMap tmapB,
                           const GemmArgs g, const ModTables T) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = total_tiles(g);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4 * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmapA);
    tma_prefetch_desc(&tmapB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t lim = g.wait_limit_ns;

  if (warp == 0) {
    // ---------------------------------------------------------- producer --
    if (elect_one()) {
      uint32_t j = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const Tile tl = decode_tile(tile, g);
        for (int kb = 0; kb < tl.nk; kb++, j++) {
          const uint32_t s = j % STAGES, ph = (j / STAGES) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, lim, g.status, kWaitEmpty) || *abort_flag) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const bool second = kb >= g.nkb;
          const int z = second ? tl.z1 : tl.z0;
          const int kx = (second ? kb - g.nkb : kb) * BK;
          mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
          tma_load_3d(sA + s * A_BYTES, &tmapA, kx, tl.m0, z, &full_bar[s]);
          tma_load_3d(sB + s * B_BYTES, &tmapB, kx, tl.n0, z, &full_bar[s]);
        }
      }
      // Drain: every copy this thread issued has landed before the CTA exits.
      const uint32_t first = j > (uint32_t)STAGES ? j - STAGES : 0;
      for (uint32_t jj = first; jj < j; jj++)
        mbar_wait(&full_bar[jj % STAGES], (jj / STAGES) & 1, drain_limit(lim), g.status, kWaitDrain);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer --
    if (elect_one()) {
      uint32_t j = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, it++) {
        const Tile tl = decode_tile(tile, g);
        const uint32_t a = it & 1, aph = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[a], aph ^ 1, lim, g.status, kWaitAccEmpty) || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BN;
        for (int kb = 0; kb < tl.nk; kb++, j++) {
          const uint32_t s = j % STAGES, ph = (j / STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, lim, g.status, kWaitFull) || *abort_flag) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * A_BYTES), b_addr = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 32; kk++)
            mma_i8(d_tmem, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32), IDESC,
                   (kb | kk) != 0);
          tc_commit(&empty_bar[s]);
        }
        if (ok) tc_commit(&acc_full[a]);
      }
      // Drain: all MMAs issued by this thread complete before TMEM is freed.
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, drain_limit(lim), g.status, kWaitDrain);
    }
  } else {
    // ----------------------------------------------------------- epilogue --
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_l = q * 32 + lane;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, it++) {
      const Tile tl = decode_tile(tile, g);
      const uint32_t a = it & 1, aph = (it >> 1) & 1;
      if (!mbar_wait(&acc_full[a], aph, lim, g.status, kWaitAccFull) || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = tl.m0 + row_l;
      const bool row_ok = row < g.M;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + a * BN;
      if (tl.kind == 0) {
        const uint32_t p = T.p[tl.t], md = T.mdiv[tl.t], off = T.off[tl.t];
        int8_t* orow = g.res + tl.out + (int64_t)row * g.ldn;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c * 32, v);
          tmem_wait_ld();
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; i++) {
            uint32_t x = 0;
#pragma unroll
            for (int e = 0; e < 4; e++)
              x |= (uint32_t)(uint8_t)(int8_t)bal_mod_s32((int)v[4 * i + e], p, md, off) << (8 * e);
            w[i] = x;
          }
          const int col = tl.n0 + c * 32;
          if (row_ok && col < g.ldn && in_span(orow + col, 16, g.res_span, g.status, kBoundsGemmStore))
            *reinterpret_cast<uint4*>(orow + col) = make_uint4(w[0], w[1], w[2], w[3]);
          if (row_ok && col + 16 < g.ldn &&
              in_span(orow + col + 16, 16, g.res_span, g.status, kBoundsGemmStore))
            *reinterpret_cast<uint4*>(orow + col + 16) = make_uint4(w[4], w[5], w[6], w[7]);
        }
      } else {
        int32_t* orow = g.corr + tl.out + (int64_t)row * g.ldn;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c * 32, v);
          tmem_wait_ld();
          const int col = tl.n0 + c * 32;
#pragma unroll
          for (int i = 0; i < 8; i++)
            if (row_ok && col + 4 * i < g.ldn &&
                in_span(orow + col + 4 * i, 16, g.corr_span, g.status, kBoundsGemmStore))
              *reinterpret_cast<uint4*>(orow + col + 4 * i) = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2],
                                                                         v[4 * i + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair form (cta_group::2): a cluster of two CTAs on two SMs computes a
// 256 x 256 tile.  CTA r loads A rows [m0 + 128 r, +128) and B rows
// [n0 + 128 r, +128) into its own shared memory (no multicast); both loads
// complete on the leader's (rank 0) full barrier; the leader's MMA thread
// issues M=256, N=256, K=32 tcgen05.mma over both CTAs' tiles and commits
// stage releases and finished accumulators to both CTAs at once.  Each
// CTA's epilogue drains its own 128 TMEM lanes and signals the leader.
// Per SM this halves the B-operand traffic through shared memory, which at
// the INT8 MMA rate is what limits the one-CTA 128 x 256 tile.
namespace {
constexpr int PBM = 256, PHALF = 128, PSTAGES = 6, PGROUP_M = 8;
constexpr uint32_t PA_BYTES = PHALF * BK, PB_BYTES = PHALF * BK, PSTAGE_BYTES = PA_BYTES + PB_BYTES;
constexpr size_t PSMEM_BYTES = 1024 + (size_t)PSTAGES * PSTAGE_BYTES + 256;
constexpr uint32_t PIDESC = idesc_i8(PBM, BN);
}  // namespace

__global__ void __launch_bounds__(NUM_THREADS, 1)
    residue_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmapA, const __grid_constant__ CUtensorMap tmapB,
                             const GemmArgs g, const ModTables T) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  uint8_t* sA = smem;
  uint8_t* sB = smem + PSTAGES * PA_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + PSTAGES * PSTAGE_BYTES);
  uint64_t* empty_bar = full_bar + PSTAGES;
  uint64_t* acc_full = empty_bar + PSTAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile uint32_t* peer_issued = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);  // leader: peer's stage count

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int ntiles = total_tiles<PBM>(g);

  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; s++) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * 4);  // one elected lane per epilogue warp of both CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *peer_issued = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmapA);
    tma_prefetch_desc(&tmapB);
  }
  __syncwarp();
  // TMEM of the pair: both CTAs' warp 1 allocate collectively, and only once
  // both CTAs are running (the first cluster barrier); the permit is given up
  // after the second, when both allocations have completed.  Measured on
  // B200: allocating before the peer CTA was known to be live, or giving up
  // the pair's permit right after one's own allocation, occasionally left the
  // peer's allocation blocked for good (a stalled product, no wait run out).
  cluster_sync();
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncwarp();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_relinquish_pair();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t lim = g.wait_limit_ns;
  const uint32_t full0 = mapa_shared(smem_u32(&full_bar[0]), 0);     // leader's full barriers
  const uint32_t accempty0 = mapa_shared(smem_u32(&acc_empty[0]), 0);  // leader's accumulator-empty

  uint32_t issued = 0;    // stages this CTA's producer thread issued
  bool producer = false;  // this thread is that producer
  if (warp == 0) {
    // ---------------------------------------------------------- producer --
    producer = elect_one();
    if (producer) {
      uint32_t j = 0;
      bool ok = true;
      for (int tile = cluster; tile < ntiles && ok; tile += nclusters) {
        const Tile tl = decode_tile<PBM, PGROUP_M>(tile, g);
        for (int kb = 0; kb < tl.nk; kb++, j++) {
          const uint32_t s = j % PSTAGES, ph = (j / PSTAGES) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, lim, g.status, kWaitEmpty) || *abort_flag) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const bool second = kb >= g.nkb;
          const int z = second ? tl.z1 : tl.z0;
          const int kx = (second ? kb - g.nkb : kb) * BK;
          if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * PSTAGE_BYTES);
          tma_load_3d_pair(sA + s * PA_BYTES, &tmapA, kx, tl.m0 + PHALF * (int)rank, z, full0 + 8 * s);
          tma_load_3d_pair(sB + s * PB_BYTES, &tmapB, kx, tl.n0 + PHALF * (int)rank, z, full0 + 8 * s);
        }
      }
      issued = j;
      // The leader drains the copies of both CTAs (its full barriers count
      // both halves) after the first cluster barrier below; it needs the
      // peer's count, which may differ from its own by up to PSTAGES stages
      // when a wait ran out.
      if (!leader) st_cluster_u32(mapa_shared(smem_u32((const void*)peer_issued), 0), j);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer --
    if (leader && elect_one()) {
      uint32_t j = 0, it = 0;
      bool ok = true;
      for (int tile = cluster; tile < ntiles && ok; tile += nclusters, it++) {
        const Tile tl = decode_tile<PBM, PGROUP_M>(tile, g);
        const uint32_t a = it & 1, aph = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[a], aph ^ 1, lim, g.status, kWaitAccEmpty) || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BN;
        for (int kb = 0; kb < tl.nk; kb++, j++) {
          const uint32_t s = j % PSTAGES, ph = (j / PSTAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, lim, g.status, kWaitFull) || *abort_flag) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * PA_BYTES), b_addr = smem_u32(sB + s * PB_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 32; kk++)
            mma_i8_pair(d_tmem, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32), PIDESC,
                        (kb | kk) != 0);
          tc_commit_pair(&empty_bar[s], 0x3);
        }
        if (ok) tc_commit_pair(&acc_full[a], 0x3);
      }
      tc_commit_pair(drain_bar, 0x1);
      mbar_wait(drain_bar, 0, drain_limit(lim), g.status, kWaitDrain);
    }
  } else {
    // ----------------------------------------------------------- epilogue --
    const int q = warp & 3;
    const int row_l = q * 32 + lane;
    uint32_t it = 0;
    for (int tile = cluster; tile < ntiles; tile += nclusters, it++) {
      const Tile tl = decode_tile<PBM, PGROUP_M>(tile, g);
      const uint32_t a = it & 1, aph = (it >> 1) & 1;
      if (!mbar_wait(&acc_full[a], aph, lim, g.status, kWaitAccFull) || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = tl.m0 + PHALF * (int)rank + row_l;
      const bool row_ok = row < g.M;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + a * BN;
      if (tl.kind == 0) {
        const uint32_t p = T.p[tl.t], md = T.mdiv[tl.t], off = T.off[tl.t];
        int8_t* orow = g.res + tl.out + (int64_t)row * g.ldn;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c * 32, v);
          tmem_wait_ld();
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; i++) {
            uint32_t x = 0;
#pragma unroll
            for (int e = 0; e < 4; e++)
              x |= (uint32_t)(uint8_t)(int8_t)bal_mod_s32((int)v[4 * i + e], p, md, off) << (8 * e);
            w[i] = x;
          }
          const int col = tl.n0 + c * 32;
          if (row_ok && col < g.ldn && in_span(orow + col, 16, g.res_span, g.status, kBoundsGemmStore))
            *reinterpret_cast<uint4*>(orow + col) = make_uint4(w[0], w[1], w[2], w[3]);
          if (row_ok && col + 16 < g.ldn &&
              in_span(orow + col + 16, 16, g.res_span, g.status, kBoundsGemmStore))
            *reinterpret_cast<uint4*>(orow + col + 16) = make_uint4(w[4], w[5], w[6], w[7]);
        }
      } else {
        int32_t* orow = g.corr + tl.out + (int64_t)row * g.ldn;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c * 32, v);
          tmem_wait_ld();
          const int col = tl.n0 + c * 32;
#pragma unroll
          for (int i = 0; i < 8; i++)
            if (row_ok && col + 4 * i < g.ldn &&
                in_span(orow + col + 4 * i, 16, g.corr_span, g.status, kBoundsGemmStore))
              *reinterpret_cast<uint4*>(orow + col + 4 * i) = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2],
                                                                         v[4 * i + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(accempty0 + 8 * a);
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync();   // the peer's stage count is visible; the leader's MMAs have drained
  if (producer && leader) {
    // Every copy of the pair lands before either CTA releases its shared
    // memory.  Both producers issue a stage only after the MMAs that freed it
    // completed, so neither runs more than PSTAGES stages ahead of the other
    // and every stage older than the last PSTAGES issued by either is complete.
    // A stage only the peer issued gets the leader's missing arrival (for the
    // peer's half of the bytes); a stage only the leader issued gets the
    // peer's half of the bytes as a complete-tx, since that copy never comes.
    const uint32_t jp = *peer_issued;
    const uint32_t jmax = issued > jp ? issued : jp;
    const uint32_t lo = jmax > (uint32_t)PSTAGES ? jmax - PSTAGES : 0;
    for (uint32_t jj = lo; jj < jmax; jj++) {
      const uint32_t s = jj % PSTAGES;
      if (jj >= issued) mbar_arrive_expect_tx(&full_bar[s], PSTAGE_BYTES);
      else if (jj >= jp) mbar_complete_tx(&full_bar[s], PSTAGE_BYTES);
      mbar_wait(&full_bar[s], (jj / PSTAGES) & 1, drain_limit(lim), g.status, kWaitDrain);
    }
  }
  __syncwarp();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// 3-D tensor map over K-major planes [zdim][rows][Kp] (uint8), box
// (128 bytes of K) x box_rows x 1, 128-byte swizzle, zero fill outside.
bool encode_plane_map(CUtensorMap* map, const void* base, int64_t zdim, int64_t rows, int64_t Kp, int box_rows,
                      int64_t zrows) {
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeFn>(f);
  }();
  if (!fn) return false;
  const cuuint64_t gdim[3] = {(cuuint64_t)Kp, (cuuint64_t)rows, (cuuint64_t)zdim};
  const cuuint64_t gstride[2] = {(cuuint64_t)Kp, (cuuint64_t)((zrows > 0 ? zrows : rows) * Kp)};
  const cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), gdim, gstride, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int gemm_block_rows_a() { return BM; }
int gemm_block_rows_b() { return BN; }
int gemm_pair_block_rows() { return PHALF; }
bool gemm_use_pair(int M) { return M > BM; }

// One thread waits, with the GEMM's bounded wait, on an mbarrier that nothing
// arrives at: the wait runs out after limit_ns and records kWaitSelfTest in
// the status word.  Nothing else is in flight, so the kernel simply returns.
__global__ void wait_selftest_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  mbar_wait(&bar, 0, limit_ns, status, kWaitSelfTest);
}

cudaError_t launch_wait_selftest(int* status, uint64_t limit_ns, cudaStream_t s) {
  wait_selftest_kernel<<<1, 1, 0, s>>>(status, limit_ns);
  return cudaGetLastError();
}

cudaError_t launch_residue_gemm(const CUtensorMap& tA, const CUtensorMap& tB, const GemmArgs& g, const ModTables& T,
                                int num_sms, cudaStream_t s) {
  const int ntm = (g.M + BM - 1) / BM, ntn = (g.N + BN - 1) / BN;
  const int ncs = g.corr_mode == 1 ? g.batch : (g.corr_mode == 2 ? 2 * g.batch : 0);
  const int64_t tiles = (int64_t)ntm * ntn * (g.P * g.batch + ncs);
  if (tiles <= 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    // the shared-memory opt-in is a per-device attribute of the kernel
    static std::mutex mtx;
    static std::set<int> done;
    std::lock_guard<std::mutex> lk(mtx);
    if (!done.count(dev)) {
      e = cudaFuncSetAttribute(residue_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
      if (e != cudaSuccess) return e;
      done.insert(dev);
    }
  }
  const int grid = (int)std::min<int64_t>(tiles, num_sms);
  residue_gemm_tc_kernel<<<grid, NUM_THREADS, SMEM_BYTES, s>>>(tA, tB, g, T);
  return cudaGetLastError();
}

cudaError_t launch_residue_gemm_pair(const CUtensorMap& tA, const CUtensorMap& tB, const GemmArgs& g,
                                     const ModTables& T, int num_sms, cudaStream_t s) {
  const int64_t tiles = total_tiles<PBM>(g);
  if (tiles <= 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  // per device: the shared-memory opt-in and the resident cluster count
  static std::mutex mtx;
  static std::map<int, int> clusters_of;
  std::unique_lock<std::mutex> lk(mtx);
  int& max_clusters = clusters_of.emplace(dev, -1).first->second;
  if (max_clusters < 0) {
    e = cudaFuncSetAttribute(residue_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PSMEM_BYTES);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = PSMEM_BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, residue_gemm_pair_kernel, &cfg);
    if (e != cudaSuccess) return e;
    max_clusters = std::max(n, 1);
  }
  const int clusters = (int)std::min<int64_t>(tiles, max_clusters);
  lk.unlock();
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = PSMEM_BYTES;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, residue_gemm_pair_kernel, tA, tB, g, T);
}

}  // namespace f64e
