// CTA-pair (2-CTA cluster, tcgen05 cta_group::2) variant of the persistent
// tcgen05 GEMM, for large 16-bit GEMMs with a K-major B operand (the
// nn.Linear weight layout: DiT block linears, the square sweep).
//
//   D[256 x BN tile] = A[256 x K] * B[BN x K]^T, fp32 accumulation in TMEM.
//
// Why a pair: a 1-CTA 128 x 256 tile streams 48 KB of operands through
// shared memory per 64-deep k-block (16 KB of A, 32 KB of B) for 512 tensor
// cycles.  In a pair each CTA holds its own 128 rows of A and HALF of the
// B rows; one M = 256 MMA issued by the even CTA reads both CTAs' shared
// memory, so each SM stages 16 KB + BN/2 x 128 B per k-block (32 KB at
// BN = 256): a third less shared-memory and L2 traffic per FLOP, and room
// for 6 operand stages instead of 4.
//
// Roles (320 threads per CTA, one CTA per SM, persistent over pair tiles):
//   warp 0      TMA producer in BOTH CTAs: loads this CTA's A rows and B half
//               into its own ring; completion bytes of both CTAs are counted
//               on the even CTA's full barrier (the even producer arms it
//               with the pair's total).
//   warp 1      TMEM allocation in both CTAs (cta_group::2, same columns in
//               both); in the even CTA lane 0 also issues the M = 256 MMAs
//               and commits stage releases and accumulator-ready signals to
//               the mbarriers of both CTAs.
//   warps 2-9   epilogue in both CTAs: each drains its own TMEM (its 128
//               accumulator rows) exactly as the 1-CTA kernel does and
//               signals "accumulator free" to the even CTA's barrier.
//
// Every wait is bounded (global timer); an expired wait records an error
// code, and both CTAs still meet at the final cluster barrier before the
// TMEM is released.  The loads never read another GPU's memory and carry no
// cluster-wide delivery qualifier: each CTA fetches its own tiles.
#pragma once
#include "gemm_tc.cuh"

namespace sf {

template <int BN_, int STAGES_, int FMT_>
struct Tc2Cfg {
  static constexpr int BM = 128;                   // rows per CTA; the pair covers 256
  static constexpr int PAIR_M = 256;
  static constexpr int BN = BN_;                   // accumulator columns (whole pair)
  static constexpr int BN_HALF = BN_ / 2;          // B rows staged by each CTA
  static constexpr int STAGES = STAGES_;
  static constexpr int FMT = FMT_;                 // 0 f16, 1 bf16
  static constexpr int BK = 64;
  static constexpr int UMMA_K = 16;
  static constexpr int KSTEPS = BK / UMMA_K;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN_HALF * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_SLOT_BYTES = 4096;
  static constexpr int STAGING_BYTES = 8 * EPI_SLOT_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + 1024;
  static constexpr int ACC_COLS = BN;
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + EPI_WARPS * 32;
  static constexpr int CH = 32;
  static_assert(FMT == 0 || FMT == 1, "16-bit operands");
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "pair tile width");
  static_assert(BN_HALF % 8 == 0, "B half is whole 8-row swizzle atoms");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

// Operand-ring depth per pair tile width: as many stages of 16 KB + BN/2 rows
// as fit next to the 32 KB of epilogue staging (at most 12).
template <int BN>
constexpr int tc2_stages() {
  constexpr int stage = 128 * 128 + (BN / 2) * 128;
  constexpr int n = (227 * 1024 - 8 * 4096 - 1024 - 512) / stage;
  return n > 12 ? 12 : n;
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const GemmTcArgs p) {
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, STAGES = Cfg::STAGES;
  constexpr int CH = Cfg::CH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  __shared__ __align__(8) uint64_t full_bar[STAGES];   // used in the even CTA
  __shared__ __align__(8) uint64_t empty_bar[STAGES];  // both CTAs
  __shared__ __align__(8) uint64_t tfull_bar[2];       // both CTAs
  __shared__ __align__(8) uint64_t tempty_bar[2];      // used in the even CTA
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * Cfg::EPI_WARPS);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.tma_store) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  volatile int* abortp = &abort_flag;

  const int cluster_id = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;
  const int units = p.total_tiles;

  if (warp == 0) {
    // ───────────── TMA producer (both CTAs) ─────────────
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(&full_bar[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = cluster_id; u < units && ok; u += clusters) {
        int mb, nb, b0, b1;
        tile_coords(u, p, mb, nb, b0, b1);
        const int arow = mb * Cfg::PAIR_M + static_cast<int>(rank) * BM;
        const int brow = nb * BN + static_cast<int>(rank) * Cfg::BN_HALF;
        // A boxes of a_box_rows rows; a CTA whose 128 rows lie wholly past M
        // loads no A (its accumulator rows are never stored, so the stale
        // shared memory it multiplies is harmless).
        const bool load_a = arow < p.M;
        const uint32_t a_bytes = static_cast<uint32_t>(p.a_box_rows) * 128u;
        const int base = mb * Cfg::PAIR_M;
        const uint32_t tx_bytes = (base < p.M ? a_bytes : 0u) + (base + BM < p.M ? a_bytes : 0u) +
                                  2u * static_cast<uint32_t>(Cfg::B_BYTES);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.err, kDevTimeoutProducer, abortp)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], tx_bytes);
          const uint32_t fb = full0 + static_cast<uint32_t>(stage * 8);
          if (load_a) tma_load_4d_pair(sa, &tmA, fb, kb * BK, arow, b0, b1);
          tma_load_4d_pair(sb, &tmB, fb, kb * BK, brow, b0, b1);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        if (leader) {
          // Abort: wait (bounded) for the copies of the stages this CTA armed.
          const int n = issued < STAGES ? issued : STAGES;
          int s = stage;
          uint32_t ph = phase;
          for (int j = 0; j < n; ++j) {
            if (--s < 0) {
              s = STAGES - 1;
              ph ^= 1u;
            }
            if (!mbar_wait_quiet(&full_bar[s], ph, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
          }
        } else {
          // The odd CTA's copies complete on the even CTA's barriers; give
          // copies still in flight time to land before the CTA retires.
          const unsigned long long t0 = global_timer_ns();
          while (global_timer_ns() - t0 < 1000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ───────────── MMA issuer (even CTA) ─────────────
    if (leader && lane == 0) {
      const uint32_t idesc = make_idesc(Cfg::FMT == 1 ? 1u : 0u, Cfg::PAIR_M, BN, 0u, 0u);
      const uint32_t empty_own = smem_u32(&empty_bar[0]);
      const uint32_t empty_peer = mapa_shared(empty_own, 1);
      const uint32_t tfull_own = smem_u32(&tfull_bar[0]);
      const uint32_t tfull_peer = mapa_shared(tfull_own, 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int u = cluster_id; u < units && ok; u += clusters) {
        if (!mbar_wait_cluster(&tempty_bar[acc], acc_phase ^ 1u, p.err, kDevTimeoutMma, abortp)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::ACC_COLS);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, p.err, kDevTimeoutMma, abortp)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < Cfg::KSTEPS; ++ks) {
            const uint64_t ad = make_sw128_desc(a_addr + ks * 32, 16, 1024);
            const uint64_t bd = make_sw128_desc(b_addr + ks * 32, 16, 1024);
            umma_f16_pair(d_tmem, ad, bd, idesc, (kb > 0 || ks > 0) ? 1u : 0u);
          }
          issued_any = true;
          umma_commit_pair(empty_own + static_cast<uint32_t>(stage * 8));
          umma_commit_pair(empty_peer + static_cast<uint32_t>(stage * 8));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_own + static_cast<uint32_t>(acc * 8));
        umma_commit_pair(tfull_peer + static_cast<uint32_t>(acc * 8));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        // Abort: no MMA may still write either CTA's TMEM when it is released.
        umma_commit_pair(smem_u32(&drain_bar));
        if (!mbar_wait_quiet(&drain_bar, 0, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
      }
    }
  } else {
    // ───────────── epilogue (warps 2..9, both CTAs) ─────────────
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quad * 32 + lane;
    uint8_t* slot = smem + STAGES * Cfg::STAGE_BYTES + (warp - 2) * Cfg::EPI_SLOT_BYTES;
    const bool tma_out = p.tma_store != 0;
    const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty_bar[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = cluster_id; u < units; u += clusters) {
      int mb, nb, b0, b1;
      tile_coords(u, p, mb, nb, b0, b1);
      const int row0 = mb * Cfg::PAIR_M + static_cast<int>(rank) * BM;
      const int i = row0 + row;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, p.err, kDevTimeoutEpilogue, abortp)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * Cfg::ACC_COLS);
      const bool rows_live = row0 + quad * 32 < p.M;
#pragma unroll 1
      for (int c = half * CH; c < BN; c += 2 * CH) {
        float v[CH];
        tmem_load_chunk<CH>(tbase + c, v);
        const int j0 = nb * BN + c;
        if (j0 < p.N && rows_live) {
          if (tma_out)
            epilogue_store_tma<CH>(p, &tmC, slot, lane, i, row0 + quad * 32, j0, b0, b1, v);
          else
            epilogue_store<CH>(p, i, j0, b0, b1, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + static_cast<uint32_t>(acc * 8));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  if (warp >= 2 && p.tma_store && lane == 0) bulk_wait_group0();
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's MMAs and remote signals are finished
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace sf
