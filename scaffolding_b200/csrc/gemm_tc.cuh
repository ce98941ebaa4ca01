// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[tile] = A[BM x K] * B[BN x K]^T   (fp32 accumulation in TMEM)
//
// Replaces the cuBLAS calls of the reference matmul path:
//   cuda_sgemm / cuda_sgemm_batched      _cuda_kernels.cu:1175-1243
//   (dev_matmul, dev_matmul_nt, dev_batched_matmul[_nt], dev_linear_forward:
//    _cuda_ops.pyx:1088-1190, :1278-1302)
// with the bias add (_cuda_kernels.cu:1490-1527), activation and scale
// (_cuda_kernels.cu:237-277, :384, :428) fused into the epilogue.
//
// CTA layout (320 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: one lane streams A/B k-blocks into a STAGES-deep
//               ring of 128B-swizzled shared-memory stages (each CTA loads its own tiles).
//   warp 1      TMEM owner + MMA issuer: one lane issues tcgen05.mma
//               (M=128, N=BN, K=16 or 8 per instruction) into one of two
//               TMEM accumulators, committing stage releases and
//               accumulator-ready signals to mbarriers.
//   warps 2-9   epilogue: two warps per 32-lane TMEM quadrant (a warp may
//               only touch the quadrant warp_id % 4); the pair splits the
//               tile's columns in interleaved 32-column chunks, loads them
//               with tcgen05.ld, applies alpha/bias/activation/residual,
//               converts and stores.
// Two TMEM accumulators let the epilogue of tile t overlap the MMAs of t+1.
//
// PROMOTE mode (fp32-accurate 3xTF32): the MMA accumulates at most
// PROMOTE_KB k-blocks into a TMEM accumulator, then hands it to the
// epilogue warps, which add it into fp32 registers with IEEE adds and
// release it.  The tensor core's own accumulation is not IEEE
// round-to-nearest, so long K reductions held entirely in TMEM drift by
// ~1e-5 relative; short TMEM chunks + register accumulation keep fp32
// accuracy.
//
// Operand forms: A is always K-major (rows of K contiguous).  B is K-major
// (the nn.Linear weight layout [N, K]) or, for 16-bit inputs, MN-major
// (row-major [K, N], e.g. V in P.V), selected by B_MN.
//
// Split-K (k_splits > 1): each work unit covers a slice of the k-blocks of
// one tile and adds its fp32 partial tile into a zero-initialised fp32
// workspace with red.global.add; a finaliser kernel applies the epilogue.
//
// Tile rasterisation: tiles are visited in groups of `group_m` M-blocks
// sweeping all N-blocks, so concurrently running CTAs share A and B panels
// in L2.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "epilogue.cuh"
#include "ptx.cuh"

namespace sf {

struct GemmTcArgs {
  int M, N, K;          // tile-orientation problem: A is M x K, B is N x K
  int nb0, nb1;         // batch extents (inner, outer); batch z = b1 * nb0 + b0
  int m_tiles, n_tiles, k_blocks;
  int total_tiles;
  int group_m;
  int k_splits, kb_per_split;
  // output, in OUTPUT orientation: element (row r, col c) of batch (b0, b1)
  // lives at C[b0*c_stride0 + b1*c_stride1 + r*ldc + c]
  void* C;
  int out_dtype;
  int64_t ldc, c_stride0, c_stride1;
  int c_trans;          // 1: tile element (i, j) is output (row j, col i) (swap-AB)
  int vec_ok;           // 16-byte vector stores legal for the non-transposed path
  int tma_store;        // 1: stores go through shared memory + TMA (map tmC)
  float* ws;            // split-K fp32 accumulation buffer (output orientation)
  int64_t ldw;
  int64_t ws_slice;     // 0: splits red.add into ws; > 0: split s stores into ws + s * ws_slice
  EpilogueArgs epi;
  int* err;             // device error word
  int a_box_rows;       // pair kernel: rows per A box (128, or fewer for skinny M)
  // Programmatic dependent launch (host: launch with the attribute when pdl
  // is set).  Before waiting for the previous grid the producer prefetches
  // the first pdl_pf k-blocks of its first unit's weight operand (A when
  // pdl_pf_b == 0, else a K-major B) into L2; operands the previous kernel
  // may write are read, and outputs written, only after the wait.
  int pdl, pdl_pf, pdl_pf_b;
};

// Work units of one CTA as (tile, k-block range [kb0, kb1)): unit
// u = blockIdx.x + i * gridDim.x over total_tiles * k_splits (k_splits > 1:
// split-K slices of a tile).
struct WorkIter {
  int u, units;
  __device__ __forceinline__ explicit WorkIter(const GemmTcArgs& p)
      : u(blockIdx.x), units(p.total_tiles * p.k_splits) {}
  __device__ __forceinline__ bool next(const GemmTcArgs& p, int& tile, int& kb0, int& kb1) {
    if (u >= units) return false;
    tile = u / p.k_splits;
    const int split = u - tile * p.k_splits;
    kb0 = split * p.kb_per_split;
    kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
    u += gridDim.x;
    return true;
  }
};

template <int BN_, int STAGES_, int FMT_, bool B_MN_, int PROMOTE_KB_ = 0>
struct TcCfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int STAGES = STAGES_;
  static constexpr int FMT = FMT_;                 // 0 f16, 1 bf16, 2 tf32
  static constexpr bool B_MN = B_MN_;
  static constexpr int PROMOTE_KB = PROMOTE_KB_;   // 0: accumulate the whole K in TMEM
  static constexpr int ELEM = (FMT == 2) ? 4 : 2;
  static constexpr int BK = 128 / ELEM;            // one 128-byte swizzle row of K
  static constexpr int UMMA_K = 32 / ELEM;         // K per tcgen05.mma
  static constexpr int KSTEPS = BK / UMMA_K;       // 4
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_SLOT_BYTES = 4096;       // per epilogue warp: 32 rows x <= 128 B
  static constexpr int STAGING_BYTES = 8 * EPI_SLOT_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + 1024;  // + alignment slack
  static constexpr int ACC_COLS = BN;
  static constexpr int TMEM_COLS = (2 * BN <= 32)    ? 32
                                   : (2 * BN <= 64)  ? 64
                                   : (2 * BN <= 128) ? 128
                                   : (2 * BN <= 256) ? 256
                                                     : 512;
  static constexpr int EPI_WARPS = 8;
  static constexpr int EPI_THREADS = EPI_WARPS * 32;
  static constexpr int THREADS = 64 + EPI_THREADS;
  static constexpr int CH = BN < 32 ? BN : 32;      // epilogue column chunk
  // columns owned per epilogue thread (PROMOTE register accumulator)
  static constexpr int OWN = (BN + 2 * CH - 1) / (2 * CH) * CH;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
  static_assert(!B_MN || (BN % 64 == 0 && ELEM == 2), "MN-major B: 64-wide 16-bit slabs");
  static_assert(PROMOTE_KB == 0 || BN % (2 * CH) == 0, "promotion needs an even chunk split");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

// Operand-ring depth per N tile: ~180-196 KB of stages plus 32 KB of
// epilogue staging fit the 227 KB per-CTA shared memory.
template <int BN>
constexpr int tc_stages() {
  return BN >= 192 ? 4 : BN >= 128 ? 6 : BN >= 64 ? 8 : BN >= 32 ? 9 : 10;
}

__device__ __forceinline__ void tile_coords(int tile, const GemmTcArgs& p, int& mb, int& nb,
                                            int& b0, int& b1) {
  const int per_batch = p.m_tiles * p.n_tiles;
  const int bz = tile / per_batch;
  const int r = tile - bz * per_batch;
  b0 = bz % p.nb0;
  b1 = bz / p.nb0;
  const int group = p.group_m * p.n_tiles;
  const int g = r / group;
  const int first_m = g * p.group_m;
  const int gm = min(p.m_tiles - first_m, p.group_m);
  const int rr = r - g * group;
  mb = first_m + rr % gm;
  nb = rr / gm;
}

// Load CH consecutive values of a 16-bit or fp32 row into floats (vectorised
// when `vec`; scalar otherwise).  Only called for chunks fully inside the row.
template <int CH>
__device__ __forceinline__ void load_row_chunk(const void* base, int64_t idx, int dtype, bool vec,
                                               float* out) {
  if (vec) {
    if (dtype == kF32) {
      const float4* s = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
#pragma unroll
      for (int q = 0; q < CH / 4; ++q) {
        const float4 f = s[q];
        out[4 * q] = f.x; out[4 * q + 1] = f.y; out[4 * q + 2] = f.z; out[4 * q + 3] = f.w;
      }
    } else {
      const uint4* s = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + idx);
#pragma unroll
      for (int q = 0; q < CH / 8; ++q) {
        const uint4 u = s[q];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          if (dtype == kBF16) {
            out[8 * q + 2 * h] = __uint_as_float(w[h] << 16);
            out[8 * q + 2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
          } else {
            const __half2 hv = *reinterpret_cast<const __half2*>(&w[h]);
            const float2 f = __half22float2(hv);
            out[8 * q + 2 * h] = f.x;
            out[8 * q + 2 * h + 1] = f.y;
          }
        }
      }
    }
  } else {
#pragma unroll
    for (int t = 0; t < CH; ++t) out[t] = load_as_f32(base, idx + t, dtype);
  }
}

// Epilogue arithmetic for CH consecutive output columns [j0, j0+CH) of tile
// row i (non-transposed output):  v = act(alpha * acc + bias) + beta * res.
// Every data-dependent choice is made once per chunk, outside the per-element
// loops.
template <int CH>
__device__ __forceinline__ void epilogue_compute(const GemmTcArgs& p, int i, int j0, int64_t roff,
                                                 const float* acc, float* v) {
  const EpilogueArgs& e = p.epi;
  const bool full = j0 + CH <= p.N;
#pragma unroll
  for (int t = 0; t < CH; ++t) v[t] = e.alpha * acc[t];
  if (e.bias) {
    float b[CH];
    if (full) {
      load_row_chunk<CH>(e.bias, j0, e.bias_dtype, e.bias_vec != 0, b);
    } else {
#pragma unroll
      for (int t = 0; t < CH; ++t) b[t] = (j0 + t < p.N) ? load_as_f32(e.bias, j0 + t, e.bias_dtype) : 0.0f;
    }
#pragma unroll
    for (int t = 0; t < CH; ++t) v[t] += b[t];
  }
  if (e.act != kActNone) {
    if (e.fast_act) {
#pragma unroll
      for (int t = 0; t < CH; ++t) v[t] = act_apply_fast(v[t], e.act);
    } else {
#pragma unroll
      for (int t = 0; t < CH; ++t) v[t] = act_apply(v[t], e.act);
    }
  }
  if (e.residual && i < p.M) {
    float r[CH];
    const int64_t ridx = roff + (int64_t)i * e.ldr + j0;
    if (full) {
      load_row_chunk<CH>(e.residual, ridx, e.residual_dtype, e.res_vec != 0, r);
    } else {
#pragma unroll
      for (int t = 0; t < CH; ++t)
        r[t] = (j0 + t < p.N) ? load_as_f32(e.residual, ridx + t, e.residual_dtype) : 0.0f;
    }
#pragma unroll
    for (int t = 0; t < CH; ++t) v[t] += e.beta * r[t];
  }
}

// Apply the epilogue to CH consecutive tile columns [j0, j0+CH) of tile row i
// and store them with per-thread global stores (split-K, swap-AB, and
// outputs TMA cannot describe).
template <int CH>
__device__ __forceinline__ void epilogue_store(const GemmTcArgs& p, int i, int j0, int b0, int b1,
                                               const float* acc, int split = 0) {
  const EpilogueArgs& e = p.epi;
  if (i >= p.M) return;
  if (p.k_splits > 1) {
    // Partial sums: raw accumulator into the fp32 workspace, added into one
    // buffer or stored into this split's own slice (no zeroing needed).
    float* const ws = p.ws + (p.ws_slice > 0 ? split * p.ws_slice : 0);
#pragma unroll
    for (int t = 0; t < CH; ++t) {
      const int j = j0 + t;
      if (j < p.N) {
        float* dst = p.c_trans ? ws + (int64_t)j * p.ldw + i : ws + (int64_t)i * p.ldw + j;
        if (p.ws_slice > 0)
          *dst = acc[t];
        else
          atomicAdd(dst, acc[t]);
      }
    }
    return;
  }
  const int64_t coff = (int64_t)b0 * p.c_stride0 + (int64_t)b1 * p.c_stride1;
  const int64_t roff = (int64_t)b0 * e.r_stride0 + (int64_t)b1 * e.r_stride1;
  if (p.c_trans) {
    // Output (row j, col i): bias by output column i; lanes hold consecutive i,
    // so every store instruction is coalesced across the warp.
    const float bias_v = e.bias ? load_as_f32(e.bias, i, e.bias_dtype) : 0.0f;
#pragma unroll
    for (int t = 0; t < CH; ++t) {
      const int j = j0 + t;
      if (j < p.N) {
        const float res_v =
            e.residual ? load_as_f32(e.residual, roff + (int64_t)j * e.ldr + i, e.residual_dtype)
                       : 0.0f;
        store_from_f32(p.C, coff + (int64_t)j * p.ldc + i, p.out_dtype,
                       epilogue_value(acc[t], e, bias_v, res_v));
      }
    }
    return;
  }
  float v[CH];
  epilogue_compute<CH>(p, i, j0, roff, acc, v);
  const bool full = j0 + CH <= p.N;
  const int64_t base = coff + (int64_t)i * p.ldc + j0;
  if (p.vec_ok && full) {
    if (p.out_dtype == kF32) {
      float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.C) + base);
#pragma unroll
      for (int q = 0; q < CH / 4; ++q)
        dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.C) + base);
      const int dt = p.out_dtype;
#pragma unroll
      for (int q = 0; q < CH / 8; ++q)
        dst[q] = make_uint4(pack2(v[8 * q], v[8 * q + 1], dt), pack2(v[8 * q + 2], v[8 * q + 3], dt),
                            pack2(v[8 * q + 4], v[8 * q + 5], dt), pack2(v[8 * q + 6], v[8 * q + 7], dt));
    }
  } else {
#pragma unroll
    for (int t = 0; t < CH; ++t)
      if (j0 + t < p.N) store_from_f32(p.C, base + t, p.out_dtype, v[t]);
  }
}

// Same epilogue, stored through the warp's shared-memory slot with one TMA
// bulk tensor store per 32-row x CH-column chunk (warp-collective).  The slot
// holds the chunk in the swizzled layout the tensor map of C declares
// (128/64/32-byte swizzle for 128/64/32-byte rows), which also keeps the
// row-per-lane shared-memory writes free of bank conflicts.  The box is
// clipped by the hardware at the matrix edges.
template <int CH>
__device__ __forceinline__ void epilogue_store_tma(const GemmTcArgs& p, const CUtensorMap* tmC,
                                                   uint8_t* slot, int lane, int i, int box_row0,
                                                   int j0, int b0, int b1, const float* acc) {
  const EpilogueArgs& e = p.epi;
  const int64_t roff = (int64_t)b0 * e.r_stride0 + (int64_t)b1 * e.r_stride1;
  float v[CH];
  epilogue_compute<CH>(p, i, j0, roff, acc, v);
  if (lane == 0) bulk_wait_group_read0();  // previous store from this slot has read it
  __syncwarp();
  if (p.out_dtype == kF32) {
    constexpr int R = CH * 4;
    uint8_t* row = slot + lane * R;
    const int sw = (R == 128) ? (lane & 7) : (R == 64) ? ((lane >> 1) & 3) : ((lane >> 2) & 1);
#pragma unroll
    for (int q = 0; q < R / 16; ++q)
      *reinterpret_cast<float4*>(row + ((q ^ sw) << 4)) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
    constexpr int R = CH * 2;
    uint8_t* row = slot + lane * R;
    const int sw = (R == 128) ? (lane & 7) : (R == 64) ? ((lane >> 1) & 3) : ((lane >> 2) & 1);
    const int dt = p.out_dtype;
#pragma unroll
    for (int q = 0; q < R / 16; ++q)
      *reinterpret_cast<uint4*>(row + ((q ^ sw) << 4)) =
          make_uint4(pack2(v[8 * q], v[8 * q + 1], dt), pack2(v[8 * q + 2], v[8 * q + 3], dt),
                     pack2(v[8 * q + 4], v[8 * q + 5], dt), pack2(v[8 * q + 6], v[8 * q + 7], dt));
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_4d(tmC, slot, j0, box_row0, b0, b1);
    bulk_commit_group();
  }
}

template <int CH>
__device__ __forceinline__ void tmem_load_chunk(uint32_t taddr, float* out) {
  uint32_t r[CH];
  if constexpr (CH == 32) {
    tmem_ld32(taddr, r);
  } else {
    uint32_t (&r16)[16] = *reinterpret_cast<uint32_t(*)[16]>(r);
    tmem_ld16(taddr, r16);
  }
  tmem_ld_wait();
#pragma unroll
  for (int t = 0; t < CH; ++t) out[t] = __uint_as_float(r[t]);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmTcArgs p) {
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, STAGES = Cfg::STAGES;
  constexpr int CH = Cfg::CH;
  constexpr int PKB = Cfg::PROMOTE_KB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], Cfg::EPI_THREADS);
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
    tmem_alloc(&tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  volatile int* abortp = &abort_flag;

  if (warp == 0) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      if (p.pdl_pf > 0) {
        WorkIter it0(p);
        int t0, k0, k1, mb, nb, b0, b1;
        if (it0.next(p, t0, k0, k1)) {
          tile_coords(t0, p, mb, nb, b0, b1);
          for (int kb = k0; kb < min(k1, k0 + p.pdl_pf); ++kb) {
            if (!p.pdl_pf_b)
              tma_prefetch_l2_4d(&tmA, kb * BK, mb * BM, b0, b1);
            else if constexpr (!Cfg::B_MN)
              tma_prefetch_l2_4d(&tmB, kb * BK, nb * BN, b0, b1);
          }
        }
      }
      pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      WorkIter it(p);
      int tile, kb0, kb1;
      while (ok && it.next(p, tile, kb0, kb1)) {
        int mb, nb, b0, b1;
        tile_coords(tile, p, mb, nb, b0, b1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.err, kDevTimeoutProducer, abortp)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          tma_load_4d(sa, &tmA, &full_bar[stage], kb * BK, mb * BM, b0, b1);
          if constexpr (!Cfg::B_MN) {
            tma_load_4d(sb, &tmB, &full_bar[stage], kb * BK, nb * BN, b0, b1);
          } else {
#pragma unroll
            for (int s = 0; s < BN / 64; ++s)
              tma_load_4d(sb + s * 8192, &tmB, &full_bar[stage], nb * BN + s * 64, kb * BK, b0,
                          b1);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Abort: wait (bounded) for the copies this thread still has in flight.
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
      }
    }
  } else if (warp == 1) {
    // ───────────── MMA issuer ─────────────
    if (lane == 0) {
      const uint32_t idesc = make_idesc(Cfg::FMT == 2 ? 2u : (Cfg::FMT == 1 ? 1u : 0u), BM, BN, 0u,
                                        Cfg::B_MN ? 1u : 0u);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      WorkIter it(p);
      int tile, kb0, kb1;
      while (ok && it.next(p, tile, kb0, kb1)) {
        const int chunk = PKB > 0 ? PKB : max(kb1 - kb0, 1);
        for (int kc = kb0; kc < kb1 && ok; kc += chunk) {
          const int kce = min(kb1, kc + chunk);
          if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, p.err, kDevTimeoutMma, abortp)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::ACC_COLS);
          for (int kb = kc; kb < kce; ++kb) {
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
              const uint64_t bd = Cfg::B_MN ? make_sw128_desc(b_addr + ks * 2048, 8192, 1024)
                                            : make_sw128_desc(b_addr + ks * 32, 16, 1024);
              const uint32_t accum = (kb > kc || ks > 0) ? 1u : 0u;
              if constexpr (Cfg::FMT == 2)
                umma_tf32(d_tmem, ad, bd, idesc, accum);
              else
                umma_f16(d_tmem, ad, bd, idesc, accum);
            }
            issued_any = true;
            umma_commit(&empty_bar[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(&tfull_bar[acc]);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
      }
      if (!ok && issued_any) {
        // Abort: make sure no tcgen05.mma is still writing TMEM before dealloc.
        umma_commit(&drain_bar);
        if (!mbar_wait_quiet(&drain_bar, 0, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
      }
    }
  } else {
    // ───────────── epilogue (warps 2..9) ─────────────
    pdl_wait();  // outputs (and residual inputs) belong to the previous grid until it completes
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quad * 32 + lane;
    uint8_t* slot = smem + STAGES * Cfg::STAGE_BYTES + (warp - 2) * Cfg::EPI_SLOT_BYTES;
    const bool tma_out = p.tma_store != 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    WorkIter it(p);
    int tile, kb0, kb1;
    while (ok && it.next(p, tile, kb0, kb1)) {
      int mb, nb, b0, b1;
      tile_coords(tile, p, mb, nb, b0, b1);
      const int i = mb * BM + row;
      // Warp-uniform: does any row of this warp's 32-row quadrant exist?
      const bool rows_live = mb * BM + quad * 32 < p.M;
      if constexpr (PKB == 0) {
        if (!mbar_wait(&tfull_bar[acc], acc_phase, p.err, kDevTimeoutEpilogue, abortp))
          break;
        tc_fence_after();
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                               static_cast<uint32_t>(acc * Cfg::ACC_COLS);
#pragma unroll 1
        for (int c = half * CH; c < BN; c += 2 * CH) {
          float v[CH];
          tmem_load_chunk<CH>(tbase + c, v);
          const int j0 = nb * BN + c;
          if (j0 < p.N && rows_live) {
            if (tma_out)
              epilogue_store_tma<CH>(p, &tmC, slot, lane, i, mb * BM + quad * 32, j0, b0, b1, v);
            else
              epilogue_store<CH>(p, i, j0, b0, b1, v, kb0 / p.kb_per_split);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      } else {
        // Promotion: sum TMEM chunks of <= PKB k-blocks into fp32 registers.
        constexpr int OWN = Cfg::OWN;
        float racc[OWN];
#pragma unroll
        for (int t = 0; t < OWN; ++t) racc[t] = 0.0f;
        for (int kc = kb0; kc < kb1; kc += PKB) {
          if (!mbar_wait(&tfull_bar[acc], acc_phase, p.err, kDevTimeoutEpilogue, abortp)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                 static_cast<uint32_t>(acc * Cfg::ACC_COLS);
#pragma unroll
          for (int q = 0; q < OWN / CH; ++q) {
            float v[CH];
            tmem_load_chunk<CH>(tbase + half * CH + q * 2 * CH, v);
#pragma unroll
            for (int t = 0; t < CH; ++t) racc[q * CH + t] += v[t];
          }
          tc_fence_before();
          mbar_arrive(&tempty_bar[acc]);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        if (!ok) break;
        for (int q = 0; q < OWN / CH; ++q) {
          const int j0 = nb * BN + half * CH + q * 2 * CH;
          if (j0 < p.N && rows_live) {
            if (tma_out)
              epilogue_store_tma<CH>(p, &tmC, slot, lane, i, mb * BM + quad * 32, j0, b0, b1,
                                     &racc[q * CH]);
            else
              epilogue_store<CH>(p, i, j0, b0, b1, &racc[q * CH], kb0 / p.kb_per_split);
          }
        }
      }
    }
  }

  if (warp >= 2 && p.tma_store && lane == 0) bulk_wait_group0();
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace sf
