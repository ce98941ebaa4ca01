// Fused attention forward for sm_100a (flash-style, tcgen05):
//
//   O[b, h] = softmax(scale * Q[b, h] K[b, h]^T) V[b, h],   head_dim = 64,
//
// with the scores S and probabilities P kept on chip.  Replaces the unfused
// chain of the reference's scaled_dot_product_attention
// (nn/functional.py:310-321: dev_batched_matmul_nt -> dev_muls -> dev_softmax
// -> dev_batched_matmul) and of the DiT attention einsum
// (diffusion/models.py:529-536), whose fp32 score matrix makes the unfused
// path HBM-bound.
//
// One CTA per (128-query block, head, batch), two CTAs per SM by default
// (AttnCfg<1>); 192 threads:
//   warp 0      TMA producer: Q once, then K and V blocks of 128 keys into a
//               KV_STAGES-deep ring (K-major 128B-swizzled tiles; V's tile is
//               the MN-major B operand of P.V).
//   warp 1      TMEM owner + MMA issuer: S_j = Q K_j^T (M 128, N 128, K 64)
//               into a TMEM score buffer, then O_{j-1} = P_{j-1} V_{j-1}
//               (M 128, N 64, K 128) into one of two TMEM output buffers,
//               so the P.V of one block overlaps the softmax of the next.
//   warps 2-5   softmax, one thread per query row (TMEM lane): two passes
//               over the row's 128 scores (row max, then exp2 / sum / bf16
//               P into a swizzled shared-memory A tile), online rescaling
//               in the log2 domain, and the running output accumulated in
//               fp32 registers from each O_j (o = o * alpha + O_j).
// Keys past kv_len (the ragged last block; TMA zero-fills them) are masked
// to -inf; query rows past q_len are computed and not stored.
//
// Every wait is bounded (global timer): an expired wait records an error
// code in the device error word, the CTA drains its copies and MMAs and
// exits, so a broken pipeline returns a status instead of hanging.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ptx.cuh"

namespace sf {

struct AttnArgs {
  int q_len, kv_len, heads, batch;
  float scale_log2;      // softmax scale * log2(e)
  void* o;               // output, 16-bit
  int out_dtype;         // kBF16 / kF16
  int64_t ldo, o_bstride;  // elements
  int* err;
  // attention_fwd2_kernel only: keys [skip_lo, skip_hi) are left out (none
  // when skip_lo == skip_hi == kv_len), and part_mode selects the output:
  //   0  normalised 16-bit O;
  //   1  write the partial result: unnormalised fp32 O to part_o and the
  //      row's (integer base m, sum l) to part_ml;
  //   2  merge with the partial result in part_o / part_ml, then write the
  //      normalised 16-bit O.
  // part_o is [batch][q_len][heads][64] fp32, part_ml [batch][q_len][heads][2].
  int skip_lo, skip_hi;
  int part_mode;
  float* part_o;
  float* part_ml;
  // Split dispatch (attention_fwd2_kernel; part_mode 0 or 2), so that the
  // last wave of CTAs is not mostly empty: a 1-D grid whose blocks
  // [0, split_first) are whole units u (query block u % nqb, head
  // (u / nqb) % heads, batch u / (nqb * heads)); block split_first + j is
  // piece j % split_k of unit split_first + j / split_k, a contiguous share
  // of the key blocks, and writes its unnormalised fp32 O rows and (m, l)
  // to slot j of ws_o [slot][128][64] / ws_ml [slot][128][2] (zeros and
  // m = -inf when all its keys are skipped); attention_merge_kernel then
  // combines the pieces of each split unit (and part_o / part_ml in mode 2).
  int split_first;  // -1: 3-D grid (query block, head, batch), no pieces
  int split_k;
  int nqb;
  float* ws_o;
  float* ws_ml;
};

constexpr int kAttnBlock = 128;   // queries per CTA and keys per block
constexpr int kAttnD = 64;        // head dim
constexpr int kAttnThreads = 192;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

// Packed fp32x2 arithmetic: two lanes of fma / add per instruction.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1,
                                     float c0, float c1) {
  asm("{\n\t.reg .b64 a, b, c, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
      "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1) {
  asm("{\n\t.reg .b64 a, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 d, {%0, %1};\n\t"
      "add.rn.f32x2 d, d, a;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1));
}

// 2^x for a pair of arguments on the FMA pipe instead of the transcendental
// unit.  Range reduction 2^x = 2^n * 2^f with n = round(x) (the 1.5 * 2^23
// rounding trick) and f = x - n in [-0.5, 0.5]; 2^f = e^(f ln 2) from its
// Taylor series to degree 5 (coefficients (ln 2)^k / k!; truncation error
// below 2.5e-6 relative for |f ln 2| <= 0.35); the exponent n is added to the
// result's exponent field.  Arguments are clamped at -126 (results below
// 2^-126 flush to zero, as ex2.approx.ftz does).
__device__ __forceinline__ void exp2_poly2(float& y0, float& y1, float x0, float x1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float c1 = 0.6931471805599453f, c2 = 0.2402265069591007f,
                  c3 = 0.05550410866482158f, c4 = 0.009618129107628477f,
                  c5 = 0.0013333558146428443f;
  x0 = fmaxf(x0, -126.0f);
  x1 = fmaxf(x1, -126.0f);
  float j0 = x0, j1 = x1;
  add2(j0, j1, kRound, kRound);              // n in the low mantissa bits
  float n0 = j0, n1 = j1;
  add2(n0, n1, -kRound, -kRound);            // n as a float
  float f0 = x0, f1 = x1;
  add2(f0, f1, -n0, -n1);                    // f = x - n
  float p0, p1;
  fma2(p0, p1, f0, f1, c5, c5, c4, c4);
  fma2(p0, p1, p0, p1, f0, f1, c3, c3);
  fma2(p0, p1, p0, p1, f0, f1, c2, c2);
  fma2(p0, p1, p0, p1, f0, f1, c1, c1);
  fma2(p0, p1, p0, p1, f0, f1, 1.0f, 1.0f);
  const int e0 = __float_as_int(j0) - 0x4B400000;  // n
  const int e1 = __float_as_int(j1) - 0x4B400000;
  y0 = __int_as_float(__float_as_int(p0) + (e0 << 23));
  y1 = __int_as_float(__float_as_int(p1) + (e1 << 23));
}

__device__ __forceinline__ uint32_t pack_16bit(float a, float b, bool bf16) {
  if (bf16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// ─────────────── second kernel: O in TMEM, lazily rescaled integer bases ───────────────
//
// Same roles and tiles as attention_fwd_kernel, with two changes that take
// the output row out of the softmax threads' registers and most of the
// per-block synchronisation off their path:
//   * O lives in TMEM and the P.V MMAs accumulate into it (accumulate = 0
//     for the first key block only).
//   * Each row's exponent base m is an integer (ceil of c * row max) and is
//     raised only when a block's c * max exceeds it by more than
//     kAttnRescaleLog2 (p then stays below 2^8).  Only then is the row of O
//     in TMEM scaled by 2^(m_old - m_new) (a warp-collective TMEM load,
//     multiply and store, with factor 1 for the warp's other rows).  Because
//     the base is an integer, the 16-bit rounding of p does not depend on
//     which base is used (a change of base is an exact power-of-two scale),
//     so the result equals the eager per-block rescale up to fp32 rounding.
// With 64-key blocks a CTA needs 128 TMEM columns and ~64 KB of shared
// memory, so three CTAs share an SM (three softmax warps per scheduler).
//
// PT (P in tensor memory, 64-key blocks only): the softmax warps store the
// 16-bit P of block j over the first 32 columns of its own score buffer
// (two values per 32-bit column) and P.V reads its A operand from TMEM.
// The MMA warp issues P.V_j before S_{j+1} (tcgen05.mma of one thread run
// in issue order, so S_{j+1} overwrites P_j only after P.V_j has read it),
// and the commit that signals S_{j+1} also covers P.V_j: the softmax warps
// wait on one barrier per block, and O is final in TMEM whenever a score
// block is ready.  Without the P tile a CTA needs ~49 KB of shared memory,
// so four CTAs share an SM.
//
// PT with 32-key blocks: two score buffers (S_j in buffer j % 2) and O fit
// the same 128 columns.  S_{j+1} is computed while block j's softmax runs;
// the MMA warp issues P.V_{j-1} before S_{j+1} (which overwrites P_{j-1}).
// The softmax of block j reads its 32 scores once, and when its row base
// rises it waits for P.V_{j-1} (o_full, one phase per P.V) before scaling
// O; the final wait is on o_last, signalled by the last P.V only.
constexpr float kAttnRescaleLog2 = 8.0f;

template <int KB_, int ST_, bool PT_ = false>
struct Attn2Cfg {
  static constexpr int KB = KB_;
  static constexpr int KV_STAGES = ST_;
  static constexpr bool PT = PT_;
  static constexpr int NS = KB == 32 ? 2 : 1;            // score buffers
  static constexpr int TILE = kAttnBlock * 128;          // Q tile / one P atom (64 keys)
  static constexpr int KV_TILE = KB * 128;
  static constexpr int P_ATOMS = PT ? 0 : KB / 64;
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = TILE;
  static constexpr int P_OFF = KV_OFF + KV_STAGES * 2 * KV_TILE;
  static constexpr int BAR_OFF = P_OFF + P_ATOMS * TILE;
  static constexpr int BYTES = BAR_OFF + 256;
  static constexpr uint32_t O_COL = NS * KB;            // S in [0, NS * KB), O in the next 64
  static constexpr uint32_t TMEM_COLS = NS * KB + 64 <= 128 ? 128 : 256;
  static constexpr int MIN_BLOCKS = PT ? 4 : (KB == 64 ? 3 : 2);
  static constexpr int CHUNKS = KB / 32;
  static_assert(KB == 32 || KB == 64 || KB == 128, "key block");
  static_assert(PT ? KB <= 64 : KB >= 64, "P in TMEM: 32- or 64-key blocks; P in smem: 64 or 128");
  static_assert((1 + 2 * KV_STAGES + 2 * NS + 4) * 8 + 8 <= 192, "barrier area");
  static constexpr int DESC_OFF = BAR_OFF + 192;        // the CTA's work description (10 ints)
};

// EMU of every four exp2 pairs of a full block go through exp2_poly2.
template <bool BF16, class Cfg, int EMU>
__global__ void __launch_bounds__(kAttnThreads, Cfg::MIN_BLOCKS)
    attention_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int ST = Cfg::KV_STAGES, KB = Cfg::KB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t& q_full = bars[0];
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ST;
  constexpr int NS = Cfg::NS;
  // One score-ready and one P-ready barrier per score buffer, so that each
  // wait is on a phase that is at most one behind (block j + NS, the next
  // user of a buffer, cannot start before P.V_j has been issued).
  uint64_t* s_full = kv_empty + ST;
  uint64_t* p_full = s_full + NS;
  uint64_t& s_free = p_full[NS];
  uint64_t& o_full = p_full[NS + 1];
  uint64_t& o_last = p_full[NS + 2];
  uint64_t& drain_bar = p_full[NS + 3];
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(&p_full[NS + 4]);
  int& abort_flag = *(reinterpret_cast<int*>(&p_full[NS + 4]) + 1);
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadConfig);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Work description, computed by thread 0 into shared memory (read where
  // used rather than held in registers): query block, head, batch, workspace
  // slot (-1: none) and the key blocks over [k0, e0) then [s1, k1), where
  // [k0, k1) is the CTA's key range and [e0, s1) the skipped keys in it.
  int* desc = reinterpret_cast<int*>(smem + Cfg::DESC_OFF);
  enum { kQb, kH, kB, kSlot, kK0, kK1, kE0, kS1, kNb0, kNblk };
  if (threadIdx.x == 0) {
    int u = static_cast<int>(blockIdx.x), k0 = 0, k1 = p.kv_len, slot = -1;
    if (p.split_first < 0) {
      desc[kQb] = blockIdx.x;
      desc[kH] = blockIdx.y;
      desc[kB] = blockIdx.z;
    } else {
      if (u >= p.split_first) {
        const int j = u - p.split_first;
        const int piece = j % p.split_k;
        const int nkb = (p.kv_len + KB - 1) / KB;
        u = p.split_first + j / p.split_k;
        k0 = (piece * nkb / p.split_k) * KB;
        k1 = min(p.kv_len, ((piece + 1) * nkb / p.split_k) * KB);
        slot = j;
      }
      desc[kQb] = u % p.nqb;
      desc[kH] = (u / p.nqb) % p.heads;
      desc[kB] = u / (p.nqb * p.heads);
    }
    const int e0 = min(k1, p.skip_lo), s1 = max(k0, p.skip_hi);
    const int nb0 = e0 > k0 ? (e0 - k0 + KB - 1) / KB : 0;
    desc[kSlot] = slot;
    desc[kK0] = k0;
    desc[kK1] = k1;
    desc[kE0] = e0;
    desc[kS1] = s1;
    desc[kNb0] = nb0;
    desc[kNblk] = nb0 + (k1 > s1 ? (k1 - s1 + KB - 1) / KB : 0);
  }
  auto block_start = [&](int j) {
    const int nb0 = desc[kNb0];
    return j < nb0 ? desc[kK0] + j * KB : desc[kS1] + (j - nb0) * KB;
  };
  auto block_valid = [&](int j) {
    return min(KB, (j < desc[kNb0] ? desc[kE0] : desc[kK1]) - block_start(j));
  };

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(&s_free, 4);
    mbar_init(&o_full, 1);
    mbar_init(&o_last, 1);
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
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
  const int nblk = desc[kNblk];

  if (warp == 0) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      bool ok = true;
      int issued = 0, stage = 0;
      uint32_t phase = 0;
      const int h = desc[kH], b = desc[kB];
      mbar_arrive_expect_tx(&q_full, Cfg::TILE);
      tma_load_4d(smem + Cfg::Q_OFF, &tmQ, &q_full, 0, desc[kQb] * kAttnBlock, h, b);
      for (int j = 0; j < nblk; ++j) {
        if (!mbar_wait(&kv_empty[stage], phase ^ 1u, p.err, kDevTimeoutProducer, abortp)) {
          ok = false;
          break;
        }
        uint8_t* kt = smem + Cfg::KV_OFF + stage * 2 * Cfg::KV_TILE;
        mbar_arrive_expect_tx(&kv_full[stage], 2 * Cfg::KV_TILE);
        tma_load_4d(kt, &tmK, &kv_full[stage], 0, block_start(j), h, b);
        tma_load_4d(kt + Cfg::KV_TILE, &tmV, &kv_full[stage], 0, block_start(j), h, b);
        ++issued;
        if (++stage == ST) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!mbar_wait_quiet(&q_full, 0, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
      if (!ok) {
        const int n = issued < ST ? issued : ST;
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < n; ++i) {
          if (--s < 0) {
            s = ST - 1;
            ph ^= 1u;
          }
          if (!mbar_wait_quiet(&kv_full[s], ph, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
        }
      }
    }
  } else if (warp == 1) {
    // ───────────── MMA issuer ─────────────
    if (lane == 0) {
      const uint32_t fmt = BF16 ? 1u : 0u;
      const uint32_t idesc_s = make_idesc(fmt, 128, KB, 0u, 0u);
      const uint32_t idesc_o = make_idesc(fmt, 128, 64, 0u, 1u);
      const uint32_t q_addr = smem_u32(smem + Cfg::Q_OFF);
      const uint32_t p_addr = smem_u32(smem + Cfg::P_OFF);
      bool ok = mbar_wait(&q_full, 0, p.err, kDevTimeoutMma, abortp);
      bool issued_any = false;
      int stage = 0, pv_stage = 0;
      uint32_t phase = 0;
      auto issue_pv = [&](int jj) -> bool {
        if (!mbar_wait(&p_full[jj % NS], static_cast<uint32_t>(jj / NS) & 1u, p.err, kDevTimeoutMma,
                       abortp))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + Cfg::KV_OFF + pv_stage * 2 * Cfg::KV_TILE +
                                         Cfg::KV_TILE);
#pragma unroll
        for (int ks = 0; ks < KB / 16; ++ks) {
          const uint64_t bd = make_sw128_desc(v_addr + ks * 2048, 8192, 1024);
          if constexpr (Cfg::PT) {
            umma_f16_tmem_a(tmem_base + Cfg::O_COL, tmem_base + (jj % NS) * KB + ks * 8, bd,
                            idesc_o, (jj > 0 || ks > 0) ? 1u : 0u);
          } else {
            const uint64_t ad =
                make_sw128_desc(p_addr + (ks >> 2) * Cfg::TILE + (ks & 3) * 32, 16, 1024);
            umma_f16(tmem_base + Cfg::O_COL, ad, bd, idesc_o, (jj > 0 || ks > 0) ? 1u : 0u);
          }
        }
        if (!Cfg::PT || NS == 2) umma_commit(&o_full);
        if (Cfg::PT && jj == nblk - 1) umma_commit(&o_last);
        umma_commit(&kv_empty[pv_stage]);
        if (++pv_stage == ST) pv_stage = 0;
        return true;
      };
      for (int j = 0; j < nblk && ok; ++j) {
        if (!mbar_wait(&kv_full[stage], phase, p.err, kDevTimeoutMma, abortp)) {
          ok = false;
          break;
        }
        if constexpr (Cfg::PT) {
          // P.V_{j-NS} first: S_j overwrites the P_{j-NS} it reads.
          if (j >= NS && !issue_pv(j - NS)) {
            ok = false;
            break;
          }
        } else if (!mbar_wait(&s_free, (static_cast<uint32_t>(j) & 1u) ^ 1u, p.err, kDevTimeoutMma,
                              abortp)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + Cfg::KV_OFF + stage * 2 * Cfg::KV_TILE);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t ad = make_sw128_desc(q_addr + ks * 32, 16, 1024);
          const uint64_t bd = make_sw128_desc(k_addr + ks * 32, 16, 1024);
          umma_f16(tmem_base + (j % NS) * KB, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
        }
        issued_any = true;
        umma_commit(&s_full[j % NS]);
        if (++stage == ST) {
          stage = 0;
          phase ^= 1u;
        }
        if (!Cfg::PT && j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if constexpr (Cfg::PT) {
        for (int jj = nblk > NS ? nblk - NS : 0; jj < nblk && ok; ++jj)
          if (!issue_pv(jj)) ok = false;
      } else if (ok && nblk > 0 && !issue_pv(nblk - 1)) {
        ok = false;
      }
      if (!ok && issued_any) {
        umma_commit(&drain_bar);
        if (!mbar_wait_quiet(&drain_bar, 0, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
      }
    }
  } else {
    // ───────────── softmax (warps 2..5): one thread per query row ─────────────
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_base;
    const uint32_t o_addr = tmem_base + lane_base + Cfg::O_COL;
    float m_run = -INFINITY, l_run = 0.0f;  // m_run: integer-valued base (log2 domain)
    const float c = p.scale_log2;
    bool ok = true;
    uint32_t r[32];
    // O row scaling by alpha (warp-collective; factor 1 on the warp's other rows).
    auto rescale_o = [&](float alpha) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(o_addr + half * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
        tmem_st32(o_addr + half * 32, r);
      }
    };
    for (int j = 0; j < nblk; ++j) {
      // Waits end the loop for the whole warp together: the TMEM loads and
      // stores that follow are warp-collective.
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[j % NS], static_cast<uint32_t>(j / NS) & 1u,
                                             p.err, kDevTimeoutEpilogue, abortp))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb_addr = s_addr + (j % NS) * KB;
      const int valid = block_valid(j);
      const bool full = valid == KB;
      float mxc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int ch = 0; ch < Cfg::CHUNKS; ++ch) {
        tmem_ld32(sb_addr + ch * 32, r);
        tmem_ld_wait();
        if (full) {
#pragma unroll
          for (int t = 0; t < 32; t += 2)
            mxc[(t >> 1) & 3] = max3f(mxc[(t >> 1) & 3], __uint_as_float(r[t]), __uint_as_float(r[t + 1]));
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (ch * 32 + t < valid) mxc[0] = fmaxf(mxc[0], __uint_as_float(r[t]));
        }
      }
      const float mx = max3f(mxc[0], mxc[1], fmaxf(mxc[2], mxc[3]));
      const float cand = ceilf(mx * c);
      const bool need = cand > m_run + kAttnRescaleLog2;  // always on the first block
      const float alpha = need ? ex2_approx(m_run - cand) : 1.0f;
      const bool rescale = j >= 1 && __any_sync(0xffffffffu, need);
      if constexpr (!Cfg::PT) {
        // P.V of the previous block must be done: it reads the P tile this
        // block overwrites, and its sum is in the O rows a rescale touches.
        if (j >= 1) {
          if (!__all_sync(0xffffffffu, mbar_wait(&o_full, static_cast<uint32_t>(j - 1) & 1u, p.err,
                                                 kDevTimeoutEpilogue, abortp))) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (rescale) {
            rescale_o(alpha);
            tmem_st_wait();
          }
        }
      }
      if (need) {
        l_run *= alpha;
        m_run = cand;
      }
      uint8_t* pbase = smem + Cfg::P_OFF;
      float sp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const float nm = -m_run;
#pragma unroll
      for (int ch = 0; ch < Cfg::CHUNKS; ++ch) {
        if (Cfg::CHUNKS > 1) {  // one chunk: the scores are still in r
          tmem_ld32(sb_addr + ch * 32, r);
          tmem_ld_wait();
        }
        float* pv = reinterpret_cast<float*>(r);
        if (full) {
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            float x0, x1;
            fma2(x0, x1, pv[t], pv[t + 1], c, c, nm, nm);
            if (((t >> 1) & 3) < EMU) {
              exp2_poly2(pv[t], pv[t + 1], x0, x1);
            } else {
              pv[t] = ex2_approx(x0);
              pv[t + 1] = ex2_approx(x1);
            }
            add2(sp[(t >> 1) & 2], sp[((t >> 1) & 2) + 1], pv[t], pv[t + 1]);
          }
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const float e = ex2_approx(fmaf(pv[t], c, nm));
            pv[t] = ch * 32 + t < valid ? e : 0.0f;
            sp[t & 3] += pv[t];
          }
        }
        if constexpr (Cfg::PT) {
          // Keys ch*32 + 2c, +2c+1 go to column ch*16 + c (low half first),
          // over score columns this thread has already read.
          uint32_t pk[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) pk[t] = pack_16bit(pv[2 * t], pv[2 * t + 1], BF16);
          tmem_st16(sb_addr + ch * 16, pk);
        } else {
          uint8_t* rowp = pbase + (ch >> 1) * Cfg::TILE + row * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = (ch & 1) * 4 + q;
            *reinterpret_cast<uint4*>(rowp + ((chunk ^ (row & 7)) << 4)) =
                make_uint4(pack_16bit(pv[8 * q], pv[8 * q + 1], BF16),
                           pack_16bit(pv[8 * q + 2], pv[8 * q + 3], BF16),
                           pack_16bit(pv[8 * q + 4], pv[8 * q + 5], BF16),
                           pack_16bit(pv[8 * q + 6], pv[8 * q + 7], BF16));
          }
        }
      }
      l_run += (sp[0] + sp[1]) + (sp[2] + sp[3]);
      if constexpr (Cfg::PT) {
        // O is scaled after P is stored (r is free again) and before P.V_j is
        // issued.  One score buffer: S_j's barrier already covers P.V_{j-1}.
        // Two: wait for P.V_{j-1} on o_full (at most one phase behind).
        if (rescale) {
          if (NS == 2 &&
              !__all_sync(0xffffffffu, mbar_wait(&o_full, static_cast<uint32_t>(j - 1) & 1u, p.err,
                                                 kDevTimeoutEpilogue, abortp))) {
            ok = false;
            break;
          }
          tc_fence_after();
          rescale_o(alpha);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      if constexpr (!Cfg::PT) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if constexpr (!Cfg::PT) mbar_arrive(&s_free);
        mbar_arrive(&p_full[j % NS]);
      }
    }
    // With P in TMEM the last P.V alone signals o_last.
    if (ok && nblk > 0)
      ok = __all_sync(0xffffffffu,
                      Cfg::PT ? mbar_wait(&o_last, 0u, p.err, kDevTimeoutEpilogue, abortp)
                              : mbar_wait(&o_full, static_cast<uint32_t>(nblk - 1) & 1u, p.err,
                                          kDevTimeoutEpilogue, abortp));
    const int qrow = desc[kQb] * kAttnBlock + row;
    if (ok) {
      tc_fence_after();
      const int h = desc[kH], b = desc[kB], slot = desc[kSlot];
      const bool live = qrow < p.q_len;
      const int64_t prow = (static_cast<int64_t>(b) * p.q_len + qrow) * p.heads + h;
      // A split piece writes its partial result to its workspace slot.
      const int mode = slot >= 0 ? 1 : p.part_mode;
      float* const pml = slot >= 0 ? p.ws_ml + (static_cast<int64_t>(slot) * kAttnBlock + row) * 2
                                   : p.part_ml + 2 * prow;
      float* const pob = slot >= 0 ? p.ws_o + (static_cast<int64_t>(slot) * kAttnBlock + row) * kAttnD
                                   : p.part_o + prow * kAttnD;
      // Merge with a partial result over other keys: both bases are integers,
      // so the rescale factors are exact powers of two.
      float a_own = 1.0f, a_part = 0.0f;
      if (mode == 2 && live) {
        const float m_p = pml[0], l_p = pml[1];
        const float m = fmaxf(m_run, m_p);
        a_own = nblk > 0 ? ex2_approx(m_run - m) : 0.0f;
        a_part = ex2_approx(m_p - m);
        l_run = (nblk > 0 ? l_run * a_own : 0.0f) + l_p * a_part;
      }
      if (mode == 1 && live) {
        pml[0] = m_run;
        pml[1] = l_run;
      }
      const float inv = 1.0f / l_run;
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.o) +
                     (static_cast<int64_t>(b) * p.o_bstride + static_cast<int64_t>(qrow) * p.ldo +
                      static_cast<int64_t>(h) * kAttnD) * 2;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(o_addr + half * 32, r);
        tmem_ld_wait();
        if (!live) continue;
        if (mode == 1) {
          float4* po = reinterpret_cast<float4*>(pob + half * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            po[q] = nblk > 0 ? make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                           __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]))
                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          continue;
        }
        float ov[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) ov[t] = nblk > 0 ? __uint_as_float(r[t]) : 0.0f;
        if (mode == 2) {
          const float4* po = reinterpret_cast<const float4*>(pob + half * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 v = po[q];
            ov[4 * q] = ov[4 * q] * a_own + v.x * a_part;
            ov[4 * q + 1] = ov[4 * q + 1] * a_own + v.y * a_part;
            ov[4 * q + 2] = ov[4 * q + 2] * a_own + v.z * a_part;
            ov[4 * q + 3] = ov[4 * q + 3] * a_own + v.w * a_part;
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<uint4*>(dst)[half * 4 + q] =
              make_uint4(pack_16bit(ov[8 * q] * inv, ov[8 * q + 1] * inv, BF16),
                         pack_16bit(ov[8 * q + 2] * inv, ov[8 * q + 3] * inv, BF16),
                         pack_16bit(ov[8 * q + 4] * inv, ov[8 * q + 5] * inv, BF16),
                         pack_16bit(ov[8 * q + 6] * inv, ov[8 * q + 7] * inv, BF16));
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Combines the split_k pieces of each split unit, and in part_mode 2 the
// partial result in part_o / part_ml (one CTA per unit of ROWS query rows,
// one thread per row): with integer bases m_p, m = max m_p,
// O = sum 2^(m_p - m) O_p / sum 2^(m_p - m) l_p, written as 16-bit O.
// Workspace slot s holds ws_o[s][ROWS][64] and ws_ml[s][ROWS][2].
template <bool BF16, int ROWS>
__global__ void __launch_bounds__(ROWS) attention_merge_kernel(const AttnArgs p) {
  const int u = p.split_first + static_cast<int>(blockIdx.x);
  const int qb = u % p.nqb, h = (u / p.nqb) % p.heads, b = u / (p.nqb * p.heads);
  const int row = threadIdx.x;
  const int qrow = qb * ROWS + row;
  if (qrow >= p.q_len) return;
  const int64_t slot0 = static_cast<int64_t>(blockIdx.x) * p.split_k;
  const int64_t prow = (static_cast<int64_t>(b) * p.q_len + qrow) * p.heads + h;
  const int n_in = p.split_k + (p.part_mode == 2 ? 1 : 0);
  // input i < split_k: workspace slot slot0 + i; i == split_k: the partial result
  auto ml_of = [&](int i) -> const float* {
    return i < p.split_k ? p.ws_ml + ((slot0 + i) * ROWS + row) * 2 : p.part_ml + 2 * prow;
  };
  auto o_of = [&](int i) -> const float* {
    return i < p.split_k ? p.ws_o + ((slot0 + i) * ROWS + row) * kAttnD
                         : p.part_o + prow * kAttnD;
  };
  float m = -INFINITY;
  for (int i = 0; i < n_in; ++i) m = fmaxf(m, ml_of(i)[0]);
  float l = 0.0f;
  float acc[kAttnD];
#pragma unroll
  for (int t = 0; t < kAttnD; ++t) acc[t] = 0.0f;
  for (int i = 0; i < n_in; ++i) {
    const float* ml = ml_of(i);
    if (ml[0] == -INFINITY) continue;  // every key of this piece skipped
    const float a = ex2_approx(ml[0] - m);
    l += ml[1] * a;
    const float4* po = reinterpret_cast<const float4*>(o_of(i));
#pragma unroll
    for (int q = 0; q < kAttnD / 4; ++q) {
      const float4 v = po[q];
      acc[4 * q] += v.x * a;
      acc[4 * q + 1] += v.y * a;
      acc[4 * q + 2] += v.z * a;
      acc[4 * q + 3] += v.w * a;
    }
  }
  const float inv = 1.0f / l;
  uint4* dst = reinterpret_cast<uint4*>(
      reinterpret_cast<uint8_t*>(p.o) +
      (static_cast<int64_t>(b) * p.o_bstride + static_cast<int64_t>(qrow) * p.ldo +
       static_cast<int64_t>(h) * kAttnD) * 2);
#pragma unroll
  for (int q = 0; q < kAttnD / 8; ++q)
    dst[q] = make_uint4(pack_16bit(acc[8 * q] * inv, acc[8 * q + 1] * inv, BF16),
                        pack_16bit(acc[8 * q + 2] * inv, acc[8 * q + 3] * inv, BF16),
                        pack_16bit(acc[8 * q + 4] * inv, acc[8 * q + 5] * inv, BF16),
                        pack_16bit(acc[8 * q + 6] * inv, acc[8 * q + 7] * inv, BF16));
}

}  // namespace sf
