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
  int sleep_ns;          // poll back-off of the softmax warps' waits (0 = spin)
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
};

constexpr int kAttnBlock = 128;   // queries per CTA and keys per block
constexpr int kAttnD = 64;        // head dim
constexpr int kAttnThreads = 192;

// Configuration: KB keys per block; NS score buffers (TMEM), NP probability
// tiles (shared memory), NO output buffers (TMEM), ST K/V ring stages.
//   AttnCfg<128, 1, 1, 2, 2>  256 TMEM columns, ~113 KB: two CTAs per SM;
//                             S_{j+1} waits for the softmax of block j.
//   AttnCfg<96, 2, 1, 1, 2>   256 TMEM columns, ~97 KB: two CTAs per SM and
//                             double-buffered scores, so S_{j+1} is computed
//                             while block j's softmax runs (96-key blocks
//                             keep 2 x 96 score + 64 output columns in 256).
//   AttnCfg<128, 2, 2, 2, 4>  512 TMEM columns: one CTA per SM.
template <int KB_, int NS_, int NP_, int NO_, int ST_>
struct AttnCfg {
  static constexpr int KB = KB_;
  static constexpr int NS = NS_, NP = NP_, NO = NO_;
  static constexpr int KV_STAGES = ST_;
  static constexpr int TILE = kAttnBlock * 128;          // Q tile / P atom: 128 rows x 128 B
  static constexpr int KV_TILE = KB * 128;               // K or V tile: KB rows x 128 B
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = TILE;                    // stage s: K at +2s*KV_TILE, V after it
  static constexpr int P_OFF = KV_OFF + KV_STAGES * 2 * KV_TILE;  // NP tiles x 2 atoms
  static constexpr int BAR_OFF = P_OFF + NP * 2 * TILE;         // mbarriers and flags
  static constexpr int BYTES = BAR_OFF + 256;
  static constexpr uint32_t O_COL = NS * KB;             // NO 64-column O buffers follow S
  static constexpr uint32_t COLS_USED = NS * KB + NO * 64;
  static constexpr uint32_t TMEM_COLS = COLS_USED <= 256 ? 256 : 512;
  static constexpr int MIN_BLOCKS = TMEM_COLS <= 256 ? 2 : 1;
  static constexpr int CHUNKS = KB / 32;
  static_assert(KB % 32 == 0 && KB <= 128 && KB_ % 16 == 0, "key block");
  static_assert(KV_TILE % 1024 == 0 && P_OFF % 1024 == 0, "1024-byte aligned tiles");
  static_assert(COLS_USED <= 512, "TMEM budget");
  static_assert(NP == 1 || NP == NS, "P tiles follow the score buffers");
  static_assert((1 + 2 * KV_STAGES + 2 * NS + NP + 2 * NO + 2) * 8 <= 256, "barrier area");
};

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

// EMU of every four exp2 pairs of a full block go through exp2_poly2.
template <bool BF16, class Cfg, int EMU>
__global__ void __launch_bounds__(kAttnThreads, Cfg::MIN_BLOCKS)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
  // All shared memory is dynamic (no static part), declared 1024-byte
  // aligned for the 128B-swizzled tiles; the mbarriers sit after the tiles.
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int ST = Cfg::KV_STAGES, KB = Cfg::KB, NS = Cfg::NS, NP = Cfg::NP, NO = Cfg::NO;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t& q_full = bars[0];
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* s_full = kv_empty + ST;
  uint64_t* s_free = s_full + NS;
  uint64_t* p_full = s_free + NS;
  uint64_t* o_full = p_full + NP;
  uint64_t* o_free = o_full + NO;
  uint64_t& drain_bar = o_free[NO];
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(&o_free[NO + 1]);
  int& abort_flag = *(reinterpret_cast<int*>(&o_free[NO + 1]) + 1);
  if ((smem_u32(smem) & 1023u) != 0) {
    // The swizzled tile layout needs 1024-byte alignment; never guess.
    if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadConfig);
    return;
  }

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nblk = (p.kv_len + KB - 1) / KB;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    for (int i = 0; i < NP; ++i) mbar_init(&p_full[i], 4);
    for (int i = 0; i < NO; ++i) {
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
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
  // TMEM columns: NS score buffers of KB columns, then NO 64-column O buffers.

  if (warp == 0) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      bool ok = true;
      int issued = 0, stage = 0;
      uint32_t phase = 0;
      mbar_arrive_expect_tx(&q_full, Cfg::TILE);
      tma_load_4d(smem + Cfg::Q_OFF, &tmQ, &q_full, 0, qb * kAttnBlock, h, b);
      for (int j = 0; j < nblk; ++j) {
        if (!mbar_wait(&kv_empty[stage], phase ^ 1u, p.err, kDevTimeoutProducer, abortp)) {
          ok = false;
          break;
        }
        uint8_t* kt = smem + Cfg::KV_OFF + stage * 2 * Cfg::KV_TILE;
        mbar_arrive_expect_tx(&kv_full[stage], 2 * Cfg::KV_TILE);
        tma_load_4d(kt, &tmK, &kv_full[stage], 0, j * KB, h, b);
        tma_load_4d(kt + Cfg::KV_TILE, &tmV, &kv_full[stage], 0, j * KB, h, b);
        ++issued;
        if (++stage == ST) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Wait (bounded) for every copy this thread issued before the CTA may
      // retire: on the normal path they have all been consumed already.
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
      const uint32_t idesc_s = make_idesc(fmt, 128, KB, 0u, 0u);   // K-major A and B
      const uint32_t idesc_o = make_idesc(fmt, 128, 64, 0u, 1u);   // P K-major, V MN-major
      const uint32_t q_addr = smem_u32(smem + Cfg::Q_OFF);
      bool ok = mbar_wait(&q_full, 0, p.err, kDevTimeoutMma, abortp);
      bool issued_any = false;
      int stage = 0;
      uint32_t phase = 0;
      int pv_stage = 0;
      auto issue_pv = [&](int jj) -> bool {
        const int pb = jj % NP;
        const uint32_t ppar = (static_cast<uint32_t>(jj / NP)) & 1u;
        const int ob = jj % NO;
        const uint32_t opar = (static_cast<uint32_t>(jj / NO)) & 1u;
        if (!mbar_wait(&p_full[pb], ppar, p.err, kDevTimeoutMma, abortp)) return false;
        if (!mbar_wait(&o_free[ob], opar ^ 1u, p.err, kDevTimeoutMma, abortp)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + Cfg::P_OFF + pb * 2 * Cfg::TILE);
        const uint32_t v_addr = smem_u32(smem + Cfg::KV_OFF + pv_stage * 2 * Cfg::KV_TILE +
                                         Cfg::KV_TILE);
        const uint32_t d_tmem = tmem_base + Cfg::O_COL + static_cast<uint32_t>(ob * 64);
#pragma unroll
        for (int ks = 0; ks < KB / 16; ++ks) {
          const uint64_t ad =
              make_sw128_desc(p_addr + (ks >> 2) * Cfg::TILE + (ks & 3) * 32, 16, 1024);
          const uint64_t bd = make_sw128_desc(v_addr + ks * 2048, 8192, 1024);
          umma_f16(d_tmem, ad, bd, idesc_o, ks > 0 ? 1u : 0u);
        }
        umma_commit(&o_full[ob]);
        umma_commit(&kv_empty[pv_stage]);  // K and V of this block are consumed
        if (++pv_stage == ST) pv_stage = 0;
        return true;
      };
      for (int j = 0; j < nblk && ok; ++j) {
        const int buf = j % NS;
        const uint32_t par = (static_cast<uint32_t>(j / NS)) & 1u;
        if (!mbar_wait(&kv_full[stage], phase, p.err, kDevTimeoutMma, abortp) ||
            !mbar_wait(&s_free[buf], par ^ 1u, p.err, kDevTimeoutMma, abortp)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + Cfg::KV_OFF + stage * 2 * Cfg::KV_TILE);
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * KB);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t ad = make_sw128_desc(q_addr + ks * 32, 16, 1024);
          const uint64_t bd = make_sw128_desc(k_addr + ks * 32, 16, 1024);
          umma_f16(d_tmem, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
        }
        issued_any = true;
        umma_commit(&s_full[buf]);
        if (++stage == ST) {
          stage = 0;
          phase ^= 1u;
        }
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && nblk > 0 && !issue_pv(nblk - 1)) ok = false;
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
    float o_acc[kAttnD];
#pragma unroll
    for (int t = 0; t < kAttnD; ++t) o_acc[t] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f, alpha_prev = 0.0f;
    const float c = p.scale_log2;
    bool ok = true;
    auto consume_o = [&](int jj, float alpha) -> bool {
      const int buf = jj % NO;
      const uint32_t par = (static_cast<uint32_t>(jj / NO)) & 1u;
      if (!mbar_wait(&o_full[buf], par, p.err, kDevTimeoutEpilogue, abortp, kWaitLimitNs,
                     p.sleep_ns))
        return false;
      tc_fence_after();
      uint32_t r[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem_base + lane_base + Cfg::O_COL + static_cast<uint32_t>(buf * 64 + half * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; t += 2)
          fma2(o_acc[half * 32 + t], o_acc[half * 32 + t + 1], o_acc[half * 32 + t],
               o_acc[half * 32 + t + 1], alpha, alpha, __uint_as_float(r[t]),
               __uint_as_float(r[t + 1]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[buf]);
      return true;
    };
    for (int j = 0; j < nblk; ++j) {
      const int buf = j % NS;
      const uint32_t par = (static_cast<uint32_t>(j / NS)) & 1u;
      if (!mbar_wait(&s_full[buf], par, p.err, kDevTimeoutEpilogue, abortp, kWaitLimitNs,
                     p.sleep_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tmem_base + lane_base + static_cast<uint32_t>(buf * KB);
      const int valid = min(KB, p.kv_len - j * KB);
      // pass 1: row maximum of the (masked) scores; four independent chains
      // of three-input max
      const bool full = valid == KB;
      float mxc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      uint32_t r[32];
#pragma unroll
      for (int ch = 0; ch < Cfg::CHUNKS; ++ch) {
        tmem_ld32(s_addr + ch * 32, r);
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
      const float m_new = fmaxf(m_run, mx * c);
      const float alpha = ex2_approx(m_run - m_new);  // 0 on the first block
      // Fold O_{j-1} (its P.V has then also released P tile (j-1) % NP,
      // which is this block's tile when NP = 1, and O buffer (j-1) % NO).
      if (j >= 1 && !consume_o(j - 1, alpha_prev)) {
        ok = false;
        break;
      }
      // pass 2: P = exp2(c*s - m_new) as 16-bit into the swizzled A tile
      const int pbuf = j % NP;
      uint8_t* pbase = smem + Cfg::P_OFF + pbuf * 2 * Cfg::TILE;
      float sp[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // two packed partial-sum pairs
      const float nm = -m_new;
#pragma unroll
      for (int ch = 0; ch < Cfg::CHUNKS; ++ch) {
        tmem_ld32(s_addr + ch * 32, r);
        tmem_ld_wait();
        float pv[32];
        if (full) {
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            float x0, x1;
            fma2(x0, x1, __uint_as_float(r[t]), __uint_as_float(r[t + 1]), c, c, nm, nm);
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
            const float e = ex2_approx(fmaf(__uint_as_float(r[t]), c, nm));
            pv[t] = ch * 32 + t < valid ? e : 0.0f;
            sp[t & 3] += pv[t];
          }
        }
        // keys [ch*32, ch*32+32): atom ch/2, 16-byte chunks (ch%2)*4 .. +3
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
      const float sum = (sp[0] + sp[1]) + (sp[2] + sp[3]);
      l_run = fmaf(l_run, alpha, sum);
      m_run = m_new;
      tc_fence_before();
      fence_proxy_async_smem();  // P writes -> tensor-core (async proxy) reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_free[buf]);
        mbar_arrive(&p_full[pbuf]);
      }
      alpha_prev = alpha;
    }
    if (ok && nblk > 0) ok = consume_o(nblk - 1, alpha_prev);
    const int qrow = qb * kAttnBlock + row;
    if (ok && qrow < p.q_len) {
      const float inv = 1.0f / l_run;
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.o) +
                     (static_cast<int64_t>(b) * p.o_bstride + static_cast<int64_t>(qrow) * p.ldo +
                      static_cast<int64_t>(h) * kAttnD) * 2;
#pragma unroll
      for (int q = 0; q < kAttnD / 8; ++q)
        reinterpret_cast<uint4*>(dst)[q] =
            make_uint4(pack_16bit(o_acc[8 * q] * inv, o_acc[8 * q + 1] * inv, BF16),
                       pack_16bit(o_acc[8 * q + 2] * inv, o_acc[8 * q + 3] * inv, BF16),
                       pack_16bit(o_acc[8 * q + 4] * inv, o_acc[8 * q + 5] * inv, BF16),
                       pack_16bit(o_acc[8 * q + 6] * inv, o_acc[8 * q + 7] * inv, BF16));
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
constexpr float kAttnRescaleLog2 = 8.0f;

template <int KB_, int ST_, bool PT_ = false>
struct Attn2Cfg {
  static constexpr int KB = KB_;
  static constexpr int KV_STAGES = ST_;
  static constexpr bool PT = PT_;
  static constexpr int TILE = kAttnBlock * 128;          // Q tile / one P atom (64 keys)
  static constexpr int KV_TILE = KB * 128;
  static constexpr int P_ATOMS = PT ? 0 : KB / 64;
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = TILE;
  static constexpr int P_OFF = KV_OFF + KV_STAGES * 2 * KV_TILE;
  static constexpr int BAR_OFF = P_OFF + P_ATOMS * TILE;
  static constexpr int BYTES = BAR_OFF + 256;
  static constexpr uint32_t O_COL = KB;                 // S in [0, KB), O in [KB, KB + 64)
  static constexpr uint32_t TMEM_COLS = KB + 64 <= 128 ? 128 : 256;
  static constexpr int MIN_BLOCKS = PT ? 4 : (KB == 64 ? 3 : 2);
  static constexpr int CHUNKS = KB / 32;
  static_assert(KB == 64 || KB == 128, "key block");
  static_assert(!PT || KB == 64, "P in TMEM: 64-key blocks");
  static_assert((1 + 2 * KV_STAGES + 5) * 8 + 8 <= 256, "barrier area");
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
  uint64_t& s_full = kv_empty[ST];
  uint64_t& s_free = kv_empty[ST + 1];
  uint64_t& p_full = kv_empty[ST + 2];
  uint64_t& o_full = kv_empty[ST + 3];
  uint64_t& drain_bar = kv_empty[ST + 4];
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(&kv_empty[ST + 5]);
  int& abort_flag = *(reinterpret_cast<int*>(&kv_empty[ST + 5]) + 1);
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadConfig);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  // Key blocks over [0, skip_lo) then [skip_hi, kv_len).
  const int nb0 = (p.skip_lo + KB - 1) / KB;
  const int nblk = nb0 + (p.kv_len - p.skip_hi + KB - 1) / KB;
  auto block_start = [&](int j) { return j < nb0 ? j * KB : p.skip_hi + (j - nb0) * KB; };
  auto block_valid = [&](int j) {
    return j < nb0 ? min(KB, p.skip_lo - j * KB) : min(KB, p.kv_len - block_start(j));
  };

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_free, 4);
    mbar_init(&p_full, 4);
    mbar_init(&o_full, 1);
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

  if (warp == 0) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      bool ok = true;
      int issued = 0, stage = 0;
      uint32_t phase = 0;
      mbar_arrive_expect_tx(&q_full, Cfg::TILE);
      tma_load_4d(smem + Cfg::Q_OFF, &tmQ, &q_full, 0, qb * kAttnBlock, h, b);
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
        if (!mbar_wait(&p_full, static_cast<uint32_t>(jj) & 1u, p.err, kDevTimeoutMma, abortp))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + Cfg::KV_OFF + pv_stage * 2 * Cfg::KV_TILE +
                                         Cfg::KV_TILE);
#pragma unroll
        for (int ks = 0; ks < KB / 16; ++ks) {
          const uint64_t bd = make_sw128_desc(v_addr + ks * 2048, 8192, 1024);
          if constexpr (Cfg::PT) {
            umma_f16_tmem_a(tmem_base + Cfg::O_COL, tmem_base + ks * 8, bd, idesc_o,
                            (jj > 0 || ks > 0) ? 1u : 0u);
          } else {
            const uint64_t ad =
                make_sw128_desc(p_addr + (ks >> 2) * Cfg::TILE + (ks & 3) * 32, 16, 1024);
            umma_f16(tmem_base + Cfg::O_COL, ad, bd, idesc_o, (jj > 0 || ks > 0) ? 1u : 0u);
          }
        }
        if (!Cfg::PT || jj == nblk - 1) umma_commit(&o_full);
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
          // P.V_{j-1} first: S_j overwrites the P_{j-1} it reads.
          if (j >= 1 && !issue_pv(j - 1)) {
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
          umma_f16(tmem_base, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
        }
        issued_any = true;
        umma_commit(&s_full);
        if (++stage == ST) {
          stage = 0;
          phase ^= 1u;
        }
        if (!Cfg::PT && j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && nblk > 0 && !issue_pv(nblk - 1)) ok = false;
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
    for (int j = 0; j < nblk; ++j) {
      // Waits end the loop for the whole warp together: the TMEM loads and
      // stores that follow are warp-collective.
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full, static_cast<uint32_t>(j) & 1u, p.err,
                                             kDevTimeoutEpilogue, abortp))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int valid = block_valid(j);
      const bool full = valid == KB;
      float mxc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int ch = 0; ch < Cfg::CHUNKS; ++ch) {
        tmem_ld32(s_addr + ch * 32, r);
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
      // P.V of the previous block must be done: it reads the P tile this block
      // overwrites, and its sum is in the O rows a rescale touches.
      // (With P in TMEM the score barrier already covers P.V of the previous block.)
      if (j >= 1) {
        if (!Cfg::PT &&
            !__all_sync(0xffffffffu, mbar_wait(&o_full, static_cast<uint32_t>(j - 1) & 1u, p.err,
                                               kDevTimeoutEpilogue, abortp))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tmem_ld32(o_addr + half * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
            tmem_st32(o_addr + half * 32, r);
          }
          tmem_st_wait();
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
        tmem_ld32(s_addr + ch * 32, r);
        tmem_ld_wait();
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
          tmem_st16(s_addr + ch * 16, pk);
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
      if constexpr (Cfg::PT) tmem_st_wait();
      tc_fence_before();
      if constexpr (!Cfg::PT) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if constexpr (!Cfg::PT) mbar_arrive(&s_free);
        mbar_arrive(&p_full);
      }
    }
    // With P in TMEM only the last P.V signals o_full (phase 0).
    if (ok && nblk > 0)
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&o_full, Cfg::PT ? 0u : static_cast<uint32_t>(nblk - 1) & 1u,
                                p.err, kDevTimeoutEpilogue, abortp));
    const int qrow = qb * kAttnBlock + row;
    if (ok) {
      tc_fence_after();
      const bool live = qrow < p.q_len;
      const int64_t prow = (static_cast<int64_t>(b) * p.q_len + qrow) * p.heads + h;
      // Merge with a partial result over other keys: both bases are integers,
      // so the rescale factors are exact powers of two.
      float a_own = 1.0f, a_part = 0.0f;
      if (p.part_mode == 2 && live) {
        const float m_p = p.part_ml[2 * prow], l_p = p.part_ml[2 * prow + 1];
        const float m = fmaxf(m_run, m_p);
        a_own = nblk > 0 ? ex2_approx(m_run - m) : 0.0f;
        a_part = ex2_approx(m_p - m);
        l_run = (nblk > 0 ? l_run * a_own : 0.0f) + l_p * a_part;
      }
      if (p.part_mode == 1 && live) {
        p.part_ml[2 * prow] = m_run;
        p.part_ml[2 * prow + 1] = l_run;
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
        if (p.part_mode == 1) {
          float4* po = reinterpret_cast<float4*>(p.part_o + prow * kAttnD + half * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            po[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
          continue;
        }
        float ov[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) ov[t] = nblk > 0 ? __uint_as_float(r[t]) : 0.0f;
        if (p.part_mode == 2) {
          const float4* po = reinterpret_cast<const float4*>(p.part_o + prow * kAttnD + half * 32);
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

}  // namespace sf
