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
};

constexpr int kAttnBlock = 128;   // queries per CTA and keys per block
constexpr int kAttnD = 64;        // head dim
constexpr int kAttnThreads = 192;

// Buffering: SB = 2 double-buffers the scores (TMEM) and P (shared memory)
// with a 4-stage K/V ring (one CTA per SM, 512 TMEM columns); SB = 1
// single-buffers them with a 2-stage ring so that two CTAs share an SM
// (256 TMEM columns and ~113 KB of shared memory each), the second CTA's
// MMAs and softmax filling the first one's gaps.
template <int SB>
struct AttnCfg {
  static constexpr int KV_STAGES = SB == 2 ? 4 : 2;
  static constexpr int TILE = kAttnBlock * 128;          // 128 rows x 128 B = 16 KB
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = TILE;                    // stage s: K at +2s*TILE, V at +(2s+1)*TILE
  static constexpr int P_OFF = KV_OFF + KV_STAGES * 2 * TILE;  // SB buffers x 2 atoms
  static constexpr int BAR_OFF = P_OFF + SB * 2 * TILE;        // mbarriers and flags
  static constexpr int BYTES = BAR_OFF + 256;
  static constexpr uint32_t TMEM_COLS = SB == 2 ? 512 : 256;
  static constexpr uint32_t O_COL = 128 * SB;            // two 64-column O buffers follow S
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_16bit(float a, float b, bool bf16) {
  if (bf16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <bool BF16, int SB>
__global__ void __launch_bounds__(kAttnThreads, SB == 1 ? 2 : 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
  // All shared memory is dynamic (no static part), declared 1024-byte
  // aligned for the 128B-swizzled tiles; the mbarriers sit after the tiles.
  extern __shared__ __align__(1024) uint8_t smem[];
  using Cfg = AttnCfg<SB>;
  constexpr int ST = Cfg::KV_STAGES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t& q_full = bars[0];
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* s_full = kv_empty + ST;
  uint64_t* s_free = s_full + SB;
  uint64_t* p_full = s_free + SB;
  uint64_t* o_full = p_full + SB;
  uint64_t* o_free = o_full + 2;
  uint64_t& drain_bar = o_free[2];
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(&o_free[3]);
  int& abort_flag = *(reinterpret_cast<int*>(&o_free[3]) + 1);
  static_assert((1 + 2 * ST + 3 * SB + 4 + 2) * 8 <= 256, "barrier area");
  if ((smem_u32(smem) & 1023u) != 0) {
    // The swizzled tile layout needs 1024-byte alignment; never guess.
    if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadConfig);
    return;
  }

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nblk = (p.kv_len + kAttnBlock - 1) / kAttnBlock;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < SB; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
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
  // TMEM columns: S buffers [0, 128*SB), then two 64-column O buffers.

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
        uint8_t* kt = smem + Cfg::KV_OFF + stage * 2 * Cfg::TILE;
        mbar_arrive_expect_tx(&kv_full[stage], 2 * Cfg::TILE);
        tma_load_4d(kt, &tmK, &kv_full[stage], 0, j * kAttnBlock, h, b);
        tma_load_4d(kt + Cfg::TILE, &tmV, &kv_full[stage], 0, j * kAttnBlock, h, b);
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
      const uint32_t idesc_s = make_idesc(fmt, 128, 128, 0u, 0u);  // K-major A and B
      const uint32_t idesc_o = make_idesc(fmt, 128, 64, 0u, 1u);   // P K-major, V MN-major
      const uint32_t q_addr = smem_u32(smem + Cfg::Q_OFF);
      bool ok = mbar_wait(&q_full, 0, p.err, kDevTimeoutMma, abortp);
      bool issued_any = false;
      int stage = 0;
      uint32_t phase = 0;
      int pv_stage = 0;
      auto issue_pv = [&](int jj) -> bool {
        const int pb = jj % SB;
        const uint32_t ppar = (static_cast<uint32_t>(jj / SB)) & 1u;
        const int ob = jj & 1;
        const uint32_t opar = (static_cast<uint32_t>(jj) >> 1) & 1u;
        if (!mbar_wait(&p_full[pb], ppar, p.err, kDevTimeoutMma, abortp)) return false;
        if (!mbar_wait(&o_free[ob], opar ^ 1u, p.err, kDevTimeoutMma, abortp)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + Cfg::P_OFF + pb * 2 * Cfg::TILE);
        const uint32_t v_addr = smem_u32(smem + Cfg::KV_OFF + pv_stage * 2 * Cfg::TILE +
                                         Cfg::TILE);
        const uint32_t d_tmem = tmem_base + Cfg::O_COL + static_cast<uint32_t>(ob * 64);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
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
        const int buf = j % SB;
        const uint32_t par = (static_cast<uint32_t>(j / SB)) & 1u;
        if (!mbar_wait(&kv_full[stage], phase, p.err, kDevTimeoutMma, abortp) ||
            !mbar_wait(&s_free[buf], par ^ 1u, p.err, kDevTimeoutMma, abortp)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + Cfg::KV_OFF + stage * 2 * Cfg::TILE);
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * 128);
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
      const int buf = jj & 1;
      const uint32_t par = (static_cast<uint32_t>(jj) >> 1) & 1u;
      if (!mbar_wait(&o_full[buf], par, p.err, kDevTimeoutEpilogue, abortp)) return false;
      tc_fence_after();
      uint32_t r[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem_base + lane_base + Cfg::O_COL + static_cast<uint32_t>(buf * 64 + half * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t)
          o_acc[half * 32 + t] = fmaf(o_acc[half * 32 + t], alpha, __uint_as_float(r[t]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[buf]);
      return true;
    };
    for (int j = 0; j < nblk; ++j) {
      const int buf = j % SB;
      const uint32_t par = (static_cast<uint32_t>(j / SB)) & 1u;
      if (!mbar_wait(&s_full[buf], par, p.err, kDevTimeoutEpilogue, abortp)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tmem_base + lane_base + static_cast<uint32_t>(buf * 128);
      const int valid = min(kAttnBlock, p.kv_len - j * kAttnBlock);
      // pass 1: row maximum of the (masked) scores
      float mx = -INFINITY;
      uint32_t r[32];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        tmem_ld32(s_addr + ch * 32, r);
        tmem_ld_wait();
        if (valid == kAttnBlock) {
#pragma unroll
          for (int t = 0; t < 32; ++t) mx = fmaxf(mx, __uint_as_float(r[t]));
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (ch * 32 + t < valid) mx = fmaxf(mx, __uint_as_float(r[t]));
        }
      }
      const float m_new = fmaxf(m_run, mx * c);
      const float alpha = ex2_approx(m_run - m_new);  // 0 on the first block
      // Fold O_{j-1} (its P.V has then also released P buffer (j-1) % SB,
      // which is this block's buffer when SB = 1).
      if (j >= 1 && !consume_o(j - 1, alpha_prev)) {
        ok = false;
        break;
      }
      // pass 2: P = exp2(c*s - m_new) as 16-bit into the swizzled A tile
      uint8_t* pbase = smem + Cfg::P_OFF + buf * 2 * Cfg::TILE;
      float sum = 0.0f;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        tmem_ld32(s_addr + ch * 32, r);
        tmem_ld_wait();
        float pv[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const float e = ex2_approx(fmaf(__uint_as_float(r[t]), c, -m_new));
          pv[t] = (valid == kAttnBlock || ch * 32 + t < valid) ? e : 0.0f;
          sum += pv[t];
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
      l_run = fmaf(l_run, alpha, sum);
      m_run = m_new;
      tc_fence_before();
      fence_proxy_async_smem();  // P writes -> tensor-core (async proxy) reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_free[buf]);
        mbar_arrive(&p_full[buf]);
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

}  // namespace sf
