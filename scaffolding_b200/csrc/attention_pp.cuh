// Fused attention forward, head_dim 64, NT query tiles of 128 rows per CTA
// sharing every K/V block.
//
//   O[b, :, h] = softmax(scale * Q[b, :, h] K[b, :, h]^T) V[b, :, h]
//
// A CTA works on a unit of NT * 128 query rows of one (head, batch): tiles
// t = 0 .. NT-1 that share every block of KB keys.  NT * 4 + 2 warps:
//   warps 4t .. 4t+3   softmax of tile t, one thread per query row (TMEM lane);
//   warp 4 NT          TMA producer: the Q tiles once, then K and V blocks of
//                      KB keys into a KV_STAGES-deep ring (K-major 128B-swizzled
//                      tiles; V's tile is the MN-major B operand of P.V);
//   warp 4 NT + 1      TMEM owner and MMA issuer.
// TMEM: S_t (fp32 scores) in columns [t KB, (t+1) KB), O_t (fp32 output
// accumulator) in [NT KB + 64 t, NT KB + 64 (t+1)); a CTA allocates 256 or
// 512 columns, so two or one CTAs share an SM.  The engine's configuration
// is NT = 2, KB = 64: 256 columns and ~96 KB of shared memory, two CTAs
// (four tiles, sixteen softmax warps) per SM, each K/V block loaded once
// for two tiles.  Measured on B200 it is the fastest of the shapes tried:
// one CTA per SM with two tiles of 128-key blocks (eight softmax warps per
// SM) leaves the softmax warps latency-bound, and four tiles per CTA queue
// behind the single MMA thread.
//
// For each tile t and key block j the MMA thread issues
//     O_t += P_t(j-1) V(j-1),  S_t(j) = Q_t K(j)^T
// as soon as P_t(j-1) is stored and K/V block j is loaded (tiles in any order),
// where P_t(j-1) is the 16-bit probability block the softmax warps of tile t
// stored over the first KB/2 columns of S_t (two values per 32-bit column)
// and P.V reads its A operand from TMEM.  tcgen05.mma instructions of one
// thread execute in issue order, so S_t(j) overwrites P_t(j-1) only after P.V
// has read it, and the commit that signals S_t(j) also covers
// O_t += P_t(j-1) V: the softmax warps of a tile wait on one barrier per
// block and find O_t final whenever their score block is ready.  While the
// tensor core works on one tile's products, the other tiles' softmax warps
// run, so the exp2 unit (16 results per clock per SM, twice the
// tensor-core time per score at head_dim 64) and the tensor core overlap.
//
// Softmax (per row, log2 domain, c = scale * log2(e)): the row's integer
// exponent base m is set by its first block (ceil(c * max)).  After that a
// warp works sum-first: p = 2^(c s - m) is formed with the current base
// (packed to 16 bits as it is formed, stored after the checks), and the base
// changes only when a block's p sum to kAttnSumLimit (2^8) or more: m then
// rises by k = floor(log2 sum) + 1, taken from the sum's exponent bits, and
// the block's p, packed P and sum, the row's l and its row of O_t in TMEM all
// scale by the exact power of two 2^-k (O: warp-collective load, multiply,
// store; factor 1 on the warp's other rows).  No row max is computed.  A sum
// too large to scale that way, or not finite (huge or non-finite scores),
// switches the warp to max-first for the rest of its unit: the scores are
// read from TMEM again, and from then on every block takes the row max first
// and raises m to ceil(c * max) only when that exceeds m by more than
// kAttnRescaleLog2.  Because m is an integer, the 16-bit rounding of p does
// not depend on which base is in force (a change of base is an exact
// power-of-two scale), and every stored p is below 2^8.

// Tiles of a unit that hold no query rows (past q_len) are skipped.  Keys
// past kv_len (TMA zero-fills them) and skipped keys are masked to p = 0;
// query rows past q_len are computed and not stored.  The partial modes,
// key-range skips and stream-K tail parts are those of AttnArgs, with units
// of NT * 128 rows (ws_o is [slot][NT * 128][64]).
//
// Every wait is bounded (global timer): an expired wait records an error
// code in the device error word, the CTA drains its copies and MMAs and
// exits, so a broken pipeline returns a status instead of hanging.
#pragma once
#include "attention.cuh"

namespace sf {

template <int NT_, int KB_, int ST_>
struct AttnPpCfg {
  static constexpr int NT = NT_;                        // query tiles of 128 rows per CTA
  static constexpr int KB = KB_;                        // keys per block
  static constexpr int KV_STAGES = ST_;
  static constexpr int ROWS = NT * 128;                 // query rows per unit
  static constexpr int THREADS = (4 * NT + 2) * 32;
  static constexpr int TMA_WARP = 4 * NT;
  static constexpr int MMA_WARP = 4 * NT + 1;
  static constexpr int CHUNKS = KB / 32;                // 32-score chunks per block
  static constexpr int Q_TILE = 128 * 128;              // 128 rows x 128 B
  static constexpr int KV_TILE = KB * 128;              // KB keys x 128 B
  static constexpr int Q_OFF = 0;                       // tile t at Q_OFF + t * Q_TILE
  static constexpr int KV_OFF = NT * Q_TILE;            // stage s: K, then V
  static constexpr int BAR_OFF = KV_OFF + KV_STAGES * 2 * KV_TILE;
  static constexpr int BYTES = BAR_OFF + 512;
  static constexpr uint32_t S_COL = 0;                  // S_t at t * KB
  static constexpr uint32_t O_COL = NT * KB;            // O_t at O_COL + t * 64
  static constexpr uint32_t TMEM_COLS = NT * (KB + 64) <= 256 ? 256 : 512;
  static constexpr int MIN_BLOCKS = 512 / TMEM_COLS;    // CTAs per SM the TMEM allows
  static_assert(KB == 64 || KB == 128, "key block");
  static_assert(NT * (KB + 64) <= 512, "TMEM budget");
  static_assert(KV_TILE % 1024 == 0 && KV_OFF % 1024 == 0, "1024-byte aligned tiles");
  static_assert((1 + 2 * KV_STAGES + 3 * NT + 2) * 8 + 8 <= 512, "barrier area");
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

// One segment of a CTA's work: query rows [qb * ROWS, +ROWS) of head h,
// batch b, and the unit's effective key blocks [ea, eb) -- block i < nkb_a
// starts at key i * KB, block i >= nkb_a at skip_hi + (i - nkb_a) * KB --
// as nblk blocks [k0, e0) then [s1, k1), KB keys each.  slot >= 0: a part of
// a split tail unit, written to workspace slot `slot`.
template <int KB>
struct PpSeg {
  int qb, h, b, slot, k0, e0, s1, k1, nb0, nblk;
  __device__ __forceinline__ int start(int j) const { return j < nb0 ? k0 + j * KB : s1 + (j - nb0) * KB; }
  __device__ __forceinline__ int valid(int j) const { return min(KB, (j < nb0 ? e0 : k1) - start(j)); }
};

// Segments of tail CTA blockIdx.x: one or two (its block range is at most one
// unit long, so it meets at most two units; none when the range is empty).
__device__ __forceinline__ int pp_nseg(const AttnArgs& p) {
  const int c = static_cast<int>(blockIdx.x);
  const int64_t lo = attn_tail_lo(p, c), hi = attn_tail_lo(p, c + 1);
  if (hi <= lo) return 0;
  return static_cast<int>((hi - 1) / p.nkb_e - lo / p.nkb_e) + 1;
}

// Segment i of tail CTA blockIdx.x: a part (or the whole) of tail unit
// split_first + ur, effective key blocks [ea, eb).
template <int KB>
__device__ __forceinline__ PpSeg<KB> pp_tail_seg(const AttnArgs& p, int i) {
  PpSeg<KB> w;
  const int c = static_cast<int>(blockIdx.x);
  const int64_t lo = attn_tail_lo(p, c), hi = attn_tail_lo(p, c + 1);
  const int64_t ur = lo / p.nkb_e + i, u0 = ur * p.nkb_e;
  const int ea = static_cast<int>(max(lo, u0) - u0);
  const int eb = static_cast<int>(min(hi, u0 + p.nkb_e) - u0);
  const int u = p.split_first + static_cast<int>(ur);
  w.slot = (ea > 0 || eb < p.nkb_e) ? 2 * c + i : -1;
  w.qb = u % p.nqb;
  w.h = (u / p.nqb) % p.heads;
  w.b = u / (p.nqb * p.heads);
  const int na = p.nkb_a;
  w.nb0 = max(0, min(eb, na) - ea);
  w.k0 = ea * KB;
  w.e0 = min(min(eb, na) * KB, p.skip_lo);
  w.s1 = p.skip_hi + (max(ea, na) - na) * KB;
  w.k1 = min(p.kv_len, p.skip_hi + (eb - na) * KB);
  w.nblk = eb - ea;
  return w;
}

// A whole unit: the 3-D grid (query unit, head, batch), or unit blockIdx.x
// of the 1-D grid of the first split_first units when a stream-K tail runs
// the rest; every key but [skip_lo, skip_hi).
template <int KB>
__device__ __forceinline__ PpSeg<KB> pp_unit(const AttnArgs& p) {
  PpSeg<KB> w;
  if (p.split_first < 0) {
    w.qb = blockIdx.x;
    w.h = blockIdx.y;
    w.b = blockIdx.z;
  } else {
    const int u = static_cast<int>(blockIdx.x);
    w.qb = u % p.nqb;
    w.h = (u / p.nqb) % p.heads;
    w.b = u / (p.nqb * p.heads);
  }
  w.slot = -1;
  w.k0 = 0;
  w.k1 = p.kv_len;
  w.e0 = min(w.k1, p.skip_lo);
  w.s1 = max(w.k0, p.skip_hi);
  w.nb0 = w.e0 > w.k0 ? (w.e0 - w.k0 + KB - 1) / KB : 0;
  w.nblk = w.nb0 + (w.k1 > w.s1 ? (w.k1 - w.s1 + KB - 1) / KB : 0);
  return w;
}

// Query tiles of a segment that hold rows (past q_len they are skipped; a
// unit is never empty).
template <class Cfg, int KB>
__device__ __forceinline__ int pp_tiles(const AttnArgs& p, const PpSeg<KB>& w) {
  return min(Cfg::NT, (p.q_len - w.qb * Cfg::ROWS + 127) / 128);
}

// The softmax warps' part of a unit (or of a segment of one), one query row
// per thread: key blocks 0 .. nblk-1 of w, sum-first then max-first as the
// header describes.  s_full_t / p_full_t: the tile's score-ready and
// P-stored barriers, with sbase phases completed before this segment;
// s_addr / o_addr: the warp's score and output columns in TMEM; r: scratch
// registers (at least 64).  m_run and l_run end as the row's base and sum.
// Returns false when a wait expired.
template <bool BF16, int KB, int CHUNKS>
__device__ __forceinline__ bool pp_softmax_rows(const AttnArgs& p, const PpSeg<KB>& w, int nblk,
                                                int sbase, uint64_t* s_full_t, uint64_t* p_full_t,
                                                uint32_t s_addr, uint32_t o_addr, int lane,
                                                volatile int* abortp, float& m_run, float& l_run,
                                                uint32_t* r) {
  const float c = p.scale_log2;
  bool ok = true;
  // O row scaling by alpha (warp-collective; factor 1 on the warp's other rows).
  auto rescale_o = [&](float alpha) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      tmem_ld32(o_addr + half * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
      tmem_st32(o_addr + half * 32, r);
    }
  };
  // P of a block: keys 2i, 2i+1 packed in pk[i]; sp: partial row sums.
  uint32_t pk[KB / 2];
  float sp[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
  auto row_sum = [&]() {
    return ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
  };
  // p = 2^(c s - m) of the block's valid keys, from the scores in r.
  auto p_block = [&](float nm, int valid) {
    if (valid == KB) {
#pragma unroll
      for (int i = 0; i < KB; i += 2) {
        float x0, x1, e0, e1;
        fma2(x0, x1, __uint_as_float(r[i]), __uint_as_float(r[i + 1]), c, c, nm, nm);
        e0 = ex2_approx(x0);
        e1 = ex2_approx(x1);
        if ((i & 2) == 0 && i < 16) {  // first keys of each pair of sums
          sp[(i >> 1) & 6] = e0;
          sp[((i >> 1) & 6) + 1] = e1;
        } else {
          add2(sp[(i >> 1) & 6], sp[((i >> 1) & 6) + 1], e0, e1);
        }
        pk[i >> 1] = pack_16bit(e0, e1, BF16);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) sp[i] = 0.0f;
#pragma unroll
      for (int i = 0; i < KB; i += 2) {
        const float e0 = i < valid ? ex2_approx(fmaf(__uint_as_float(r[i]), c, nm)) : 0.0f;
        const float e1 = i + 1 < valid ? ex2_approx(fmaf(__uint_as_float(r[i + 1]), c, nm)) : 0.0f;
        sp[i & 7] += e0;
        sp[(i + 1) & 7] += e1;
        pk[i >> 1] = pack_16bit(e0, e1, BF16);
      }
    }
  };
  // Waits end the loop for the whole warp together: the TMEM loads and
  // stores that follow are warp-collective.
  auto wait_scores = [&](int j) -> bool {
    if (!__all_sync(0xffffffffu, mbar_wait(s_full_t, static_cast<uint32_t>(sbase + j) & 1u, p.err,
                                           kDevTimeoutEpilogue, abortp)))
      return false;
    tc_fence_after();
    return true;
  };
  auto load_scores = [&]() {
#pragma unroll
    for (int ch = 0; ch < CHUNKS; ++ch) tmem_ld32(s_addr + ch * 32, r + ch * 32);
    tmem_ld_wait();
  };
  // Max-first block: the row max; the base rises to ceil(c * max) when that
  // exceeds it by more than kAttnRescaleLog2 (always on the first block);
  // then p.  Returns whether some row of the warp raised its base.
  auto max_first = [&](int j, int valid, float& alpha) -> bool {
    float mx;
    if (valid == KB) {
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < KB; i += 8) {
        m4[0] = max3f(m4[0], __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
        m4[1] = max3f(m4[1], __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
        m4[2] = max3f(m4[2], __uint_as_float(r[i + 4]), __uint_as_float(r[i + 5]));
        m4[3] = max3f(m4[3], __uint_as_float(r[i + 6]), __uint_as_float(r[i + 7]));
      }
      mx = max3f(m4[0], m4[1], fmaxf(m4[2], m4[3]));
    } else {
      mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < KB; ++i)
        if (i < valid) mx = fmaxf(mx, __uint_as_float(r[i]));
    }
    const float cand = ceilf(mx * c);
    const bool need = cand > m_run + kAttnRescaleLog2;  // always on the first block
    alpha = need ? ex2_approx(m_run - cand) : 1.0f;
    const bool raised = j >= 1 && __any_sync(0xffffffffu, need);
    if (need) {
      l_run *= alpha;
      m_run = cand;
    }
    p_block(-m_run, valid);
    return raised;
  };
  // Store P over the scores already read (keys ch*32 + 2i, +2i+1 in column
  // ch*16 + i), add the block to l, rescale O if a base rose, and hand P to
  // the MMA warp: O_t is final up to P_t(j-1) V (S_t(j)'s barrier covers it)
  // and P_t(j) V is issued only after the arrival.
  auto finish = [&](bool raised, float alpha, float sum) {
#pragma unroll
    for (int ch = 0; ch < CHUNKS; ++ch) tmem_st16(s_addr + ch * 16, pk + ch * 16);
    l_run += sum;
    if (raised) rescale_o(alpha);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_full_t);
  };
  int j = 0;
  // Sum-first blocks: the first block max-first, then p with the current base
  // (no row max).  Leaves for the max-first loop below at the first block
  // whose sum is too large to scale by a power of two (or infinite).
  for (; j < nblk; ++j) {
    if (!wait_scores(j)) {
      ok = false;
      break;
    }
    load_scores();
    const int valid = w.valid(j);
    float alpha = 1.0f;
    bool raised = false, leave = false;
    float sum = 0.0f;  // the block's row sum as stored
    if (j == 0) {
      raised = max_first(j, valid, alpha);
      sum = row_sum();
    } else {
      p_block(-m_run, valid);
      const float bs = row_sum();
      sum = bs;
      if (!__all_sync(0xffffffffu, bs < kAttnSumLimit)) {
        // A NaN sum (non-finite scores) raises nothing: its row is NaN anyway.
        if (__all_sync(0xffffffffu, bs < (BF16 ? 0x1p120f : 0x1p15f) || bs != bs)) {
          const bool need = bs >= kAttnSumLimit;
          const int k = need ? static_cast<int>((__float_as_uint(bs) >> 23) & 0xffu) - 126 : 0;
          alpha = __uint_as_float(static_cast<uint32_t>(127 - k) << 23);
          raised = __any_sync(0xffffffffu, need);
          if (need) {
            l_run *= alpha;
            m_run += static_cast<float>(k);
          }
          sum = bs * alpha;  // exact: alpha is a power of two (1 where no row raised)
          if (raised) {
            const uint32_t a2 = pack_16bit(alpha, alpha, BF16);
#pragma unroll
            for (int i = 0; i < KB / 2; ++i) pk[i] = mul_16bit2(pk[i], a2, BF16);
          }
        } else {
          load_scores();
          raised = max_first(j, valid, alpha);
          sum = row_sum();
          leave = true;
        }
      }
    }
    finish(raised, alpha, sum);
    if (leave) {
      ++j;
      break;
    }
  }
  // Max-first blocks: the rest of the unit after a sum too large to scale.
  for (; ok && j < nblk; ++j) {
    if (!wait_scores(j)) {
      ok = false;
      break;
    }
    load_scores();
    float alpha = 1.0f;
    const bool raised = max_first(j, w.valid(j), alpha);
    const float sum = row_sum();
    finish(raised, alpha, sum);
  }
  return ok;
}

// The output rows of a finished unit (or segment), one query row per
// thread, O read from TMEM: normalised 16-bit O (mode 0), merged first with
// the partial result over other keys (mode 2), or the unnormalised fp32 O
// with the row's (m, l) as a partial result (mode 1, and every part of a
// split tail unit, which writes its workspace slot).
template <bool BF16, class Cfg, int KB>
__device__ __forceinline__ void pp_write_rows(const AttnArgs& p, const PpSeg<KB>& w, int t, int row,
                                              uint32_t o_addr, float m_run, float l_run, int nblk,
                                              uint32_t* r) {
  const int qrow = w.qb * Cfg::ROWS + t * 128 + row;
  const bool live = qrow < p.q_len;
  const int64_t prow = (static_cast<int64_t>(w.b) * p.q_len + qrow) * p.heads + w.h;
  // A part of a split unit writes its partial result to its workspace slot.
  const int mode = w.slot >= 0 ? 1 : p.part_mode;
  const int urow = t * 128 + row;
  float* const pml = w.slot >= 0 ? p.ws_ml + (static_cast<int64_t>(w.slot) * Cfg::ROWS + urow) * 2
                                 : p.part_ml + 2 * prow;
  float* const pob = w.slot >= 0
                         ? p.ws_o + (static_cast<int64_t>(w.slot) * Cfg::ROWS + urow) * kAttnD
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
                 (static_cast<int64_t>(w.b) * p.o_bstride + static_cast<int64_t>(qrow) * p.ldo +
                  static_cast<int64_t>(w.h) * kAttnD) * 2;
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
    for (int i = 0; i < 32; ++i) ov[i] = nblk > 0 ? __uint_as_float(r[i]) : 0.0f;
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

// Whole units, one per CTA (pp_unit).  When a stream-K tail runs, this is
// launched after the tail kernel with programmatic stream serialisation and
// takes the SM slots the tail CTAs leave; it reads nothing they write.
template <bool BF16, class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, Cfg::MIN_BLOCKS)
    attention_pp_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int ST = Cfg::KV_STAGES, NT = Cfg::NT, KB = Cfg::KB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t& q_full = bars[0];
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* s_full = kv_empty + ST;   // [NT]: S_t(j) ready (covers O_t += P_t(j-1) V)
  uint64_t* p_full = s_full + NT;     // [NT]: P_t(j) stored (4 warp arrivals)
  uint64_t* o_last = p_full + NT;     // [NT]: the last P.V of tile t done
  uint64_t& drain_bar = o_last[NT];
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(&o_last[NT + 1]);
  int& abort_flag = *(reinterpret_cast<int*>(&o_last[NT + 1]) + 1);
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadConfig);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const PpSeg<KB> w = pp_unit<KB>(p);
  const int nblk = w.nblk;
  // Only tiles that hold query rows run (the unit is never empty).
  const int ntiles = min(NT, (p.q_len - w.qb * Cfg::ROWS + 127) / 128);

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_last[t], 1);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == Cfg::TMA_WARP && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == Cfg::MMA_WARP) {
    tmem_alloc(&tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  volatile int* abortp = &abort_flag;

  if (warp == Cfg::TMA_WARP) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      bool ok = true;
      int issued = 0, stage = 0;
      uint32_t phase = 0;
      mbar_arrive_expect_tx(&q_full, ntiles * Cfg::Q_TILE);
      for (int t = 0; t < ntiles; ++t)
        tma_load_4d(smem + Cfg::Q_OFF + t * Cfg::Q_TILE, &tmQ, &q_full, 0,
                    w.qb * Cfg::ROWS + t * 128, w.h, w.b);
      for (int j = 0; j < nblk; ++j) {
        if (!mbar_wait(&kv_empty[stage], phase ^ 1u, p.err, kDevTimeoutProducer, abortp)) {
          ok = false;
          break;
        }
        uint8_t* kt = smem + Cfg::KV_OFF + stage * 2 * Cfg::KV_TILE;
        mbar_arrive_expect_tx(&kv_full[stage], 2 * Cfg::KV_TILE);
        const int ks = w.start(j);
        tma_load_4d(kt, &tmK, &kv_full[stage], 0, ks, w.h, w.b);
        tma_load_4d(kt + Cfg::KV_TILE, &tmV, &kv_full[stage], 0, ks, w.h, w.b);
        ++issued;
        if (++stage == ST) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!mbar_wait_quiet(&q_full, 0, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
      if (!ok) {
        // Wait for the copies still in flight before the CTA exits.
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
  } else if (warp == Cfg::MMA_WARP) {
    // ───────────── MMA issuer ─────────────
    // Tiles are served out of order: whenever tile t's P for block j-1 is
    // stored and block j's K/V are loaded, O_t += P_t(j-1) V(j-1) and
    // S_t(j) are issued for it, whatever the other tiles are doing, so a
    // slow tile never holds back the others.  A K/V stage is released once
    // every running tile has issued its P.V on it (the commit covers all
    // MMAs issued before it).  Tiles can drift apart by up to KV_STAGES-1
    // blocks; the producer refills stages in block order.
    if (lane == 0) {
      const uint32_t fmt = BF16 ? 1u : 0u;
      const uint32_t idesc_s = make_idesc(fmt, 128, KB, 0u, 0u);
      const uint32_t idesc_o = make_idesc(fmt, 128, 64, 0u, 1u);
      bool ok = nblk == 0 || mbar_wait(&q_full, 0, p.err, kDevTimeoutMma, abortp);
      bool issued_any = false;
      int jt[NT];                 // next block each tile issues S for (P.V of jt-1 with it)
      int pv_done[ST];            // tiles that have issued their P.V on each stage's block
#pragma unroll
      for (int t = 0; t < NT; ++t) jt[t] = 0;
#pragma unroll
      for (int s2 = 0; s2 < ST; ++s2) pv_done[s2] = 0;
      int finished = 0;
      unsigned long long t_last = 0;  // start of the current idle period
      int idle = 0;
      while (ok && finished < ntiles) {
        bool progress = false;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t >= ntiles) continue;
          const int j = jt[t];
          if (j > nblk) continue;
          if (j > 0 && !mbar_test(&p_full[t], static_cast<uint32_t>(j - 1) & 1u)) continue;
          if (j < nblk && !mbar_test(&kv_full[j % ST], static_cast<uint32_t>(j / ST) & 1u)) continue;
          tc_fence_after();
          if (j > 0) {
            // O_t += P_t(j-1) V(j-1), P from TMEM, V MN-major from its stage.
            const int ps = (j - 1) % ST;
            const uint32_t v_addr = smem_u32(smem + Cfg::KV_OFF + ps * 2 * Cfg::KV_TILE + Cfg::KV_TILE);
#pragma unroll
            for (int ks = 0; ks < KB / 16; ++ks) {
              const uint64_t bd = make_sw128_desc(v_addr + ks * 2048, Cfg::KV_TILE, 1024);
              umma_f16_tmem_a(tmem_base + Cfg::O_COL + t * 64,
                              tmem_base + Cfg::S_COL + t * KB + ks * 8, bd, idesc_o,
                              (j > 1 || ks > 0) ? 1u : 0u);
            }
            if (++pv_done[ps] == ntiles) {
              pv_done[ps] = 0;
              umma_commit(&kv_empty[ps]);
            }
            if (j == nblk) umma_commit(&o_last[t]);
          }
          if (j < nblk) {
            const uint32_t q_addr = smem_u32(smem + Cfg::Q_OFF + t * Cfg::Q_TILE);
            const uint32_t k_addr = smem_u32(smem + Cfg::KV_OFF + (j % ST) * 2 * Cfg::KV_TILE);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t ad = make_sw128_desc(q_addr + ks * 32, 16, 1024);
              const uint64_t bd = make_sw128_desc(k_addr + ks * 32, 16, 1024);
              umma_f16(tmem_base + Cfg::S_COL + t * KB, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
            }
            issued_any = true;
            umma_commit(&s_full[t]);
          }
          jt[t] = j + 1;
          if (j == nblk) ++finished;
          progress = true;
        }
        if (progress) {
          idle = 0;
        } else {
          // Nothing ready: back off briefly (the thread shares its scheduler
          // with softmax warps) and check the abort flag and the time limit
          // every 16 idle passes.
          if (idle == 0) t_last = global_timer_ns();
          if ((++idle & 15) == 0) {
            if (*abortp) {
              ok = false;
            } else if (global_timer_ns() - t_last > kWaitLimitNs) {
              *abortp = 1;
              atomicCAS(p.err, 0, kDevTimeoutMma);
              ok = false;
            }
          }
          __nanosleep(20);
        }
      }
      if (!ok && issued_any) {
        umma_commit(&drain_bar);
        if (!mbar_wait_quiet(&drain_bar, 0, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
      }
    }
  } else if ((warp >> 2) < ntiles) {
    // ───────────── softmax of tile t: one thread per query row ─────────────
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;                 // row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_base + Cfg::S_COL + t * KB;
    const uint32_t o_addr = tmem_base + lane_base + Cfg::O_COL + t * 64;
    float m_run = -INFINITY, l_run = 0.0f;  // m_run: integer-valued base (log2 domain)
    uint32_t r[KB > 64 ? KB : 64];
    bool ok = pp_softmax_rows<BF16, KB, Cfg::CHUNKS>(p, w, nblk, 0, &s_full[t], &p_full[t], s_addr,
                                                     o_addr, lane, abortp, m_run, l_run, r);
    if (ok && nblk > 0)
      ok = __all_sync(0xffffffffu, mbar_wait(&o_last[t], 0u, p.err, kDevTimeoutEpilogue, abortp));
    if (ok) {
      tc_fence_after();
      pp_write_rows<BF16, Cfg>(p, w, t, row, o_addr, m_run, l_run, nblk, r);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == Cfg::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Stream-K tail CTA blockIdx.x: one or two segments (pp_nseg, pp_tail_seg)
// through the same barriers.  Launched before the whole units' kernel, which
// it lets start at once (its CTAs take the slots this kernel leaves).
template <bool BF16, class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, Cfg::MIN_BLOCKS)
    attention_pp_tail_kernel(const __grid_constant__ CUtensorMap tmQ,
                             const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (threadIdx.x == 0) pdl_launch_dependents();
  constexpr int ST = Cfg::KV_STAGES, NT = Cfg::NT, KB = Cfg::KB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t& q_full = bars[0];
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* s_full = kv_empty + ST;   // [NT]: S_t(j) ready (covers O_t += P_t(j-1) V)
  uint64_t* p_full = s_full + NT;     // [NT]: P_t(j) stored (4 warp arrivals)
  uint64_t* o_last = p_full + NT;     // [NT]: the last P.V of tile t's segment done
  uint64_t& drain_bar = o_last[NT];
  uint64_t& q_empty = o_last[NT + 1]; // a segment's S MMAs done: its Q tiles are free
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(&o_last[NT + 2]);
  int& abort_flag = *(reinterpret_cast<int*>(&o_last[NT + 2]) + 1);
  const int nseg = pp_nseg(p);
  if (nseg == 0) return;  // a tail CTA without blocks (the whole CTA)
  if ((smem_u32(smem) & 1023u) != 0 || nseg > 2) {
    if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadConfig);
    return;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_last[t], 1);
    }
    mbar_init(&drain_bar, 1);
    mbar_init(&q_empty, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == Cfg::TMA_WARP && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == Cfg::MMA_WARP) {
    tmem_alloc(&tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  volatile int* abortp = &abort_flag;

  // Segments run one after another through the same barriers; every
  // barrier's phase parity is taken from a count that runs across them:
  // q_full / q_empty per segment with blocks, kv_full / kv_empty per K/V
  // block, s_full / p_full per block of tile t, o_last per segment of tile t.
  if (warp == Cfg::TMA_WARP) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      bool ok = true;
      int issued = 0, stage = 0, nq = 0;
      uint32_t phase = 0;
      for (int si = 0; si < nseg && ok; ++si) {
        const PpSeg<KB> w = pp_tail_seg<KB>(p, si);
        if (w.nblk == 0) continue;
        const int nt = pp_tiles<Cfg>(p, w);
        if (nq > 0 && !mbar_wait(&q_empty, static_cast<uint32_t>(nq - 1) & 1u, p.err,
                                 kDevTimeoutProducer, abortp)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full, nt * Cfg::Q_TILE);
        for (int t = 0; t < nt; ++t)
          tma_load_4d(smem + Cfg::Q_OFF + t * Cfg::Q_TILE, &tmQ, &q_full, 0,
                      w.qb * Cfg::ROWS + t * 128, w.h, w.b);
        ++nq;
        for (int j = 0; j < w.nblk; ++j) {
          if (!mbar_wait(&kv_empty[stage], phase ^ 1u, p.err, kDevTimeoutProducer, abortp)) {
            ok = false;
            break;
          }
          uint8_t* kt = smem + Cfg::KV_OFF + stage * 2 * Cfg::KV_TILE;
          mbar_arrive_expect_tx(&kv_full[stage], 2 * Cfg::KV_TILE);
          const int ks = w.start(j);
          tma_load_4d(kt, &tmK, &kv_full[stage], 0, ks, w.h, w.b);
          tma_load_4d(kt + Cfg::KV_TILE, &tmV, &kv_full[stage], 0, ks, w.h, w.b);
          ++issued;
          if (++stage == ST) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (nq > 0 && !mbar_wait_quiet(&q_full, static_cast<uint32_t>(nq - 1) & 1u, 200000000ull))
        atomicCAS(p.err, 0, kDevTimeoutDrain);
      if (!ok) {
        // Wait for the copies still in flight before the CTA exits.
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
  } else if (warp == Cfg::MMA_WARP) {
    // ───────────── MMA issuer ─────────────
    // Tiles are served out of order: whenever tile t's P for block j-1 is
    // stored and block j's K/V are loaded, O_t += P_t(j-1) V(j-1) and
    // S_t(j) are issued for it, whatever the other tiles are doing, so a
    // slow tile never holds back the others.  A K/V stage is released once
    // every running tile has issued its P.V on it (the commit covers all
    // MMAs issued before it).  Tiles can drift apart by up to KV_STAGES-1
    // blocks; the producer refills stages in block order.  The first P.V of
    // a segment overwrites O_t: the softmax warps of tile t have read the
    // previous segment's O_t before they store the P that lets it issue.
    if (lane == 0) {
      const uint32_t fmt = BF16 ? 1u : 0u;
      const uint32_t idesc_s = make_idesc(fmt, 128, KB, 0u, 0u);
      const uint32_t idesc_o = make_idesc(fmt, 128, 64, 0u, 1u);
      bool ok = true, issued_any = false;
      int pbase[NT];              // p_full phases of tile t before this segment
      int pv_done[ST];            // tiles that have issued their P.V on each stage's block
#pragma unroll
      for (int t = 0; t < NT; ++t) pbase[t] = 0;
#pragma unroll
      for (int s2 = 0; s2 < ST; ++s2) pv_done[s2] = 0;
      int g0 = 0, nq = 0;         // K/V blocks and Q loads of the earlier segments
      for (int si = 0; si < nseg && ok; ++si) {
        const PpSeg<KB> w = pp_tail_seg<KB>(p, si);
        const int nblk = w.nblk;
        if (nblk == 0) continue;
        const int nt = pp_tiles<Cfg>(p, w);
        if (!mbar_wait(&q_full, static_cast<uint32_t>(nq) & 1u, p.err, kDevTimeoutMma, abortp)) {
          ok = false;
          break;
        }
        int jt[NT];               // next block each tile issues S for (P.V of jt-1 with it)
#pragma unroll
        for (int t = 0; t < NT; ++t) jt[t] = 0;
        int finished = 0;
        unsigned long long t_last = 0;  // start of the current idle period
        int idle = 0;
        while (ok && finished < nt) {
          bool progress = false;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t >= nt) continue;
            const int j = jt[t];
            if (j > nblk) continue;
            if (j > 0 && !mbar_test(&p_full[t], static_cast<uint32_t>(pbase[t] + j - 1) & 1u)) continue;
            const int g = g0 + j;
            if (j < nblk && !mbar_test(&kv_full[g % ST], static_cast<uint32_t>(g / ST) & 1u)) continue;
            tc_fence_after();
            if (j > 0) {
              // O_t += P_t(j-1) V(j-1), P from TMEM, V MN-major from its stage.
              const int ps = (g - 1) % ST;
              const uint32_t v_addr = smem_u32(smem + Cfg::KV_OFF + ps * 2 * Cfg::KV_TILE + Cfg::KV_TILE);
#pragma unroll
              for (int ks = 0; ks < KB / 16; ++ks) {
                const uint64_t bd = make_sw128_desc(v_addr + ks * 2048, Cfg::KV_TILE, 1024);
                umma_f16_tmem_a(tmem_base + Cfg::O_COL + t * 64,
                                tmem_base + Cfg::S_COL + t * KB + ks * 8, bd, idesc_o,
                                (j > 1 || ks > 0) ? 1u : 0u);
              }
              if (++pv_done[ps] == nt) {
                pv_done[ps] = 0;
                umma_commit(&kv_empty[ps]);
              }
              if (j == nblk) umma_commit(&o_last[t]);
            }
            if (j < nblk) {
              const uint32_t q_addr = smem_u32(smem + Cfg::Q_OFF + t * Cfg::Q_TILE);
              const uint32_t k_addr = smem_u32(smem + Cfg::KV_OFF + (g % ST) * 2 * Cfg::KV_TILE);
#pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                const uint64_t ad = make_sw128_desc(q_addr + ks * 32, 16, 1024);
                const uint64_t bd = make_sw128_desc(k_addr + ks * 32, 16, 1024);
                umma_f16(tmem_base + Cfg::S_COL + t * KB, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
              }
              issued_any = true;
              umma_commit(&s_full[t]);
            }
            jt[t] = j + 1;
            if (j == nblk) ++finished;
            progress = true;
          }
          if (progress) {
            idle = 0;
          } else {
            // Nothing ready: back off briefly (the thread shares its scheduler
            // with softmax warps) and check the abort flag and the time limit
            // every 16 idle passes.
            if (idle == 0) t_last = global_timer_ns();
            if ((++idle & 15) == 0) {
              if (*abortp) {
                ok = false;
              } else if (global_timer_ns() - t_last > kWaitLimitNs) {
                *abortp = 1;
                atomicCAS(p.err, 0, kDevTimeoutMma);
                ok = false;
              }
            }
            __nanosleep(20);
          }
        }
        if (!ok) break;
        // Every S MMA of the segment is issued: its Q tiles free once they complete.
        umma_commit(&q_empty);
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < nt) pbase[t] += nblk;
        g0 += nblk;
        ++nq;
      }
      if (!ok && issued_any) {
        umma_commit(&drain_bar);
        if (!mbar_wait_quiet(&drain_bar, 0, 200000000ull)) atomicCAS(p.err, 0, kDevTimeoutDrain);
      }
    }
  } else {
    // ───────────── softmax of tile t: one thread per query row ─────────────
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;                 // row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_base + Cfg::S_COL + t * KB;
    const uint32_t o_addr = tmem_base + lane_base + Cfg::O_COL + t * 64;
    bool ok = true;
    int sbase = 0, ocnt = 0;  // s_full phases and finished segments of this tile so far
    uint32_t r[KB > 64 ? KB : 64];
    for (int si = 0; si < nseg && ok; ++si) {
      const PpSeg<KB> w = pp_tail_seg<KB>(p, si);
      if (t >= pp_tiles<Cfg>(p, w)) continue;
      const int nblk = w.nblk;
      float m_run = -INFINITY, l_run = 0.0f;  // m_run: integer-valued base (log2 domain)
      ok = pp_softmax_rows<BF16, KB, Cfg::CHUNKS>(p, w, nblk, sbase, &s_full[t], &p_full[t], s_addr,
                                                  o_addr, lane, abortp, m_run, l_run, r);
      if (ok && nblk > 0)
        ok = __all_sync(0xffffffffu, mbar_wait(&o_last[t], static_cast<uint32_t>(ocnt) & 1u, p.err,
                                               kDevTimeoutEpilogue, abortp));
      sbase += nblk;
      if (nblk > 0) ++ocnt;
      if (!ok) break;
      tc_fence_after();
      pp_write_rows<BF16, Cfg>(p, w, t, row, o_addr, m_run, l_run, nblk, r);
      // This tile's O_t reads are complete (pp_write_rows waits for its TMEM
      // loads) before its next P arrival lets the next segment's first P.V
      // overwrite O_t.
      tc_fence_before();
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == Cfg::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace sf
