// GEMM / softmax / elementwise entry points of the C ABI and their dispatch.
//
// Dispatch policy (sf_gemm / sf_gemm_batched):
//   16-bit inputs, TMA-describable layout  -> tcgen05 GEMM
//       * B stored [N,K] (trans_b = 1, nn.Linear weights): K-major B
//       * B stored [K,N] (trans_b = 0): MN-major B, 64-wide swizzled slabs
//       * M <= 256, unbatched, K-major B: swap-AB ("skinny-M"): the weight
//         rows fill the 128-row UMMA tile, the few activation rows become
//         the UMMA N extent, outputs are stored transposed; split-K over a
//         zeroed fp32 workspace when there are too few tiles to cover the SMs
//   fp32 inputs:
//       * SF_FP32_ACCURATE (default): 3xTF32 -- operands are split into
//         K-concatenated TF32 hi/lo panels in the workspace and multiplied
//         by the tcgen05 kernel in kind::tf32
//       * SF_FP32_TF32: single TF32 pass (direct when K-major and aligned)
//       * SF_FP32_FFMA: IEEE fp32 SIMT kernel
//   anything else (transposed A, strides TMA cannot describe) -> SIMT kernel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "common.h"
#include "gemm_simt.cuh"
#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "gemv.cuh"
#include "rowwise.cuh"
#include "tma_host.h"

namespace sf {


// ───────────────────────────── problem / plan ─────────────────────────────

struct Problem {
  int64_t M, N, K;
  const void* A;
  int64_t lda;
  int ta;
  const void* B;
  int64_t ldb;
  int tb;
  void* C;
  int64_t ldc;
  int in_dt, out_dt;
  sf_epilogue epi;
  int64_t nb0, nb1, as0, as1, bs0, bs1, cs0, cs1;
  void* ws;
  size_t ws_bytes;
  cudaStream_t stream;
};

enum PlanKind { kPlanSimt, kPlanTc, kPlanTcSwap, kPlanTf32Split, kPlanTf32Direct, kPlanGemv };

struct Plan {
  PlanKind kind = kPlanSimt;
  int bn = 128;
  bool b_mn = false;
  int splits = 1;
  bool ws_slices = false; // split-K partials stored per split (no zeroing) and summed by the finaliser
  bool promote = false; // fp32-accurate: chunked TMEM accumulation promoted to registers
  bool pair = false;    // 2-CTA cluster (cta_group::2) kernel, 256-row pair tiles
  int a_box_rows = 128; // pair kernel: rows per A box (fewer for skinny M)
  int64_t kk = 0;       // reduction length seen by the TC kernel (3K for 3xTF32)
  int64_t ld_split = 0; // leading dimension of the split panels
  size_t ws_bytes = 0;
};


static int pick_bn(int64_t n) {
  if (n <= 16) return 16;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  // One 192-wide tile covers N <= 192; wider outputs take 256-wide tiles even
  // where 192 would pad less.  Measured on B200 (bf16, K = 1920 and 7680,
  // M = 4444 .. 35552): at N = 1920 (ten 192-wide tiles exactly, or eight
  // 256-wide with 6.7 % padding) the 256-wide tiles are 13-25 % faster.
  return n <= 192 ? 192 : 256;
}

// Skinny pair GEMMs (M <= 256: one 256-row pair tile holds every activation
// row, so each weight byte is read once): the pair tile width whose tile
// count best fills the SM pairs, counting column padding as waste.
static int pick_bn_pair_skinny(int64_t n, int clusters) {
  static const int kCand[] = {64, 96, 128, 160, 192, 256};
  int best = 256;
  double best_eff = -1.0;
  for (int bn : kCand) {
    const int64_t tiles = ceil_div(n, bn);
    const int64_t rounds = ceil_div(tiles, clusters);
    const double eff = static_cast<double>(tiles) / static_cast<double>(rounds * clusters) *
                       static_cast<double>(n) / static_cast<double>(tiles * bn);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = bn;
    }
  }
  return best;
}

// Reduction length from which narrow 16-bit GEMMs promote their accumulators.
constexpr int64_t kPromoteMinK = 8192;


// `have_ptrs` = false when only sizing the workspace (pointers unknown, assumed aligned).
static Plan make_plan(const Problem& p, int sm_count, bool have_ptrs) {
  Plan pl;
  const int ovr = kernel_override();
  const int64_t batch = p.nb0 * p.nb1;
  if (p.in_dt == kF32) {
    const int mode = fp32_mode();
    if (mode == SF_FP32_FFMA || ovr == SF_KERNEL_SIMT) return pl;
    if (mode == SF_FP32_TF32) {
      const bool direct = p.ta == 0 && p.tb == 1 && bytes16(p.lda, 4) && bytes16(p.ldb, 4) &&
                          bytes16(p.as0, 4) && bytes16(p.as1, 4) && bytes16(p.bs0, 4) &&
                          bytes16(p.bs1, 4) &&
                          (!have_ptrs || (aligned16(p.A) && aligned16(p.B)));
      if (direct) {
        pl.kind = kPlanTf32Direct;
        pl.kk = p.K;
        pl.bn = pick_bn(p.N);
        return pl;
      }
      pl.kk = p.K;
    } else {
      pl.kk = 3 * p.K;
      pl.promote = true;
    }
    pl.kind = kPlanTf32Split;
    pl.ld_split = (pl.kk + 3) & ~int64_t(3);
    pl.bn = pl.promote ? (p.N <= 64 ? 64 : 128) : pick_bn(p.N);
    pl.ws_bytes = static_cast<size_t>(batch) * static_cast<size_t>(p.M + p.N) *
                  static_cast<size_t>(pl.ld_split) * 4u;
    return pl;
  }
  // 16-bit inputs
  if (ovr == SF_KERNEL_SIMT || p.ta != 0) return pl;
  const bool a_ok = bytes16(p.lda, 2) && bytes16(p.as0, 2) && bytes16(p.as1, 2) &&
                    (!have_ptrs || aligned16(p.A));
  const bool b_ok = bytes16(p.ldb, 2) && bytes16(p.bs0, 2) && bytes16(p.bs1, 2) &&
                    (!have_ptrs || aligned16(p.B));
  if (!a_ok || !b_ok) return pl;
  if (p.tb == 0) {
    pl.kind = kPlanTc;
    pl.b_mn = true;
    pl.bn = pick_bn(p.N) < 64 ? 64 : pick_bn(p.N);
    // Long reductions into narrow outputs (attention P.V: K = keys, N = head
    // dim) average thousands of small terms; keep them IEEE-accurate by
    // promoting TMEM partial sums into fp32 registers every 4 k-blocks.
    if (p.K >= kPromoteMinK && pl.bn <= 128) pl.promote = true;
    return pl;
  }
  // The balanced GEMV kernel (K % 256 == 0) for M <= 2 (from M = 3 the
  // swap-AB tensor-core path streams the weights faster on B200), the plain
  // GEMV kernel for M <= 4 otherwise.  Test hook: SF_GEMV_MAX_M (<= 8) widens
  // the balanced kernel's range so its code paths for M up to 8 are covered.
  const int gemv_max_m = (p.K % 256 == 0) ? std::min(8, env_int("SF_GEMV_MAX_M", 2)) : 4;
  if (batch == 1 && p.M <= gemv_max_m && p.K % 8 == 0 && p.lda % 8 == 0 && p.ldb % 8 == 0 &&
      ovr != SF_KERNEL_TCGEN05 && ovr != SF_KERNEL_TCGEN05_1CTA) {
    // Decode-style shapes: a pure weight stream, served by the GEMV kernel.
    pl.kind = kPlanGemv;
    return pl;
  }
  // Skinny M on B200 (graph-replayed, K = 4096): with k-balanced split-K the
  // swap-AB kernel (weights fill the 128-row MMA side) is fastest up to
  // M = 128, and at N = 4096 up to M = 256; wide outputs with M = 129..256
  // run on CTA pairs holding every activation row in one pair tile.  Test
  // hooks: SF_SKINNY_PAIR=0 and SF_SKINNY_PAIR_MIN_M / _MIN_N move shapes
  // between the two paths so that both are checked on every skinny shape.
  const int pair_min_m = env_int("SF_SKINNY_PAIR_MIN_M", 129);
  const int pair_min_n = env_int("SF_SKINNY_PAIR_MIN_N", 8192);
  if (batch == 1 && p.M <= 256 && p.M >= pair_min_m && p.N >= std::max(1024, pair_min_n) &&
      p.K >= 64 &&
      ovr != SF_KERNEL_TCGEN05_1CTA && env_int("SF_SKINNY_PAIR", 1)) {
    // Skinny M on CTA pairs: activations = A (one pair tile), weights = B
    // split into ~one tile per SM pair.
    pl.kind = kPlanTc;
    pl.pair = true;
    pl.bn = pick_bn_pair_skinny(p.N, std::max(1, sm_count / 2));
    pl.a_box_rows = static_cast<int>(std::min<int64_t>(128, (p.M + 7) / 8 * 8));
    return pl;
  }
  if (batch == 1 && p.M <= 256 && p.N >= 256) {
    pl.kind = kPlanTcSwap;
    pl.bn = pick_bn(p.M);
    const int64_t tiles = ceil_div(p.N, 128);
    const int64_t kb = ceil_div(p.K, 64);
    int64_t splits = 1;
    if (kb >= 8) {
      // The weight stream is shared evenly only when every SM has the same
      // number of k-blocks: pick the split count s (>= 4 k-blocks per split)
      // minimising the busiest SM's k-blocks, ceil(tiles*s / SMs) * ceil(kb/s),
      // plus the partials' write + read (s*M*N*8 bytes over all SMs, in units
      // of one 16 KB weight k-block per SM).
      double best = static_cast<double>(ceil_div(tiles, sm_count) * kb);
      for (int64_t s = 2; s <= kb / 4; ++s) {
        const int64_t per = ceil_div(kb, s);
        const int64_t ss = ceil_div(kb, per);
        const double t = static_cast<double>(ceil_div(tiles * ss, sm_count) * per) +
                         static_cast<double>(ss * p.M * p.N * 8) / (16384.0 * sm_count);
        if (t < best - 1e-9) {
          best = t;
          splits = ss;
        }
      }
      pl.ws_slices = splits > 1;
    } else if (tiles * 2 <= sm_count && kb >= 8) {
      splits = std::min<int64_t>(kb / 4, sm_count / tiles);
      splits = std::max<int64_t>(splits, 1);
      const int64_t per = ceil_div(kb, splits);
      splits = ceil_div(kb, per);
    }
    pl.splits = static_cast<int>(splits);
    if (pl.splits > 1)
      pl.ws_bytes = static_cast<size_t>(p.M) * static_cast<size_t>(p.N) * 4u *
                    static_cast<size_t>(pl.ws_slices ? pl.splits : 1);
    return pl;
  }
  pl.kind = kPlanTc;
  pl.bn = pick_bn(p.N);
  if (pl.bn < 64 && p.M > 4096) pl.bn = 64;
  // CTA pairs over 256-row tiles: a third less operand traffic per SM than
  // 1-CTA 128-row tiles.  Measured on B200 they pay only for wide (BN = 256),
  // tall GEMMs with long reductions (the square 16384 shape); on the DiT
  // linears (K = 1920 and 7680, M = 8888 .. 35552, 256-wide tiles) the 1-CTA
  // kernel is 0-13 % faster, so AUTO picks pairs for that class only.  Test
  // hook: SF_PAIR=1 puts every eligible GEMM on the pair kernel (parity of
  // its code paths).
  if (pl.bn >= 128 && p.M >= 1024 && p.K >= 256 && ovr != SF_KERNEL_TCGEN05_1CTA) {
    const int knob = env_int("SF_PAIR", -1);
    if (knob == 1 ||
        (knob < 0 && pl.bn == 256 && p.N >= 4096 && p.M >= 16384 && p.K >= 8192))
      pl.pair = true;
  }
  return pl;
}

static EpilogueArgs to_epi(const sf_epilogue& e, int out_dt) {
  EpilogueArgs a;
  a.alpha = e.alpha;
  a.beta = e.beta;
  a.fast_act = out_dt != kF32 ? 1 : 0;
  a.bias_vec = (e.bias && (reinterpret_cast<uintptr_t>(e.bias) & 15u) == 0) ? 1 : 0;
  {
    const int res = e.residual_dtype == kF32 ? 4 : 2;
    a.res_vec = (e.residual && (reinterpret_cast<uintptr_t>(e.residual) & 15u) == 0 &&
                 ((e.ldr * res) & 15) == 0 && ((e.r_stride0 * res) & 15) == 0 &&
                 ((e.r_stride1 * res) & 15) == 0)
                    ? 1
                    : 0;
  }
  a.bias = e.bias;
  a.bias_dtype = e.bias_dtype;
  a.bias_on_rows = 0;
  a.act = e.activation;
  a.residual = e.residual;
  a.residual_dtype = e.residual_dtype;
  a.ldr = e.ldr;
  a.r_stride0 = e.r_stride0;
  a.r_stride1 = e.r_stride1;
  return a;
}

// ───────────────────────────── launchers ─────────────────────────────

// C-operand map for the TMA-store epilogue (set by run_tc before launching).
static thread_local CUtensorMap t_map_c;

template <class Cfg>
static int32_t launch_tc_cfg(const CUtensorMap& ma, const CUtensorMap& mb, const GemmTcArgs& a,
                             int grid, cudaStream_t s, int device) {
  static bool attr_set[64] = {false};
  if (device < 64 && !attr_set[device]) {
    SF_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Cfg::SMEM_BYTES));
    attr_set[device] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  SF_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<Cfg>, ma, mb, t_map_c, a));
  return SF_OK;
}

// Launch of a kernel that waits for its predecessor with griddepcontrol
// (programmatic dependent launch when `pdl`).
template <class... KArgs, class... Args>
static int32_t launch_maybe_pdl(bool pdl, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                void (*kernel)(KArgs...), Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  return SF_OK;
}

// Stage counts per N tile: keep ~192-216 KB of operand ring per CTA.
template <int FMT, bool BMN, int PKB>
static int32_t launch_tc(int bn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmTcArgs& a,
                         int grid, cudaStream_t s, int device) {
  if constexpr (PKB > 0) {
    switch (bn) {
      case 64: return launch_tc_cfg<TcCfg<64, tc_stages<64>(), FMT, false, PKB>>(ma, mb, a, grid, s, device);
      case 128: return launch_tc_cfg<TcCfg<128, tc_stages<128>(), FMT, false, PKB>>(ma, mb, a, grid, s, device);
      default: return fail(SF_ERR_UNSUPPORTED, "promoted tile width %d", bn);
    }
  } else if constexpr (BMN) {
    switch (bn) {
      case 64: return launch_tc_cfg<TcCfg<64, tc_stages<64>(), FMT, true>>(ma, mb, a, grid, s, device);
      case 128: return launch_tc_cfg<TcCfg<128, tc_stages<128>(), FMT, true>>(ma, mb, a, grid, s, device);
      case 192: return launch_tc_cfg<TcCfg<192, tc_stages<192>(), FMT, true>>(ma, mb, a, grid, s, device);
      case 256: return launch_tc_cfg<TcCfg<256, tc_stages<256>(), FMT, true>>(ma, mb, a, grid, s, device);
      default: return fail(SF_ERR_UNSUPPORTED, "MN-major B tile width %d", bn);
    }
  } else {
    switch (bn) {
      case 16: return launch_tc_cfg<TcCfg<16, tc_stages<16>(), FMT, false>>(ma, mb, a, grid, s, device);
      case 32: return launch_tc_cfg<TcCfg<32, tc_stages<32>(), FMT, false>>(ma, mb, a, grid, s, device);
      case 64: return launch_tc_cfg<TcCfg<64, tc_stages<64>(), FMT, false>>(ma, mb, a, grid, s, device);
      case 128: return launch_tc_cfg<TcCfg<128, tc_stages<128>(), FMT, false>>(ma, mb, a, grid, s, device);
      case 192: return launch_tc_cfg<TcCfg<192, tc_stages<192>(), FMT, false>>(ma, mb, a, grid, s, device);
      case 256: return launch_tc_cfg<TcCfg<256, tc_stages<256>(), FMT, false>>(ma, mb, a, grid, s, device);
      default: return fail(SF_ERR_UNSUPPORTED, "tile width %d", bn);
    }
  }
}

template <int FMT>
static int32_t launch_tc_mn_promoted(int bn, const CUtensorMap& ma, const CUtensorMap& mb,
                                     const GemmTcArgs& a, int grid, cudaStream_t s, int device) {
  switch (bn) {
    case 64: return launch_tc_cfg<TcCfg<64, tc_stages<64>(), FMT, true, 4>>(ma, mb, a, grid, s, device);
    case 128: return launch_tc_cfg<TcCfg<128, tc_stages<128>(), FMT, true, 4>>(ma, mb, a, grid, s, device);
    default: return fail(SF_ERR_UNSUPPORTED, "promoted MN-major tile width %d", bn);
  }
}

static int32_t dispatch_tc(int fmt, bool bmn, bool promote, int bn, const CUtensorMap& ma,
                           const CUtensorMap& mb, const GemmTcArgs& a, int grid, cudaStream_t s,
                           int device) {
  if (fmt == kBF16) {
    if (bmn && promote) return launch_tc_mn_promoted<1>(bn, ma, mb, a, grid, s, device);
    return bmn ? launch_tc<1, true, 0>(bn, ma, mb, a, grid, s, device)
               : launch_tc<1, false, 0>(bn, ma, mb, a, grid, s, device);
  }
  if (fmt == kF16) {
    if (bmn && promote) return launch_tc_mn_promoted<0>(bn, ma, mb, a, grid, s, device);
    return bmn ? launch_tc<0, true, 0>(bn, ma, mb, a, grid, s, device)
               : launch_tc<0, false, 0>(bn, ma, mb, a, grid, s, device);
  }
  if (bmn) return fail(SF_ERR_UNSUPPORTED, "MN-major TF32 operand");
  return promote ? launch_tc<2, false, 4>(bn, ma, mb, a, grid, s, device)
                 : launch_tc<2, false, 0>(bn, ma, mb, a, grid, s, device);
}

// CTA-pair launch: clusters of 2 along x, one cluster per SM pair, persistent
// over the pair tiles.  The number of co-resident clusters comes from the
// occupancy calculator (SMs that cannot host a whole pair stay idle).
template <class Cfg>
static int32_t launch_tc2_cfg(const CUtensorMap& ma, const CUtensorMap& mb, const GemmTcArgs& a,
                              int64_t tiles, cudaStream_t s, int device) {
  static int max_clusters[64] = {0};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (device >= 64) return fail(SF_ERR_UNSUPPORTED, "device index %d", device);
  if (max_clusters[device] == 0) {
    SF_CUDA_TRY(cudaFuncSetAttribute(gemm_tc2_kernel<Cfg>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    cfg.gridDim = dim3(2, 1, 1);
    int n = 0;
    SF_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<Cfg>, &cfg));
    if (n < 1) return fail(SF_ERR_UNSUPPORTED, "no co-resident CTA pair for this kernel");
    max_clusters[device] = n;
  }
  const int64_t clusters = std::min<int64_t>(tiles, max_clusters[device]);
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters), 1, 1);
  SF_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<Cfg>, ma, mb, t_map_c, a));
  return SF_OK;
}

template <int FMT>
static int32_t launch_tc2(int bn, const CUtensorMap& ma, const CUtensorMap& mb,
                          const GemmTcArgs& a, int64_t tiles, cudaStream_t s, int device) {
  switch (bn) {
    case 64: return launch_tc2_cfg<Tc2Cfg<64, tc2_stages<64>(), FMT>>(ma, mb, a, tiles, s, device);
    case 96: return launch_tc2_cfg<Tc2Cfg<96, tc2_stages<96>(), FMT>>(ma, mb, a, tiles, s, device);
    case 128: return launch_tc2_cfg<Tc2Cfg<128, tc2_stages<128>(), FMT>>(ma, mb, a, tiles, s, device);
    case 160: return launch_tc2_cfg<Tc2Cfg<160, tc2_stages<160>(), FMT>>(ma, mb, a, tiles, s, device);
    case 192: return launch_tc2_cfg<Tc2Cfg<192, tc2_stages<192>(), FMT>>(ma, mb, a, tiles, s, device);
    case 256: return launch_tc2_cfg<Tc2Cfg<256, tc2_stages<256>(), FMT>>(ma, mb, a, tiles, s, device);
    default: return fail(SF_ERR_UNSUPPORTED, "pair tile width %d", bn);
  }
}

static int32_t dispatch_tc2(int fmt, int bn, const CUtensorMap& ma, const CUtensorMap& mb,
                            const GemmTcArgs& a, int64_t tiles, cudaStream_t s, int device) {
  if (fmt == kBF16) return launch_tc2<1>(bn, ma, mb, a, tiles, s, device);
  if (fmt == kF16) return launch_tc2<0>(bn, ma, mb, a, tiles, s, device);
  return fail(SF_ERR_UNSUPPORTED, "pair kernel needs 16-bit operands");
}

static int grid_for(int64_t n, int sm_count) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), sm_count * 8LL)));
}

static int32_t run_simt(const Problem& p) {
  GemmSimtArgs a;
  a.M = static_cast<int>(p.M);
  a.N = static_cast<int>(p.N);
  a.K = static_cast<int>(p.K);
  a.nb0 = static_cast<int>(p.nb0);
  a.nb1 = static_cast<int>(p.nb1);
  a.A = p.A;
  a.a_dtype = p.in_dt;
  a.a_rs = p.ta ? 1 : p.lda;
  a.a_cs = p.ta ? p.lda : 1;
  a.a_s0 = p.as0;
  a.a_s1 = p.as1;
  a.B = p.B;
  a.b_dtype = p.in_dt;
  a.b_ks = p.tb ? 1 : p.ldb;
  a.b_ns = p.tb ? p.ldb : 1;
  a.b_s0 = p.bs0;
  a.b_s1 = p.bs1;
  a.C = p.C;
  a.out_dtype = p.out_dt;
  a.ldc = p.ldc;
  a.c_s0 = p.cs0;
  a.c_s1 = p.cs1;
  a.epi = to_epi(p.epi, p.out_dt);
  const int64_t batch = p.nb0 * p.nb1;
  if (batch > 65535) return fail(SF_ERR_UNSUPPORTED, "SIMT GEMM batch %lld > 65535", (long long)batch);
  dim3 grid(static_cast<unsigned>(ceil_div(p.N, kSimtBN)), static_cast<unsigned>(ceil_div(p.M, kSimtBM)),
            static_cast<unsigned>(batch));
  if (grid.y > 65535) return fail(SF_ERR_UNSUPPORTED, "SIMT GEMM M too large");
  gemm_simt_kernel<<<grid, kSimtThreads, 0, p.stream>>>(a);
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}

static int32_t run_tc(const Problem& p, const Plan& pl, const DeviceInfo& dev, int device) {
  const bool swap = pl.kind == kPlanTcSwap;
  const bool tf32 = pl.kind == kPlanTf32Split || pl.kind == kPlanTf32Direct;
  const int fmt = tf32 ? kF32 : p.in_dt;
  const int es = tf32 ? 4 : 2;
  const int bk = 128 / es;
  const int64_t kk = tf32 ? pl.kk : p.K;

  // Tile-orientation operands.
  const void* ta_ptr = swap ? p.B : p.A;
  int64_t ta_ld = swap ? p.ldb : p.lda;
  int64_t ta_s0 = swap ? p.bs0 : p.as0, ta_s1 = swap ? p.bs1 : p.as1;
  const void* tb_ptr = swap ? p.A : p.B;
  int64_t tb_ld = swap ? p.lda : p.ldb;
  int64_t tb_s0 = swap ? p.as0 : p.bs0, tb_s1 = swap ? p.as1 : p.bs1;
  const int64_t tM = swap ? p.N : p.M;
  const int64_t tN = swap ? p.M : p.N;

  if (pl.kind == kPlanTf32Split) {
    // Split / repack both operands into dense K-major TF32 panels.
    float* ap = static_cast<float*>(p.ws);
    float* bp = ap + static_cast<size_t>(p.nb0 * p.nb1) * p.M * pl.ld_split;
    const int pattern_a = (pl.kk == p.K) ? 2 : 0;
    const int pattern_b = (pl.kk == p.K) ? 2 : 1;
    for (int64_t b1 = 0; b1 < p.nb1; ++b1)
      for (int64_t b0 = 0; b0 < p.nb0; ++b0) {
        const int64_t z = b1 * p.nb0 + b0;
        const float* asrc = static_cast<const float*>(p.A) + b0 * p.as0 + b1 * p.as1;
        const float* bsrc = static_cast<const float*>(p.B) + b0 * p.bs0 + b1 * p.bs1;
        tf32_split_kernel<<<grid_for(p.M * p.K, dev.sm_count), 256, 0, p.stream>>>(
            asrc, p.ta ? 1 : p.lda, p.ta ? p.lda : 1, static_cast<int>(p.M), static_cast<int>(p.K),
            ap + z * p.M * pl.ld_split, pl.ld_split, pattern_a);
        tf32_split_kernel<<<grid_for(p.N * p.K, dev.sm_count), 256, 0, p.stream>>>(
            bsrc, p.tb ? p.ldb : 1, p.tb ? 1 : p.ldb, static_cast<int>(p.N), static_cast<int>(p.K),
            bp + z * p.N * pl.ld_split, pl.ld_split, pattern_b);
        SF_CUDA_TRY(cudaGetLastError());
      }
    ta_ptr = ap;
    ta_ld = pl.ld_split;
    ta_s0 = p.M * pl.ld_split;
    ta_s1 = p.nb0 * p.M * pl.ld_split;
    tb_ptr = bp;
    tb_ld = pl.ld_split;
    tb_s0 = p.N * pl.ld_split;
    tb_s1 = p.nb0 * p.N * pl.ld_split;
  }

  CUtensorMap ma, mbm;
  MapSpec sa{ta_ptr, es, tma_dtype(fmt), static_cast<uint64_t>(kk), static_cast<uint64_t>(tM),
             static_cast<uint64_t>(p.nb0), static_cast<uint64_t>(p.nb1), ta_ld, ta_s0, ta_s1,
             static_cast<uint32_t>(bk), static_cast<uint32_t>(pl.pair ? pl.a_box_rows : 128)};
  int32_t st = encode_map(&ma, sa);
  if (st != SF_OK) return st;
  if (pl.b_mn) {
    MapSpec sb{tb_ptr, es, tma_dtype(fmt), static_cast<uint64_t>(tN), static_cast<uint64_t>(kk),
               static_cast<uint64_t>(p.nb0), static_cast<uint64_t>(p.nb1), tb_ld, tb_s0, tb_s1,
               64u, static_cast<uint32_t>(bk)};
    st = encode_map(&mbm, sb);
  } else {
    MapSpec sb{tb_ptr, es, tma_dtype(fmt), static_cast<uint64_t>(kk), static_cast<uint64_t>(tN),
               static_cast<uint64_t>(p.nb0), static_cast<uint64_t>(p.nb1), tb_ld, tb_s0, tb_s1,
               static_cast<uint32_t>(bk), static_cast<uint32_t>(pl.pair ? pl.bn / 2 : pl.bn)};
    st = encode_map(&mbm, sb);
  }
  if (st != SF_OK) return st;

  GemmTcArgs a;
  a.M = static_cast<int>(tM);
  a.N = static_cast<int>(tN);
  a.K = static_cast<int>(kk);
  a.nb0 = static_cast<int>(p.nb0);
  a.nb1 = static_cast<int>(p.nb1);
  a.m_tiles = static_cast<int>(ceil_div(tM, pl.pair ? 256 : 128));
  a.n_tiles = static_cast<int>(ceil_div(tN, pl.bn));
  a.k_blocks = static_cast<int>(ceil_div(kk, bk));
  const int64_t total = int64_t(a.m_tiles) * a.n_tiles * p.nb0 * p.nb1;
  if (total * pl.splits > INT32_MAX) return fail(SF_ERR_UNSUPPORTED, "too many tiles");
  a.total_tiles = static_cast<int>(total);
  a.group_m = 8;  // raster group height
  a.k_splits = pl.splits;
  a.kb_per_split = static_cast<int>(ceil_div(a.k_blocks, pl.splits));
  a.C = p.C;
  a.out_dtype = p.out_dt;
  a.ldc = p.ldc;
  a.c_stride0 = p.cs0;
  a.c_stride1 = p.cs1;
  a.c_trans = swap ? 1 : 0;
  const int oes = esize(p.out_dt);
  a.vec_ok = (!swap && aligned16(p.C) && bytes16(p.ldc, oes) && bytes16(p.cs0, oes) &&
              bytes16(p.cs1, oes))
                 ? 1
                 : 0;
  a.ws = nullptr;
  a.ldw = 0;
  a.ws_slice = 0;
  a.epi = to_epi(p.epi, p.out_dt);
  a.err = dev.err_word;
  a.a_box_rows = pl.pair ? pl.a_box_rows : 128;
  a.tma_store = 0;
  // Programmatic dependent launch of the 1-CTA kernel; skinny shapes prefetch
  // their first 8 weight k-blocks into L2 before waiting for the previous grid.
  a.pdl = pl.pair ? 0 : 1;
  a.pdl_pf = p.M <= 256 ? 8 : 0;
  a.pdl_pf_b = swap ? 0 : 1;
  memset(&t_map_c, 0, sizeof(t_map_c));
  if (!swap && pl.splits == 1 && a.vec_ok) {
    // Epilogue chunks of CH columns x 32 rows, stored by TMA with the swizzle
    // matching the chunk's row bytes.
    const int ch = pl.bn < 32 ? pl.bn : 32;
    const int row_bytes = ch * oes;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    const uint64_t e = static_cast<uint64_t>(oes);
    uint64_t st1 = static_cast<uint64_t>(p.ldc) * e;
    uint64_t st2 = p.nb0 > 1 ? static_cast<uint64_t>(p.cs0) * e : st1 * static_cast<uint64_t>(p.M);
    uint64_t st3 = p.nb1 > 1 ? static_cast<uint64_t>(p.cs1) * e : st2 * static_cast<uint64_t>(p.nb0);
    st2 = (st2 + 15) & ~15ull;
    st3 = (st3 + 15) & ~15ull;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(p.N), static_cast<cuuint64_t>(p.M),
                          static_cast<cuuint64_t>(p.nb0), static_cast<cuuint64_t>(p.nb1)};
    cuuint64_t strides[3] = {st1, st2, st3};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(ch), 32u, 1u, 1u};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapSwizzle sw = row_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                    : CU_TENSOR_MAP_SWIZZLE_32B;
    CUresult r = fn(&t_map_c, tma_dtype(p.out_dt), 4, p.C, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled (C) failed (%d)", static_cast<int>(r));
    a.tma_store = 1;
  }
  if (pl.splits > 1) {
    a.ws = static_cast<float*>(p.ws);
    a.ldw = p.N;  // output orientation [M][N]
    if (pl.ws_slices)
      a.ws_slice = p.M * p.N;
    else
      SF_CUDA_TRY(cudaMemsetAsync(p.ws, 0, static_cast<size_t>(p.M) * p.N * 4u, p.stream));
  }
  const int64_t units = total * pl.splits;
  if (pl.pair) return dispatch_tc2(fmt, pl.bn, ma, mbm, a, total, p.stream, device);
  const int grid = static_cast<int>(std::min<int64_t>(units, dev.sm_count));
  st = dispatch_tc(fmt, pl.b_mn, pl.promote, pl.bn, ma, mbm, a, grid, p.stream, device);
  if (st != SF_OK) return st;
  if (pl.splits > 1) {
    st = launch_maybe_pdl(a.pdl != 0, dim3(static_cast<unsigned>(grid_for(p.M * p.N, dev.sm_count))),
                          dim3(256), 0, p.stream, epilogue_finalize_kernel,
                          static_cast<const float*>(p.ws), static_cast<int64_t>(p.N),
                          static_cast<int>(p.M), static_cast<int>(p.N), p.C, static_cast<int>(p.out_dt),
                          static_cast<int64_t>(p.ldc), to_epi(p.epi, p.out_dt),
                          pl.ws_slices ? pl.splits : 1, static_cast<int64_t>(a.ws_slice));
    if (st != SF_OK) return st;
  }
  return SF_OK;
}

template <int MM, int R>
static void launch_gemv_mr(const Problem& p, const EpilogueArgs& e, cudaStream_t s) {
  const int warps = static_cast<int>(ceil_div(p.N, R));
  const int grid = static_cast<int>(ceil_div(warps, kGemvWarps));
  const uint16_t* x = static_cast<const uint16_t*>(p.A);
  const uint16_t* w = static_cast<const uint16_t*>(p.B);
  if (p.in_dt == kBF16)
    gemv_kernel<MM, R, true><<<grid, kGemvWarps * 32, 0, s>>>(
        x, p.lda, w, p.ldb, p.C, p.out_dt, p.ldc, static_cast<int>(p.N), static_cast<int>(p.K), e);
  else
    gemv_kernel<MM, R, false><<<grid, kGemvWarps * 32, 0, s>>>(
        x, p.lda, w, p.ldb, p.C, p.out_dt, p.ldc, static_cast<int>(p.N), static_cast<int>(p.K), e);
}

template <int MM>
static void launch_gemv_m(const Problem& p, const EpilogueArgs& e, cudaStream_t s, int sm_count) {
  // Four weight rows per warp when that still gives >= 2 CTAs per SM, else two.
  if (ceil_div(p.N, 4 * kGemvWarps) >= 2 * sm_count)
    launch_gemv_mr<MM, 4>(p, e, s);
  else
    launch_gemv_mr<MM, 2>(p, e, s);
}

// Balanced GEMV: one CTA per SM, contiguous row ranges (shared-memory row sums
// of ceil(N/G) x M floats; the grid grows past one CTA per SM only when
// that would exceed 48 KB).
template <int MM, int R, int U>
static int32_t launch_gemv_seg(const Problem& p, const EpilogueArgs& e, int sm_count) {
  int64_t G = sm_count;
  const int64_t max_rows = (48 * 1024) / (MM * 4);
  if (ceil_div(p.N, G) > max_rows) G = ceil_div(p.N, max_rows);
  G = std::min<int64_t>(G, p.N);
  const size_t smem = static_cast<size_t>(ceil_div(p.N, G)) * MM * 4;
  const uint16_t* x = static_cast<const uint16_t*>(p.A);
  const uint16_t* w = static_cast<const uint16_t*>(p.B);
  // Programmatic dependent launch: each warp prefetches its first 8 weight
  // units into L2 before waiting for the previous grid.
  const bool pdl = true;
  const int pf_units = 8;
  const int n = static_cast<int>(p.N), k = static_cast<int>(p.K);
  const dim3 grid(static_cast<unsigned>(G)), block(kSegWarps * 32);
  if (p.in_dt == kBF16)
    return launch_maybe_pdl(pdl, grid, block, smem, p.stream, gemv_seg_kernel<MM, R, U, true>, x,
                            p.lda, w, p.ldb, p.C, static_cast<int>(p.out_dt), p.ldc, n, k, e, pf_units);
  return launch_maybe_pdl(pdl, grid, block, smem, p.stream, gemv_seg_kernel<MM, R, U, false>, x,
                          p.lda, w, p.ldb, p.C, static_cast<int>(p.out_dt), p.ldc, n, k, e, pf_units);
}

static bool gemv_seg_ok(const Problem& p) {
  return p.K % 256 == 0 && aligned16(p.A) && aligned16(p.B);
}

static int32_t run_gemv(const Problem& p, const DeviceInfo& dev) {
  const EpilogueArgs e = to_epi(p.epi, p.out_dt);
  if (gemv_seg_ok(p)) {
    switch (p.M) {
      case 1: return launch_gemv_seg<1, 4, 4>(p, e, dev.sm_count);
      case 2: return launch_gemv_seg<2, 4, 4>(p, e, dev.sm_count);
      case 3: return launch_gemv_seg<3, 4, 2>(p, e, dev.sm_count);
      case 4: return launch_gemv_seg<4, 4, 2>(p, e, dev.sm_count);
      case 5: return launch_gemv_seg<5, 2, 2>(p, e, dev.sm_count);
      case 6: return launch_gemv_seg<6, 2, 2>(p, e, dev.sm_count);
      case 7: return launch_gemv_seg<7, 2, 2>(p, e, dev.sm_count);
      case 8: return launch_gemv_seg<8, 2, 2>(p, e, dev.sm_count);
      default: return fail(SF_ERR_UNSUPPORTED, "GEMV path needs M <= 8");
    }
  }
  switch (p.M) {
    case 1: launch_gemv_m<1>(p, e, p.stream, dev.sm_count); break;
    case 2: launch_gemv_m<2>(p, e, p.stream, dev.sm_count); break;
    case 3: launch_gemv_m<3>(p, e, p.stream, dev.sm_count); break;
    case 4: launch_gemv_m<4>(p, e, p.stream, dev.sm_count); break;
    default: return fail(SF_ERR_UNSUPPORTED, "row-per-warp GEMV path needs M <= 4");
  }
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}

static int32_t validate(const Problem& p) {
  if (p.M < 0 || p.N < 0 || p.K < 0) return fail(SF_ERR_INVALID_ARGUMENT, "negative dimension");
  if (p.M > INT32_MAX || p.N > INT32_MAX || p.K > INT32_MAX)
    return fail(SF_ERR_UNSUPPORTED, "dimension exceeds 2^31-1");
  if (p.nb0 < 1 || p.nb1 < 1) return fail(SF_ERR_INVALID_ARGUMENT, "batch counts must be >= 1");
  for (int dt : {p.in_dt, p.out_dt})
    if (dt != kF32 && dt != kF16 && dt != kBF16)
      return fail(SF_ERR_INVALID_ARGUMENT, "unknown dtype %d", dt);
  if (p.ta != 0 && p.ta != 1) return fail(SF_ERR_INVALID_ARGUMENT, "trans_a must be 0 or 1");
  if (p.tb != 0 && p.tb != 1) return fail(SF_ERR_INVALID_ARGUMENT, "trans_b must be 0 or 1");
  if (p.epi.activation < SF_ACT_NONE || p.epi.activation > SF_ACT_GELU_TANH)
    return fail(SF_ERR_INVALID_ARGUMENT, "unknown activation %d", p.epi.activation);
  if (p.M == 0 || p.N == 0) return SF_OK;
  if (!p.C) return fail(SF_ERR_INVALID_ARGUMENT, "null C");
  if (p.K > 0 && (!p.A || !p.B)) return fail(SF_ERR_INVALID_ARGUMENT, "null A or B");
  if (p.ldc < p.N) return fail(SF_ERR_INVALID_ARGUMENT, "ldc %lld < N %lld", (long long)p.ldc, (long long)p.N);
  if (p.K > 0) {
    if (p.lda < (p.ta ? p.M : p.K)) return fail(SF_ERR_INVALID_ARGUMENT, "lda too small");
    if (p.ldb < (p.tb ? p.K : p.N)) return fail(SF_ERR_INVALID_ARGUMENT, "ldb too small");
  }
  if (p.epi.bias && p.epi.bias_dtype != kF32 && p.epi.bias_dtype != kF16 && p.epi.bias_dtype != kBF16)
    return fail(SF_ERR_INVALID_ARGUMENT, "unknown bias dtype");
  if (p.epi.residual && p.epi.ldr < p.N) return fail(SF_ERR_INVALID_ARGUMENT, "ldr < N");
  return SF_OK;
}

static int32_t gemm_impl(Problem& p) {
  int32_t st = validate(p);
  if (st != SF_OK) return st;
  if (p.M == 0 || p.N == 0) return SF_OK;
  DeviceInfo* dev = nullptr;
  int device = 0;
  st = current_device_info(&dev, &device);
  if (st != SF_OK) return st;
  if (p.K == 0) {
    // Empty reduction: D = epilogue(0) per batch.
    for (int64_t b1 = 0; b1 < p.nb1; ++b1)
      for (int64_t b0 = 0; b0 < p.nb0; ++b0) {
        EpilogueArgs e = to_epi(p.epi, p.out_dt);
        if (e.residual) {
          const int res_es = esize(e.residual_dtype);
          e.residual = static_cast<const char*>(e.residual) + (b0 * e.r_stride0 + b1 * e.r_stride1) * res_es;
        }
        void* c = static_cast<char*>(p.C) + (b0 * p.cs0 + b1 * p.cs1) * esize(p.out_dt);
        epilogue_finalize_kernel<<<grid_for(p.M * p.N, dev->sm_count), 256, 0, p.stream>>>(
            nullptr, 0, static_cast<int>(p.M), static_cast<int>(p.N), c, p.out_dt, p.ldc, e);
      }
    SF_CUDA_TRY(cudaGetLastError());
    return SF_OK;
  }
  const Plan pl = make_plan(p, dev->sm_count, true);
  if (pl.ws_bytes > 0 && (p.ws == nullptr || p.ws_bytes < pl.ws_bytes))
    return fail(SF_ERR_WORKSPACE, "workspace of %zu bytes required (%zu given)", pl.ws_bytes,
                p.ws ? p.ws_bytes : size_t(0));
  if (pl.kind == kPlanGemv) return run_gemv(p, *dev);
  if (pl.kind == kPlanSimt) {
    if (kernel_override() == SF_KERNEL_TCGEN05)
      return fail(SF_ERR_UNSUPPORTED, "layout not supported by the tcgen05 kernel");
    return run_simt(p);
  }
  return run_tc(p, pl, *dev, device);
}

static Problem make_problem(const sf_batch* batch, int64_t M, int64_t N, int64_t K, const void* A,
                            int64_t lda, int32_t trans_a, const void* B, int64_t ldb,
                            int32_t trans_b, void* C, int64_t ldc, int32_t in_dtype,
                            int32_t out_dtype, const sf_epilogue* epi, void* ws, size_t ws_bytes,
                            void* stream) {
  Problem p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.A = A;
  p.lda = lda;
  p.ta = trans_a;
  p.B = B;
  p.ldb = ldb;
  p.tb = trans_b;
  p.C = C;
  p.ldc = ldc;
  p.in_dt = in_dtype;
  p.out_dt = out_dtype;
  if (epi) {
    p.epi = *epi;
  } else {
    p.epi = sf_epilogue{};
    p.epi.alpha = 1.0f;
  }
  if (batch) {
    p.nb0 = batch->count0;
    p.nb1 = batch->count1;
    p.as0 = batch->a_stride0;
    p.as1 = batch->a_stride1;
    p.bs0 = batch->b_stride0;
    p.bs1 = batch->b_stride1;
    p.cs0 = batch->c_stride0;
    p.cs1 = batch->c_stride1;
  } else {
    p.nb0 = p.nb1 = 1;
    p.as0 = p.as1 = p.bs0 = p.bs1 = p.cs0 = p.cs1 = 0;
  }
  p.ws = ws;
  p.ws_bytes = ws_bytes;
  p.stream = static_cast<cudaStream_t>(stream);
  return p;
}

}  // namespace sf

using namespace sf;

extern "C" {

int32_t sf_gemm(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, int32_t trans_a,
                const void* B, int64_t ldb, int32_t trans_b, void* C, int64_t ldc,
                int32_t in_dtype, int32_t out_dtype, const sf_epilogue* epi, void* workspace,
                size_t workspace_bytes, void* stream) {
  Problem p = make_problem(nullptr, M, N, K, A, lda, trans_a, B, ldb, trans_b, C, ldc, in_dtype,
                           out_dtype, epi, workspace, workspace_bytes, stream);
  return gemm_impl(p);
}

int32_t sf_gemm_batched(const sf_batch* batch, int64_t M, int64_t N, int64_t K, const void* A,
                        int64_t lda, int32_t trans_a, const void* B, int64_t ldb, int32_t trans_b,
                        void* C, int64_t ldc, int32_t in_dtype, int32_t out_dtype,
                        const sf_epilogue* epi, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (!batch) return fail(SF_ERR_INVALID_ARGUMENT, "null batch descriptor");
  Problem p = make_problem(batch, M, N, K, A, lda, trans_a, B, ldb, trans_b, C, ldc, in_dtype,
                           out_dtype, epi, workspace, workspace_bytes, stream);
  return gemm_impl(p);
}

int32_t sf_gemm_workspace_size(const sf_batch* batch, int64_t M, int64_t N, int64_t K,
                               int32_t trans_a, int32_t trans_b, int32_t in_dtype,
                               int32_t out_dtype, size_t* bytes) {
  if (!bytes) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  *bytes = 0;
  const int64_t lda = trans_a ? M : K, ldb = trans_b ? K : N;
  Problem p = make_problem(batch, M, N, K, nullptr, lda, trans_a, nullptr, ldb, trans_b, nullptr,
                           N, in_dtype, out_dtype, nullptr, nullptr, 0, nullptr);
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return SF_OK;
  int sm = 148;
  DeviceInfo* dev = nullptr;
  int cnt = 0;
  if (cudaGetDeviceCount(&cnt) == cudaSuccess && cnt > 0 && current_device_info(&dev, nullptr) == SF_OK)
    sm = dev->sm_count;
  else
    cudaGetLastError();
  *bytes = make_plan(p, sm, false).ws_bytes;
  return SF_OK;
}

int32_t sf_softmax_rows(const void* x, int32_t x_dtype, int64_t ldx, void* y, int32_t y_dtype,
                        int64_t ldy, int64_t rows, int64_t cols, float scale, void* stream) {
  if (rows < 0 || cols < 0) return fail(SF_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0 || cols == 0) return SF_OK;
  if (!x || !y) return fail(SF_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldx < cols || ldy < cols) return fail(SF_ERR_INVALID_ARGUMENT, "leading dimension < cols");
  if (rows > INT32_MAX || cols > INT32_MAX) return fail(SF_ERR_UNSUPPORTED, "softmax size");
  for (int dt : {x_dtype, y_dtype})
    if (dt != kF32 && dt != kF16 && dt != kBF16) return fail(SF_ERR_INVALID_ARGUMENT, "dtype %d", dt);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = x_dtype == kF32 && (cols % 4) == 0 && aligned16(x) && (ldx % 4) == 0 &&
                   (y_dtype == kF32 ? (aligned16(y) && ldy % 4 == 0)
                                    : ((reinterpret_cast<uintptr_t>(y) & 7u) == 0 && ldy % 4 == 0));
  const unsigned grid = static_cast<unsigned>(rows);
  if (vec) {
    const float* xf = static_cast<const float*>(x);
    if (y_dtype == kF32)
      softmax_rows_online_kernel<false><<<grid, kSoftmaxOnlineThreads, 0, s>>>(
          xf, ldx, y, y_dtype, ldy, static_cast<int>(cols), scale);
    else
      softmax_rows_online_kernel<true><<<grid, kSoftmaxOnlineThreads, 0, s>>>(
          xf, ldx, y, y_dtype, ldy, static_cast<int>(cols), scale);
  } else {
    softmax_rows_generic_kernel<<<grid, kSoftmaxThreads, 0, s>>>(x, x_dtype, ldx, y, y_dtype, ldy,
                                                                 static_cast<int>(cols), scale);
  }
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}

int32_t sf_unary(const void* x, int32_t x_dtype, void* y, int32_t y_dtype, int64_t n, float alpha,
                 int32_t activation, void* stream) {
  if (n < 0) return fail(SF_ERR_INVALID_ARGUMENT, "negative size");
  if (n == 0) return SF_OK;
  if (!x || !y) return fail(SF_ERR_INVALID_ARGUMENT, "null pointer");
  if (activation < SF_ACT_NONE || activation > SF_ACT_GELU_TANH)
    return fail(SF_ERR_INVALID_ARGUMENT, "unknown activation %d", activation);
  for (int dt : {x_dtype, y_dtype})
    if (dt != kF32 && dt != kF16 && dt != kBF16) return fail(SF_ERR_INVALID_ARGUMENT, "dtype %d", dt);
  DeviceInfo* dev = nullptr;
  int32_t st = current_device_info(&dev, nullptr);
  if (st != SF_OK) return st;
  unary_act_kernel<<<grid_for(n, dev->sm_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_dtype, y, y_dtype, n, alpha, activation);
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}

int32_t sf_selftest_bounded_wait(int64_t limit_ns, int32_t* device_code, void* stream) {
  if (!device_code) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  if (limit_ns <= 0 || limit_ns > 10000000000LL)
    return fail(SF_ERR_INVALID_ARGUMENT, "limit must be in (0, 10 s]");
  DeviceInfo* dev = nullptr;
  int32_t st = current_device_info(&dev, nullptr);
  if (st != SF_OK) return st;
  int* word = dev->err_word + 32;  // private slot, separate from the GEMM error word
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SF_CUDA_TRY(cudaMemsetAsync(word, 0, sizeof(int), s));
  bounded_wait_selftest_kernel<<<1, 32, 0, s>>>(word, static_cast<unsigned long long>(limit_ns));
  SF_CUDA_TRY(cudaGetLastError());
  int v = 0;
  SF_CUDA_TRY(cudaMemcpyAsync(&v, word, sizeof(int), cudaMemcpyDeviceToHost, s));
  SF_CUDA_TRY(cudaStreamSynchronize(s));
  *device_code = v;
  return SF_OK;
}

int32_t sf_fill_normal(void* x, int32_t dtype, int64_t n, uint64_t seed, float mean, float std,
                       void* stream) {
  if (n < 0) return fail(SF_ERR_INVALID_ARGUMENT, "negative size");
  if (n == 0) return SF_OK;
  if (!x) return fail(SF_ERR_INVALID_ARGUMENT, "null pointer");
  if (dtype != kF32 && dtype != kF16 && dtype != kBF16) return fail(SF_ERR_INVALID_ARGUMENT, "dtype %d", dtype);
  DeviceInfo* dev = nullptr;
  int32_t st = current_device_info(&dev, nullptr);
  if (st != SF_OK) return st;
  fill_normal_kernel<<<grid_for(n, dev->sm_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, dtype, n, seed, mean, std);
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}

}  // extern "C"
