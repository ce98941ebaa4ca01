// sf_linear_skinny_noalloc: the skinny-M linear (swap-AB tcgen05 GEMM with
// split-K) for callers that cannot allocate device memory.
//
// Who needs it: a host program that hands all of the GPU's memory to its own
// allocator at start-up (a serving process that reserves HBM for its caches),
// or that must not call cudaMalloc on its latency path (cudaMalloc can
// synchronise the device), cannot give the engine a workspace or let it
// allocate one.  sf_gemm needs a caller workspace for the split-K partial
// sums of small-M problems; this entry point keeps those partial sums in a
// fixed array compiled into the library instead, so the only device memory
// it touches is the caller's inputs and outputs plus that array.
//
// The scratch array: kNoAllocScratchFloats fp32 values (4 MiB), a
// file-scope __device__ array.  Every GPU that loads the library holds one
// copy of it until the process exits.  All calls on a device share it, and it
// keeps what the previous call left there: each call zeroes the part it
// accumulates into before use.  Calls whose GPU work overlaps (on different
// streams, or from different host threads without ordering) race on the
// array and produce wrong results -- order them on one stream.
//
// Errors: a bounded wait of these kernels that expires records its code in
// a static device word of this file (not the runtime's per-device word,
// which is cudaMalloc'd); sf_device_error_status reports both.
//
// Set-up: the first call on each device (with that device current) looks up
// the array's device address with cudaGetSymbolAddress and sets the kernels'
// shared-memory attributes.  Make that first call before any stream capture
// on the device.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "common.h"
#include "gemm_tc.cuh"
#include "rowwise.cuh"

namespace sf {
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;  // M * N limit (4 MiB of fp32)

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) int g_noalloc_err[64];

struct NoAllocDevice {
  bool ready = false;
  float* scratch = nullptr;
  int* err = nullptr;
  int sm_count = 0;
};
std::mutex g_mu;
NoAllocDevice g_dev[64];

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

template <class Cfg>
int32_t set_smem_attr() {
  SF_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cfg::SMEM_BYTES));
  return SF_OK;
}

template <int FMT>
int32_t set_attrs_fmt() {
  int32_t st = set_smem_attr<TcCfg<16, tc_stages<16>(), FMT, false>>();
  if (st == SF_OK) st = set_smem_attr<TcCfg<32, tc_stages<32>(), FMT, false>>();
  if (st == SF_OK) st = set_smem_attr<TcCfg<64, tc_stages<64>(), FMT, false>>();
  if (st == SF_OK) st = set_smem_attr<TcCfg<128, tc_stages<128>(), FMT, false>>();
  if (st == SF_OK) st = set_smem_attr<TcCfg<256, tc_stages<256>(), FMT, false>>();
  return st;
}

// Once per device, with `device` current.
int32_t setup(int device, NoAllocDevice** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= 64) return fail(SF_ERR_INVALID_ARGUMENT, "device %d out of range", device);
  NoAllocDevice& d = g_dev[device];
  if (!d.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(no-alloc scratch)");
    d.scratch = static_cast<float*>(p);
    e = cudaGetSymbolAddress(&p, g_noalloc_err);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(no-alloc error word)");
    d.err = static_cast<int*>(p);
    SF_CUDA_TRY(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, device));
    int32_t st = set_attrs_fmt<0>();
    if (st == SF_OK) st = set_attrs_fmt<1>();
    if (st != SF_OK) return st;
    d.ready = true;
  }
  *out = &d;
  return SF_OK;
}

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

// 2-D K-major operand [rows, K] with row stride ld (elements), as a 4-D map.
int32_t encode_rows(CUtensorMap* m, const void* base, int dtype, uint64_t K, uint64_t rows,
                    int64_t ld, uint32_t box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const uint64_t row_bytes = static_cast<uint64_t>(ld) * 2u;
  const uint64_t plane = (row_bytes * rows + 15) & ~15ull;
  cuuint64_t dims[4] = {K, rows, 1, 1};
  cuuint64_t strides[3] = {row_bytes, plane, plane};
  cuuint32_t box[4] = {64u, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return SF_OK;
}

template <int FMT>
int32_t launch(int bn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmTcArgs& a, int grid,
               cudaStream_t s) {
#define SF_NOALLOC_LAUNCH(BN)                                                               \
  gemm_tc_kernel<TcCfg<BN, tc_stages<BN>(), FMT, false>>                                      \
      <<<grid, TcCfg<BN, tc_stages<BN>(), FMT, false>::THREADS,                              \
         TcCfg<BN, tc_stages<BN>(), FMT, false>::SMEM_BYTES, s>>>(ma, mb, ma, a)
  switch (bn) {
    case 16: SF_NOALLOC_LAUNCH(16); break;
    case 32: SF_NOALLOC_LAUNCH(32); break;
    case 64: SF_NOALLOC_LAUNCH(64); break;
    case 128: SF_NOALLOC_LAUNCH(128); break;
    case 256: SF_NOALLOC_LAUNCH(256); break;
    default: return fail(SF_ERR_UNSUPPORTED, "tile width %d", bn);
  }
#undef SF_NOALLOC_LAUNCH
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}

}  // namespace

int32_t noalloc_error_word(int* value, bool clear) {
  int v = 0;
  SF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_noalloc_err, sizeof(int)));
  if (clear && v != 0) {
    const int zero = 0;
    SF_CUDA_TRY(cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(int)));
  }
  *value = v;
  return SF_OK;
}

}  // namespace sf

using namespace sf;

extern "C" int32_t sf_linear_skinny_noalloc(int64_t M, int64_t N, int64_t K, const void* x,
                                            int64_t ldx, const void* W, int64_t ldw,
                                            const void* bias, int32_t bias_dtype, void* y,
                                            int64_t ldy, int32_t in_dtype, int32_t out_dtype,
                                            int32_t activation, void* stream) {
  // ── argument checks (nothing is launched or looked up before these pass)
  if (M < 1 || M > 256)
    return fail(SF_ERR_INVALID_ARGUMENT, "sf_linear_skinny_noalloc: M = %lld outside [1, 256]", (long long)M);
  if (N < 1 || K < 1 || N > INT32_MAX || K > INT32_MAX)
    return fail(SF_ERR_INVALID_ARGUMENT, "sf_linear_skinny_noalloc: N = %lld, K = %lld", (long long)N,
                (long long)K);
  if (static_cast<size_t>(M) * static_cast<size_t>(N) > kNoAllocScratchFloats)
    return fail(SF_ERR_INVALID_ARGUMENT,
                "sf_linear_skinny_noalloc: M*N = %lld exceeds the fixed scratch of %zu fp32 values "
                "(4 MiB); use sf_gemm with a workspace",
                (long long)(M * N), kNoAllocScratchFloats);
  if (in_dtype != kBF16 && in_dtype != kF16)
    return fail(SF_ERR_INVALID_ARGUMENT, "sf_linear_skinny_noalloc: inputs must be bf16 or fp16");
  if (out_dtype != kF32 && out_dtype != kF16 && out_dtype != kBF16)
    return fail(SF_ERR_INVALID_ARGUMENT, "sf_linear_skinny_noalloc: unknown output dtype %d", out_dtype);
  if (bias && bias_dtype != kF32 && bias_dtype != kF16 && bias_dtype != kBF16)
    return fail(SF_ERR_INVALID_ARGUMENT, "sf_linear_skinny_noalloc: unknown bias dtype %d", bias_dtype);
  if (activation < SF_ACT_NONE || activation > SF_ACT_GELU_TANH)
    return fail(SF_ERR_INVALID_ARGUMENT, "sf_linear_skinny_noalloc: unknown activation %d", activation);
  if (!x || !W || !y) return fail(SF_ERR_INVALID_ARGUMENT, "sf_linear_skinny_noalloc: null pointer");
  if (ldx < K || ldw < K || ldy < N)
    return fail(SF_ERR_INVALID_ARGUMENT, "sf_linear_skinny_noalloc: leading dimension too small");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(W) & 15u) ||
      ((ldx * 2) & 15) || ((ldw * 2) & 15))
    return fail(SF_ERR_UNSUPPORTED,
                "sf_linear_skinny_noalloc: x and W need 16-byte aligned bases and row strides");

  int device = 0;
  SF_CUDA_TRY(cudaGetDevice(&device));
  NoAllocDevice* d = nullptr;
  int32_t st = setup(device, &d);
  if (st != SF_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // ── plan: weights are the 128-row UMMA M side, the M activation rows the N side
  const int bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const int64_t tiles = (N + 127) / 128;
  const int64_t kb = (K + 63) / 64;
  int64_t splits = std::max<int64_t>(2, std::min<int64_t>(kb / 4, d->sm_count / tiles));
  splits = std::min<int64_t>(splits, kb);
  const int64_t per = (kb + splits - 1) / splits;
  splits = (kb + per - 1) / per;

  CUtensorMap ma, mb;
  st = encode_rows(&ma, W, in_dtype, K, N, ldw, 128u);
  if (st == SF_OK) st = encode_rows(&mb, x, in_dtype, K, M, ldx, static_cast<uint32_t>(bn));
  if (st != SF_OK) return st;

  EpilogueArgs e{};
  e.alpha = 1.0f;
  e.beta = 1.0f;
  e.fast_act = out_dtype != kF32 ? 1 : 0;
  e.bias = bias;
  e.bias_dtype = bias_dtype;
  e.bias_vec = (bias && (reinterpret_cast<uintptr_t>(bias) & 15u) == 0) ? 1 : 0;
  e.act = activation;

  GemmTcArgs a{};
  a.M = static_cast<int>(N);
  a.N = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.nb0 = a.nb1 = 1;
  a.m_tiles = static_cast<int>(tiles);
  a.n_tiles = 1;
  a.k_blocks = static_cast<int>(kb);
  a.total_tiles = static_cast<int>(tiles);
  a.group_m = 8;
  a.k_splits = static_cast<int>(splits);
  a.kb_per_split = static_cast<int>(per);
  a.C = y;
  a.out_dtype = out_dtype;
  a.ldc = ldy;
  a.c_trans = 1;
  a.vec_ok = 0;
  a.tma_store = 0;  // transposed (swap-AB) output: per-thread stores
  a.epi = e;
  a.err = d->err;
  const int grid = static_cast<int>(std::min<int64_t>(tiles * splits, d->sm_count));

  if (splits > 1) {
    // Partial sums accumulate into the fixed scratch: zero the M x N part first.
    a.ws = d->scratch;
    a.ldw = N;
    SF_CUDA_TRY(cudaMemsetAsync(d->scratch, 0, static_cast<size_t>(M) * N * sizeof(float), s));
  }
  st = in_dtype == kBF16 ? launch<1>(bn, ma, mb, a, grid, s) : launch<0>(bn, ma, mb, a, grid, s);
  if (st != SF_OK) return st;
  if (splits > 1) {
    const int64_t total = M * N;
    const int fgrid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256,
                                                                               d->sm_count * 8LL)));
    epilogue_finalize_kernel<<<fgrid, 256, 0, s>>>(d->scratch, N, static_cast<int>(M),
                                                   static_cast<int>(N), y, out_dtype, ldy, e);
    SF_CUDA_TRY(cudaGetLastError());
  }
  return SF_OK;
}
