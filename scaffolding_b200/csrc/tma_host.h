// Host-side helpers shared by the engine's translation units: TMA tensor-map
// encoding (the driver's cuTensorMapEncodeTiled, resolved once through the
// runtime), dtype facts, alignment checks and the tuning-knob reader.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "common.h"
#include "epilogue.cuh"
#include "ptx.cuh"

namespace sf {

// ───────────────────────────── TMA descriptors ─────────────────────────────

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

// 4-D view: element (i0, i1, i2, i3) at base + i1*s1 + i2*s2 + i3*s3 (elements),
// i0 contiguous.  Extent-1 batch dims get a packed stride.
struct MapSpec {
  const void* base;
  int esize;
  CUtensorMapDataType dt;
  uint64_t d0, d1, d2, d3;
  int64_t s1, s2, s3;
  uint32_t box0, box1;
};

inline int32_t encode_map(CUtensorMap* m, const MapSpec& s) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const uint64_t e = static_cast<uint64_t>(s.esize);
  uint64_t st1 = static_cast<uint64_t>(s.s1) * e;
  uint64_t st2 = s.d2 > 1 ? static_cast<uint64_t>(s.s2) * e : st1 * s.d1;
  uint64_t st3 = s.d3 > 1 ? static_cast<uint64_t>(s.s3) * e : st2 * s.d2;
  st2 = (st2 + 15) & ~15ull;
  st3 = (st3 + 15) & ~15ull;
  cuuint64_t dims[4] = {s.d0, s.d1, s.d2, s.d3};
  cuuint64_t strides[3] = {st1, st2, st3};
  cuuint32_t box[4] = {s.box0, s.box1, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, s.dt, 4, const_cast<void*>(s.base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SF_ERR_CUDA,
                "cuTensorMapEncodeTiled failed (%d): dims {%llu,%llu,%llu,%llu} strides "
                "{%llu,%llu,%llu} box {%u,%u}",
                static_cast<int>(r), (unsigned long long)s.d0, (unsigned long long)s.d1,
                (unsigned long long)s.d2, (unsigned long long)s.d3, (unsigned long long)st1,
                (unsigned long long)st2, (unsigned long long)st3, s.box0, s.box1);
  return SF_OK;
}

inline CUtensorMapDataType tma_dtype(int dt) {
  return dt == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
         : dt == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}

inline int esize(int dt) { return dt == kF32 ? 4 : 2; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool bytes16(int64_t elems, int es) { return ((elems * es) & 15) == 0; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

}  // namespace sf
