// LayerNorm with the adaptive (adaLN) scale / shift of the DiT blocks, as one
// bandwidth kernel in front of the QKV and FFN-up GEMMs:
//
//   y[r, :] = ((x[r, :] - mean) / sqrt(var + eps) * gamma + beta) * (1 + scale[g]) + shift[g]
//
// with mean and var (population) over the row's C columns, g = r / group_rows
// the sample the row belongs to, and scale[g] = mod[g, 0:C],
// shift[g] = mod[g, C:2C] the output of the block's modulation linear
// (AdaLayerNorm.forward, diffusion/models.py:478-487: norm, then
// `h * (params[..., :C] + 1) + params[..., C:]`).  Without `mod` it is the
// plain LayerNorm of cuda_layer_norm_f32 (_cuda_kernels.cu:1070-1093,
// nn/layers.py:470-493), any of fp32 / bf16 / fp16 in and out.
//
// One warp per row; the row is held in registers (16-byte vector loads,
// NV vectors per lane), so x is read from HBM once and y written once:
// 4 B per element for 16-bit in and out.  The row stays packed as loaded and
// is unpacked in each pass (half the registers for 16-bit rows).  The
// per-group scale / shift rows and gamma / beta are read as 16-byte vectors
// too (they stay in L1 / L2).  Mean, then the sum of squared deviations (two
// passes over the registers, as the reference kernel and NumPy's var do),
// fp32 throughout; rows wider than the register budget take a loop that
// re-reads the row from L1/L2 instead.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.h"
#include "epilogue.cuh"
#include "tma_host.h"

namespace sf {
namespace {

struct NormArgs {
  int64_t rows;
  int cols;
  const void* x;
  int x_dtype;
  int64_t ldx;
  const float* gamma;  // [cols] or null
  const float* beta;   // [cols] or null
  float eps;
  const void* mod;     // [groups][2 * cols] or null
  int mod_dtype;
  int64_t ld_mod;
  int64_t group_rows;
  void* y;
  int y_dtype;
  int64_t ldy;
};

__device__ __forceinline__ float load_elem(const void* p, int dt, int64_t i) {
  if (dt == kF32) return static_cast<const float*>(p)[i];
  if (dt == kBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void store_elem(void* p, int dt, int64_t i, float v) {
  if (dt == kF32)
    static_cast<float*>(p)[i] = v;
  else if (dt == kBF16)
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half*>(p)[i] = __float2half_rn(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Unpacks 16 bytes of elements (4 x fp32 when E == 4, else 8 x bf16 / fp16).
template <int E, bool BF16>
__device__ __forceinline__ void unpack16(const uint4& u, float* f) {
  if constexpr (E == 4) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (BF16) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      } else {
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
      }
    }
  }
}

// Row held in registers: NV 16-byte vectors per lane of E elements each;
// each warp loads RPW rows at once (more bytes in flight per warp).  x, y
// and the modulation rows share one element type (fp32 when E == 4, else
// bf16 / fp16 as BF16 says).
template <int E, bool BF16, int NV, int RPW>
__global__ void __launch_bounds__(256, 2) layernorm_mod_vec_kernel(const NormArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int nvec = a.cols / E;  // vectors per row
  const float inv_c = 1.0f / static_cast<float>(a.cols);
  constexpr int ES = E == 4 ? 4 : 2;
  for (int64_t r0 = warp0 * RPW; r0 < a.rows; r0 += nwarps * RPW) {
    uint4 raw[RPW][NV];  // the rows, packed as loaded
#pragma unroll
    for (int q = 0; q < RPW; ++q) {
      const int64_t r = r0 + q;
      const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const char*>(a.x) + r * a.ldx * ES);
#pragma unroll
      for (int k = 0; k < NV; ++k)
        if (r < a.rows && lane + 32 * k < nvec) raw[q][k] = __ldg(xr + lane + 32 * k);
    }
#pragma unroll
    for (int q = 0; q < RPW; ++q) {
      const int64_t r = r0 + q;
      if (r >= a.rows) break;
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < NV; ++k)
        if (lane + 32 * k < nvec) {
          float f[E];
          unpack16<E, BF16>(raw[q][k], f);
#pragma unroll
          for (int e = 0; e < E; ++e) s += f[e];
        }
      const float mean = warp_sum(s) * inv_c;
      float ss = 0.0f;
#pragma unroll
      for (int k = 0; k < NV; ++k)
        if (lane + 32 * k < nvec) {
          float f[E];
          unpack16<E, BF16>(raw[q][k], f);
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const float d = f[e] - mean;
            ss += d * d;
          }
        }
      const float rstd = 1.0f / sqrtf(warp_sum(ss) * inv_c + a.eps);
      // scale / shift rows of this row's group (16-byte vectors, from L1 / L2)
      const uint4* msc = a.mod ? reinterpret_cast<const uint4*>(static_cast<const char*>(a.mod) +
                                                                (r / a.group_rows) * a.ld_mod * ES)
                               : nullptr;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int vi = lane + 32 * k;
        if (vi >= nvec) continue;
        float v[E];
        unpack16<E, BF16>(raw[q][k], v);
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = (v[e] - mean) * rstd;
        if (a.gamma) {
#pragma unroll
          for (int e = 0; e < E; e += 4) {
            const float4 g4 = __ldg(reinterpret_cast<const float4*>(a.gamma + vi * E + e));
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(a.beta + vi * E + e));
            v[e] = v[e] * g4.x + b4.x;
            v[e + 1] = v[e + 1] * g4.y + b4.y;
            v[e + 2] = v[e + 2] * g4.z + b4.z;
            v[e + 3] = v[e + 3] * g4.w + b4.w;
          }
        }
        if (msc) {
          float sc[E], sh[E];
          unpack16<E, BF16>(__ldg(msc + vi), sc);
          unpack16<E, BF16>(__ldg(msc + nvec + vi), sh);
#pragma unroll
          for (int e = 0; e < E; ++e) v[e] = v[e] * (sc[e] + 1.0f) + sh[e];
        }
        char* yr = static_cast<char*>(a.y) + (r * a.ldy + static_cast<int64_t>(vi) * E) * ES;
        if constexpr (E == 4) {
          *reinterpret_cast<float4*>(yr) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            if constexpr (BF16) {
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[e], v[e + 1]);
              w[e / 2] = *reinterpret_cast<const uint32_t*>(&h2);
            } else {
              const __half2 h2 = __floats2half2_rn(v[e], v[e + 1]);
              w[e / 2] = *reinterpret_cast<const uint32_t*>(&h2);
            }
          }
          *reinterpret_cast<uint4*>(yr) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
}

// Any width, alignment and dtype: the row is re-read (from L1/L2) per pass.
__global__ void __launch_bounds__(256) layernorm_mod_generic_kernel(const NormArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const float inv_c = 1.0f / static_cast<float>(a.cols);
  for (int64_t r = warp0; r < a.rows; r += nwarps) {
    float s = 0.0f;
    for (int c = lane; c < a.cols; c += 32) s += load_elem(a.x, a.x_dtype, r * a.ldx + c);
    const float mean = warp_sum(s) * inv_c;
    float q = 0.0f;
    for (int c = lane; c < a.cols; c += 32) {
      const float d = load_elem(a.x, a.x_dtype, r * a.ldx + c) - mean;
      q += d * d;
    }
    const float rstd = 1.0f / sqrtf(warp_sum(q) * inv_c + a.eps);
    const int64_t g = a.mod ? r / a.group_rows : 0;
    for (int c = lane; c < a.cols; c += 32) {
      float h = (load_elem(a.x, a.x_dtype, r * a.ldx + c) - mean) * rstd;
      if (a.gamma) h *= a.gamma[c];
      if (a.beta) h += a.beta[c];
      if (a.mod)
        h = h * (load_elem(a.mod, a.mod_dtype, g * a.ld_mod + c) + 1.0f) +
            load_elem(a.mod, a.mod_dtype, g * a.ld_mod + a.cols + c);
      store_elem(a.y, a.y_dtype, r * a.ldy + c, h);
    }
  }
}

template <int E, bool BF16>
void launch_vec(const NormArgs& a, int nv, unsigned grid, cudaStream_t s) {
  switch (nv) {
    case 1: layernorm_mod_vec_kernel<E, BF16, 1, 4><<<grid, 256, 0, s>>>(a); break;
    case 2: layernorm_mod_vec_kernel<E, BF16, 2, 4><<<grid, 256, 0, s>>>(a); break;
    case 4: layernorm_mod_vec_kernel<E, BF16, 4, 2><<<grid, 256, 0, s>>>(a); break;
    case 8: layernorm_mod_vec_kernel<E, BF16, 8, 2><<<grid, 256, 0, s>>>(a); break;
    default: layernorm_mod_vec_kernel<E, BF16, 16, 1><<<grid, 256, 0, s>>>(a); break;
  }
}

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" int32_t sf_layernorm_modulate(int64_t rows, int64_t cols, const void* x, int32_t x_dtype,
                                         int64_t ldx, const float* gamma, const float* beta,
                                         float eps, const void* mod, int32_t mod_dtype,
                                         int64_t ld_mod, int64_t group_rows, void* y,
                                         int32_t y_dtype, int64_t ldy, void* stream) {
  if (rows < 0 || cols < 0) return fail(SF_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0 || cols == 0) return SF_OK;
  if (cols > (1 << 24)) return fail(SF_ERR_UNSUPPORTED, "layer norm over %lld columns", (long long)cols);
  if (!x || !y) return fail(SF_ERR_INVALID_ARGUMENT, "null pointer");
  for (int dt : {x_dtype, y_dtype})
    if (dt != kF32 && dt != kF16 && dt != kBF16) return fail(SF_ERR_INVALID_ARGUMENT, "dtype %d", dt);
  if (ldx < cols || ldy < cols) return fail(SF_ERR_INVALID_ARGUMENT, "leading dimension < cols");
  if (!(eps >= 0.0f)) return fail(SF_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (mod) {
    if (mod_dtype != kF32 && mod_dtype != kF16 && mod_dtype != kBF16)
      return fail(SF_ERR_INVALID_ARGUMENT, "modulation dtype %d", mod_dtype);
    if (group_rows < 1) return fail(SF_ERR_INVALID_ARGUMENT, "group_rows must be >= 1");
    if (ld_mod < 2 * cols) return fail(SF_ERR_INVALID_ARGUMENT, "modulation row < 2 * cols");
  }
  DeviceInfo* dev = nullptr;
  int32_t st = current_device_info(&dev, nullptr);
  if (st != SF_OK) return st;
  NormArgs a{rows, static_cast<int>(cols), x, x_dtype, ldx, gamma, beta, eps, mod, mod_dtype, ld_mod,
             group_rows, y, y_dtype, ldy};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // 8 warps per CTA, at most 16 CTAs per SM, grid-stride over the rows.
  const unsigned grid = static_cast<unsigned>(
      std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, 8), dev->sm_count * 16LL)));
  // Register-resident rows need 16-byte vectors on both sides: one element
  // type in and out, 16-byte aligned bases and row strides.
  const int es = x_dtype == kF32 ? 4 : 2;
  const int E = 16 / es;
  // The modulation rows are read as vectors of x's type; gamma / beta as float4.
  const bool vec = x_dtype == y_dtype && cols % E == 0 && aligned16(x) &&
                   aligned16(y) && bytes16(ldx, es) && bytes16(ldy, es) &&
                   (!mod || (mod_dtype == x_dtype && aligned16(mod) && bytes16(ld_mod, es))) &&
                   (!gamma || (aligned16(gamma) && aligned16(beta)));
  const int64_t per_lane = ceil_div(cols / E, 32);
  if (vec && per_lane <= 16) {
    const int nv = per_lane <= 1 ? 1 : per_lane <= 2 ? 2 : per_lane <= 4 ? 4 : per_lane <= 8 ? 8 : 16;
    if (x_dtype == kF32)
      launch_vec<4, false>(a, nv, grid, s);
    else if (x_dtype == kBF16)
      launch_vec<8, true>(a, nv, grid, s);
    else
      launch_vec<8, false>(a, nv, grid, s);
  } else {
    layernorm_mod_generic_kernel<<<grid, 256, 0, s>>>(a);
  }
  if (st != SF_OK) return st;
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}
