// Fused GEMM epilogue math: alpha scale, bias, activation, residual, and
// fp32 -> fp32/bf16/fp16 conversion.  Shared by the tcgen05 GEMM, the FFMA
// GEMM, the split-K finaliser and the standalone elementwise kernels so that
// every path applies bit-identical arithmetic.
//
// Reference arithmetic being fused (all fp32):
//   bias add      C[i,j] += b[j]                     _cuda_kernels.cu:1490-1527
//   SiLU          x * (1 / (1 + exp(-x)))            nn/functional.py:57-59
//   GELU (tanh)   0.5x(1+tanh(sqrt(2/pi)(x+0.044715x^3)))  nn/functional.py:79-82
//   scalar mul    y = s * x                          _cuda_kernels.cu:237-277
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace sf {

enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };
enum Act : int { kActNone = 0, kActSilu = 1, kActGeluTanh = 2 };

__device__ __forceinline__ float act_apply(float z, int act) {
  if (act == kActSilu) {
    const float sig = 1.0f / (1.0f + expf(-z));
    return z * sig;
  }
  if (act == kActGeluTanh) {
    const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
    return 0.5f * z * (1.0f + tanhf(k0 * (z + 0.044715f * z * z * z)));
  }
  return z;
}

// Fast forms for 16-bit outputs, where the result is rounded to 8 (bf16) or
// 11 (fp16) significant bits anyway.  GELU-tanh uses the identity
// 0.5 * (1 + tanh(u)) = 1 / (1 + exp(-2u)); both use the hardware exp2
// intrinsic and a fast divide.
__device__ __forceinline__ float act_apply_fast(float z, int act) {
  if (act == kActSilu) return __fdividef(z, 1.0f + __expf(-z));
  if (act == kActGeluTanh) {
    const float u = 0.7978845608028654f * (z + 0.044715f * z * z * z);
    return __fdividef(z, 1.0f + __expf(-2.0f * u));
  }
  return z;
}

__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int dtype) {
  if (dtype == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_f32(void* p, int64_t i, int dtype, float v) {
  if (dtype == kBF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == kF16)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int dtype) {
  if (dtype == kBF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Parameters of the fused epilogue  D = act(alpha * acc + bias) + beta * R.
struct EpilogueArgs {
  float alpha;
  float beta;
  int fast_act;          // 1: act_apply_fast (16-bit outputs)
  int bias_vec;          // 1: bias rows may be read with 16-byte vector loads
  int res_vec;           // 1: residual rows may be read with 16-byte vector loads
  const void* bias;      // indexed by output column (or by output row if bias_on_rows)
  int bias_dtype;
  int bias_on_rows;
  int act;
  const void* residual;  // same indexing as the output, own leading dimension
  int residual_dtype;
  int64_t ldr;
  int64_t r_stride0, r_stride1;  // batch strides of the residual
};

__device__ __forceinline__ float epilogue_value(float acc, const EpilogueArgs& e, float bias_v,
                                                float res_v) {
  float v = e.alpha * acc + bias_v;
  v = e.fast_act ? act_apply_fast(v, e.act) : act_apply(v, e.act);
  if (e.residual != nullptr) v += e.beta * res_v;
  return v;
}

}  // namespace sf
