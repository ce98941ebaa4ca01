// Shared parts of the fused attention forward for sm_100a (head_dim 64):
// the launch arguments (AttnArgs), the packed fp32x2 / exp2 / 16-bit packing
// helpers the softmax uses, and the merge kernel of the split dispatch.  The
// kernel itself is attention_pp_kernel (attention_pp.cuh).
//
// The fused attention computes O[b, h] = softmax(scale * Q[b, h] K[b, h]^T)
// V[b, h] with the scores S and probabilities P kept on chip.  It replaces
// the unfused chain of the reference's scaled_dot_product_attention
// (nn/functional.py:310-321: dev_batched_matmul_nt -> dev_muls ->
// dev_softmax -> dev_batched_matmul) and the DiT attention einsum
// (diffusion/models.py:529-536), whose fp32 score matrix makes the unfused
// path HBM-bound.
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
  // Keys [skip_lo, skip_hi) are left out (none
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
  // Split dispatch (part_mode 0 or 2), so that the
  // last wave of CTAs is not mostly empty: a 1-D grid whose blocks
  // [0, split_first) are whole units u (query block u % nqb, head
  // (u / nqb) % heads, batch u / (nqb * heads)); block split_first + j is
  // piece j % split_k of unit split_first + j / split_k, a contiguous share
  // of the key blocks, and writes its unnormalised fp32 O rows and (m, l)
  // to slot j of ws_o [slot][rows][64] / ws_ml [slot][rows][2] (zeros and
  // m = -inf when all its keys are skipped); attention_merge_kernel then
  // combines the pieces of each split unit (and part_o / part_ml in mode 2).
  int split_first;  // -1: 3-D grid (query unit, head, batch), no pieces
  int split_k;
  int nqb;
  float* ws_o;
  float* ws_ml;
};

constexpr int kAttnBlock = 128;   // query rows per tile
constexpr int kAttnD = 64;        // head dim

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

__device__ __forceinline__ uint32_t pack_16bit(float a, float b, bool bf16) {
  if (bf16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Row exponent bases are raised only when a block's ceil(c * max) exceeds
// them by more than this (p then stays below 2^8 before the rescale).
constexpr float kAttnRescaleLog2 = 8.0f;

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
