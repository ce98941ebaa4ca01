// Shared parts of the fused attention forward for sm_100a (head_dim 64):
// the launch arguments (AttnArgs), the packed fp32x2 / exp2 / 16-bit packing
// helpers the softmax uses, and the merge kernel of the stream-K tail.  The
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
  // Key blocks of a unit: nkb_a blocks of KB keys from key 0 cover
  // [0, skip_lo), then blocks from skip_hi cover [skip_hi, kv_len); nkb_e
  // blocks in all (the unit's effective blocks).
  int nkb_a, nkb_e;
  // Stream-K tail, so that the last wave of CTAs is not partly empty: the
  // tail kernel's tail_ctas CTAs share the effective key blocks of the last
  // tail_units units laid end to end, and the whole-unit kernel runs the first
  // split_first units on a 1-D grid (unit u = query block u % nqb, head
  // (u / nqb) % heads, batch u / (nqb * heads)) on the slots they leave: tail CTA c takes blocks
  // [c W / T, (c + 1) W / T) (W = tail_units * nkb_e, T = tail_ctas >=
  // tail_units), one or two segments (parts of consecutive units).  A
  // segment that covers a whole unit writes its output as usual; a part of
  // a unit writes its unnormalised fp32 O rows and (m, l) to workspace slot
  // 2 c + (segment index) of ws_o [slot][rows][64] / ws_ml [slot][rows][2],
  // and attention_merge_kernel combines the parts of each split unit (with
  // part_o / part_ml in mode 2, into part_o / part_ml in mode 1).
  int split_first;  // -1: 3-D grid (query unit, head, batch), no tail
  int tail_ctas, tail_units;
  int nqb;
  float* ws_o;
  float* ws_ml;
};

constexpr int kAttnBlock = 128;   // query rows per tile
constexpr int kAttnD = 64;        // head dim

// First effective block (within the tail's blocks laid end to end) of tail
// CTA c; c = tail_ctas gives the end.
__device__ __forceinline__ int64_t attn_tail_lo(const AttnArgs& p, int c) {
  return static_cast<int64_t>(c) * (static_cast<int64_t>(p.tail_units) * p.nkb_e) / p.tail_ctas;
}

// The tail CTA whose block range holds tail block g: the largest c with
// attn_tail_lo(c) <= g.
__device__ __forceinline__ int attn_tail_cta(const AttnArgs& p, int64_t g) {
  const int64_t w = static_cast<int64_t>(p.tail_units) * p.nkb_e;
  return static_cast<int>(((g + 1) * p.tail_ctas - 1) / w);
}

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

// Two 16-bit products a * b (bf16x2 or f16x2, round to nearest).
__device__ __forceinline__ uint32_t mul_16bit2(uint32_t a, uint32_t b, bool bf16) {
  if (bf16) {
    const __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                     *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// Sum-first softmax: a row keeps its integer exponent base while the
// p = 2^(c s - m) of a key block sum to less than this; a block that reaches
// it raises the base by floor(log2 sum) + 1.
constexpr float kAttnSumLimit = 256.0f;

// Max-first softmax: the base is raised to ceil(c * block max) only when that
// exceeds it by more than this (p then stays below 2^8 before the rescale).
constexpr float kAttnRescaleLog2 = 8.0f;

// Combines the parts of each split tail unit, and in part_mode 2 the
// partial result in part_o / part_ml (one CTA per tail unit of ROWS query
// rows, one thread per row): with integer bases m_i, m = max m_i,
// O = sum 2^(m_i - m) O_i / sum 2^(m_i - m) l_i, written as 16-bit O; in
// part_mode 1 the combined unnormalised sum and (m, l) go to part_o /
// part_ml instead.  A unit that one CTA ran whole was written by it.
template <bool BF16, int ROWS>
__global__ void __launch_bounds__(ROWS) attention_merge_kernel(const AttnArgs p) {
  const int i = static_cast<int>(blockIdx.x);
  const int64_t ne = p.nkb_e;
  const int c0 = attn_tail_cta(p, i * ne), c1 = attn_tail_cta(p, (i + 1) * ne - 1);
  if (c0 == c1) return;
  const int u = p.split_first + i;
  const int qb = u % p.nqb, h = (u / p.nqb) % p.heads, b = u / (p.nqb * p.heads);
  const int row = threadIdx.x;
  const int qrow = qb * ROWS + row;
  if (qrow >= p.q_len) return;
  const int64_t prow = (static_cast<int64_t>(b) * p.q_len + qrow) * p.heads + h;
  // input c in [c0, c1]: the part tail CTA c ran (its first or second
  // segment); c1 + 1: the partial result of mode 2
  const int n_in = c1 + 1 + (p.part_mode == 2 ? 1 : 0);
  auto slot_of = [&](int c) -> int64_t {
    return 2 * c + (attn_tail_lo(p, c) / ne == i ? 0 : 1);
  };
  auto ml_of = [&](int c) -> const float* {
    return c <= c1 ? p.ws_ml + (slot_of(c) * ROWS + row) * 2 : p.part_ml + 2 * prow;
  };
  auto o_of = [&](int c) -> const float* {
    return c <= c1 ? p.ws_o + (slot_of(c) * ROWS + row) * kAttnD : p.part_o + prow * kAttnD;
  };
  float m = -INFINITY;
  for (int c = c0; c < n_in; ++c) m = fmaxf(m, ml_of(c)[0]);
  float l = 0.0f;
  float acc[kAttnD];
#pragma unroll
  for (int t = 0; t < kAttnD; ++t) acc[t] = 0.0f;
  for (int c = c0; c < n_in; ++c) {
    const float* ml = ml_of(c);
    if (ml[0] == -INFINITY) continue;  // every key of this input skipped
    const float a = ex2_approx(ml[0] - m);
    l += ml[1] * a;
    const float4* po = reinterpret_cast<const float4*>(o_of(c));
#pragma unroll
    for (int q = 0; q < kAttnD / 4; ++q) {
      const float4 v = po[q];
      acc[4 * q] += v.x * a;
      acc[4 * q + 1] += v.y * a;
      acc[4 * q + 2] += v.z * a;
      acc[4 * q + 3] += v.w * a;
    }
  }
  if (p.part_mode == 1) {
    p.part_ml[2 * prow] = m;
    p.part_ml[2 * prow + 1] = l;
    float4* po = reinterpret_cast<float4*>(p.part_o + prow * kAttnD);
#pragma unroll
    for (int q = 0; q < kAttnD / 4; ++q)
      po[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
    return;
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
