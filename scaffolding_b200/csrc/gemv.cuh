// Skinny-M linear as a bandwidth-bound GEMV:  y[m, n] = epi(sum_k x[m, k] W[n, k])
// for M <= 4 activation rows, 16-bit x and W (nn.Linear weight layout [N, K]).
//
// The decode-style shape of benchmark config 3 (M = 1 .. 4, K = 4096,
// N = 4096 / 11008) is a pure weight stream: every weight byte is used M
// times, so the kernel is bound by HBM, not by the tensor cores.  Design:
//   * each warp owns R consecutive weight rows; a lane reads 16 bytes
//     (8 elements) of each row per step, so one warp-wide load instruction
//     covers 512 contiguous bytes of a row (fully coalesced), with R
//     independent loads in flight per lane per step;
//   * the M activation rows (a few KB) are read through the read-only cache
//     and reused by every warp of the SM;
//   * fp32 accumulation, then a butterfly warp-shuffle reduction and the
//     fused epilogue (alpha, bias, activation, residual, cast) by R*M lanes;
//   * no workspace, one launch.
// Replaces, for this shape, the cuBLAS SGEMM + bias + activation launches of
// dev_linear_forward (_cuda_ops.pyx:1278-1302).
#pragma once
#include <cstdint>

#include "epilogue.cuh"

namespace sf {

constexpr int kGemvWarps = 8;

__device__ __forceinline__ void unpack8(const uint4 u, bool bf16, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    if (bf16) {
      f[2 * h] = __uint_as_float(w[h] << 16);
      f[2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
    } else {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[h]));
      f[2 * h] = v.x;
      f[2 * h + 1] = v.y;
    }
  }
}

// MM activation rows, R weight rows per warp.  Requires K % 8 == 0 and
// 16-byte aligned rows of x and W (checked by the dispatcher).
template <int MM, int R, bool BF16>
static __global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_kernel(const uint16_t* __restrict__ x, int64_t ldx, const uint16_t* __restrict__ W,
                int64_t ldw, void* __restrict__ y, int out_dtype, int64_t ldy, int N, int K,
                EpilogueArgs e) {
  const int lane = threadIdx.x & 31;
  const int warp_global = blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
  const int n0 = warp_global * R;
  if (n0 >= N) return;  // warp-uniform
  const int chunks = K >> 3;  // 8-element (16-byte) chunks per row

  float acc[R][MM];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MM; ++m) acc[r][m] = 0.0f;

  const uint4* wrow[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int n = min(n0 + r, N - 1);  // rows past N repeat the last row; never stored
    wrow[r] = reinterpret_cast<const uint4*>(W + (int64_t)n * ldw);
  }
  const uint4* xrow[MM];
#pragma unroll
  for (int m = 0; m < MM; ++m) xrow[m] = reinterpret_cast<const uint4*>(x + (int64_t)m * ldx);

#pragma unroll 2
  for (int c = lane; c < chunks; c += 32) {
    uint4 wv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) wv[r] = __ldcs(wrow[r] + c);  // streamed once: evict-first
    float xf[MM][8];
#pragma unroll
    for (int m = 0; m < MM; ++m) unpack8(__ldg(xrow[m] + c), BF16, xf[m]);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float wf[8];
      unpack8(wv[r], BF16, wf);
#pragma unroll
      for (int m = 0; m < MM; ++m)
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[r][m] = fmaf(wf[t], xf[m][t], acc[r][m]);
    }
  }

  // Butterfly reduction: every lane ends with every sum.
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MM; ++m)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);

  // Lane t stores output (r, m) = (t / MM, t % MM).
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MM; ++m) {
      if (lane == r * MM + m) {
        const int n = n0 + r;
        if (n < N) {
          const float bias_v = e.bias ? load_as_f32(e.bias, n, e.bias_dtype) : 0.0f;
          const float res_v =
              e.residual ? load_as_f32(e.residual, (int64_t)m * e.ldr + n, e.residual_dtype) : 0.0f;
          store_from_f32(y, (int64_t)m * ldy + n, out_dtype,
                         epilogue_value(acc[r][m], e, bias_v, res_v));
        }
      }
    }
}

}  // namespace sf
