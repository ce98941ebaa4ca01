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
#include "ptx.cuh"

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

// ───────────────────────── balanced (segmented) GEMV ─────────────────────────
//
// One CTA of kSegWarps warps per SM.  CTA c owns the contiguous weight rows
// [c*N/G, (c+1)*N/G) (G = grid size), so every SM streams the same number
// of bytes to within one row.  Inside the CTA the work is cut into units of
// (group of R rows) x (512-byte column step); warp w takes the contiguous
// unit range [w*U/W, (w+1)*U/W), so warps are balanced to one unit instead of
// one row.  A warp folds each finished row group into per-row fp32 sums in
// shared memory (warp butterfly + one shared atomic per row and activation
// row); after a CTA barrier the fused epilogue writes the CTA's outputs.
// Requires K % 256 == 0 and 16-byte aligned rows of x and W.
//
// Programmatic dependent launch: the kernel lets the next one in the stream
// start at once, and before it waits for the previous grid (griddepcontrol)
// it only zeroes its shared memory and prefetches the first `pf_units` units
// of each warp's weights into L2 -- the weights are not written by any
// kernel on the path, while x and y are touched only after the wait.  Back to
// back launches so overlap one kernel's launch, prologue and first weight
// bytes with the previous kernel's tail.
constexpr int kSegWarps = 16;

template <int MM, int R, int U, bool BF16>
static __global__ void __launch_bounds__(kSegWarps * 32, 1)
    gemv_seg_kernel(const uint16_t* __restrict__ x, int64_t ldx, const uint16_t* __restrict__ W,
                    int64_t ldw, void* __restrict__ y, int out_dtype, int64_t ldy, int N, int K,
                    EpilogueArgs e, int pf_units) {
  extern __shared__ float sacc[];  // [rows of this CTA][MM]
  pdl_launch_dependents();
  const int G = gridDim.x;
  const int r0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * N / G);
  const int r1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * N / G);
  const int rows = r1 - r0;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int spr = K >> 8;                       // 512-byte steps per row
  const int groups = (rows + R - 1) / R;
  const int total = groups * spr;
  const int u0 = static_cast<int>(static_cast<int64_t>(warp) * total / kSegWarps);
  const int u1 = static_cast<int>(static_cast<int64_t>(warp + 1) * total / kSegWarps);
  // L2 prefetch of this warp's first units: lane l takes row l % R of unit l / R.
  for (int l = lane; l < pf_units * R; l += 32) {
    const int uu = u0 + l / R;
    const int g = uu / spr;
    const int row = r0 + g * R + l % R;
    if (uu < u1 && row < r1)
      prefetch_l2_bulk(W + static_cast<int64_t>(row) * ldw + (uu - g * spr) * 256, 512);
  }
  for (int t = threadIdx.x; t < rows * MM; t += blockDim.x) sacc[t] = 0.0f;
  pdl_wait();
  __syncthreads();

  float acc[R][MM];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MM; ++m) acc[r][m] = 0.0f;

  auto flush = [&](int g) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MM; ++m) {
        float v = acc[r][m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][m] = 0.0f;
        const int row = g * R + r;
        if (lane == 0 && row < rows) atomicAdd(&sacc[row * MM + m], v);
      }
  };

  int cur_g = u0 < u1 ? u0 / spr : 0;
  for (int u = u0; u < u1; u += U) {
    uint4 wv[U][R];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int uu = u + j;
      const int g = uu / spr;
      const int col = (uu - g * spr) * 32 + lane;  // 16-byte chunk index within the row
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = r0 + g * R + r;
        wv[j][r] = (uu < u1 && row < r1)
                       ? __ldcs(reinterpret_cast<const uint4*>(W + static_cast<int64_t>(row) * ldw) + col)
                       : make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int uu = u + j;
      if (uu >= u1) break;  // warp-uniform
      const int g = uu / spr;
      if (g != cur_g) {     // warp-uniform
        flush(cur_g);
        cur_g = g;
      }
      const int col = (uu - g * spr) * 32 + lane;
      float xf[MM][8];
#pragma unroll
      for (int m = 0; m < MM; ++m)
        unpack8(__ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(m) * ldx) + col), BF16,
                xf[m]);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float wf[8];
        unpack8(wv[j][r], BF16, wf);
#pragma unroll
        for (int m = 0; m < MM; ++m)
#pragma unroll
          for (int t = 0; t < 8; ++t) acc[r][m] = fmaf(wf[t], xf[m][t], acc[r][m]);
      }
    }
  }
  if (u0 < u1) flush(cur_g);
  __syncthreads();

  // Epilogue: consecutive threads take consecutive output columns n.
  for (int t = threadIdx.x; t < rows * MM; t += blockDim.x) {
    const int m = t / rows;
    const int rr = t - m * rows;
    const int n = r0 + rr;
    const float bias_v = e.bias ? load_as_f32(e.bias, n, e.bias_dtype) : 0.0f;
    const float res_v =
        e.residual ? load_as_f32(e.residual, static_cast<int64_t>(m) * e.ldr + n, e.residual_dtype) : 0.0f;
    store_from_f32(y, static_cast<int64_t>(m) * ldy + n, out_dtype,
                   epilogue_value(sacc[rr * MM + m], e, bias_v, res_v));
  }
}

}  // namespace sf
