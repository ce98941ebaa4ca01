// SIMT FFMA GEMM for any layout and input dtype, fp32 accumulation.
//
// Serves two roles:
//   * the exact-fp32 "FFMA" mode of the fp32 path (IEEE fp32 multiply-add,
//     no TF32 rounding anywhere), matching the default non-TF32 cuBLAS SGEMM
//     math the reference uses (_cuda_kernels.cu:1175-1220, TF32 off by
//     default per backends/cuda.py:20-35);
//   * shapes/layouts the tcgen05 kernel cannot take through TMA (row strides
//     that are not 16-byte multiples, transposed A, misaligned bases).
//
// Tile 128x128x8, 256 threads, each thread owns an 8x8 micro-tile
// (two 4x4 quadrants at stride 64 to keep shared-memory reads conflict-free);
// global->shared staging is register double-buffered.
#pragma once
#include <cstdint>

#include "epilogue.cuh"

namespace sf {

struct GemmSimtArgs {
  int M, N, K;
  int nb0, nb1;
  // element (m, k) of A at A[b0*a_s0 + b1*a_s1 + m*a_rs + k*a_cs]
  const void* A;
  int a_dtype;
  int64_t a_rs, a_cs, a_s0, a_s1;
  // element (k, n) of B at B[b0*b_s0 + b1*b_s1 + k*b_ks + n*b_ns]
  const void* B;
  int b_dtype;
  int64_t b_ks, b_ns, b_s0, b_s1;
  void* C;
  int out_dtype;
  int64_t ldc, c_s0, c_s1;
  EpilogueArgs epi;
};

constexpr int kSimtBM = 128, kSimtBN = 128, kSimtBK = 8, kSimtThreads = 256;

static __global__ void __launch_bounds__(kSimtThreads)
    gemm_simt_kernel(const GemmSimtArgs p) {
  __shared__ float As[2][kSimtBK][kSimtBM];
  __shared__ float Bs[2][kSimtBK][kSimtBN];

  const int bz = blockIdx.z;
  const int b0 = bz % p.nb0, b1 = bz / p.nb0;
  const int m0 = blockIdx.y * kSimtBM, n0 = blockIdx.x * kSimtBN;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;

  const int64_t aoff = (int64_t)b0 * p.a_s0 + (int64_t)b1 * p.a_s1;
  const int64_t boff = (int64_t)b0 * p.b_s0 + (int64_t)b1 * p.b_s1;

  // Each thread stages 4 A values and 4 B values per k-tile.
  float ra[4], rb[4];
  auto load_tile = [&](int k0) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int idx = tid + t * kSimtThreads;  // 0..1023
      // A: 128 rows x 8 k; consecutive threads walk k fastest when A is K-contiguous.
      const int am = idx >> 3, ak = idx & 7;
      const int gm = m0 + am, gk = k0 + ak;
      ra[t] = (gm < p.M && gk < p.K)
                  ? load_as_f32(p.A, aoff + (int64_t)gm * p.a_rs + (int64_t)gk * p.a_cs, p.a_dtype)
                  : 0.0f;
      // B: 8 k x 128 n.
      int bk, bn;
      if (p.b_ns == 1) {
        bk = idx >> 7;
        bn = idx & 127;
      } else {
        bn = idx >> 3;
        bk = idx & 7;
      }
      const int gn = n0 + bn, gk2 = k0 + bk;
      rb[t] = (gn < p.N && gk2 < p.K)
                  ? load_as_f32(p.B, boff + (int64_t)gk2 * p.b_ks + (int64_t)gn * p.b_ns, p.b_dtype)
                  : 0.0f;
    }
  };
  auto store_tile = [&](int buf) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int idx = tid + t * kSimtThreads;
      const int am = idx >> 3, ak = idx & 7;
      As[buf][ak][am] = ra[t];
      int bk, bn;
      if (p.b_ns == 1) {
        bk = idx >> 7;
        bn = idx & 127;
      } else {
        bn = idx >> 3;
        bk = idx & 7;
      }
      Bs[buf][bk][bn] = rb[t];
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  const int ktiles = (p.K + kSimtBK - 1) / kSimtBK;
  load_tile(0);
  store_tile(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load_tile((kt + 1) * kSimtBK);
#pragma unroll
    for (int kk = 0; kk < kSimtBK; ++kk) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4 + 64]);
      const float4 c0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 c1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4 + 64]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = c0.x; b[1] = c0.y; b[2] = c0.z; b[3] = c0.w;
      b[4] = c1.x; b[5] = c1.y; b[6] = c1.z; b[7] = c1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) store_tile(buf ^ 1);
    __syncthreads();
  }

  const EpilogueArgs& e = p.epi;
  const int64_t coff = (int64_t)b0 * p.c_s0 + (int64_t)b1 * p.c_s1;
  const int64_t roff = (int64_t)b0 * e.r_stride0 + (int64_t)b1 * e.r_stride1;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + ty * 4 + (i & 3) + (i >> 2) * 64;
    if (gm >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + tx * 4 + (j & 3) + (j >> 2) * 64;
      if (gn >= p.N) continue;
      const float bias_v = e.bias ? load_as_f32(e.bias, gn, e.bias_dtype) : 0.0f;
      const float res_v =
          e.residual ? load_as_f32(e.residual, roff + (int64_t)gm * e.ldr + gn, e.residual_dtype)
                     : 0.0f;
      store_from_f32(p.C, coff + (int64_t)gm * p.ldc + gn, p.out_dtype,
                     epilogue_value(acc[i][j], e, bias_v, res_v));
    }
  }
}

}  // namespace sf
