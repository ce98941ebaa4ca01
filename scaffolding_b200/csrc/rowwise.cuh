// Bandwidth-bound companions of the GEMMs: row softmax, elementwise
// activation/scale, the split-K finaliser, the 3xTF32 operand splitter and
// the K == 0 epilogue.
#pragma once
#include <cstdint>

#include "epilogue.cuh"
#include "ptx.cuh"

namespace sf {

// ─────────────────────────── row softmax ───────────────────────────────────
// y[r, :] = softmax(scale * x[r, :]) in fp32: max-subtract, exp, sum, divide,
// as nn/functional.py:131-136 and the device kernels of
// _cuda_kernels.cu:473-640 (there fused with the separate dev_muls scale of
// nn/functional.py:315).  One CTA per row; the row is held in registers
// (VPT float4 per thread) so HBM sees exactly one read of x and one write
// of y.  Rows longer than the register budget use the three-pass variant.

constexpr int kSoftmaxThreads = 512;

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? red[l] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ void store4(void* y, int64_t idx, int dtype, float a, float b, float c,
                                       float d) {
  if (dtype == kF32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + idx) = make_float4(a, b, c, d);
  } else {
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(y) + idx) =
        make_uint2(pack2(a, b, dtype), pack2(c, d, dtype));
  }
}

// Two-pass streaming softmax for long fp32 rows (cols % 4 == 0, aligned):
// pass 1 streams the row once from HBM keeping a running (max, sum of exp)
// pair per thread -- on a new maximum the sum is rescaled by exp(old - new) --
// and reduces the pairs across the block; pass 2 re-reads the row (from L2)
// and writes exp(x - max) / sum.  HBM sees one read and one write of the row
// while each CTA holds no row in registers, so many rows are in flight per
// SM.  The exponentials of pass 2 are the reference's exp(x - max) exactly;
// only the sum's rounding order differs.  FAST (16-bit outputs) uses the
// hardware exp2 intrinsic (__expf) and a reciprocal multiply.
constexpr int kSoftmaxOnlineThreads = 256;

template <bool FAST>
__device__ __forceinline__ float sm_exp(float v) {
  return FAST ? __expf(v) : expf(v);
}

template <bool FAST>
__device__ __forceinline__ void sm_combine(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;  // both empty
  const float a = (m == -INFINITY) ? 0.0f : s * sm_exp<FAST>(m - mn);
  const float b = (m2 == -INFINITY) ? 0.0f : s2 * sm_exp<FAST>(m2 - mn);
  m = mn;
  s = a + b;
}

template <bool FAST>
static __global__ void __launch_bounds__(kSoftmaxOnlineThreads)
    softmax_rows_online_kernel(const float* __restrict__ x, int64_t ldx, void* __restrict__ y,
                               int y_dtype, int64_t ldy, int cols, float scale) {
  __shared__ float red_m[32], red_s[32];
  __shared__ float fin[2];
  const int64_t r = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + r * ldx);
  const int nv = cols >> 2;
  float m = -INFINITY, s = 0.0f;
#pragma unroll 4
  for (int c = threadIdx.x; c < nv; c += kSoftmaxOnlineThreads) {
    const float4 q = __ldcg(xr + c);
    const float a = q.x * scale, b = q.y * scale, cc = q.z * scale, d = q.w * scale;
    const float lm = fmaxf(fmaxf(a, b), fmaxf(cc, d));
    if (lm > m) {
      s = (m == -INFINITY) ? 0.0f : s * sm_exp<FAST>(m - lm);
      m = lm;
    }
    s += (sm_exp<FAST>(a - m) + sm_exp<FAST>(b - m)) + (sm_exp<FAST>(cc - m) + sm_exp<FAST>(d - m));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    sm_combine<FAST>(m, s, m2, s2);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    red_m[w] = m;
    red_s[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    m = (l < kSoftmaxOnlineThreads / 32) ? red_m[l] : -INFINITY;
    s = (l < kSoftmaxOnlineThreads / 32) ? red_s[l] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      sm_combine<FAST>(m, s, m2, s2);
    }
    if (l == 0) {
      fin[0] = m;
      fin[1] = s;
    }
  }
  __syncthreads();
  const float mx = fin[0], sum = fin[1];
  const float inv = 1.0f / sum;
#pragma unroll 4
  for (int c = threadIdx.x; c < nv; c += kSoftmaxOnlineThreads) {
    const float4 q = __ldcs(xr + c);
    float e0 = sm_exp<FAST>(q.x * scale - mx), e1 = sm_exp<FAST>(q.y * scale - mx);
    float e2 = sm_exp<FAST>(q.z * scale - mx), e3 = sm_exp<FAST>(q.w * scale - mx);
    if (FAST) {
      e0 *= inv; e1 *= inv; e2 *= inv; e3 *= inv;
    } else {
      e0 /= sum; e1 /= sum; e2 /= sum; e3 /= sum;
    }
    store4(y, r * ldy + 4 * (int64_t)c, y_dtype, e0, e1, e2, e3);
  }
}

// General three-pass softmax (any cols, any alignment, any input dtype).
static __global__ void __launch_bounds__(kSoftmaxThreads)
    softmax_rows_generic_kernel(const void* __restrict__ x, int x_dtype, int64_t ldx,
                                void* __restrict__ y, int y_dtype, int64_t ldy, int cols,
                                float scale) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  float m = -INFINITY;
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    m = fmaxf(m, scale * load_as_f32(x, r * ldx + c, x_dtype));
  m = block_reduce_max(m, red);
  float s = 0.0f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    s += expf(scale * load_as_f32(x, r * ldx + c, x_dtype) - m);
  s = block_reduce_sum(s, red);
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    store_from_f32(y, r * ldy + c, y_dtype, expf(scale * load_as_f32(x, r * ldx + c, x_dtype) - m) / s);
}

// ─────────────────────── elementwise activation ───────────────────────────
// y = act(alpha * x)  (dev_silu / dev_gelu / dev_muls of _cuda_ops.pyx:944-998)
static __global__ void unary_act_kernel(const void* __restrict__ x, int x_dtype, void* __restrict__ y,
                                 int y_dtype, int64_t n, float alpha, int act) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    store_from_f32(y, i, y_dtype, act_apply(alpha * load_as_f32(x, i, x_dtype), act));
}

// ─────────────────────────── split-K finaliser ─────────────────────────────
// out[r, c] = epilogue(ws[r, c]) for the split-K / K == 0 paths (ws == null => 0).
static __global__ void epilogue_finalize_kernel(const float* __restrict__ ws, int64_t ldw, int rows,
                                         int cols, void* __restrict__ out, int out_dtype,
                                         int64_t ldc, EpilogueArgs e, int slices = 1,
                                         int64_t slice = 0) {
  pdl_launch_dependents();
  pdl_wait();  // the partials come from the previous grid
  const int64_t total = (int64_t)rows * cols;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(t / cols), c = (int)(t - (t / cols) * cols);
    float acc = 0.0f;  // sum of the split slices, in split order
    if (ws)
      for (int s = 0; s < slices; ++s) acc += ws[s * slice + (int64_t)r * ldw + c];
    const float bias_v = e.bias ? load_as_f32(e.bias, c, e.bias_dtype) : 0.0f;
    const float res_v =
        e.residual ? load_as_f32(e.residual, (int64_t)r * e.ldr + c, e.residual_dtype) : 0.0f;
    store_from_f32(out, (int64_t)r * ldc + c, out_dtype, epilogue_value(acc, e, bias_v, res_v));
  }
}

// ─────────────────────────── 3xTF32 splitter ───────────────────────────────
// For an fp32 operand X (rows x K, element (r,k) at X[r*rs + k*ks]) write a
// dense K-major panel with leading dimension ld_out:
//   pattern 0: [X_hi | X_lo | X_hi]     pattern 1: [X_hi | X_hi | X_lo]
//   pattern 2: [X]  (plain repack, single-pass TF32)
// X_hi = tf32(X), X_lo = tf32(X - X_hi).  A'.B'^T over the 3K-long reduction
// of (pattern 0, pattern 1) panels equals A_hi.B_hi + A_lo.B_hi + A_hi.B_lo,
// the 3xTF32 product; the dropped A_lo.B_lo term is ~2^-22 relative.
// Reading X through (rs, ks) lets the same pass transpose an MN-major operand
// into K-major form.
__device__ __forceinline__ float to_tf32(float f) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(f));
  return __uint_as_float(r);
}

static __global__ void tf32_split_kernel(const float* __restrict__ X, int64_t rs, int64_t ks, int rows,
                                  int K, float* __restrict__ out, int64_t ld_out, int pattern) {
  const int64_t total = (int64_t)rows * K;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(t / K), k = (int)(t - (t / K) * K);
    const float v = X[(int64_t)r * rs + (int64_t)k * ks];
    float* o = out + (int64_t)r * ld_out;
    if (pattern == 2) {
      o[k] = v;
      continue;
    }
    const float hi = to_tf32(v);
    const float lo = to_tf32(v - hi);
    o[k] = hi;
    o[K + k] = pattern == 0 ? lo : hi;
    o[2 * K + k] = pattern == 0 ? hi : lo;
  }
}

// ─────────────────────────── seeded normal fill ─────────────────────────────
// Counter-based: element i gets a standard normal sample from two 32-bit
// uniforms produced by the SplitMix64 finaliser applied to (seed, i), turned
// into a normal by the Box-Muller transform.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static __global__ void fill_normal_kernel(void* x, int dtype, int64_t n, uint64_t seed, float mean,
                                          float stdv) {
  const uint64_t key = splitmix64(seed);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t r = splitmix64(key ^ static_cast<uint64_t>(i));
    const float u1 = (static_cast<float>(r >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = static_cast<float>((r >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
    const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    store_from_f32(x, i, dtype, mean + stdv * z);
  }
}

// Dense K-major copy of a strided 16-bit operand (used when a layout cannot
// be described to TMA directly).
static __global__ void repack_k_major_kernel(const uint16_t* __restrict__ X, int64_t rs, int64_t ks,
                                      int rows, int K, uint16_t* __restrict__ out, int64_t ld_out) {
  const int64_t total = (int64_t)rows * K;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(t / K), k = (int)(t - (t / K) * K);
    out[(int64_t)r * ld_out + k] = X[(int64_t)r * rs + (int64_t)k * ks];
  }
}

}  // namespace sf

namespace sf {
// Waits on an mbarrier nothing ever arrives on, with a short limit: proves
// that an expired wait records its code and returns instead of hanging.
static __global__ void bounded_wait_selftest_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile int* ab = &abort_flag;
    mbar_wait(&bar, 0, err, kDevTimeoutSelftest, ab, limit_ns);
  }
  __syncthreads();
}
}  // namespace sf
