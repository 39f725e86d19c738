// split.cu -- K2: operand packing for the tensor-core contractions.
//
// The reference packs its operands before the FMA micro-kernels (A panels
// with alpha folded in, src/gemm.cpp:50-59; B panels, src/gemm.cpp:60-78;
// W^T into 16x16 tiles, include/pack_16x16.h:9-25).  The tcgen05 kernels want
// instead K-major fp32 rows padded to a multiple of 32 elements (one 128-byte
// swizzle row per 32 K values), and for 3xTF32 each value x split into
//   hi = tf32_round(x)     (low 13 mantissa bits zero: exact as a tf32 operand)
//   lo = x - hi            (exact in fp32; |lo| <= 2^-11 |x|)
// so that x*y ~= hi_x*hi_y + hi_x*lo_y + lo_x*hi_y with an error near 2^-22.
// These kernels are HBM-bound streaming passes.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace attnb {
namespace {

__device__ __forceinline__ void split_value(float x, bool split3, float& hi, float& lo) {
  hi = tf32_round(x);
  lo = split3 ? (x - hi) : 0.f;
}

// src[rows, cols] (row pitch ld) -> hi/lo[rows, kp], cols..kp-1 zero.
// One thread writes 4 consecutive output columns (one 16-byte store each).
__global__ void pack_rows_kernel(const float* __restrict__ src, int64_t ld, int rows, int cols,
                                 int kp, float* __restrict__ hi, float* __restrict__ lo,
                                 int split3) {
  const int kp4 = kp >> 2;
  const int64_t n = (int64_t)rows * kp4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(i / kp4);
    const int c = static_cast<int>(i % kp4) * 4;
    const float* s = src + r * ld;
    float4 h, l;
    float x0 = c + 0 < cols ? s[c + 0] : 0.f;
    float x1 = c + 1 < cols ? s[c + 1] : 0.f;
    float x2 = c + 2 < cols ? s[c + 2] : 0.f;
    float x3 = c + 3 < cols ? s[c + 3] : 0.f;
    split_value(x0, split3, h.x, l.x);
    split_value(x1, split3, h.y, l.y);
    split_value(x2, split3, h.z, l.z);
    split_value(x3, split3, h.w, l.w);
    reinterpret_cast<float4*>(hi + (int64_t)r * kp)[c >> 2] = h;
    if (split3) reinterpret_cast<float4*>(lo + (int64_t)r * kp)[c >> 2] = l;
  }
}

// src[K, N] (row pitch ld) -> hi/lo[N, kp] (transposed), k in [K, kp) zero.
// 32x32 tiles through shared memory; block (32, 8).
__global__ void pack_transpose_kernel(const float* __restrict__ src, int64_t ld, int K, int N,
                                      int kp, float* __restrict__ hi, float* __restrict__ lo,
                                      int split3) {
  __shared__ float tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int k = k0 + j, n = n0 + threadIdx.x;
    tile[j][threadIdx.x] = (k < K && n < N) ? src[(int64_t)k * ld + n] : 0.f;
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int n = n0 + j, k = k0 + threadIdx.x;
    if (n < N && k < kp) {
      float h, l;
      split_value(tile[threadIdx.x][j], split3, h, l);
      hi[(int64_t)n * kp + k] = h;
      if (split3) lo[(int64_t)n * kp + k] = l;
    }
  }
}

// 3-D strided src[h, r, c] (r < R, c < C) -> hi/lo[h, r, cp] scaled by `scale`,
// columns C..cp-1 zero.  One thread writes 4 output columns.
__global__ void pack3_kernel(const float* __restrict__ src, int64_t sH, int64_t sR, int64_t sC,
                             int H, int R, int C, int cp, float scale, float* __restrict__ hi,
                             float* __restrict__ lo, int split3) {
  const int cp4 = cp >> 2;
  const int64_t n = (int64_t)H * R * cp4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t hr = i / cp4;
    const int c = static_cast<int>(i % cp4) * 4;
    const int h = static_cast<int>(hr / R), r = static_cast<int>(hr % R);
    const float* s = src + h * sH + r * sR;
    float x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = (c + j < C) ? s[(c + j) * sC] * scale : 0.f;
    float4 h4, l4;
    split_value(x[0], split3, h4.x, l4.x);
    split_value(x[1], split3, h4.y, l4.y);
    split_value(x[2], split3, h4.z, l4.z);
    split_value(x[3], split3, h4.w, l4.w);
    reinterpret_cast<float4*>(hi + hr * cp)[c >> 2] = h4;
    if (split3) reinterpret_cast<float4*>(lo + hr * cp)[c >> 2] = l4;
  }
}

// 3-D strided src[h, t, d] (t < T, d < D) -> hi/lo[h, d, tp] for d < dp
// (transposed per head), zero outside t < T, d < D.  32x32 tiles, block (32, 8).
__global__ void pack3_transpose_kernel(const float* __restrict__ src, int64_t sH, int64_t sT,
                                       int64_t sD, int T, int D, int tp, int dp,
                                       float* __restrict__ hi, float* __restrict__ lo,
                                       int split3) {
  __shared__ float tile[32][33];
  const int h = blockIdx.z;
  const int d0 = blockIdx.x * 32, t0 = blockIdx.y * 32;
  const float* s = src + h * sH;
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int t = t0 + j, d = d0 + threadIdx.x;
    tile[j][threadIdx.x] = (t < T && d < D) ? s[t * sT + d * sD] : 0.f;
  }
  __syncthreads();
  float* oh = hi + (int64_t)h * dp * tp;
  float* ol = split3 ? lo + (int64_t)h * dp * tp : nullptr;
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int d = d0 + j, t = t0 + threadIdx.x;
    if (d < dp && t < tp) {
      float hv, lv;
      split_value(tile[threadIdx.x][j], split3, hv, lv);
      oh[(int64_t)d * tp + t] = hv;
      if (split3) ol[(int64_t)d * tp + t] = lv;
    }
  }
}

}  // namespace

void pack3_launch(const float* src, int64_t sH, int64_t sR, int64_t sC, int H, int R, int C,
                  int cp, float scale, float* hi, float* lo, bool split3, cudaStream_t s) {
  const int64_t n = (int64_t)H * R * (cp / 4);
  if (n <= 0) return;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  pack3_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(src, sH, sR, sC, H, R, C, cp, scale,
                                                              hi, lo, split3 ? 1 : 0);
}

void pack3_transpose_launch(const float* src, int64_t sH, int64_t sT, int64_t sD, int H, int T,
                            int D, int tp, int dp, float* hi, float* lo, bool split3,
                            cudaStream_t s) {
  if (H <= 0 || tp <= 0 || dp <= 0) return;
  const dim3 grid((dp + 31) / 32, (tp + 31) / 32, H);
  pack3_transpose_kernel<<<grid, dim3(32, 8), 0, s>>>(src, sH, sT, sD, T, D, tp, dp, hi, lo,
                                                      split3 ? 1 : 0);
}

void pack_rows_launch(const float* src, int64_t ld, int rows, int cols, int kp, float* hi,
                      float* lo, bool split3, cudaStream_t s) {
  if (rows <= 0) return;
  const int64_t n = (int64_t)rows * (kp / 4);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((n + threads - 1) / threads, 148 * 16);
  pack_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(src, ld, rows, cols, kp, hi,
                                                                    lo, split3 ? 1 : 0);
}

void pack_transpose_launch(const float* src, int64_t ld, int K, int N, int kp, float* hi,
                           float* lo, bool split3, cudaStream_t s) {
  if (N <= 0 || kp <= 0) return;
  const dim3 grid((N + 31) / 32, (kp + 31) / 32);
  pack_transpose_kernel<<<grid, dim3(32, 8), 0, s>>>(src, ld, K, N, kp, hi, lo, split3 ? 1 : 0);
}

}  // namespace attnb
