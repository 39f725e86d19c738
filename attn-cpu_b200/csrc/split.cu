// split.cu -- K2: operand packing for the tensor-core contractions.
//
// The reference packs its operands before the FMA micro-kernels (A panels
// with alpha folded in, src/gemm.cpp:50-59; B panels, src/gemm.cpp:60-78;
// W^T into 16x16 tiles, include/pack_16x16.h:9-25; K transposed per head,
// include/layout.h:9-42).  The tcgen05 kernels want instead K-major fp32 rows
// padded to a multiple of 32 elements (one 128-byte swizzle row per 32 K
// values), and for 3xTF32 each value x split into
//   hi = tf32_round(x)     (low 13 mantissa bits zero: exact as a tf32 operand)
//   lo = x - hi            (exact in fp32; |lo| <= 2^-11 |x|)
// so that x*y ~= hi_x*hi_y + hi_x*lo_y + lo_x*hi_y with an error near 2^-22.
//
// One launch packs every operand of a contraction (up to three jobs: e.g. Q,
// K and V^T of an attention call), each job a strided 3-D source written
// either in place ([h][r][c], columns padded) or transposed per head
// ([h][c][r]).  It releases the dependent kernel early (programmatic dependent launch) so that
// kernel's prologue overlaps the packing.  HBM-bound streaming pass.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace attnb {
namespace {

constexpr int kThreads = 256;

struct PackArgs {
  PackJob job[kMaxPackJobs];
  int start[kMaxPackJobs + 1];  // first block of each job
  int njobs;
  int split3;
};

__device__ __forceinline__ void split_value(float x, bool split3, float& hi, float& lo) {
  hi = tf32_round(x);
  lo = split3 ? (x - hi) : 0.f;
}

// Rows are spread over the lanes of a warp: `lpr` lanes per row (32 for long
// rows, fewer for short ones so no lane idles), each lane four columns at a
// time, with 16-byte loads when the source row is contiguous and aligned.
__device__ __forceinline__ int lanes_per_row(int cp4) {
  return cp4 >= 32 ? 32 : cp4 >= 16 ? 16 : cp4 >= 8 ? 8 : 4;
}

__device__ void pack_rows(const PackJob& j, bool split3, int lb, int nb) {
  constexpr int kWarps = kThreads / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cp4 = j.cols_out >> 2;
  const int lpr = lanes_per_row(cp4), rpw = 32 / lpr;
  const int sub = lane / lpr, sl = lane % lpr;
  const int64_t nrows = (int64_t)j.H * j.R;
  const bool vec = j.sC == 1 && (j.sR & 3) == 0 && (j.sH & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(j.src) & 15u) == 0;
  for (int64_t hr = ((int64_t)lb * kWarps + warp) * rpw + sub; hr < nrows;
       hr += (int64_t)nb * kWarps * rpw) {
    const int h = static_cast<int>(hr / j.R), r = static_cast<int>(hr % j.R);
    const float* s = j.src + h * j.sH + r * j.sR;
    float4* oh = reinterpret_cast<float4*>(j.hi + hr * j.cols_out);
    float4* ol = split3 ? reinterpret_cast<float4*>(j.lo + hr * j.cols_out) : nullptr;
#pragma unroll 4
    for (int c4 = sl; c4 < cp4; c4 += lpr) {
      const int c = c4 * 4;
      float x[4];
      if (vec && c + 3 < j.C) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(s + c));
        x[0] = v.x;
        x[1] = v.y;
        x[2] = v.z;
        x[3] = v.w;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = (c + k < j.C) ? s[(int64_t)(c + k) * j.sC] : 0.f;
      }
      float4 h4, l4;
      split_value(x[0] * j.scale, split3, h4.x, l4.x);
      split_value(x[1] * j.scale, split3, h4.y, l4.y);
      split_value(x[2] * j.scale, split3, h4.z, l4.z);
      split_value(x[3] * j.scale, split3, h4.w, l4.w);
      oh[c4] = h4;
      if (split3) ol[c4] = l4;
    }
  }
}

// out[h][c][r] = src[h][r][c] through 64x64 shared-memory tiles (row pitch
// 65: the transposed writes spread over the banks).  Sixteen threads cover a
// 64-wide row with 16-byte accesses on both sides when the source allows.
constexpr int kTile = 64;
constexpr int kTilePitch = kTile + 1;

__device__ void pack_transposed(const PackJob& j, bool split3, int lb, int nb, float* tile) {
  const int tiles_c = (j.rows_out + kTile - 1) / kTile, tiles_r = (j.cols_out + kTile - 1) / kTile;
  const int64_t ntiles = (int64_t)j.H * tiles_c * tiles_r;
  const int t16 = threadIdx.x & 15, row_in = threadIdx.x >> 4;  // 16 rows per pass
  const bool vec = j.sC == 1 && (j.sR & 3) == 0 && (j.sH & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(j.src) & 15u) == 0;
  const bool vec_out = (j.cols_out & 3) == 0;
  for (int64_t t = lb; t < ntiles; t += nb) {
    const int h = static_cast<int>(t / ((int64_t)tiles_c * tiles_r));
    const int rem = static_cast<int>(t % ((int64_t)tiles_c * tiles_r));
    const int c0 = (rem % tiles_c) * kTile, r0 = (rem / tiles_c) * kTile;
    const float* s = j.src + h * j.sH;
    __syncthreads();  // the previous tile has been written out
    // Load: source rows r0.. (columns c0 + 4*t16 ..), stored transposed.
#pragma unroll
    for (int p = 0; p < kTile / 16; ++p) {
      const int y = p * 16 + row_in, r = r0 + y, c = c0 + 4 * t16;
      float x[4] = {0.f, 0.f, 0.f, 0.f};
      if (r < j.R) {
        const float* sr = s + (int64_t)r * j.sR;
        if (vec && c + 3 < j.C) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(sr + c));
          x[0] = v.x;
          x[1] = v.y;
          x[2] = v.z;
          x[3] = v.w;
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (c + k < j.C) x[k] = sr[(int64_t)(c + k) * j.sC];
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) tile[(4 * t16 + k) * kTilePitch + y] = x[k] * j.scale;
    }
    __syncthreads();
    // Store: output rows c0.. (columns r0 + 4*t16 ..), split into hi / lo.
    float* oh = j.hi + (int64_t)h * j.rows_out * j.cols_out;
    float* ol = split3 ? j.lo + (int64_t)h * j.rows_out * j.cols_out : nullptr;
#pragma unroll
    for (int p = 0; p < kTile / 16; ++p) {
      const int y = p * 16 + row_in, c = c0 + y, r = r0 + 4 * t16;
      if (c >= j.rows_out) continue;
      float hv[4], lv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) split_value(tile[y * kTilePitch + 4 * t16 + k], split3, hv[k], lv[k]);
      const int64_t o = (int64_t)c * j.cols_out + r;
      if (vec_out && r + 3 < j.cols_out) {
        *reinterpret_cast<float4*>(oh + o) = make_float4(hv[0], hv[1], hv[2], hv[3]);
        if (split3) *reinterpret_cast<float4*>(ol + o) = make_float4(lv[0], lv[1], lv[2], lv[3]);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (r + k < j.cols_out) {
            oh[o + k] = hv[k];
            if (split3) ol[o + k] = lv[k];
          }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) pack_kernel(const __grid_constant__ PackArgs a) {
  __shared__ float tile[kTile * kTilePitch];
  // Let the dependent tensor-core kernel start its prologue now; it waits
  // (griddepcontrol.wait) for this grid's writes before reading them.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int b = blockIdx.x;
  int j = 0;
  while (j + 1 < a.njobs && b >= a.start[j + 1]) ++j;
  const int lb = b - a.start[j], nb = a.start[j + 1] - a.start[j];
  if (a.job[j].transpose) pack_transposed(a.job[j], a.split3 != 0, lb, nb, tile);
  else pack_rows(a.job[j], a.split3 != 0, lb, nb);
}

}  // namespace

void pack_launch(const PackJob* jobs, int njobs, bool split3, int num_sms, cudaStream_t s) {
  if (njobs < 1 || njobs > kMaxPackJobs) fail(ATTNB_ERR_RUNTIME, "internal: bad pack job count");
  PackArgs a{};
  a.njobs = njobs;
  a.split3 = split3 ? 1 : 0;
  int total = 0;
  for (int i = 0; i < njobs; ++i) {
    const PackJob& j = jobs[i];
    a.job[i] = j;
    a.start[i] = total;
    int64_t blocks;
    if (j.transpose) {
      blocks = (int64_t)j.H * ((j.rows_out + kTile - 1) / kTile) * ((j.cols_out + kTile - 1) / kTile);
    } else {
      const int cp4 = j.cols_out / 4;
      const int rpw = 32 / (cp4 >= 32 ? 32 : cp4 >= 16 ? 16 : cp4 >= 8 ? 8 : 4);
      const int64_t rows_per_block = (int64_t)(kThreads / 32) * rpw;
      blocks = ((int64_t)j.H * j.R + rows_per_block - 1) / rows_per_block;
    }
    blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)num_sms * 8));
    total += static_cast<int>(blocks);
  }
  a.start[njobs] = total;
  pack_kernel<<<total, kThreads, 0, s>>>(a);
  ATTNB_CUDA(cudaGetLastError());
}

}  // namespace attnb
