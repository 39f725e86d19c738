// attn_simt.cu -- generic prefill attention on CUDA cores (attn::attn_block_dense
// for shapes the tensor-core kernel does not take).
//
// Reference: src/attn_block.cpp:104-241 (two-pass exact softmax per (h, l) row,
// causal keys t <= l) and the per-query online kernels
// include/kernels/attn_dh16_m1_generic.h:8-267 / include/attn_generic_m1.h:7-37
// (running max / sum, valid_len = l + 1 when causal).  One warp owns one query
// row: lane i holds dims i, i+32, ... of q and of the output accumulator, four
// keys are scored per step (butterfly-reduced dot products), and the running
// (m, l) update of include/online_softmax.h:8-17 folds them in.  Any strides,
// any head size up to 512; fp32 FMA throughout.
#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace attnb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <int DPL>  // dims per lane: Dh <= 32 * DPL
__global__ void __launch_bounds__(256) attn_rows_kernel(
    const float* __restrict__ Q, int64_t qsH, int64_t qsT, int64_t qsD,
    const float* __restrict__ K, int64_t ksH, int64_t ksT, int64_t ksD,
    const float* __restrict__ V, int64_t vsH, int64_t vsT, int64_t vsD, float* __restrict__ O,
    int64_t osH, int64_t osT, int64_t osD, int H, int L, int T, int Dh, int causal,
    float qscale) {
  constexpr int U = 4;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= (int64_t)H * L) return;
  const int h = static_cast<int>(row / L), l = static_cast<int>(row % L);
  const int len = causal ? min(l + 1, T) : T;

  float q[DPL], acc[DPL];
#pragma unroll
  for (int j = 0; j < DPL; ++j) {
    const int d = lane + 32 * j;
    q[j] = d < Dh ? Q[h * qsH + l * qsT + d * qsD] * qscale : 0.f;
    acc[j] = 0.f;
  }
  const float* Kh = K + h * ksH;
  const float* Vh = V + h * vsH;
  float m = -INFINITY, lsum = 0.f;
  for (int t0 = 0; t0 < len; t0 += U) {
    float s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float p = 0.f;
      if (t0 + u < len) {
        const float* kr = Kh + (int64_t)(t0 + u) * ksT;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
          const int d = lane + 32 * j;
          if (d < Dh) p = fmaf(q[j], kr[d * ksD], p);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
      s[u] = (t0 + u < len) ? p : -INFINITY;
    }
    float bm = s[0];
#pragma unroll
    for (int u = 1; u < U; ++u) bm = fmaxf(bm, s[u]);
    const float m_new = fmaxf(m, bm);
    const float alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
    lsum *= alpha;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] *= alpha;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (t0 + u < len) {
        const float p = fast_exp2(s[u] - m_new);
        lsum += p;
        const float* vr = Vh + (int64_t)(t0 + u) * vsT;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
          const int d = lane + 32 * j;
          if (d < Dh) acc[j] = fmaf(p, vr[d * vsD], acc[j]);
        }
      }
    }
    m = m_new;
  }
  const float inv = 1.f / lsum;
#pragma unroll
  for (int j = 0; j < DPL; ++j) {
    const int d = lane + 32 * j;
    if (d < Dh) O[h * osH + l * osT + d * osD] = acc[j] * inv;
  }
}

template <int DPL>
void launch_rows(const View3& Q, const View3& K, const View3& V, const MView3& O, bool causal,
                 float qscale, cudaStream_t s) {
  const int64_t rows = (int64_t)Q.H * Q.T;
  const int per_block = 8;
  const unsigned blocks = static_cast<unsigned>((rows + per_block - 1) / per_block);
  attn_rows_kernel<DPL><<<blocks, 32 * per_block, 0, s>>>(
      Q.data, Q.sH, Q.sT, Q.sD, K.data, K.sH, K.sT, K.sD, V.data, V.sH, V.sT, V.sD, O.data, O.sH,
      O.sT, O.sD, Q.H, Q.T, K.T, Q.Dh, causal ? 1 : 0, qscale);
}

}  // namespace

void attn_block_simt_launch(const View3& Q, const View3& K, const View3& V, const MView3& O,
                            bool causal, cudaStream_t stream) {
  if ((int64_t)Q.H * Q.T == 0) return;
  const float qscale = kLog2e / std::sqrt(static_cast<float>(Q.Dh));
  const int Dh = Q.Dh;
  ProfScope prof("attn_simt", stream);
  if (Dh <= 32) launch_rows<1>(Q, K, V, O, causal, qscale, stream);
  else if (Dh <= 64) launch_rows<2>(Q, K, V, O, causal, qscale, stream);
  else if (Dh <= 128) launch_rows<4>(Q, K, V, O, causal, qscale, stream);
  else if (Dh <= 256) launch_rows<8>(Q, K, V, O, causal, qscale, stream);
  else launch_rows<16>(Q, K, V, O, causal, qscale, stream);
}

}  // namespace attnb
