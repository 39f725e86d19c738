// decode.cu -- K4: the M=1 decode step (attn::attn_step_dense) on CUDA cores.
//
// Reference: src/attn_dense.cpp:21-73 computes, per head, an exact two-pass
// softmax over T keys (logits + max, then exp / sum / V-mix / 1/sum).  The same
// function is computed here as a split-KV online softmax, the running (m, l)
// update of include/online_softmax.h:8-17:
//
//   * the grid is (nsplit, H): each CTA streams one contiguous key range of one
//     head; each warp takes U keys per step with 128-bit loads (one float4 of
//     K and of V per lane per key), reduces the U dot products with butterfly
//     shuffles and folds them into its running max m, sum l and accumulator;
//   * the warps of a CTA merge (m, l, acc) through shared memory;
//   * with nsplit > 1 each CTA writes its partial (m, l, acc) to scratch and a
//     second tiny kernel merges the splits: m = max m_s,
//     O = sum_s 2^(m_s - m) acc_s / sum_s 2^(m_s - m) l_s.
//
// Logits are kept in base-2 units (q is pre-scaled by log2(e)/sqrt(Dh)) so the
// exponentials are single ex2 instructions.  The path is HBM-bound: it moves
// K and V once (2*H*T*Dh*4 bytes) plus q and o.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace attnb {
namespace {

constexpr int kThreads = 256;  // 8 warps per CTA
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Merge the per-warp (m, l, acc[Dh]) of the CTA held in shared memory and
// write either the final output (nsplit == 1) or the split's partial.
__device__ void cta_merge_and_store(const float* sm_m, const float* sm_l, const float* sm_acc,
                                    int nwarps, int Dh, float* out_final, int64_t osD,
                                    float* part_o, float2* part_ml) {
  float M = -INFINITY;
  for (int w = 0; w < nwarps; ++w) M = fmaxf(M, sm_m[w]);
  float L = 0.f;
  for (int w = 0; w < nwarps; ++w) L += (sm_m[w] == -INFINITY) ? 0.f : fast_exp2(sm_m[w] - M) * sm_l[w];
  for (int d = threadIdx.x; d < Dh; d += blockDim.x) {
    float o = 0.f;
    for (int w = 0; w < nwarps; ++w)
      if (sm_m[w] != -INFINITY) o += fast_exp2(sm_m[w] - M) * sm_acc[w * Dh + d];
    if (out_final) out_final[d * osD] = o / L;
    else part_o[d] = o;
  }
  if (!out_final && threadIdx.x == 0) *part_ml = make_float2(M, L);
}

// Vector path: NV float4 per lane covers Dh <= 128 * NV; U keys per warp step.
template <int NV, int U>
__global__ void __launch_bounds__(kThreads, 2) decode_vec_kernel(
    const float* __restrict__ Q, int64_t qsH, const float* __restrict__ K, int64_t ksH,
    int64_t ksT, const float* __restrict__ V, int64_t vsH, int64_t vsT, int T, int Dh,
    int keys_per_split, float qscale, float* __restrict__ O, int64_t osH, int64_t osD,
    float* __restrict__ part_o, float2* __restrict__ part_ml) {
  extern __shared__ float smem[];
  const int nwarps = kThreads / 32;
  float* sm_m = smem;
  float* sm_l = smem + nwarps;
  float* sm_acc = smem + 2 * nwarps;

  const int split = blockIdx.x, h = blockIdx.y, nsplit = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Dh4 = Dh >> 2;
  const int t_begin = split * keys_per_split;
  const int t_end = min(T, t_begin + keys_per_split);

  float4 q[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int i = lane + 32 * v;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < Dh4) x = *reinterpret_cast<const float4*>(Q + h * qsH + 4 * i);
    q[v] = make_float4(x.x * qscale, x.y * qscale, x.z * qscale, x.w * qscale);
  }
  const float* Kh = K + h * ksH;
  const float* Vh = V + h * vsH;

  float m = -INFINITY, l = 0.f;
  float4 acc[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);

  for (int t0 = t_begin + warp * U; t0 < t_end; t0 += nwarps * U) {
    float4 kr[U][NV], vr[U][NV];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool ok = (t0 + u) < t_end;
      const float* kp = Kh + (int64_t)(t0 + u) * ksT;
      const float* vp = Vh + (int64_t)(t0 + u) * vsT;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const int i = lane + 32 * v;
        if (ok && i < Dh4) {
          kr[u][v] = __ldg(reinterpret_cast<const float4*>(kp + 4 * i));
          vr[u][v] = __ldg(reinterpret_cast<const float4*>(vp + 4 * i));
        } else {
          kr[u][v] = make_float4(0.f, 0.f, 0.f, 0.f);
          vr[u][v] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    float s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float p = 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v)
        p += q[v].x * kr[u][v].x + q[v].y * kr[u][v].y + q[v].z * kr[u][v].z + q[v].w * kr[u][v].w;
      s[u] = warp_sum(p);
      if (t0 + u >= t_end) s[u] = -INFINITY;
    }
    float bm = s[0];
#pragma unroll
    for (int u = 1; u < U; ++u) bm = fmaxf(bm, s[u]);
    const float m_new = fmaxf(m, bm);  // s[0] is a valid key, so m_new is finite
    const float alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
    l *= alpha;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      acc[v].x *= alpha; acc[v].y *= alpha; acc[v].z *= alpha; acc[v].w *= alpha;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float p = (s[u] == -INFINITY) ? 0.f : fast_exp2(s[u] - m_new);
      l += p;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        acc[v].x = fmaf(p, vr[u][v].x, acc[v].x);
        acc[v].y = fmaf(p, vr[u][v].y, acc[v].y);
        acc[v].z = fmaf(p, vr[u][v].z, acc[v].z);
        acc[v].w = fmaf(p, vr[u][v].w, acc[v].w);
      }
    }
    m = m_new;
  }

  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int i = lane + 32 * v;
    if (i < Dh4) *reinterpret_cast<float4*>(sm_acc + warp * Dh + 4 * i) = acc[v];
  }
  __syncthreads();
  const size_t pidx = (size_t)h * nsplit + split;
  cta_merge_and_store(sm_m, sm_l, sm_acc, nwarps, Dh, nsplit == 1 ? O + h * osH : nullptr, osD,
                      part_o ? part_o + pidx * Dh : nullptr, part_ml ? part_ml + pidx : nullptr);
  grid_dep_launch();  // the split merge may be scheduled once every CTA gets here
}

// Any strides / head size: scores of the key range go to shared memory, then
// one exact softmax over the range (this is the reference's two-pass order).
__global__ void __launch_bounds__(kThreads) decode_generic_kernel(
    const float* __restrict__ Q, int64_t qsH, int64_t qsD, const float* __restrict__ K,
    int64_t ksH, int64_t ksT, int64_t ksD, const float* __restrict__ V, int64_t vsH,
    int64_t vsT, int64_t vsD, int T, int Dh, int keys_per_split, float qscale,
    float* __restrict__ O, int64_t osH, int64_t osD, float* __restrict__ part_o,
    float2* __restrict__ part_ml) {
  extern __shared__ float smem[];
  float* sc = smem;  // keys_per_split scores
  __shared__ float red[32];
  __shared__ float s_max, s_sum;

  const int split = blockIdx.x, h = blockIdx.y, nsplit = gridDim.x;
  const int t_begin = split * keys_per_split;
  const int n = min(T, t_begin + keys_per_split) - t_begin;
  const float* q = Q + h * qsH;

  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float* kr = K + h * ksH + (int64_t)(t_begin + j) * ksT;
    float dot = 0.f;
    for (int d = 0; d < Dh; ++d) dot = fmaf(q[d * qsD], kr[d * ksD], dot);
    sc[j] = dot * qscale;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < n; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v = fmaxf(v, red[w]);
    s_max = v;
  }
  __syncthreads();
  const float M = s_max;
  float sum = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float p = fast_exp2(sc[j] - M);
    sc[j] = p;
    sum += p;
  }
  sum = warp_sum(sum);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += red[w];
    s_sum = v;
  }
  __syncthreads();
  const float L = s_sum;
  const size_t pidx = (size_t)h * nsplit + split;
  for (int d = threadIdx.x; d < Dh; d += blockDim.x) {
    float o = 0.f;
    const float* vc = V + h * vsH + (int64_t)t_begin * vsT + d * vsD;
    for (int j = 0; j < n; ++j) o = fmaf(sc[j], vc[(int64_t)j * vsT], o);
    if (nsplit == 1) O[h * osH + d * osD] = o / L;
    else part_o[pidx * Dh + d] = o;
  }
  if (nsplit > 1 && threadIdx.x == 0) part_ml[pidx] = make_float2(M, L);
}

// Merge the nsplit partials of each head (one CTA of kMergeThreads per head):
//   m* = max_s m_s,  w_s = 2^(m_s - m*),  L = sum_s w_s l_s,
//   O[d] = sum_s w_s acc_s[d] / L.
// The split maxima, weights and L are reductions over all threads; the sum
// over splits is spread over thread groups (each group a strided subset of
// the splits, each thread one float4 of the head), so the loads of
// different splits are in flight together rather than one after another.
constexpr int kMergeThreads = 128;
constexpr int kMergeMaxW = 1024;  // split weights kept in shared memory

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kMergeThreads / 32; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kMergeThreads) decode_merge_kernel(
    const float* __restrict__ part_o, const float2* __restrict__ part_ml, int nsplit, int Dh,
    float* __restrict__ O, int64_t osH, int64_t osD, const PeerOut peers) {
  grid_dep_wait();  // the partials come from the split kernel launched before this one
  __shared__ float red[kMergeThreads / 32];
  __shared__ float wsh[kMergeMaxW];
  __shared__ float4 part[kMergeThreads];
  const int h = blockIdx.x, t = threadIdx.x;
  const float2* ml = part_ml + (size_t)h * nsplit;
  const float* po = part_o + (size_t)h * nsplit * Dh;
  float mx = -INFINITY;
  for (int s = t; s < nsplit; s += kMergeThreads) mx = fmaxf(mx, ml[s].x);
  const float M = block_reduce(mx, true, red);
  float lsum = 0.f;
  for (int s = t; s < nsplit; s += kMergeThreads) {
    const float2 v = ml[s];
    const float w = v.x == -INFINITY ? 0.f : fast_exp2(v.x - M);
    if (s < kMergeMaxW) wsh[s] = w;
    lsum = fmaf(w, v.y, lsum);
  }
  const float invL = 1.f / block_reduce(lsum, false, red);  // also orders the wsh writes
  auto weight = [&](int s) {
    if (s < kMergeMaxW) return wsh[s];
    const float m = ml[s].x;
    return m == -INFINITY ? 0.f : fast_exp2(m - M);
  };
  auto put = [&](int d, float v) {
    const int64_t off = h * osH + d * osD;
    O[off] = v;
    // Replicas on other GPUs (the sharded decode step's output heads).
#pragma unroll
    for (int p = 0; p < kMaxPeerOut; ++p)
      if (p < peers.n) peers.dst[p][off] = v;
  };
  const int nd4 = Dh / 4;
  if (Dh % 4 == 0 && nd4 <= kMergeThreads && (reinterpret_cast<uintptr_t>(po) & 15u) == 0) {
    const int groups = kMergeThreads / nd4;
    const int d4 = t % nd4, gi = t / nd4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (gi < groups) {
#pragma unroll 4
      for (int s = gi; s < nsplit; s += groups) {
        const float w = weight(s);
        const float4 v = *reinterpret_cast<const float4*>(po + (size_t)s * Dh + 4 * d4);
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
      }
    }
    part[t] = acc;
    __syncthreads();
    if (t < nd4) {
      float4 o = part[t];
      for (int g = 1; g < groups; ++g) {
        const float4 v = part[g * nd4 + t];
        o.x += v.x;
        o.y += v.y;
        o.z += v.z;
        o.w += v.w;
      }
      put(4 * t, o.x * invL);
      put(4 * t + 1, o.y * invL);
      put(4 * t + 2, o.z * invL);
      put(4 * t + 3, o.w * invL);
    }
  } else {
    for (int d = t; d < Dh; d += kMergeThreads) {
      float o = 0.f;
#pragma unroll 4
      for (int s = 0; s < nsplit; ++s) o = fmaf(weight(s), po[(size_t)s * Dh + d], o);
      put(d, o * invL);
    }
  }
  if (peers.n > 0) __threadfence_system();
  grid_dep_launch();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

DecodePlan decode_plan(const View3& Q, const View3& K, const View3& V, int num_sms) {
  DecodePlan p{};
  const int H = K.H, T = K.T, Dh = K.Dh;
  p.fast = Q.sD == 1 && K.sD == 1 && V.sD == 1 && Dh % 4 == 0 && Dh <= 256 &&
           aligned16(Q.data) && aligned16(K.data) && aligned16(V.data) && Q.sH % 4 == 0 &&
           K.sH % 4 == 0 && K.sT % 4 == 0 && V.sH % 4 == 0 && V.sT % 4 == 0;
  // Two CTAs per SM over all heads (the kernel's residency: one wave of long
  // key ranges); each split keeps at least 64 keys so the merge stays cheap.
  // Measured with graph-replayed steps at T = 4096, Dh = 128: at 256 heads
  // 150 us against 160 us with eight per SM (several waves of shorter
  // ranges), at 32 heads 27 us against 34 us.
  int per_sm = 2;
  if (const char* e = std::getenv("ATTNB_DECODE_CTAS_PER_SM")) per_sm = std::max(1, std::atoi(e));
  const int slots = std::max(1, num_sms) * per_sm;
  int ns = std::max(1, slots / std::max(1, H));
  ns = std::min(ns, std::max(1, (T + 63) / 64));
  int kps = (T + ns - 1) / ns;
  if (!p.fast) kps = std::min(kps, 2048);  // generic path keeps a range's scores in smem
  kps = std::max(kps, 1);
  p.keys_per_split = kps;
  p.nsplit = (T + kps - 1) / kps;
  return p;
}

size_t decode_workspace_bytes(const DecodePlan& p, int H, int Dh) {
  if (p.nsplit <= 1) return 0;
  const size_t n = (size_t)H * p.nsplit;
  return n * Dh * sizeof(float) + n * sizeof(float2) + 256;
}

void decode_launch(const DecodePlan& p, const View3& Q, const View3& K, const View3& V,
                   const MView3& O, void* ws, cudaStream_t stream, const PeerOut* peers) {
  const int H = K.H, T = K.T, Dh = K.Dh;
  const float qscale = kLog2e / std::sqrt(static_cast<float>(Dh));
  float* part_o = nullptr;
  float2* part_ml = nullptr;
  if (p.nsplit > 1) {
    part_o = static_cast<float*>(ws);
    const size_t off = (((size_t)H * p.nsplit * Dh * sizeof(float)) + 255) & ~size_t(255);
    part_ml = reinterpret_cast<float2*>(static_cast<char*>(ws) + off);
  }
  const dim3 grid(p.nsplit, H);
  ProfScope prof("decode", stream);
  if (p.fast) {
    const size_t sm = (2 * (kThreads / 32) + (kThreads / 32) * Dh) * sizeof(float);
    if (Dh <= 128)
      decode_vec_kernel<1, 8><<<grid, kThreads, sm, stream>>>(
          Q.data, Q.sH, K.data, K.sH, K.sT, V.data, V.sH, V.sT, T, Dh, p.keys_per_split, qscale,
          O.data, O.sH, O.sD, part_o, part_ml);
    else
      decode_vec_kernel<2, 4><<<grid, kThreads, sm, stream>>>(
          Q.data, Q.sH, K.data, K.sH, K.sT, V.data, V.sH, V.sT, T, Dh, p.keys_per_split, qscale,
          O.data, O.sH, O.sD, part_o, part_ml);
  } else {
    const size_t sm = (size_t)p.keys_per_split * sizeof(float);
    decode_generic_kernel<<<grid, kThreads, sm, stream>>>(
        Q.data, Q.sH, Q.sD, K.data, K.sH, K.sT, K.sD, V.data, V.sH, V.sT, V.sD, T, Dh,
        p.keys_per_split, qscale, O.data, O.sH, O.sD, part_o, part_ml);
  }
  const PeerOut none{};
  if (p.nsplit > 1) {
    ATTNB_CUDA(launch_pdl(decode_merge_kernel, dim3(H), dim3(kMergeThreads), 0, stream,
                          (const float*)part_o, (const float2*)part_ml, p.nsplit, Dh, O.data,
                          O.sH, O.sD, peers ? *peers : none));
  } else if (peers) {
    // One key range per head: the attention kernel stored O itself; copy the
    // rows (unit head-dim stride, checked by the caller) to the replicas.
    for (int i = 0; i < peers->n; ++i)
      ATTNB_CUDA(cudaMemcpy2DAsync(peers->dst[i], O.sH * sizeof(float), O.data,
                                   O.sH * sizeof(float), Dh * sizeof(float), H,
                                   cudaMemcpyDeviceToDevice, stream));
  }
}

}  // namespace attnb

// ===================================================================
// attnb_attn_step_dense_noalloc -- the decode step for callers that may not
// allocate device memory.
//
// Some callers cannot call cudaMalloc at all: code running inside a custom
// allocator or memory pool that owns the whole device budget, runtimes that
// forbid allocation on their hot path, and applications that must keep their
// memory footprint fixed once they start.  For them this entry point computes
// exactly what attnb_attn_step_dense_dev computes (same plan, same kernels)
// but keeps the split-KV partials (per head and key range: the running max,
// the sum and the unnormalised output row) in a fixed, file-scope device array
// of kNoAllocScratchBytes, which every GPU that loads the library holds until
// the process exits.  The caller passes device pointers for inputs and output.
//
// Limits and rules:
//   * a call whose decode plan needs more scratch than kNoAllocScratchBytes
//     (heads x key ranges x head size x 4 bytes + 8 bytes per pair) is
//     rejected with ATTNB_ERR_INVALID_ARGUMENT before any work is enqueued;
//   * every call shares the one array, which keeps the previous call's
//     contents; nothing in it has to start at zero (each partial is written
//     before it is read), but calls whose work overlaps on the GPU (different
//     streams, or other host threads) race on it and must be ordered by the
//     caller;
//   * the first call on a device looks the array's device address up
//     (cudaGetSymbolAddress) and caches it, so make that first call before
//     any stream capture.  The cache is keyed by the device's current CUDA
//     context: after the caller destroys and recreates that context (for
//     example cudaDeviceReset), the next call looks the address up again and
//     should likewise come before any capture.
// ===================================================================
#include <mutex>

#include "runtime.h"

namespace attnb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices];
int g_noalloc_sms[kNoAllocMaxDevices];
unsigned long long g_noalloc_ctx[kNoAllocMaxDevices];  // context the address belongs to

// Unique id of the calling thread's current CUDA context (driver entry points
// looked up through the runtime, as for the tensor-map encoder), or 0 when it
// cannot be read; a context created after a reset gets a new id.
unsigned long long current_context_id() {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static const std::pair<GetCurrentFn, GetIdFn> fns = [] {
    void* a = nullptr;
    void* b = nullptr;
    cudaDriverEntryPointQueryResult qa, qb;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &a, 12000, cudaEnableDefault, &qa) !=
            cudaSuccess || qa != cudaDriverEntryPointSuccess)
      a = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &b, 12000, cudaEnableDefault, &qb) !=
            cudaSuccess || qb != cudaDriverEntryPointSuccess)
      b = nullptr;
    cudaGetLastError();
    return std::make_pair(reinterpret_cast<GetCurrentFn>(a), reinterpret_cast<GetIdFn>(b));
  }();
  if (!fns.first || !fns.second) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (fns.first(&ctx) != CUDA_SUCCESS || !ctx || fns.second(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// The reference's validate_dense_shapes (include/attn.h:54-83), same messages.
void noalloc_validate(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
                      const attnb_mtensor* O) {
  if (!Q || !K || !V || !O) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null tensor descriptor");
  if (!Q->data || !K->data || !V->data || !O->data)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
  if (Q->H <= 0 || Q->Dh <= 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "Q has invalid H/Dh");
  if (K->H != Q->H || V->H != Q->H) fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V H must match Q.H");
  if (K->Dh != Q->Dh || V->Dh != Q->Dh)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V Dh must match Q.Dh");
  if (K->T <= 0 || V->T != K->T)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V T must be positive and equal");
  if (O->H != Q->H || O->Dh != Q->Dh)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "O must be [H, Dh] matching Q");
  if (Q->strideH == 0 || Q->strideDh == 0 || K->strideH == 0 || K->strideT == 0 ||
      K->strideDh == 0 || V->strideH == 0 || V->strideT == 0 || V->strideDh == 0 ||
      O->strideH == 0 || O->strideDh == 0)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "Zero stride encountered");
}

// Device address of the fixed scratch and the SM count, looked up with the
// device current on its first call, and again whenever the device's current
// context is no longer the one the address was looked up in.
void* noalloc_scratch(int dev, int* num_sms) {
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    fail(ATTNB_ERR_RUNTIME, "device index out of range for the fixed decode scratch");
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  // Make sure the runtime has made the device's context current before its id
  // is read (the first runtime call of a thread creates it lazily).
  ATTNB_CUDA(cudaDeviceGetAttribute(num_sms, cudaDevAttrMultiProcessorCount, dev));
  const unsigned long long ctx = current_context_id();
  if (!g_noalloc_addr[dev] || ctx == 0 || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    ATTNB_CUDA(cudaGetSymbolAddress(&p, g_decode_scratch));
    g_noalloc_sms[dev] = *num_sms;
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *num_sms = g_noalloc_sms[dev];
  return g_noalloc_addr[dev];
}

}  // namespace
}  // namespace attnb

extern "C" ATTNB_API int attnb_attn_step_dense_noalloc(const attnb_tensor* Q,
                                                       const attnb_tensor* K,
                                                       const attnb_tensor* V, attnb_mtensor* O,
                                                       void* stream) {
  using namespace attnb;
  NvtxRange range(__func__);
  try {
    noalloc_validate(Q, K, V, O);
    int dev = -1;
    ATTNB_CUDA(cudaGetDevice(&dev));
    int num_sms = 0;
    void* scratch = noalloc_scratch(dev, &num_sms);
    const View3 q{Q->data, Q->H, 1, Q->Dh, Q->strideH, 0, Q->strideDh};
    const View3 k{K->data, K->H, K->T, K->Dh, K->strideH, K->strideT, K->strideDh};
    const View3 v{V->data, V->H, V->T, V->Dh, V->strideH, V->strideT, V->strideDh};
    const MView3 o{O->data, O->H, 1, O->Dh, O->strideH, 0, O->strideDh};
    const DecodePlan p = decode_plan(q, k, v, num_sms);
    const size_t need = decode_workspace_bytes(p, K->H, K->Dh);
    if (need > kNoAllocScratchBytes)
      fail(ATTNB_ERR_INVALID_ARGUMENT,
           "decode step needs " + std::to_string(need) + " bytes of scratch; the fixed scratch of "
           "attnb_attn_step_dense_noalloc holds " + std::to_string(kNoAllocScratchBytes) +
           " (use attnb_attn_step_dense_dev)");
    decode_launch(p, q, k, v, o, scratch, static_cast<cudaStream_t>(stream));
    ATTNB_CUDA(cudaGetLastError());
    return ATTNB_OK;
  } catch (const Error& e) {
    return set_last_error(e.code, e.msg);
  } catch (const std::exception& e) {
    return set_last_error(ATTNB_ERR_RUNTIME, e.what());
  }
}
