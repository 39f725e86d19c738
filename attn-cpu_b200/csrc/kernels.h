// kernels.h -- host-side launch interface of the device kernels.  Everything
// here takes device pointers and a stream; validation happens in capi.cu.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

namespace attnb {

// Strided fp32 view [H, T, Dh] (strides in elements).
struct View3 {
  const float* data;
  int H, T, Dh;
  int64_t sH, sT, sD;
};
struct MView3 {
  float* data;
  int H, T, Dh;
  int64_t sH, sT, sD;
};

// ------------------------------------------------------------ peer memory
// Replicas of an output on other GPUs (peer pointers mapped into this
// process) that a kernel writes besides the output itself: every element
// stored to the output is also stored, at the same offset from dst[i] (same
// strides), to each replica.
constexpr int kMaxPeerOut = 7;
struct PeerOut {
  float* dst[kMaxPeerOut];
  int n;
};
// Flag arrays of a cross-GPU barrier (peer.cu): `local` is this rank's array
// of n epochs followed by its own barrier count, peer[r] rank r's array as
// mapped into this process.
constexpr int kMaxRanks = 8;
struct PeerFlags {
  uint64_t* local;
  uint64_t* peer[kMaxRanks];
  int n, rank;
};
// Enqueues the next barrier on s; a wait longer than limit_ns raises the
// status word.
void peer_barrier(const PeerFlags& f, uint64_t limit_ns, int* status, cudaStream_t s);

// ------------------------------------------------------------ decode (K4)
// Split-KV plan for one decode step: how many key ranges each head is cut
// into and how long each range is.
struct DecodePlan {
  int nsplit;
  int keys_per_split;
  bool fast;  // 128-bit vector path (strideDh == 1, 16-byte aligned rows, Dh % 4 == 0, Dh <= 256)
};
DecodePlan decode_plan(const View3& Q, const View3& K, const View3& V, int num_sms);
// Scratch bytes the plan needs (0 when nsplit == 1).
size_t decode_workspace_bytes(const DecodePlan& p, int H, int Dh);
// O[h, :] for every head; `ws` holds decode_workspace_bytes(p, ...) bytes.
// With `peers`, every element of O is also stored into each replica.
void decode_launch(const DecodePlan& p, const View3& Q, const View3& K, const View3& V,
                   const MView3& O, void* ws, cudaStream_t stream,
                   const PeerOut* peers = nullptr);

// ------------------------------------------- generic prefill (CUDA cores)
// O[h,l,:] for any strides and head size; exact fp32 online softmax.
void attn_block_simt_launch(const View3& Q, const View3& K, const View3& V, const MView3& O,
                            bool causal, cudaStream_t stream);

// ---------------------------------------- tcgen05 prefill attention (K3)
struct AttnTcPlan {
  int H, L, T, Dh, dhp, tp, qtiles, nsplit, tiles_per_split;
  bool split3;
  // One key tile per CTA and dhp <= 64: when the views allow TMA reads, the
  // kernel loads and splits the raw operands itself (no packing launch).
  bool fusable;
  // 1xTF32 with at least two query tiles and two key tiles: K3p (attn_pp.cu),
  // two query tiles per CTA.  ATTNB_ATTN_PAIRS=0 keeps K3.
  bool pairs;
  // 1xTF32, non-causal, head size 128: K3q (attn_pair.cu) on CTA pairs.
  // ATTNB_ATTN_CTA_PAIRS=0 turns it off.
  bool cta_pairs;
  size_t off_q, off_k, off_v, ws_bytes;
};
// Head sizes the tensor-core kernel takes (padded to a multiple of 32, <= 128).
bool attn_tc_supported(int Dh);
AttnTcPlan attn_tc_plan(int H, int L, int T, int Dh, bool causal, int precision, int num_sms);
// `ws` holds plan.ws_bytes bytes (packed operands).
void attn_tc_run(const AttnTcPlan& p, const View3& Q, const View3& K, const View3& V,
                 const MView3& O, bool causal, void* ws, int* status, int num_sms,
                 cudaStream_t s);

// K3p: 1xTF32 prefill, two query tiles per CTA (attn_pp.cu).  Maps as built by
// attn_tc_run for the packed operands: Q [H, L, dhp] box 128 x 32, K [H, T, dhp]
// box 128 x 32, V^T [H, dhp, tp] box dhp x 32, and O box 128 x 32 (o_tma).
struct AttnPPArgs {
  int L, T, H, Dh, causal, qtiles, o_tma;
  float* O;
  int64_t osH, osT, osD;
  int* status;
};
void attn_pp_launch(int dhp, const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                    const CUtensorMap& o, const AttnPPArgs& a, cudaStream_t s);

// K3q: 1xTF32 prefill on CTA pairs (attn_pair.cu), head size 128.  Maps: Q as
// for K3p, K [H, T, dhp] box 64 x 32, V^T [H, dhp, tp] box dhp/2 x 32, O box
// 128 x 32 (o_tma).
void attn_pair_launch(int dhp, const CUtensorMap& q, const CUtensorMap& k_half,
                      const CUtensorMap& v_half, const CUtensorMap& o, const AttnPPArgs& a,
                      cudaStream_t s);

// ------------------------------------------------ operand packing (K2)
// One packing job: a strided 3-D source src[h][r][c] (r < R, c < C), times
// `scale`, written to hi (and lo when splitting) either in place as
// [H][rows_out = R][cols_out] (columns C..cols_out-1 zero) or, with
// `transpose`, as [H][rows_out][cols_out] holding src[h][r][c] at [h][c][r]
// (zero outside r < R, c < C).  cols_out % 4 == 0.
struct PackJob {
  const float* src;
  int64_t sH, sR, sC;
  int H, R, C;
  int rows_out, cols_out;
  bool transpose;
  float scale;
  float* hi;
  float* lo;
};
constexpr int kMaxPackJobs = 3;
// Packs up to kMaxPackJobs jobs in one launch.
void pack_launch(const PackJob* jobs, int njobs, bool split3, int num_sms, cudaStream_t s);

// Launches `kernel` with programmatic stream serialisation, so its prologue
// may overlap the previous kernel on the stream; the kernel must execute
// griddepcontrol.wait before reading what that kernel wrote.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// As launch_pdl, with the grid tiled into thread-block clusters of `cluster`.
template <class... KArgs, class... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t s, dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster.x;
  attr[1].val.clusterDim.y = cluster.y;
  attr[1].val.clusterDim.z = cluster.z;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// --------------------------------------------------- tcgen05 GEMM (K1)
// C[M,N] = alpha * A.B + beta * C (+ bias[n]).  A is [M,K] (a_kmajor: rows of
// K, pitch lda) or [K,M] (pitch lda); B is [N,K] (b_kmajor) or [K,N].
struct GemmPlan {
  int M, N, K, Kp;
  bool split3;
  size_t off_a_hi, off_a_lo, off_b_hi, off_b_lo, ws_bytes;
};
GemmPlan gemm_plan(int M, int N, int K, int precision);
// C[M,N] = beta * C + bias[n] (bias may be null; beta == 0 never reads C).
void gemm_scale_bias(float* C, int64_t ldc, int M, int N, float beta, const float* bias,
                     int num_sms, cudaStream_t s);
// Scratch bytes of a plan of this size.
size_t gemm_workspace_bound(int M, int N, int K, int precision);
// With pre_b_hi (and pre_b_lo in 3xTF32), B is not read: the operand comes
// already packed by gemm_pack_b for this N, K and precision.
void gemm_run(const GemmPlan& p, const float* A, int64_t lda, bool a_kmajor, const float* B,
              int64_t ldb, bool b_kmajor, float* C, int64_t ldc, float alpha, float beta,
              const float* bias, void* ws, int* status, int num_sms, cudaStream_t s,
              const PeerOut* peers = nullptr, const float* pre_b_hi = nullptr,
              const float* pre_b_lo = nullptr);
// Bytes of one packed operand of `rows` x K (hi, then lo in 3xTF32, each
// 256-byte aligned), and the packing of B ([N, K] rows when b_kmajor, else
// [K, N]) into it, as gemm_run packs B.
size_t gemm_packed_bytes(int rows, int K, bool split3);
void gemm_pack_b(const float* B, int64_t ldb, bool b_kmajor, int N, int K, bool split3,
                 float* hi, float* lo, int num_sms, cudaStream_t s);

}  // namespace attnb
