// gemm_tc.cu -- K1: persistent tcgen05 SGEMM (kind::tf32, 1xTF32 or 3xTF32).
//
// Computes C[M,N] = alpha * A.B^T' + beta * C (+ bias[n]) where both operands
// arrive K-major in HBM: A as [M, K] rows, B as [N, K] rows (split.cu packs
// them, or they are used in place when already K-major and 16-byte aligned).
// It replaces the reference's FMA micro-kernels: src/gemm.cpp:89-249
// (8x48 register tiles over KC=768 panels), src/jit_gemm.cpp:256-406 (JIT
// 8xNR tiles) and include/gemm_16x16.h:7-60 (bias-initialised row GEMM of the
// MHA projections).  Accumulation is fp32 in tensor memory over the whole K.
//
// Structure (one CTA per SM, persistent over 128 x BN output tiles):
//   warp 0      TMA producer: fills a STAGES-deep shared-memory ring with
//               128-byte-swizzled 32-wide K slices of A (and B), signalling
//               `full[s]` with the transaction byte count;
//   warp 1      allocates all 512 TMEM columns (two accumulator slots), then
//               one lane issues tcgen05.mma (4 K-steps of 8 per slice) and
//               tcgen05.commit's each slice back to the producer (`empty[s]`)
//               and each finished accumulator to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld the accumulator (lane = row), apply
//               alpha / beta / bias, store to C, release the slot.
// 1xTF32: one 128xBN accumulator per tile (BN = 256, or 128 / 64 when the
// product has too few wide tiles to occupy every SM); the two slots let the
// epilogue of tile i overlap the MMAs of tile i+1.
// 3xTF32 (128x128 or 128x64 tiles): hi*hi goes to a "big" accumulator and
// hi*lo + lo*hi to a separate "small" one, and both are drained into fp32
// registers every 256 K values, alternating slots, so the epilogue's
// round-to-nearest fp32 sums carry the long-K accumulation.
#include <algorithm>
#include <atomic>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace attnb {
namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int GROUP_M = 16;

template <int BN, bool SPLIT3>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 4;                 // 16 KB
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = (SPLIT3 ? 2 : 1) * (A_BYTES + B_BYTES);
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;    // + alignment slack
  // Peer-output form: each epilogue warp turns its 32 rows x 32 columns
  // around in shared memory (rows padded to 36 floats) before storing them.
  static constexpr int XPOSE_ROW = 36;
  static constexpr int XPOSE_BYTES = 4 * 32 * XPOSE_ROW * 4;
  static constexpr int SMEM_BCAST = SMEM + XPOSE_BYTES;
  // Two accumulator slots; in 3xTF32 mode each slot holds a "big" (hi*hi)
  // and a "small" (hi*lo + lo*hi) accumulator.
  static constexpr int SLOT_COLS = (SPLIT3 ? 2 : 1) * BN;
  static constexpr int TMEM_COLS = 2 * SLOT_COLS;
  static_assert(STAGES >= 2, "pipeline needs two stages");
  static_assert(TMEM_COLS <= 512, "TMEM has 512 columns");
};

// 3xTF32 drains its TMEM accumulators into fp32 registers every KB_CHUNK
// K-slices (256 K values): the tensor core's own accumulation truncates, so
// long K runs inside TMEM would drift by up to ~1e-5 relative at K = 4096.
constexpr int KB_CHUNK = 8;

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int per_group = GROUP_M * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * GROUP_M;
  const int gsize = min(tiles_m - first_m, GROUP_M);
  const int r = tile % per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

// Wait without the abort short-cut: used to drain copies that are in flight.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity, int* status) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > ATTNB_WAIT_LIMIT_NS) {
      raise_timeout(status);
      return;
    }
  }
}

// Epilogue for 32 consecutive columns of one output row.
__device__ __forceinline__ void store32(float* crow, int row, int col0, const float* acc, int M,
                                        int N, float alpha, float beta,
                                        const float* __restrict__ bias, bool c_vec) {
  if (row >= M) return;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = alpha * acc[j];
  if (beta != 0.f) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) v[j] = fmaf(beta, crow[col0 + j], v[j]);
  }
  if (bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) v[j] += __ldg(bias + col0 + j);
  }
  if (c_vec && col0 + 32 <= N) {
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(crow + col0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) crow[col0 + j] = v[j];
  }
}

// Peer-output epilogue for 32 consecutive columns of the 32 rows [row0,
// row0 + 32) that one warp holds (lane = row).  The values are those of
// store32; they are turned around through the warp's block of shared memory
// `xp` ([32][XROW] floats) and stored by row segments -- eight lanes write one
// row's 128 contiguous bytes -- to C and to every replica in `peers`, so each
// store instruction moves four whole 128-byte lines (whole NVLink writes for
// a replica on another GPU).
template <int XROW>
__device__ __forceinline__ void store32_bcast(float* __restrict__ C, int64_t ldc, int row0,
                                              int lane, int col0, const float* acc, int M, int N,
                                              float alpha, float beta,
                                              const float* __restrict__ bias, bool c_vec,
                                              float* xp, const PeerOut& peers) {
  const int row = row0 + lane;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = alpha * acc[j];
  if (beta != 0.f && row < M) {
    const float* crow = C + (int64_t)row * ldc;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) v[j] = fmaf(beta, crow[col0 + j], v[j]);
  }
  if (bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) v[j] += __ldg(bias + col0 + j);
  }
  __syncwarp();  // the previous chunk's reads of xp are done
  float* mine = xp + lane * XROW;
#pragma unroll
  for (int j = 0; j < 32; j += 4)
    *reinterpret_cast<float4*>(mine + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  __syncwarp();
  const int c4 = (lane & 7) * 4;
  const int col = col0 + c4;
#pragma unroll 2
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    const int grow = row0 + r;
    if (grow >= M || col >= N) continue;
    const float4 q = *reinterpret_cast<const float4*>(xp + r * XROW + c4);
    const int64_t off = (int64_t)grow * ldc + col;
    if (c_vec && col + 4 <= N) {
      *reinterpret_cast<float4*>(C + off) = q;
#pragma unroll
      for (int p = 0; p < kMaxPeerOut; ++p)
        if (p < peers.n) *reinterpret_cast<float4*>(peers.dst[p] + off) = q;
    } else {
      const float e[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (col + k >= N) break;
        C[off + k] = e[k];
#pragma unroll
        for (int p = 0; p < kMaxPeerOut; ++p)
          if (p < peers.n) peers.dst[p][off + k] = e[k];
      }
    }
  }
}

template <int BN, bool SPLIT3, bool BCAST = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA_hi,
                   const __grid_constant__ CUtensorMap tmA_lo,
                   const __grid_constant__ CUtensorMap tmB_hi,
                   const __grid_constant__ CUtensorMap tmB_lo, int M, int N, int Kp,
                   float* __restrict__ C, int64_t ldc, float alpha, float beta,
                   const float* __restrict__ bias, int* status, const PeerOut peers) {
  using Cfg = GemmCfg<BN, SPLIT3>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_tf32(BM, BN);
  // 3xTF32: A_hi.[B_hi | B_lo] as one MMA of width 2*BN (B_lo follows B_hi in
  // the stage, the small accumulator follows the big one in TMEM), then
  // A_lo.B_hi into the small accumulator: two MMAs per K step for three
  // products.
  constexpr uint32_t IDESC2 = idesc_tf32(BM, 2 * BN);

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2], tempty_bar[2], final_bar;
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tiles_base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  auto sA_hi = [&](int s) { return tiles_base + s * Cfg::STAGE_BYTES; };
  auto sA_lo = [&](int s) { return tiles_base + s * Cfg::STAGE_BYTES + Cfg::A_BYTES; };
  auto sB_hi = [&](int s) {
    return tiles_base + s * Cfg::STAGE_BYTES + (SPLIT3 ? 2 : 1) * Cfg::A_BYTES;
  };
  static_assert(!SPLIT3 || 2 * BN <= 256, "double-width MMA: N <= 256");
  auto sB_lo = [&](int s) {
    return tiles_base + s * Cfg::STAGE_BYTES + 2 * Cfg::A_BYTES + Cfg::B_BYTES;
  };

  const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = Kp / BK;
  // Accumulator hand-offs per tile: one per K chunk (3xTF32) or one per tile.
  const int nchunks = SPLIT3 ? (num_kb + KB_CHUNK - 1) / KB_CHUNK : 1;
  const int kb_per_chunk = SPLIT3 ? KB_CHUNK : num_kb;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&tfull_bar[b]), 1);
      mbar_init(smem_addr(&tempty_bar[b]), 4);
    }
    mbar_init(smem_addr(&final_bar), 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA_hi);
    tma_prefetch_desc(&tmB_hi);
    if (SPLIT3) {
      tma_prefetch_desc(&tmA_lo);
      tma_prefetch_desc(&tmB_lo);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(&tmem_base_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_slot;
  volatile int* abort_p = &abort_flag;
  grid_dep_wait();  // the packed operands come from the kernel before this one

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, tiles_m, tiles_n, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_addr(&empty_bar[stage]), phase ^ 1u, abort_p, status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_addr(&full_bar[stage]);
          mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
          tma_load_2d(sA_hi(stage), &tmA_hi, fb, kb * BK, tm * BM);
          tma_load_2d(sB_hi(stage), &tmB_hi, fb, kb * BK, tn * BN);
          if (SPLIT3) {
            tma_load_2d(sA_lo(stage), &tmA_lo, fb, kb * BK, tm * BM);
            tma_load_2d(sB_lo(stage), &tmB_lo, fb, kb * BK, tn * BN);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Copies still in flight (only possible after an abort) land before exit.
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s))
          mbar_drain(smem_addr(&full_bar[s]), (issued_parity >> s) & 1u, status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int g = 0;  // accumulator hand-offs so far
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        for (int c = 0; ok && c < nchunks; ++c, ++g) {
          const int slot = g & 1;
          const uint32_t use = (g >> 1) & 1;
          if (!mbar_wait(smem_addr(&tempty_bar[slot]), use ^ 1u, abort_p, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_big = tmem_base + slot * Cfg::SLOT_COLS;
          const uint32_t d_small = d_big + BN;
          const int kb0 = c * kb_per_chunk;
          const int kb1 = min(num_kb, kb0 + kb_per_chunk);
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(smem_addr(&full_bar[stage]), phase, abort_p, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk) {
              const uint32_t acc = (kb != kb0 || kk != 0) ? 1u : 0u;
              const uint64_t a_hi = sdesc_kmajor_sw128(sA_hi(stage) + kk * 32);
              const uint64_t b_hi = sdesc_kmajor_sw128(sB_hi(stage) + kk * 32);
              if (SPLIT3) {
                const uint64_t a_lo = sdesc_kmajor_sw128(sA_lo(stage) + kk * 32);
                mma_tf32(d_big, a_hi, b_hi, IDESC2, acc);
                mma_tf32(d_small, a_lo, b_hi, IDESC, 1u);
              } else {
                mma_tf32(d_big, a_hi, b_hi, IDESC, acc);
              }
            }
            mma_commit(smem_addr(&empty_bar[stage]));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (ok) mma_commit(smem_addr(&tfull_bar[slot]));
        }
      }
      // Every MMA issued above has finished before TMEM is released.
      mma_commit(smem_addr(&final_bar));
      mbar_drain(smem_addr(&final_bar), 0, status);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const bool c_vec = ((ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0);
    // Peer-output form: this warp's transpose block, past the operand ring.
    float* xp = nullptr;
    if constexpr (BCAST)
      xp = reinterpret_cast<float*>(smem_raw + (tiles_base - smem_addr(smem_raw)) +
                                    STAGES * Cfg::STAGE_BYTES) +
           quarter * 32 * Cfg::XPOSE_ROW;
    int g = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
      int tm, tn;
      tile_coords(tile, tiles_m, tiles_n, tm, tn);
      const int row = tm * BM + quarter * 32 + lane;
      float* crow = C + (int64_t)row * ldc;
      if constexpr (SPLIT3) {
        float acc[BN];
#pragma unroll
        for (int i = 0; i < BN; ++i) acc[i] = 0.f;
        for (int c = 0; c < nchunks; ++c, ++g) {
          const int slot = g & 1;
          const uint32_t use = (g >> 1) & 1;
          if (!mbar_wait(smem_addr(&tfull_bar[slot]), use, abort_p, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tb = tmem_base + lane_off + slot * Cfg::SLOT_COLS;
#pragma unroll
          for (int j = 0; j < BN / 32; ++j) {
            uint32_t rb[32], rs[32];
            tmem_ld32(tb + j * 32, rb);
            tmem_ld32(tb + BN + j * 32, rs);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              acc[j * 32 + i] += __uint_as_float(rb[i]) + __uint_as_float(rs[i]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_addr(&tempty_bar[slot]));
        }
        if (!ok) break;
        if constexpr (BCAST) {
#pragma unroll
          for (int j = 0; j < BN / 32; ++j)
            store32_bcast<Cfg::XPOSE_ROW>(C, ldc, tm * BM + quarter * 32, lane, tn * BN + j * 32,
                                          &acc[j * 32], M, N, alpha, beta, bias, c_vec, xp,
                                          peers);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 32; ++j)
            store32(crow, row, tn * BN + j * 32, &acc[j * 32], M, N, alpha, beta, bias, c_vec);
        }
      } else {
        const int slot = g & 1;
        const uint32_t use = (g >> 1) & 1;
        if (!mbar_wait(smem_addr(&tfull_bar[slot]), use, abort_p, status)) break;
        tc_fence_after();
        const uint32_t tb = tmem_base + lane_off + slot * Cfg::SLOT_COLS;
#pragma unroll 1
        for (int j = 0; j < BN / 32; ++j) {
          uint32_t r[32];
          tmem_ld32(tb + j * 32, r);
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          if constexpr (BCAST)
            store32_bcast<Cfg::XPOSE_ROW>(C, ldc, tm * BM + quarter * 32, lane, tn * BN + j * 32,
                                          v, M, N, alpha, beta, bias, c_vec, xp, peers);
          else
            store32(crow, row, tn * BN + j * 32, v, M, N, alpha, beta, bias, c_vec);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&tempty_bar[slot]));
        ++g;
      }
    }
    // Stores to the replicas are visible system-wide before this CTA retires,
    // so a collective that follows the kernel orders every reader after them.
    if constexpr (BCAST) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// K1f: one tile per CTA, operand split fused in.
//
// When the 128 x BN output tiles number at most the SM count, the packing pass
// and the L2 traffic of the packed copies (hi and lo, re-read by every tile of
// a row or column) cost as much as the MMAs.  This form TMA-loads the raw fp32
// slices -- A as [128 rows x 32 k]; B as [BN rows x 32 k] when K-major, or as
// (BN/32) boxes of [32 k x 32 columns] staged and transposed when N-major --
// and the four epilogue warps split them into the tf32 hi / fp32 lo operand
// slots while the MMAs run: eight warps (2-9), the four epilogue warps among
// them.  In 3xTF32 every 256-K chunk gets its own TMEM accumulator pair (at
// most 512 / (2 BN) chunks), drained once at the end, so those warps have
// nothing else to do during the loop.
constexpr int kFusedThreads = 320;
// hi = tf32 round-to-nearest of x (exact as a tf32 operand), lo = x - hi
// (exact in fp32).
__device__ __forceinline__ void split4(float4 x, float4& hi, float4& lo) {
  hi = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
  lo = make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w);
}

template <int BN, bool SPLIT3, bool B_KMAJOR>
struct FusedCfg {
  static constexpr int NPART = SPLIT3 ? 2 : 1;
  static constexpr int A_BYTES = BM * BK * 4;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int RAW_B = B_KMAJOR ? 0 : BK * BN * 4;  // N-major B staging
  static constexpr int OFF_A_LO = A_BYTES;
  static constexpr int OFF_B_HI = NPART * A_BYTES;
  static constexpr int OFF_B_LO = OFF_B_HI + B_BYTES;  // follows B_hi: one [B_hi | B_lo] operand
  static constexpr int OFF_RAW = NPART * (A_BYTES + B_BYTES);
  static constexpr int STAGE_BYTES = OFF_RAW + RAW_B;
  static constexpr int STAGES_FIT = (200 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT < 6 ? STAGES_FIT : 6;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
  static constexpr int SLOT_COLS = NPART * BN;  // one chunk's [big | small] accumulators
  static constexpr int MAX_CHUNKS = SPLIT3 ? 512 / SLOT_COLS : 1;
  static constexpr int TMEM_COLS = SPLIT3 ? 512 : (BN < 32 ? 32 : BN);
  static_assert(STAGES >= 2, "pipeline needs two stages");
};

template <int BN, bool SPLIT3, bool B_KMAJOR>
__global__ void __launch_bounds__(kFusedThreads, 1)
    gemm_fused_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
                      float* __restrict__ C, int64_t ldc, float alpha, float beta,
                      const float* __restrict__ bias, int* status) {
  using Cfg = FusedCfg<BN, SPLIT3, B_KMAJOR>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_tf32(BM, BN);
  constexpr uint32_t IDESC2 = idesc_tf32(BM, 2 * BN);  // A_hi . [B_hi | B_lo]
  static_assert(!SPLIT3 || 2 * BN <= 256, "double-width MMA: N <= 256");
  static_assert(Cfg::MAX_CHUNKS * Cfg::SLOT_COLS <= Cfg::TMEM_COLS, "chunk slots fit TMEM");

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES], conv_bar[STAGES], empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar, final_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base - smem_addr(smem_raw));
  auto stage_addr = [&](int s) { return base + s * Cfg::STAGE_BYTES; };
  const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
  int tm, tn;
  tile_coords(blockIdx.x, tiles_m, tiles_n, tm, tn);
  const int nkb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&conv_bar[s]), 8);  // one arrival per converting warp
      mbar_init(smem_addr(&empty_bar[s]), 1);
    }
    mbar_init(smem_addr(&tfull_bar), 1);
    mbar_init(smem_addr(&final_bar), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(&tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;
  grid_dep_wait();  // the operands may come from the kernel before this one

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------- producer (raw fp32)
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, issued_parity = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(smem_addr(&empty_bar[stage]), phase ^ 1u, abort_p, status)) break;
        const uint32_t fb = smem_addr(&full_bar[stage]), sa = stage_addr(stage);
        mbar_arrive_expect_tx(fb, Cfg::A_BYTES + (B_KMAJOR ? Cfg::B_BYTES : Cfg::RAW_B));
        tma_load_2d(sa, &tmA, fb, kb * BK, tm * BM);
        if (B_KMAJOR) {
          tma_load_2d(sa + Cfg::OFF_B_HI, &tmB, fb, kb * BK, tn * BN);
        } else {
#pragma unroll
          for (int bx = 0; bx < BN / 32; ++bx)
            tma_load_2d(sa + Cfg::OFF_RAW + bx * 4096, &tmB, fb, tn * BN + bx * 32, kb * BK);
        }
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Copies still in flight (only possible after an abort) land before exit.
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s))
          mbar_drain(smem_addr(&full_bar[s]), (issued_parity >> s) & 1u, status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; ok && kb < nkb; ++kb) {
        if (!mbar_wait(smem_addr(&conv_bar[stage]), phase, abort_p, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = stage_addr(stage);
        // 3xTF32: chunk kb / KB_CHUNK accumulates into its own slot.
        const int c = SPLIT3 ? kb / KB_CHUNK : 0;
        const bool first = SPLIT3 ? (kb % KB_CHUNK) == 0 : kb == 0;
        const uint32_t d_big = tmem + c * Cfg::SLOT_COLS, d_small = d_big + BN;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint32_t acc = (!first || kk != 0) ? 1u : 0u;
          const uint64_t a_hi = sdesc_kmajor_sw128(sa + kk * 32);
          const uint64_t b_hi = sdesc_kmajor_sw128(sa + Cfg::OFF_B_HI + kk * 32);
          if (SPLIT3) {
            const uint64_t a_lo = sdesc_kmajor_sw128(sa + Cfg::OFF_A_LO + kk * 32);
            mma_tf32(d_big, a_hi, b_hi, IDESC2, acc);
            mma_tf32(d_small, a_lo, b_hi, IDESC, 1u);
          } else {
            mma_tf32(d_big, a_hi, b_hi, IDESC, acc);
          }
        }
        mma_commit(smem_addr(&empty_bar[stage]));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) mma_commit(smem_addr(&tfull_bar));
      // Every MMA issued above has finished before TMEM is released.
      mma_commit(smem_addr(&final_bar));
      mbar_drain(smem_addr(&final_bar), 0, status);
    }
  } else {
    // ------------------------------------- operand split, then epilogue
    const int t = threadIdx.x - 64, cw = warp - 2;  // 0..255, converting warp 0..7
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
      // Lanes of a warp pass the same __syncwarp whatever their waits returned.
      if (ok && !mbar_wait(smem_addr(&full_bar[stage]), phase, abort_p, status)) ok = false;
      if (ok) {
        uint8_t* st = sbase + stage * Cfg::STAGE_BYTES;
        // A (and a K-major B) in place: hi over the raw value, lo beside it.
#pragma unroll 4
        for (int i = t; i < Cfg::A_BYTES / 16; i += 256) {
          float4* x = reinterpret_cast<float4*>(st + i * 16);
          float4 hi, lo;
          split4(*x, hi, lo);
          *x = hi;
          if (SPLIT3) *reinterpret_cast<float4*>(st + Cfg::OFF_A_LO + i * 16) = lo;
        }
        if (B_KMAJOR) {
#pragma unroll 4
          for (int i = t; i < Cfg::B_BYTES / 16; i += 256) {
            float4* x = reinterpret_cast<float4*>(st + Cfg::OFF_B_HI + i * 16);
            float4 hi, lo;
            split4(*x, hi, lo);
            *x = hi;
            if (SPLIT3) *reinterpret_cast<float4*>(st + Cfg::OFF_B_LO + i * 16) = lo;
          }
        } else {
          // N-major B: lane = k; a 16-byte read of four columns of row k of a
          // staged box, four 4-byte writes down the K-major rows of B.
          for (int gi = cw; gi < BN / 4; gi += 8) {
            const int bx = gi >> 3, c = gi & 7;
            const float4 x = *reinterpret_cast<const float4*>(
                st + Cfg::OFF_RAW + bx * 4096 + lane * 128 + ((c ^ (lane & 7)) << 4));
            float4 hi, lo;
            split4(x, hi, lo);
            const float hv[4] = {hi.x, hi.y, hi.z, hi.w};
            const float lv[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int n = gi * 4 + i;
              const uint32_t off = n * 128 + (((lane >> 2) ^ (n & 7)) << 4) + (lane & 3) * 4;
              *reinterpret_cast<float*>(st + Cfg::OFF_B_HI + off) = hv[i];
              if (SPLIT3) *reinterpret_cast<float*>(st + Cfg::OFF_B_LO + off) = lv[i];
            }
          }
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(smem_addr(&conv_bar[stage]));
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    // Epilogue (warps 2-5): row = TMEM lane; the chunks' big + small sums
    // (3xTF32) added in fp32 registers in chunk order.
    if (warp < 6 && ok && mbar_wait(smem_addr(&tfull_bar), 0, abort_p, status)) {
      tc_fence_after();
      const int quarter = warp & 3;
      const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
      const int row = tm * BM + quarter * 32 + lane;
      float* crow = C + (int64_t)row * ldc;
      const bool c_vec = ((ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0);
      const int nchunks = SPLIT3 ? (nkb + KB_CHUNK - 1) / KB_CHUNK : 1;
#pragma unroll 1
      for (int j = 0; j < BN / 32; ++j) {
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        for (int c = 0; c < nchunks; ++c) {
          const uint32_t tb = tmem + lane_off + c * Cfg::SLOT_COLS + j * 32;
          uint32_t rb[32], rs[32];
          if (SPLIT3) {
            tmem_ld32x2(tb, rb, tb + BN, rs);
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] += __uint_as_float(rb[i]) + __uint_as_float(rs[i]);
          } else {
            tmem_ld32(tb, rb);
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(rb[i]);
          }
        }
        store32(crow, row, tn * BN + j * 32, acc, M, N, alpha, beta, bias, c_vec);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int BN, bool SPLIT3, bool B_KMAJOR>
void launch_fused(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, float* C,
                  int64_t ldc, float alpha, float beta, const float* bias, int* status,
                  cudaStream_t s) {
  using Cfg = FusedCfg<BN, SPLIT3, B_KMAJOR>;
  static std::atomic<uint64_t> configured{0};  // one bit per device
  int dev = 0;
  ATTNB_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    ATTNB_CUDA(cudaFuncSetAttribute(gemm_fused_kernel<BN, SPLIT3, B_KMAJOR>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    configured.fetch_or(bit);
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  ATTNB_CUDA(launch_pdl(gemm_fused_kernel<BN, SPLIT3, B_KMAJOR>, dim3(tiles),
                        dim3(kFusedThreads), Cfg::SMEM, s, ta, tb, M, N, K, C, ldc, alpha, beta,
                        bias, status));
}

// C = beta * C (+ bias[n]): the alpha == 0 path of the reference
// (src/gemm.cpp:328-336) and an empty inner dimension.  beta == 0 never reads C.
__global__ void scale_c_kernel(float* C, int64_t ldc, int M, int N, float beta,
                               const float* __restrict__ bias) {
  const int64_t n = (int64_t)M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / N, c = i % N;
    float* p = C + r * ldc + c;
    const float b = bias ? bias[c] : 0.f;
    *p = (beta == 0.f) ? b : fmaf(*p, beta, b);
  }
}

template <int BN, bool SPLIT3, bool BCAST = false>
void launch_gemm(const GemmPlan& p, const CUtensorMap& a_hi, const CUtensorMap& a_lo,
                 const CUtensorMap& b_hi, const CUtensorMap& b_lo, float* C, int64_t ldc,
                 float alpha, float beta, const float* bias, int* status, int num_sms,
                 cudaStream_t s, const PeerOut& peers = PeerOut{}) {
  using Cfg = GemmCfg<BN, SPLIT3>;
  constexpr int smem = BCAST ? Cfg::SMEM_BCAST : Cfg::SMEM;
  static std::atomic<uint64_t> configured{0};  // one bit per device
  int dev = 0;
  ATTNB_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    ATTNB_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, SPLIT3, BCAST>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured.fetch_or(bit);
  }
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = std::min(tiles, num_sms);
  ATTNB_CUDA(launch_pdl(gemm_tc_kernel<BN, SPLIT3, BCAST>, dim3(grid), dim3(kThreads), smem, s,
                        a_hi, a_lo, b_hi, b_lo, p.M, p.N, p.Kp, C, ldc, alpha, beta, bias,
                        status, peers));
}

// Output tile width: the widest (256 for 1xTF32, 128 for 3xTF32, whose MMAs
// are already 2*BN wide) that still gives every SM a tile; narrower tiles for
// small products that would otherwise leave most SMs idle.
int pick_bn(int M, int N, bool split3, int num_sms) {
  const int tiles_m = (M + BM - 1) / BM;
  for (int bn = split3 ? 128 : 256; bn > 64; bn /= 2)
    if ((int64_t)tiles_m * ((N + bn - 1) / bn) >= num_sms) return bn;
  return 64;
}

}  // namespace

GemmPlan gemm_plan(int M, int N, int K, int precision) {
  GemmPlan p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.Kp = (K + BK - 1) / BK * BK;
  p.split3 = precision != ATTNB_PREC_TF32;
  // Both operands are always packed: round-to-nearest tf32 (the tensor core
  // would otherwise truncate an fp32 operand read in place, which doubles and
  // biases the 1xTF32 error), K-major, K padded to a multiple of 32.
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t a_bytes = (size_t)M * p.Kp * sizeof(float);
  const size_t b_bytes = (size_t)N * p.Kp * sizeof(float);
  p.off_a_hi = take(a_bytes);
  p.off_a_lo = p.split3 ? take(a_bytes) : 0;
  p.off_b_hi = take(b_bytes);
  p.off_b_lo = p.split3 ? take(b_bytes) : 0;
  p.ws_bytes = off;
  return p;
}

void gemm_run(const GemmPlan& p, const float* A, int64_t lda, bool a_kmajor, const float* B,
              int64_t ldb, bool b_kmajor, float* C, int64_t ldc, float alpha, float beta,
              const float* bias, void* ws, int* status, int num_sms, cudaStream_t s,
              const PeerOut* peers, const float* pre_b_hi, const float* pre_b_lo) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return;
  const bool bcast = peers != nullptr && peers->n > 0;
  const bool prepacked = pre_b_hi != nullptr;
  if (alpha == 0.f && bias == nullptr) {
    if (beta != 1.f) gemm_scale_bias(C, ldc, p.M, p.N, beta, nullptr, num_sms, s);
    if (bcast)  // no product to fuse with: copy the rows to the replicas
      for (int i = 0; i < peers->n; ++i)
        ATTNB_CUDA(cudaMemcpy2DAsync(peers->dst[i], ldc * sizeof(float), C, ldc * sizeof(float),
                                     p.N * sizeof(float), p.M, cudaMemcpyDeviceToDevice, s));
    return;
  }
  // 1xTF32, one 128x64 tile per CTA, aligned rows: the raw operands go
  // straight into the kernel (no packing pass).  3xTF32 stays on the packed
  // path: its split stages (hi and lo of A and B, plus the B staging) leave
  // only three in flight, and the fused form measured no faster there.
  {
    const int tiles64 = ((p.M + BM - 1) / BM) * ((p.N + 63) / 64);
    auto aligned = [](const float* x, int64_t ld) {
      return (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && ld % 4 == 0;
    };
    if (!bcast && !prepacked && !p.split3 && a_kmajor &&
        pick_bn(p.M, p.N, false, num_sms) == 64 &&
        tiles64 <= num_sms && aligned(A, lda) && aligned(B, ldb)) {
      const CUtensorMap ta = make_tmap_2d(A, p.M, p.K, lda, BM, BK);
      const CUtensorMap tb = b_kmajor ? make_tmap_2d(B, p.N, p.K, ldb, 64, BK)
                                      : make_tmap_2d(B, p.K, p.N, ldb, BK, 32);
      ProfScope prof("gemm_tc", s);
      const auto go = [&](auto launch) {
        launch(ta, tb, p.M, p.N, p.K, C, ldc, alpha, beta, bias, status, s);
      };
      if (b_kmajor) go(launch_fused<64, false, true>);
      else go(launch_fused<64, false, false>);
      return;
    }
  }
  char* w = static_cast<char*>(ws);
  float* a_hi = reinterpret_cast<float*>(w + p.off_a_hi);
  float* a_lo = p.split3 ? reinterpret_cast<float*>(w + p.off_a_lo) : nullptr;
  const float* b_hi = prepacked ? pre_b_hi : reinterpret_cast<float*>(w + p.off_b_hi);
  const float* b_lo = prepacked ? pre_b_lo
                                : (p.split3 ? reinterpret_cast<float*>(w + p.off_b_lo) : nullptr);
  // A -> [M, Kp] and B -> [N, Kp], K-major, in one launch (B only when it
  // does not come packed already).
  PackJob jobs[2];
  jobs[0] = a_kmajor ? PackJob{A, 0, lda, 1, 1, p.M, p.K, p.M, p.Kp, false, 1.f, a_hi, a_lo}
                     : PackJob{A, 0, lda, 1, 1, p.K, p.M, p.M, p.Kp, true, 1.f, a_hi, a_lo};
  if (!prepacked) {
    float* bh = const_cast<float*>(b_hi);
    float* bl = const_cast<float*>(b_lo);
    jobs[1] = b_kmajor ? PackJob{B, 0, ldb, 1, 1, p.N, p.K, p.N, p.Kp, false, 1.f, bh, bl}
                       : PackJob{B, 0, ldb, 1, 1, p.K, p.N, p.N, p.Kp, true, 1.f, bh, bl};
  }
  pack_launch(jobs, prepacked ? 1 : 2, p.split3, num_sms, s);
  const int bn = pick_bn(p.M, p.N, p.split3, num_sms);
  const CUtensorMap tA_hi = make_tmap_2d(a_hi, p.M, p.Kp, p.Kp, BM, BK);
  const CUtensorMap tB_hi = make_tmap_2d(b_hi, p.N, p.Kp, p.Kp, bn, BK);
  ProfScope prof("gemm_tc", s);
  const PeerOut none{};
  const PeerOut& po = bcast ? *peers : none;
  // The two forms (plain C, or C plus replicas) share the kernel's template.
  const auto run = [&](auto bcast_tag) {
    constexpr bool BC = decltype(bcast_tag)::value;
    if (p.split3) {
      const CUtensorMap tA_lo = make_tmap_2d(a_lo, p.M, p.Kp, p.Kp, BM, BK);
      const CUtensorMap tB_lo = make_tmap_2d(b_lo, p.N, p.Kp, p.Kp, bn, BK);
      if (bn == 128)
        launch_gemm<128, true, BC>(p, tA_hi, tA_lo, tB_hi, tB_lo, C, ldc, alpha, beta, bias,
                                   status, num_sms, s, po);
      else
        launch_gemm<64, true, BC>(p, tA_hi, tA_lo, tB_hi, tB_lo, C, ldc, alpha, beta, bias,
                                  status, num_sms, s, po);
    } else {
      if (bn == 256)
        launch_gemm<256, false, BC>(p, tA_hi, tA_hi, tB_hi, tB_hi, C, ldc, alpha, beta, bias,
                                    status, num_sms, s, po);
      else if (bn == 128)
        launch_gemm<128, false, BC>(p, tA_hi, tA_hi, tB_hi, tB_hi, C, ldc, alpha, beta, bias,
                                    status, num_sms, s, po);
      else
        launch_gemm<64, false, BC>(p, tA_hi, tA_hi, tB_hi, tB_hi, C, ldc, alpha, beta, bias,
                                   status, num_sms, s, po);
    }
  };
  if (bcast) run(std::true_type{});
  else run(std::false_type{});
}

void gemm_scale_bias(float* C, int64_t ldc, int M, int N, float beta, const float* bias,
                     int num_sms, cudaStream_t s) {
  if (M <= 0 || N <= 0) return;
  const int64_t n = (int64_t)M * N;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms * 8);
  scale_c_kernel<<<blocks, 256, 0, s>>>(C, ldc, M, N, beta, bias);
}

size_t gemm_workspace_bound(int M, int N, int K, int precision) {
  return gemm_plan(M, N, K, precision).ws_bytes;
}

size_t gemm_packed_bytes(int rows, int K, bool split3) {
  const int Kp = (K + BK - 1) / BK * BK;
  const size_t one = ((size_t)rows * Kp * sizeof(float) + 255) & ~size_t(255);
  return split3 ? 2 * one : one;
}

void gemm_pack_b(const float* B, int64_t ldb, bool b_kmajor, int N, int K, bool split3,
                 float* hi, float* lo, int num_sms, cudaStream_t s) {
  const int Kp = (K + BK - 1) / BK * BK;
  const PackJob job = b_kmajor ? PackJob{B, 0, ldb, 1, 1, N, K, N, Kp, false, 1.f, hi, lo}
                               : PackJob{B, 0, ldb, 1, 1, K, N, N, Kp, true, 1.f, hi, lo};
  pack_launch(&job, 1, split3, num_sms, s);
}

}  // namespace attnb
