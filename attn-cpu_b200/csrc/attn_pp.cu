// attn_pp.cu -- K3p: 1xTF32 prefill attention with two query tiles per CTA.
//
// The same function as K3 (attn_tc.cu; reference: the online softmax of
// include/kernels/attn_dhk16_m4_nocausal.h:20-293 and include/online_softmax.h:8-17),
// laid out for long key ranges in 1xTF32:
//
//   CTA = two 128-row query tiles A and B of one head (query tiles 2x, 2x+1).
//   Each K / V^T tile streamed into shared memory serves both, so every byte
//   read from L2 feeds twice the tensor-core work of K3.  Warp 0 streams Q
//   and K, warp 3 V^T, each through its own ring.  The two tiles run as
//   chains, each issued by one thread of its own warp (1 and 2; two threads
//   of one warp would wait in lockstep):
//       S_c(j) = Q_c . K_j^T  ->  softmax_c(j) writes P over S_c  ->  O_c += P . V_j
//   With rings that hold a whole K and V tile (head size <= 96) the two
//   softmaxes take turns, so the tensor core works on one tile's products
//   while the other tile's softmax runs; at head size 128 the rings are
//   shorter than a tile and the chains run in step.  TMEM: S_A, S_B (128
//   columns each), O_A, O_B (<= 128 each).
//   Warps 4-7 (tile A) and 8-11 (tile B) own one query row per thread and hold
//   the whole 128-key row of S in registers: one TMEM load, the row max, the
//   exponentials and one TMEM store per tile, with no exchange between warps.
//
//   O stays in TMEM across key tiles.  The running max m used for P only
//   moves when a tile's row max exceeds it by more than 8 (P <= 2^8); then
//   the row of O and the sum l are rescaled by 2^(m_old - m_new) before the
//   next P.V product.  Both O and l carry the same stale max, so O / l at
//   the end is exact.
//
// Operands come packed by split.cu (Q scaled by log2(e)/sqrt(Dh) and rounded
// to tf32, K, V^T), as for K3's multi-tile form.
#include <algorithm>
#include <atomic>
#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace attnb {
namespace {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // keys per K / V tile
constexpr int BK = 32;   // fp32 elements per 128-byte swizzle row
// Warp 0: Q/K loads, 1-2: MMA chains, 3: V^T loads, 4-11: softmax.  Twelve
// warps keep 168 registers per thread (three warps per SM sub-partition).
constexpr int kPPThreads = 384;
constexpr float kRescaleGap = 8.f;  // log2 of the largest P between rescales

constexpr int clamp_int(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

template <int DHP>
struct PPCfg {
  static constexpr int NKB = DHP / BK;        // 32-wide slices of the head dimension
  static constexpr int QBOX = BM * BK * 4;    // 16 KB: 128 query rows x 32 columns
  static constexpr int KBOX = BN * BK * 4;    // 16 KB: 128 keys x 32 columns
  static constexpr int VBOX = DHP * BK * 4;   // V^T rows for 32 keys
  static constexpr int Q_BYTES = NKB * QBOX;  // one query tile, resident
  static constexpr int BUDGET = 225 * 1024;
  static constexpr int REM = BUDGET - 2 * Q_BYTES;
  static constexpr int K_ST = clamp_int(REM / 2 / KBOX, 2, 8);
  static constexpr int V_ST = clamp_int((REM - K_ST * KBOX) / VBOX, 2, 8);
  static constexpr int OFF_K = 2 * Q_BYTES;
  static constexpr int OFF_V = OFF_K + K_ST * KBOX;
  static constexpr int SMEM = OFF_V + V_ST * VBOX + 1024;
  static constexpr int S_COLS = BN;       // TMEM: S_A at 0, S_B at 128
  static constexpr int O_BASE = 2 * BN;   // O_A at 256, O_B at 384
  static constexpr int O_STRIDE = 128;
  static_assert(DHP % 32 == 0 && DHP <= 128, "head size padded to 32..128");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(OFF_V + V_ST * VBOX <= BUDGET, "rings fit");
};

template <int DHP>
__global__ void __launch_bounds__(kPPThreads, 1)
    attn_pp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                   const AttnPPArgs p) {
  using Cfg = PPCfg<DHP>;
  constexpr int KST = Cfg::K_ST, VST = Cfg::V_ST;
  constexpr uint32_t IDESC_S = idesc_tf32(BM, BN);
  constexpr uint32_t IDESC_PV = idesc_tf32(BM, DHP);

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t kfull[KST], kempty[KST], vfull[VST], vempty[VST];
  __shared__ __align__(8) uint64_t q_bar, s_bar[2], p_bar[2], pv_bar[2], done_bar[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int wg_fail[2];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.z;
  const int qt0 = 2 * blockIdx.x;  // chain c takes query tile qt0 + c
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  const int n_kv = (p.T + BN - 1) / BN;
  // Key tiles of chain c (0 when its query tile lies past L).
  auto tiles_of = [&](int c) {
    const int qt = qt0 + c;
    if (qt * BM >= p.L) return 0;
    if (!p.causal) return n_kv;
    const int last_row = min(p.L, (qt + 1) * BM) - 1;
    return min(n_kv, last_row / BN + 1);
  };
  const int n_tiles[2] = {tiles_of(0), tiles_of(1)};
  const int n_load = max(n_tiles[0], n_tiles[1]);  // the producer streams this many
  auto slices_of = [&](int j) { return min(BN / BK, (p.T - j * BN + BK - 1) / BK); };

  if (threadIdx.x == 0) {
    abort_flag = 0;
    wg_fail[0] = wg_fail[1] = 0;
    // Each ring slot is released by both chains (an MMA commit, or a plain
    // arrival from a chain whose query tile does not need that key tile).
    for (int i = 0; i < KST; ++i) {
      mbar_init(smem_addr(&kfull[i]), 1);
      mbar_init(smem_addr(&kempty[i]), 2);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(smem_addr(&vfull[i]), 1);
      mbar_init(smem_addr(&vempty[i]), 2);
    }
    mbar_init(smem_addr(&q_bar), 1);
    for (int c = 0; c < 2; ++c) {
      mbar_init(smem_addr(&s_bar[c]), 1);
      mbar_init(smem_addr(&p_bar[c]), 4);  // one arrival per softmax warp of the chain
      mbar_init(smem_addr(&pv_bar[c]), 1);
      mbar_init(smem_addr(&done_bar[c]), 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(&tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;
  grid_dep_wait();  // the packed operands come from the packing launch

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ Q and K loads
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      const int nq = n_tiles[1] > 0 ? 2 : 1;
      const uint32_t qb = smem_addr(&q_bar);
      mbar_arrive_expect_tx(qb, nq * Cfg::Q_BYTES);
      for (int c = 0; c < nq; ++c)
        for (int kb = 0; kb < Cfg::NKB; ++kb)
          tma_load_3d(base + c * Cfg::Q_BYTES + kb * Cfg::QBOX, &tmQ, qb, kb * BK,
                      (qt0 + c) * BM, h);
      Ring<KST> rk;
      bool ok = true;
      for (int j = 0; ok && j < n_load; ++j) {
        for (int kb = 0; kb < Cfg::NKB; ++kb) {
          if (!mbar_wait(smem_addr(&kempty[rk.stage]), rk.phase ^ 1u, abort_p, p.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_addr(&kfull[rk.stage]);
          mbar_arrive_expect_tx(fb, Cfg::KBOX);
          tma_load_3d(base + Cfg::OFF_K + rk.stage * Cfg::KBOX, &tmK, fb, kb * BK, j * BN, h);
          rk.note_issue();
          rk.advance();
        }
      }
      // Every copy issued lands before the CTA may exit.
      drain_wait(qb, 0, p.status);
      for (int i = 0; i < KST; ++i)
        if (rk.issued_mask & (1u << i))
          drain_wait(smem_addr(&kfull[i]), (rk.issued_parity >> i) & 1u, p.status);
    }
  } else if (warp == 3) {
    if (lane == 0) {
      // ---------------------------------------------------------- V^T loads
      tma_prefetch_desc(&tmV);
      Ring<VST> rv;
      bool ok = true;
      for (int j = 0; ok && j < n_load; ++j) {
        const int nvb = slices_of(j);
        for (int vb = 0; vb < nvb; ++vb) {
          if (!mbar_wait(smem_addr(&vempty[rv.stage]), rv.phase ^ 1u, abort_p, p.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_addr(&vfull[rv.stage]);
          mbar_arrive_expect_tx(fb, Cfg::VBOX);
          tma_load_3d(base + Cfg::OFF_V + rv.stage * Cfg::VBOX, &tmV, fb, j * BN + vb * BK, 0, h);
          rv.note_issue();
          rv.advance();
        }
      }
      for (int i = 0; i < VST; ++i)
        if (rv.issued_mask & (1u << i))
          drain_wait(smem_addr(&vfull[i]), (rv.issued_parity >> i) & 1u, p.status);
    }
  } else if (warp <= 2) {
    if (lane == 0) {
      // ------------------------------------------------- MMA issuer, chain c
      const int c = warp - 1;
      const int n = n_tiles[c];
      const uint32_t sbuf = tmem + c * Cfg::S_COLS;
      const uint32_t obuf = tmem + Cfg::O_BASE + c * Cfg::O_STRIDE;
      const uint32_t qbase = base + c * Cfg::Q_BYTES;
      Ring<KST> rk;
      Ring<VST> rv;
      bool ok = n == 0 || mbar_wait(smem_addr(&q_bar), 0, abort_p, p.status);
      for (int j = 0; ok && j < n_load; ++j) {
        const bool use = j < n;
        // S_c(j) overwrites P_c(j - 1): it waits until P_c(j - 1) . V is done.
        if (use && j > 0) {
          if (!mbar_wait(smem_addr(&pv_bar[c]), (j - 1) & 1, abort_p, p.status)) break;
          tc_fence_after();
        }
        for (int kb = 0; ok && kb < Cfg::NKB; ++kb) {
          if (!mbar_wait(smem_addr(&kfull[rk.stage]), rk.phase, abort_p, p.status)) {
            ok = false;
            break;
          }
          const uint32_t empty = smem_addr(&kempty[rk.stage]);
          if (use) {
            tc_fence_after();
            const uint32_t ka = base + Cfg::OFF_K + rk.stage * Cfg::KBOX;
            const uint32_t qa = qbase + kb * Cfg::QBOX;
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk)
              mma_tf32(sbuf, sdesc_kmajor_sw128(qa + kk * 32), sdesc_kmajor_sw128(ka + kk * 32),
                       IDESC_S, (kb | kk) != 0 ? 1u : 0u);
            mma_commit(empty);
          } else {
            mbar_arrive(empty);
          }
          rk.advance();
        }
        if (!ok) break;
        if (use) {
          mma_commit(smem_addr(&s_bar[c]));
          if (!mbar_wait(smem_addr(&p_bar[c]), j & 1, abort_p, p.status)) break;
          tc_fence_after();
        }
        const int nvb = slices_of(j);
        for (int vb = 0; ok && vb < nvb; ++vb) {
          if (!mbar_wait(smem_addr(&vfull[rv.stage]), rv.phase, abort_p, p.status)) {
            ok = false;
            break;
          }
          const uint32_t empty = smem_addr(&vempty[rv.stage]);
          if (use) {
            tc_fence_after();
            const uint32_t va = base + Cfg::OFF_V + rv.stage * Cfg::VBOX;
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk)
              mma_tf32_ts(obuf, sbuf + vb * BK + kk * 8, sdesc_kmajor_sw128(va + kk * 32),
                          IDESC_PV, (j | vb | kk) != 0 ? 1u : 0u);
            mma_commit(empty);
          } else {
            mbar_arrive(empty);
          }
          rv.advance();
        }
        if (ok && use) mma_commit(smem_addr(&pv_bar[c]));
      }
      // Every product issued completes before TMEM is released.
      mma_commit(smem_addr(&done_bar[c]));
      drain_wait(smem_addr(&done_bar[c]), 0, p.status);
    }
  } else {
    // ------------------------------------------------ softmax / output, chain c
    const int c = warp >= 8 ? 1 : 0;
    const int quarter = warp & 3;  // TMEM lanes [32 * quarter, +32)
    const int r = quarter * 32 + lane;
    const int qt = qt0 + c;
    const int qrow = qt * BM + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t srow = tmem + lane_off + c * Cfg::S_COLS;
    const uint32_t orow = tmem + lane_off + Cfg::O_BASE + c * Cfg::O_STRIDE;
    const int n = n_tiles[c];
    const int kmax = p.causal ? min(p.T - 1, qrow) : p.T - 1;  // last valid key
    // One thread of the warp waits and the warp follows its result, so the
    // warp-wide TMEM accesses below are always reached by all 32 lanes.
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) {
      int got = 0;
      if (lane == 0) got = mbar_wait(smem_addr(bar), parity, abort_p, p.status) ? 1 : 0;
      return __shfl_sync(0xffffffffu, got, 0) != 0;
    };
    float m = -INFINITY, l = 0.f;
    // One tile of this chain's softmax: S from TMEM, row max, lazy rescale,
    // P (tf32) back over S, then hand P to the MMA thread.
    auto softmax_tile = [&](int j) {
      tc_fence_after();
      uint32_t s[BN];
      tmem_ld32x2(srow, *reinterpret_cast<uint32_t(*)[32]>(s),
                  srow + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
      tmem_ld32x2(srow + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64),
                  srow + 96, *reinterpret_cast<uint32_t(*)[32]>(s + 96));
      const int kb0 = j * BN;
      // Keys past the row's last valid one (the tail of the key range, the
      // causal diagonal) only occur in some tiles: the warp masks them only
      // there.
      if (__any_sync(0xffffffffu, kb0 + BN - 1 > kmax)) {
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (kb0 + i > kmax) s[i] = __float_as_uint(-INFINITY);
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < BN; ++i) mx[i & 1] = fmaxf(mx[i & 1], __uint_as_float(s[i]));
      const float tmax = fmaxf(mx[0], mx[1]);
      const bool need = tmax > m + kRescaleGap;
      const bool rescale = __any_sync(0xffffffffu, need);  // warp-uniform
      float alpha = 1.f;
      if (need) {
        alpha = m == -INFINITY ? 0.f : fast_exp2(m - tmax);
        m = tmax;
      }
      // A row with no valid key yet keeps m = -inf; its P is 0 (not NaN).
      const float m_use = m == -INFINITY ? 0.f : m;
      // P = 2^(s - m), cut to tf32 (low 13 mantissa bits cleared): the tensor
      // core and the row sum l see the same weights, so O / l carries no bias
      // from the cut.
      float ls[2] = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        const uint32_t pt = __float_as_uint(fast_exp2(__uint_as_float(s[i]) - m_use)) & 0xFFFFE000u;
        ls[i & 1] += __uint_as_float(pt);
        s[i] = pt;
      }
      l = l * alpha + (ls[0] + ls[1]);
#pragma unroll
      for (int q = 0; q < BN / 32; ++q)
        tmem_st32(srow + q * 32, *reinterpret_cast<const uint32_t(*)[32]>(s + q * 32));
      if (rescale && j > 0) {
        // O_c holds P.V up to tile j - 1 (complete: S_c(j) was issued after
        // it); the row moves to the new max before P_c(j) . V is added.
#pragma unroll 1
        for (int d = 0; d < DHP; d += 32) {
          uint32_t o[32];
          tmem_ld32(orow + d, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(orow + d, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&p_bar[c]));
    };
    // The two chains take turns at the softmax (tile j: A, then B; then A at
    // j + 1): each runs with the SM's exponent and FMA units to itself while
    // the other chain's products run.  Named barrier 3 passes the turn to B,
    // 4 back to A; both sides count the same tiles, and a warp whose wait
    // failed keeps passing turns (without work) so the other side never
    // waits for a turn that does not come.
    // Taking turns needs rings that hold a whole K and V tile: otherwise a
    // chain's products wait for the other chain's releases and the turns
    // only add waits (head size 128).
    constexpr bool TURNS = Cfg::K_ST >= Cfg::NKB && Cfg::V_ST >= BN / BK;
    const int n_other = TURNS ? n_tiles[1 - c] : 0;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (c == 0 ? (j >= 1 && j - 1 < n_other) : (j < n_other))
        named_bar_sync(c == 0 ? 4 : 3, 256);
      if (ok) ok = warp_wait(&s_bar[c], j & 1);
      if (ok) softmax_tile(j);
      if (c == 0 ? (j < n_other) : (j + 1 < n_other)) named_bar_arrive(c == 0 ? 3 : 4, 256);
    }
    // Output: O_c / l, staged in this chain's (now idle) Q area as 128-row x
    // 32-column boxes with the 128-byte swizzle and written by TMA, or stored
    // row by row when the output view does not allow a tensor map.
    if (ok && n > 0) ok = warp_wait(&pv_bar[c], (n - 1) & 1);
    if (ok && n > 0) {
      tc_fence_after();
      const float inv = 1.f / l;
      uint8_t* qarea = smem_raw + (base - smem_addr(smem_raw)) + c * Cfg::Q_BYTES;
#pragma unroll 1
      for (int d = 0; d < DHP; d += 32) {
        uint32_t o[32];
        tmem_ld32(orow + d, o);
        if (p.o_tma) {
          uint8_t* box = qarea + (d / 32) * Cfg::QBOX;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(box + r * 128 + ((q ^ (r & 7)) << 4)) =
                make_float4(__uint_as_float(o[q * 4]) * inv, __uint_as_float(o[q * 4 + 1]) * inv,
                            __uint_as_float(o[q * 4 + 2]) * inv,
                            __uint_as_float(o[q * 4 + 3]) * inv);
        } else if (qrow < p.L) {
          float* out = p.O + h * p.osH + (int64_t)qrow * p.osT;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (d + i < p.Dh) out[(int64_t)(d + i) * p.osD] = __uint_as_float(o[i]) * inv;
        }
      }
    }
    if (!ok && lane == 0) wg_fail[c] = 1;
    fence_proxy_async_smem();  // staged boxes are read by the TMA store (async proxy)
    named_bar_sync(1 + c, 128);
    if (p.o_tma && n > 0 && wg_fail[c] == 0 && quarter == 0 && lane == 0) {
      const uint32_t qa = base + c * Cfg::Q_BYTES;
#pragma unroll
      for (int bx = 0; bx < DHP / 32; ++bx)
        tma_store_3d(&tmO, qa + bx * Cfg::QBOX, bx * 32, qt * BM, h);
      bulk_commit_group();
      bulk_wait_read_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int DHP>
void launch_pp(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
               const CUtensorMap& o, const AttnPPArgs& a, cudaStream_t s) {
  using Cfg = PPCfg<DHP>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  ATTNB_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    ATTNB_CUDA(cudaFuncSetAttribute(attn_pp_kernel<DHP>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    configured.fetch_or(bit);
  }
  const dim3 grid((a.qtiles + 1) / 2, 1, a.H);
  ATTNB_CUDA(launch_pdl(attn_pp_kernel<DHP>, grid, dim3(kPPThreads), Cfg::SMEM, s, q, k, v, o, a));
}

}  // namespace

void attn_pp_launch(int dhp, const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                    const CUtensorMap& o, const AttnPPArgs& a, cudaStream_t s) {
  switch (dhp) {
    case 32: launch_pp<32>(q, k, v, o, a, s); break;
    case 64: launch_pp<64>(q, k, v, o, a, s); break;
    case 96: launch_pp<96>(q, k, v, o, a, s); break;
    case 128: launch_pp<128>(q, k, v, o, a, s); break;
    default: fail(ATTNB_ERR_RUNTIME, "internal: unsupported padded head size");
  }
}

}  // namespace attnb
