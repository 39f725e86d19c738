// attn_pair.cu -- K3q: 1xTF32 prefill attention on CTA pairs (tcgen05 cta_group::2).
//
// The same function as K3 (attn_tc.cu; reference: the online softmax of
// include/kernels/attn_dhk16_m4_nocausal.h:20-293 and include/online_softmax.h:8-17),
// for long key ranges at head size 128 in 1xTF32:
//
//   A thread-block cluster of two CTAs takes query tiles 2x (rank 0) and
//   2x + 1 (rank 1) of one head.  Rank 0 issues every product for both as
//   one M = 256 tcgen05.mma.cta_group::2: each CTA holds its 128 query rows
//   (A), half of each key tile's K rows and half of each V^T tile's rows (B,
//   split along N), and gets its own rows of S and O in its own TMEM.  So each
//   CTA streams half of K3's K/V bytes per query tile, and the shared memory
//   left beside the resident Q tile holds rings 2.5 key tiles deep.
//   TMEM per CTA: two S buffers (128 columns each) and O (DHP columns): S(j+1)
//   runs while the softmax of tile j does, and P.V(j) accumulates into O.
//
//   Warp 0: TMA loads (Q once, K and V^T halves) into its own CTA's shared
//   memory; the loads of both CTAs count on rank 0's barriers.  Warp 1: TMEM
//   allocation (both CTAs) and, on rank 0, the MMA issuer.  Warps 2-5: one
//   query row per thread, the whole 128-key row of S in registers (as in
//   K3p); P overwrites S in TMEM and is read by the P.V product from there.
//   Rank 0's product commits arrive on both CTAs' barriers at once; the
//   softmax warps of both CTAs arrive on rank 0's P barrier.
//
//   O stays in TMEM; the max m used for P moves only when a row's tile max
//   exceeds it by more than 8, and then O and l are rescaled (K3p's rule).
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

constexpr int BM = 128;    // query rows per CTA
constexpr int BN = 128;    // keys per tile (64 per CTA)
constexpr int BK = 32;     // fp32 elements per 128-byte swizzle row
constexpr int kQThreads = 192;  // warp 0 TMA, warp 1 TMEM / MMA, warps 2-5 softmax
constexpr float kGap = 8.f;     // log2 of the largest P between rescales

// ----------------------------------------------------- cta_group::2 forms
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D (+)= A(smem) . B(smem)^T over the pair: A rows split by CTA, B rows (N) split.
__device__ __forceinline__ void mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// As mma_pair with A read from each CTA's TMEM.
__device__ __forceinline__ void mma_pair_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive once on the barrier at this offset in both CTAs of the pair when the
// products issued so far are done.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(bar),
      "h"((uint16_t)0x3)
      : "memory");
}
// 3-D tiled load into this CTA's shared memory whose bytes count on the
// barrier `bar_cluster` (a shared::cluster address, here rank 0's).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}

constexpr int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

template <int DHP>
struct PairCfg {
  static constexpr int NKB = DHP / BK;          // 32-wide slices of the head dimension
  static constexpr int QBOX = BM * BK * 4;      // 16 KB: 128 query rows x 32 columns
  static constexpr int KBOX = (BN / 2) * BK * 4;  // 8 KB: this CTA's 64 keys x 32 columns
  static constexpr int VBOX = (DHP / 2) * BK * 4;  // this CTA's DHP/2 rows of V^T, 32 keys
  static constexpr int Q_BYTES = NKB * QBOX;
  static constexpr int BUDGET = 225 * 1024;
  static constexpr int REM = BUDGET - Q_BYTES;
  static constexpr int K_ST = clampi(REM / 2 / KBOX, 4, 16);
  static constexpr int V_ST = clampi((REM - K_ST * KBOX) / VBOX, 4, 16);
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + K_ST * KBOX;
  static constexpr int SMEM = OFF_V + V_ST * VBOX + 1024;
  static constexpr int O_COL = 2 * BN;  // TMEM: S0 at 0, S1 at 128, O at 256
  static_assert(DHP % 32 == 0 && DHP <= 128 && (DHP / 2) % 16 == 0, "head size");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(VBOX % 1024 == 0 && KBOX % 1024 == 0, "swizzle atoms stay aligned");
};

template <int DHP>
__global__ void __launch_bounds__(kQThreads, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                     const AttnPPArgs p) {
  using Cfg = PairCfg<DHP>;
  constexpr int KST = Cfg::K_ST, VST = Cfg::V_ST;
  constexpr uint32_t IDESC_S = idesc_tf32(2 * BM, BN);
  constexpr uint32_t IDESC_PV = idesc_tf32(2 * BM, DHP);

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t kfull[KST], kempty[KST], vfull[VST], vempty[VST];
  __shared__ __align__(8) uint64_t q_bar, s_bar[2], p_bar[2], pv_bar, done_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int wg_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 issues the products
  const int qt = blockIdx.x, h = blockIdx.z;
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  const int n = (p.T + BN - 1) / BN;  // key tiles (non-causal)
  auto slices_of = [&](int j) { return min(BN / BK, (p.T - j * BN + BK - 1) / BK); };
  // Rank 0's copy of one of this CTA's barriers.
  auto at0 = [&](uint64_t* bar) { return map_shared_rank(smem_addr(bar), 0); };

  if (threadIdx.x == 0) {
    abort_flag = 0;
    wg_fail = 0;
    for (int i = 0; i < KST; ++i) {
      mbar_init(smem_addr(&kfull[i]), 1);   // rank 0: expect_tx for both halves
      mbar_init(smem_addr(&kempty[i]), 1);  // a product commit (both CTAs)
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(smem_addr(&vfull[i]), 1);
      mbar_init(smem_addr(&vempty[i]), 1);
    }
    mbar_init(smem_addr(&q_bar), 1);
    mbar_init(smem_addr(&s_bar[0]), 1);
    mbar_init(smem_addr(&s_bar[1]), 1);
    // P(j) ready, by the parity of j: a warp may hand over P(j + 1) while
    // another is still on P(j).  Four softmax warps in each CTA.
    mbar_init(smem_addr(&p_bar[0]), 8);
    mbar_init(smem_addr(&p_bar[1]), 8);
    mbar_init(smem_addr(&pv_bar), 1);
    mbar_init(smem_addr(&done_bar), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_addr(&tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers and TMEM exist before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;
  grid_dep_wait();  // the packed operands come from the packing launch

  if (warp == 0) {
    if (lane == 0) {
      // -------------------------------------------------------- TMA loads
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const bool lead = rank == 0;
      const uint32_t qb = at0(&q_bar);
      if (lead) mbar_arrive_expect_tx(smem_addr(&q_bar), 2 * Cfg::Q_BYTES);
      for (int kb = 0; kb < Cfg::NKB; ++kb)
        tma_load_3d_pair(base + kb * Cfg::QBOX, &tmQ, qb, kb * BK, qt * BM, h);
      Ring<KST> rk;
      Ring<VST> rv;
      bool ok = true;
      // K slices of tile j, then its V^T slices: the order the products use them.
      for (int j = 0; ok && j < n; ++j) {
        for (int kb = 0; kb < Cfg::NKB; ++kb) {
          if (!mbar_wait(smem_addr(&kempty[rk.stage]), rk.phase ^ 1u, abort_p, p.status)) {
            ok = false;
            break;
          }
          if (lead) mbar_arrive_expect_tx(smem_addr(&kfull[rk.stage]), 2 * Cfg::KBOX);
          tma_load_3d_pair(base + Cfg::OFF_K + rk.stage * Cfg::KBOX, &tmK, at0(&kfull[rk.stage]),
                           kb * BK, j * BN + (int)rank * (BN / 2), h);
          rk.note_issue();
          rk.advance();
        }
        const int nvb = slices_of(j);
        for (int vb = 0; ok && vb < nvb; ++vb) {
          if (!mbar_wait(smem_addr(&vempty[rv.stage]), rv.phase ^ 1u, abort_p, p.status)) {
            ok = false;
            break;
          }
          if (lead) mbar_arrive_expect_tx(smem_addr(&vfull[rv.stage]), 2 * Cfg::VBOX);
          tma_load_3d_pair(base + Cfg::OFF_V + rv.stage * Cfg::VBOX, &tmV, at0(&vfull[rv.stage]),
                           j * BN + vb * BK, (int)rank * (DHP / 2), h);
          rv.note_issue();
          rv.advance();
        }
      }
      // Copies land before exit: rank 0 sees them on its barriers; the
      // final cluster barrier keeps rank 1 alive until rank 0 has.
      if (lead) {
        drain_wait(smem_addr(&q_bar), 0, p.status);
        for (int i = 0; i < KST; ++i)
          if (rk.issued_mask & (1u << i))
            drain_wait(smem_addr(&kfull[i]), (rk.issued_parity >> i) & 1u, p.status);
        for (int i = 0; i < VST; ++i)
          if (rv.issued_mask & (1u << i))
            drain_wait(smem_addr(&vfull[i]), (rv.issued_parity >> i) & 1u, p.status);
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      // ------------------------------------------ MMA issuer (both CTAs)
      Ring<KST> rk;
      Ring<VST> rv;
      auto issue_s = [&](int j) {
        const uint32_t sbuf = tmem + (j & 1) * BN;
        for (int kb = 0; kb < Cfg::NKB; ++kb) {
          if (!mbar_wait(smem_addr(&kfull[rk.stage]), rk.phase, abort_p, p.status)) return false;
          tc_fence_after();
          const uint32_t ka = base + Cfg::OFF_K + rk.stage * Cfg::KBOX;
          const uint32_t qa = base + kb * Cfg::QBOX;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk)
            mma_pair(sbuf, sdesc_kmajor_sw128(qa + kk * 32), sdesc_kmajor_sw128(ka + kk * 32),
                     IDESC_S, (kb | kk) != 0 ? 1u : 0u);
          commit_pair(smem_addr(&kempty[rk.stage]));
          rk.advance();
        }
        commit_pair(smem_addr(&s_bar[j & 1]));
        return true;
      };
      bool ok = mbar_wait(smem_addr(&q_bar), 0, abort_p, p.status);
      if (ok) ok = issue_s(0);
      if (ok && n > 1) ok = issue_s(1);
      for (int j = 0; ok && j < n; ++j) {
        if (!mbar_wait_cluster(smem_addr(&p_bar[j & 1]), (j >> 1) & 1, abort_p, p.status)) break;
        tc_fence_after();
        const uint32_t sbuf = tmem + (j & 1) * BN;
        const int nvb = slices_of(j);
        for (int vb = 0; ok && vb < nvb; ++vb) {
          if (!mbar_wait(smem_addr(&vfull[rv.stage]), rv.phase, abort_p, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t va = base + Cfg::OFF_V + rv.stage * Cfg::VBOX;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk)
            mma_pair_ts(tmem + Cfg::O_COL, sbuf + vb * BK + kk * 8,
                        sdesc_kmajor_sw128(va + kk * 32), IDESC_PV, (j | vb | kk) != 0 ? 1u : 0u);
          commit_pair(smem_addr(&vempty[rv.stage]));
          rv.advance();
        }
        if (!ok) break;
        commit_pair(smem_addr(&pv_bar));
        // S(j + 2) overwrites P(j): it waits until P(j) . V is done.
        if (j + 2 < n) {
          if (!mbar_wait(smem_addr(&pv_bar), j & 1, abort_p, p.status)) break;
          tc_fence_after();
          if (!issue_s(j + 2)) break;
        }
      }
      // Every product issued completes before TMEM is released.
      commit_pair(smem_addr(&done_bar));
      drain_wait(smem_addr(&done_bar), 0, p.status);
    }
  } else {
    // ---------------------------------------------- softmax / output (warps 2-5)
    const int quarter = warp & 3;  // TMEM lanes [32 * quarter, +32)
    const int r = quarter * 32 + lane;
    const int qrow = qt * BM + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t orow = tmem + lane_off + Cfg::O_COL;
    const int kmax = p.T - 1;
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) {
      int got = 0;
      if (lane == 0) got = mbar_wait(smem_addr(bar), parity, abort_p, p.status) ? 1 : 0;
      return __shfl_sync(0xffffffffu, got, 0) != 0;
    };
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; ok && j < n; ++j) {
      if (!warp_wait(&s_bar[j & 1], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t srow = tmem + lane_off + (j & 1) * BN;
      uint32_t s[BN];
      tmem_ld32x2(srow, *reinterpret_cast<uint32_t(*)[32]>(s), srow + 32,
                  *reinterpret_cast<uint32_t(*)[32]>(s + 32));
      tmem_ld32x2(srow + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64), srow + 96,
                  *reinterpret_cast<uint32_t(*)[32]>(s + 96));
      const int kb0 = j * BN;
      if (__any_sync(0xffffffffu, kb0 + BN - 1 > kmax)) {
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (kb0 + i > kmax) s[i] = __float_as_uint(-INFINITY);
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < BN; ++i) mx[i & 1] = fmaxf(mx[i & 1], __uint_as_float(s[i]));
      const float tmax = fmaxf(mx[0], mx[1]);
      const bool need = tmax > m + kGap;
      const bool rescale = __any_sync(0xffffffffu, need);
      float alpha = 1.f;
      if (need) {
        alpha = m == -INFINITY ? 0.f : fast_exp2(m - tmax);
        m = tmax;
      }
      const float m_use = m == -INFINITY ? 0.f : m;
      // P cut to tf32, so the products and l use the same weights.
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
        // O holds P.V up to tile j - 1 once that product is done.
        if (!warp_wait(&pv_bar, (j - 1) & 1)) {
          ok = false;
        } else {
          tc_fence_after();
#pragma unroll 1
          for (int d = 0; d < DHP; d += 32) {
            uint32_t o[32];
            tmem_ld32(orow + d, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(orow + d, o);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (ok && lane == 0) mbar_arrive_cluster(at0(&p_bar[j & 1]));
    }
    // Output: O / l through this CTA's (idle) Q area and TMA stores, or row
    // by row when the output view does not allow a tensor map.
    if (ok) ok = warp_wait(&done_bar, 0);
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l;
      uint8_t* qarea = smem_raw + (base - smem_addr(smem_raw));
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
    if (!ok && lane == 0) wg_fail = 1;
    fence_proxy_async_smem();
    named_bar_sync(1, 128);
    if (p.o_tma && wg_fail == 0 && qt * BM < p.L && quarter == 2 && lane == 0) {
#pragma unroll
      for (int bx = 0; bx < DHP / 32; ++bx)
        tma_store_3d(&tmO, base + bx * Cfg::QBOX, bx * 32, qt * BM, h);
      bulk_commit_group();
      bulk_wait_read_all();
    }
  }

  // Neither CTA leaves, or releases TMEM, while the other may still use it.
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

template <int DHP>
void launch_pair(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                 const CUtensorMap& o, const AttnPPArgs& a, cudaStream_t s) {
  using Cfg = PairCfg<DHP>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  ATTNB_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    ATTNB_CUDA(cudaFuncSetAttribute(attn_pair_kernel<DHP>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    configured.fetch_or(bit);
  }
  const dim3 grid((a.qtiles + 1) / 2 * 2, 1, a.H);
  ATTNB_CUDA(launch_pdl_cluster(attn_pair_kernel<DHP>, grid, dim3(kQThreads), Cfg::SMEM, s,
                                dim3(2, 1, 1), q, k, v, o, a));
}

}  // namespace

void attn_pair_launch(int dhp, const CUtensorMap& q, const CUtensorMap& k_half,
                      const CUtensorMap& v_half, const CUtensorMap& o, const AttnPPArgs& a,
                      cudaStream_t s) {
  if (dhp != 128) fail(ATTNB_ERR_RUNTIME, "internal: CTA-pair attention needs head size 128");
  launch_pair<128>(q, k_half, v_half, o, a, s);
}

}  // namespace attnb
