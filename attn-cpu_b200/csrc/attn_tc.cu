// attn_tc.cu -- K3: tcgen05 prefill attention (attn::attn_block_dense and the
// attention step of attn::mha_block_dense), 3xTF32 or 1xTF32.
//
// Reference: the flash-style online softmax of
// include/kernels/attn_dhk16_m4_nocausal.h:20-293 (per key block: block max,
// rescale a = exp(m - m_new), weights exp(s - m_new), masked denominators,
// V-FMA, stats update, final 1/l) and the causal per-query kernels
// include/attn_generic_m1.h:7-37 (keys 0..t); exact two-pass form in
// src/attn_block.cpp:104-241.  The same function, tiled for the tensor cores:
//
//   CTA = 128 query rows (one per TMEM lane) of one head, a range of 128-key
//   tiles.  Warp 0 streams, through a shared-memory ring, 32-wide slices of
//   Q and K (S phase) and of V^T (PV phase) with TMA.  Warp 1 issues
//     S  = Q.K^T          into TMEM (3xTF32: big = hi*hi, small = hi*lo + lo*hi)
//     PV = P.V            with P read straight from TMEM (tcgen05.mma A-from-TMEM)
//   Warps 2-5 (thread = query row) read S, keep the running max m and sum l,
//   write P = 2^(s - m) (split hi/lo) over S's TMEM columns, then fold the
//   finished PV tile into an fp32 register accumulator:
//     O = O * 2^(m_old - m_new) + PV.
//   Scores never leave the SM; O is normalised once at the end.  When few
//   (head, query-tile) pairs exist, the key range is split over the CTAs of a
//   thread-block cluster, which combine their (m, l, O) rows through
//   distributed shared memory.
//
// Operands arrive pre-packed by split.cu: Q scaled by log2(e)/sqrt(Dh), head
// size zero-padded to a multiple of 32, V transposed per head (K-major for the
// PV product), each split into tf32 hi + fp32 lo for 3xTF32.  When every CTA
// holds a single key tile and dhp <= 64 (short sequences, where the packing
// launch would cost as much as the attention), four extra warps do that
// conversion from the raw fp32 tensors straight into shared memory instead.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace attnb {
namespace {

constexpr int BM = 128;        // query rows per CTA
constexpr int BN = 128;        // keys per KV tile
constexpr int BK = 32;         // fp32 elements per 128-byte swizzle row
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 softmax (two groups)
// Fused form: two more warps (10 and 11) split the raw V slices as they land,
// off the softmax warps' path.  Twelve warps still leave 168 registers a
// thread (three warps per SM sub-partition, as with ten).
constexpr int kThreadsFused = 384;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxSplits = 8;  // key splits of a query tile: one portable cluster

// QRES: the CTA's Q tile is loaded once and stays in shared memory, and the
// S ring carries K slices only (deeper for the same bytes).  Used by the
// multi-tile 1xTF32 form; 3xTF32 needs the bytes for its lo parts.
template <int DHP, bool SPLIT3, bool QRESIDENT = false>
struct AttnCfg {
  static constexpr bool QRES = QRESIDENT;
  static constexpr int NKB = DHP / BK;       // K slices of the S product
  static constexpr int NPART = SPLIT3 ? 2 : 1;
  static constexpr int QBOX = BM * BK * 4;   // 16 KB
  static constexpr int KBOX = BN * BK * 4;   // 16 KB
  static constexpr int VBOX = DHP * BK * 4;  // 32 keys of V^T
  static constexpr int BUDGET = 225 * 1024;
  // Resident Q: hi slices kb at kb * QBOX, lo slices at (NKB + kb) * QBOX.
  static constexpr int Q_BYTES = QRES ? NPART * NKB * QBOX : 0;
  // Two rings: Q+K (or K) slices for the S product, V^T slices for the PV
  // product, so all of a tile's V slices can be in flight while S and the
  // softmax run.
  static constexpr int S_STAGE = QRES ? NPART * KBOX : NPART * (QBOX + KBOX);
  // S stage: [Q hi |] K hi | K lo [| Q lo], so that K hi and K lo form one
  // 256-row B operand ([Qh.Kh | Qh.Kl] in a single N = 256 MMA).
  static constexpr int OFF_KH = QRES ? 0 : QBOX;
  static constexpr int OFF_KL = OFF_KH + KBOX;
  static constexpr int OFF_QL = QBOX + 2 * KBOX;
  static constexpr int V_STAGE = NPART * VBOX;
  static constexpr int S_STAGES_FIT = (BUDGET - Q_BYTES - 4 * V_STAGE) / S_STAGE;
  static constexpr int S_STAGES = !QRES ? (SPLIT3 ? 2 : 4) : (S_STAGES_FIT < 8 ? S_STAGES_FIT : 8);
  static constexpr int V_STAGES_FIT = (BUDGET - Q_BYTES - S_STAGES * S_STAGE) / V_STAGE;
  static constexpr int V_CAP = QRES ? 8 : 4;
  static constexpr int V_STAGES = V_STAGES_FIT < V_CAP ? V_STAGES_FIT : V_CAP;
  static constexpr int S_RING = Q_BYTES;                          // offset of the S ring
  static constexpr int V_RING = S_RING + S_STAGES * S_STAGE;      // offset of the V ring
  static constexpr int RING_BYTES = V_RING + V_STAGES * V_STAGE;
  static constexpr int SMEM = RING_BYTES + 1024;
  // Fused form: raw V rows of the tile's key slices staged past the rings.
  static constexpr int SMEM_FUSED = RING_BYTES + (BN / BK) * VBOX + 1024;
  // Split merge: the CTAs of a cluster push their unnormalised rows to the
  // CTA that merges them (rows [q * rows_per, ...) to rank q) as [O (DHP
  // floats) | m | l | valid | spare] (OP floats, a multiple of 16 bytes).
  // They land in q's receive area at the start of its Q / S region, idle by
  // then, one block of rows per sending split: at most 127 rows in all.
  static constexpr int OP = DHP + 4;
  static constexpr int RECV_MAX = (BM - 1) * OP * 4;
  // Staging of the rows a CTA sends, at their row positions, behind it.
  static constexpr int STAGE_END = RECV_MAX + BM * OP * 4;
  // TMEM: NBUF S buffers ([big | small] key columns each), then NBUF P.V
  // accumulators ([big | small] head columns).  Two of each when they fit
  // (1xTF32): S(j+1) then runs during the softmax of tile j, and PV(j) is
  // folded into the output during the softmax of tile j+1.
  static constexpr int S_BUF = NPART * BN;
  static constexpr int PV_BUF = NPART * DHP;
  static constexpr int NBUF = 2 * (S_BUF + PV_BUF) <= 512 ? 2 : 1;
  static constexpr int PV_BASE = NBUF * S_BUF;
  static constexpr int S_BIG = 0;  // within an S buffer
  static constexpr int S_SMALL = BN;
  static constexpr int PV_BIG = 0;  // within a P.V accumulator
  static constexpr int PV_SMALL = DHP;
  static constexpr int TMEM_COLS = 512;
  static_assert(DHP % 32 == 0 && DHP <= 128, "head size padded to 32..128");
  static_assert(V_STAGES >= 2 && S_STAGES >= 2, "rings need two stages");
  static_assert(!QRES || !SPLIT3, "resident Q is a 1xTF32 layout");
  static_assert(BM * (DHP + 1) * 4 <= RING_BYTES, "output staging fits the rings");
  static_assert(RECV_MAX <= V_RING, "merge receive area fits the Q / S region");
  static_assert(STAGE_END <= RING_BYTES, "merge staging fits the rings");
  static_assert(NBUF * (S_BUF + PV_BUF) <= TMEM_COLS, "TMEM budget");
};

struct AttnParams {
  int L, T, H, Dh, causal, nsplit, tiles_per_split, qtiles;
  int o_tma;  // the output tile leaves through the tmO tensor map
  float* O;
  int64_t osH, osT, osD;
  // Raw operands for the fused form (the kernel splits them itself).
  const float* q;
  const float* k;
  const float* v;
  int64_t qsH, qsT, qsD, ksH, ksT, ksD, vsH, vsT, vsD;
  float qscale;
  int* status;
};

__device__ __forceinline__ void split4(float4 x, float s, float4& hi, float4& lo) {
  hi = make_float4(tf32_round(x.x * s), tf32_round(x.y * s), tf32_round(x.z * s),
                   tf32_round(x.w * s));
  lo = make_float4(x.x * s - hi.x, x.y * s - hi.y, x.z * s - hi.z, x.w * s - hi.w);
}

// Fused form, S operands: waits for the raw Q and K slices of each S stage
// (TMA-loaded into the hi slots), splits them in place (Q also scaled) and
// releases the stage to the MMA warp.  Run by the 256 threads of warps 2-9,
// `t` = 0..255.  Returns false when a wait gave up.
template <int DHP, bool SPLIT3>
__device__ __forceinline__ bool fused_split_qk(uint8_t* ring, const uint64_t* rbar,
                                               uint64_t* sfull, int t, float qscale,
                                               volatile int* abort_p, int* status) {
  using Cfg = AttnCfg<DHP, SPLIT3>;
  bool good = true;
  for (int kb = 0; kb < Cfg::NKB; ++kb) {
    // Lanes of a warp pass the same __syncwarp whatever their waits returned.
    if (good && !mbar_wait(smem_addr(&rbar[kb]), 0, abort_p, status)) good = false;
    if (!good) {
      __syncwarp();
      continue;
    }
    uint8_t* st = ring + kb * Cfg::S_STAGE;
#pragma unroll
    for (int i = t; i < Cfg::QBOX / 16; i += 256) {
      float4 hi, lo;
      float4* qv = reinterpret_cast<float4*>(st + i * 16);
      float4* kv = reinterpret_cast<float4*>(st + Cfg::OFF_KH + i * 16);
      split4(*qv, qscale, hi, lo);
      *qv = hi;
      if (SPLIT3) *reinterpret_cast<float4*>(st + Cfg::OFF_QL + i * 16) = lo;
      split4(*kv, 1.f, hi, lo);
      *kv = hi;
      if (SPLIT3) *reinterpret_cast<float4*>(st + Cfg::OFF_KL + i * 16) = lo;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if ((t & 31) == 0) mbar_arrive(smem_addr(&sfull[kb]));
  }
  return good;
}

// Fused form, PV operand: splits and transposes raw V slice `vb` (32 keys,
// staged by TMA as DHP/32 boxes of [32 keys x 32 columns], 128-byte swizzle)
// into the K-major V^T slots of V stage vb.  Lane = key: a 16-byte read of
// four columns of its row, four 4-byte writes down the V^T columns; the
// calling warp takes column groups gi = gi0, gi0 + gstep, ...
template <int DHP, bool SPLIT3>
__device__ __forceinline__ void fused_split_v_slice(uint8_t* ring, int vb, int lane, int gi0,
                                                    int gstep) {
  using Cfg = AttnCfg<DHP, SPLIT3>;
  const uint8_t* raw = ring + Cfg::RING_BYTES + vb * Cfg::VBOX;
  uint8_t* st = ring + Cfg::V_RING + vb * Cfg::V_STAGE;
#pragma unroll 4
  for (int gi = gi0; gi < DHP / 4; gi += gstep) {
    const int bx = gi >> 3, c = gi & 7;
    const float4 x =
        *reinterpret_cast<const float4*>(raw + bx * 4096 + lane * 128 + ((c ^ (lane & 7)) << 4));
    float4 hi, lo;
    split4(x, 1.f, hi, lo);
    const float hv[4] = {hi.x, hi.y, hi.z, hi.w};
    const float lv[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = gi * 4 + i;
      const uint32_t off = d * 128 + (((lane >> 2) ^ (d & 7)) << 4) + (lane & 3) * 4;
      *reinterpret_cast<float*>(st + off) = hv[i];
      if (SPLIT3) *reinterpret_cast<float*>(st + Cfg::VBOX + off) = lv[i];
    }
  }
  fence_proxy_async_smem();
}

// FUSED: every CTA owns one key tile, loaded raw by TMA and split in shared
// memory (Q/K by the softmax warps 2-9 before their softmax, V by warp 0).
// Otherwise warp 0 streams pre-packed tiles.
template <int DHP, bool SPLIT3, bool FUSED>
__global__ void __launch_bounds__(FUSED ? kThreadsFused : kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQh, const __grid_constant__ CUtensorMap tmQl,
                   const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                   const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl,
                   const __grid_constant__ CUtensorMap tmO, const AttnParams p) {
  using Cfg = AttnCfg<DHP, SPLIT3, !SPLIT3 && !FUSED>;
  constexpr int SST = Cfg::S_STAGES, VST = Cfg::V_STAGES;
  static_assert(!FUSED || (Cfg::NKB <= SST && BN / BK <= VST && Cfg::SMEM_FUSED <= 227 * 1024),
                "fused form: one stage per slice of the single key tile");
  // 3xTF32 issues two MMAs per K step where three products are needed: the
  // hi.hi and hi.lo products share one MMA of twice the width (their B
  // operands sit next to each other in shared memory, their accumulators next
  // to each other in TMEM), the lo.hi product takes a second one.
  constexpr uint32_t IDESC_S = idesc_tf32(BM, BN);
  constexpr uint32_t IDESC_S2 = idesc_tf32(BM, 2 * BN);
  constexpr uint32_t IDESC_PV = idesc_tf32(BM, DHP);
  constexpr uint32_t IDESC_PV2 = idesc_tf32(BM, 2 * DHP);
  static_assert(Cfg::S_SMALL == Cfg::S_BIG + BN && Cfg::PV_SMALL == Cfg::PV_BIG + DHP,
                "small accumulators follow the big ones");

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t sfull[SST], sempty[SST], vfull[VST], vempty[VST];
  __shared__ __align__(8) uint64_t s_bar[2], p_bar, pv_bar[2], final_bar, recv_bar, q_bar;
  __shared__ __align__(8) uint64_t ready_bar;  // split merge: peers' Q / S regions are idle
  __shared__ __align__(8) uint64_t rbar[FUSED ? 8 : 1];  // fused: raw Q/K (per slice), V slices
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int softmax_failed;  // any softmax thread saw a wait fail

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, split = blockIdx.y, h = blockIdx.z;
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  auto s_addr = [&](int st) { return base + Cfg::S_RING + st * Cfg::S_STAGE; };
  auto v_addr = [&](int st) { return base + Cfg::V_RING + st * Cfg::V_STAGE; };

  // Key tiles of this CTA.
  int n_kv = (p.T + BN - 1) / BN;
  if (p.causal) {
    const int last_row = min(p.L, (qt + 1) * BM) - 1;
    n_kv = min(n_kv, last_row / BN + 1);
  }
  const int j0 = split * p.tiles_per_split;
  const int j1 = min(n_kv, j0 + p.tiles_per_split);

  if (threadIdx.x == 32) {
    // The tensor maps' first use waits for their fetch: start it now (after
    // an L2 flush it is a DRAM round trip ahead of the first tile's).
    tma_prefetch_desc(&tmQh);
    tma_prefetch_desc(&tmKh);
    tma_prefetch_desc(&tmVh);
    if (SPLIT3 && !FUSED) {
      tma_prefetch_desc(&tmQl);
      tma_prefetch_desc(&tmKl);
      tma_prefetch_desc(&tmVl);
    }
  }
  if (threadIdx.x == 0) {
    abort_flag = 0;
    softmax_failed = 0;
    // Full barriers: one TMA arrival with a byte count, or in the fused form
    // (whose stages are each filled once) one arrival per splitting warp.
    for (int i = 0; i < SST; ++i) {
      mbar_init(smem_addr(&sfull[i]), FUSED ? 8 : 1);
      mbar_init(smem_addr(&sempty[i]), 1);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(smem_addr(&vfull[i]), FUSED ? 2 : 1);  // fused: both V-splitting warps
      mbar_init(smem_addr(&vempty[i]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&s_bar[b]), 1);
      mbar_init(smem_addr(&pv_bar[b]), 1);
    }
    mbar_init(smem_addr(&p_bar), 8);  // one arrival per softmax warp
    mbar_init(smem_addr(&final_bar), 1);
    mbar_init(smem_addr(&recv_bar), 1);
    mbar_init(smem_addr(&ready_bar), p.nsplit > 1 ? p.nsplit - 1 : 1);
    mbar_init(smem_addr(&q_bar), 1);
    if (FUSED)
      for (int i = 0; i < 8; ++i) mbar_init(smem_addr(&rbar[i]), 1);
    fence_barrier_init();
    if (p.nsplit > 1) {
      // The other splits' rows of this CTA's share: DHP floats and (m, l,
      // valid, spare) per row from each of them.
      const int rows_per = (BM + p.nsplit - 1) / p.nsplit;
      const int mine = min(rows_per, BM - (int)cluster_ctarank() * rows_per);
      mbar_arrive_expect_tx(smem_addr(&recv_bar), (p.nsplit - 1) * mine * (DHP * 4 + 16));
    }
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
  // Split cluster barrier, first phase: waited on before any access to a
  // peer's barriers or shared memory.  Every thread arrives and waits twice
  // (the second phase ends before the exit).
  if (p.nsplit > 1) cluster_arrive_relaxed();
  grid_dep_wait();  // packed operands (or, fused, the raw ones) come from earlier kernels

  if (warp == 0) {
    if constexpr (FUSED) if (j0 < j1) {
      // ----------------------------------------------- raw loads (fused form)
      // Lane 0 loads the only key tile's Q/K slices into the S stages' hi
      // slots and its V rows (32 keys x 32 columns per box) into the staging
      // area; the softmax warps split Q/K, warps 10-11 split V.
      const int j = j0;
      const int nvb = min(BN / BK, (p.T - j * BN + BK - 1) / BK);
      if (lane == 0) {
        for (int kb = 0; kb < Cfg::NKB; ++kb) {
          const uint32_t rb = smem_addr(&rbar[kb]), sa = s_addr(kb);
          mbar_arrive_expect_tx(rb, Cfg::QBOX + Cfg::KBOX);
          tma_load_3d(sa, &tmQh, rb, kb * BK, qt * BM, h);
          tma_load_3d(sa + Cfg::OFF_KH, &tmKh, rb, kb * BK, j * BN, h);
        }
        for (int vb = 0; vb < nvb; ++vb) {
          const uint32_t rb = smem_addr(&rbar[Cfg::NKB + vb]);
          const uint32_t va = base + Cfg::RING_BYTES + vb * Cfg::VBOX;
          mbar_arrive_expect_tx(rb, Cfg::VBOX);
          for (int bx = 0; bx < DHP / 32; ++bx)
            tma_load_3d(va + bx * 4096, &tmVh, rb, bx * 32, j * BN + vb * BK, h);
        }
      }
      // Every copy lands before the CTA can exit (they are never cancelled).
      if (lane == 0)
        for (int i = 0; i < Cfg::NKB + nvb; ++i) drain_wait(smem_addr(&rbar[i]), 0, p.status);
    }
    if (!FUSED && lane == 0) {
      // ------------------------------------------------------------ producer
      const bool load_q = Cfg::QRES && j0 < j1;
      if (load_q) {
        // The CTA's Q tile, once: hi slices kb at base + kb * QBOX.
        const uint32_t qb = smem_addr(&q_bar);
        mbar_arrive_expect_tx(qb, Cfg::Q_BYTES);
        for (int kb = 0; kb < Cfg::NKB; ++kb)
          tma_load_3d(base + kb * Cfg::QBOX, &tmQh, qb, kb * BK, qt * BM, h);
      }
      Ring<SST> rs;
      Ring<VST> rv;
      bool ok = true;
      for (int j = j0; ok && j < j1; ++j) {
        for (int kb = 0; kb < Cfg::NKB; ++kb) {
          if (!mbar_wait(smem_addr(&sempty[rs.stage]), rs.phase ^ 1u, abort_p, p.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_addr(&sfull[rs.stage]), sa = s_addr(rs.stage);
          mbar_arrive_expect_tx(fb, Cfg::S_STAGE);
          if (!Cfg::QRES) tma_load_3d(sa, &tmQh, fb, kb * BK, qt * BM, h);
          tma_load_3d(sa + Cfg::OFF_KH, &tmKh, fb, kb * BK, j * BN, h);
          if (SPLIT3) {
            tma_load_3d(sa + Cfg::OFF_QL, &tmQl, fb, kb * BK, qt * BM, h);
            tma_load_3d(sa + Cfg::OFF_KL, &tmKl, fb, kb * BK, j * BN, h);
          }
          rs.note_issue();
          rs.advance();
        }
        const int nvb = min(BN / BK, (p.T - j * BN + BK - 1) / BK);
        for (int vb = 0; ok && vb < nvb; ++vb) {
          if (!mbar_wait(smem_addr(&vempty[rv.stage]), rv.phase ^ 1u, abort_p, p.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_addr(&vfull[rv.stage]), va = v_addr(rv.stage);
          mbar_arrive_expect_tx(fb, Cfg::V_STAGE);
          tma_load_3d(va, &tmVh, fb, j * BN + vb * BK, 0, h);
          if (SPLIT3) tma_load_3d(va + Cfg::VBOX, &tmVl, fb, j * BN + vb * BK, 0, h);
          rv.note_issue();
          rv.advance();
        }
      }
      if (load_q) drain_wait(smem_addr(&q_bar), 0, p.status);
      // Copies still in flight (only possible after an abort) land before exit.
      for (int i = 0; i < SST; ++i)
        if (rs.issued_mask & (1u << i))
          drain_wait(smem_addr(&sfull[i]), (rs.issued_parity >> i) & 1u, p.status);
      for (int i = 0; i < VST; ++i)
        if (rv.issued_mask & (1u << i))
          drain_wait(smem_addr(&vfull[i]), (rv.issued_parity >> i) & 1u, p.status);
    }
    if (p.nsplit > 1) {
      cluster_wait_acquire();
      cluster_arrive_relaxed();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      Ring<SST> rs;
      Ring<VST> rv;
      // S(j0 + it) into S buffer it % NBUF.
      bool q_ready = !Cfg::QRES;
      auto issue_s = [&](int it) {
        const uint32_t sbuf = tmem + (it % Cfg::NBUF) * Cfg::S_BUF;
        if (!q_ready) {
          if (!mbar_wait(smem_addr(&q_bar), 0, abort_p, p.status)) return false;
          q_ready = true;
        }
        for (int kb = 0; kb < Cfg::NKB; ++kb) {
          if (!mbar_wait(smem_addr(&sfull[rs.stage]), rs.phase, abort_p, p.status)) return false;
          tc_fence_after();
          const uint32_t sa = s_addr(rs.stage);
          const uint32_t qa = Cfg::QRES ? base + kb * Cfg::QBOX : sa;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;
            const uint64_t qh = sdesc_kmajor_sw128(qa + kk * 32);
            const uint64_t kh = sdesc_kmajor_sw128(sa + Cfg::OFF_KH + kk * 32);
            if (SPLIT3) {
              // [S_BIG | S_SMALL] (+)= Qh . [Kh | Kl]^T, then S_SMALL += Ql . Kh^T.
              const uint64_t ql = sdesc_kmajor_sw128(sa + Cfg::OFF_QL + kk * 32);
              mma_tf32(sbuf + Cfg::S_BIG, qh, kh, IDESC_S2, acc);
              mma_tf32(sbuf + Cfg::S_SMALL, ql, kh, IDESC_S, 1u);
            } else {
              mma_tf32(sbuf + Cfg::S_BIG, qh, kh, IDESC_S, acc);
            }
          }
          mma_commit(smem_addr(&sempty[rs.stage]));
          rs.advance();
        }
        mma_commit(smem_addr(&s_bar[it % Cfg::NBUF]));
        return true;
      };
      // PV(j0 + it) = P . V with P (in S buffer it % NBUF) read from TMEM, into
      // P.V accumulator it % NBUF.
      auto issue_pv = [&](int it) {
        const uint32_t sbuf = tmem + (it % Cfg::NBUF) * Cfg::S_BUF;
        const uint32_t pvbuf = tmem + Cfg::PV_BASE + (it % Cfg::NBUF) * Cfg::PV_BUF;
        const int j = j0 + it;
        const int nvb = min(BN / BK, (p.T - j * BN + BK - 1) / BK);
        for (int vb = 0; vb < nvb; ++vb) {
          if (!mbar_wait(smem_addr(&vfull[rv.stage]), rv.phase, abort_p, p.status)) return false;
          tc_fence_after();
          const uint32_t sa = v_addr(rv.stage);
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const uint32_t acc = (vb | kk) != 0 ? 1u : 0u;
            const uint32_t key = vb * BK + kk * 8;
            const uint64_t vh = sdesc_kmajor_sw128(sa + kk * 32);
            if (SPLIT3) {
              // V^T hi and lo rows are contiguous: one B operand of 2*DHP rows.
              mma_tf32_ts(pvbuf + Cfg::PV_BIG, sbuf + Cfg::S_BIG + key, vh, IDESC_PV2, acc);
              mma_tf32_ts(pvbuf + Cfg::PV_SMALL, sbuf + Cfg::S_SMALL + key, vh, IDESC_PV, 1u);
            } else {
              mma_tf32_ts(pvbuf + Cfg::PV_BIG, sbuf + Cfg::S_BIG + key, vh, IDESC_PV, acc);
            }
          }
          mma_commit(smem_addr(&vempty[rv.stage]));
          rv.advance();
        }
        mma_commit(smem_addr(&pv_bar[it % Cfg::NBUF]));
        return true;
      };
      // Order: S(0); then per tile it: [S(it + 1) into the other buffer once
      // PV(it - 1) has read the P it overwrites]; PV(it) once the softmax has
      // written P(it).  With one buffer, S(it + 1) waits for PV(it) instead.
      const int n = j1 - j0;
      bool ok = n > 0 ? issue_s(0) : true;
      for (int it = 0; ok && it < n; ++it) {
        if (Cfg::NBUF == 2 && it + 1 < n) {
          if (it >= 1 && !mbar_wait(smem_addr(&pv_bar[(it - 1) % 2]), ((it - 1) / 2) & 1,
                                    abort_p, p.status))
            break;
          tc_fence_after();
          if (!issue_s(it + 1)) break;
        }
        if (!mbar_wait(smem_addr(&p_bar), it & 1, abort_p, p.status)) break;
        tc_fence_after();
        if (!issue_pv(it)) break;
        if (Cfg::NBUF == 1 && it + 1 < n) {
          if (!mbar_wait(smem_addr(&pv_bar[0]), it & 1, abort_p, p.status)) break;
          tc_fence_after();
          if (!issue_s(it + 1)) break;
        }
      }
      mma_commit(smem_addr(&final_bar));
      drain_wait(smem_addr(&final_bar), 0, p.status);
    }
    if (p.nsplit > 1) {
      cluster_wait_acquire();
      cluster_arrive_relaxed();
    }
  } else if (FUSED && warp >= 10) {
    // ------------------------------------------- V split (fused form, 2 warps)
    // Each raw V slice, as it lands, is split and transposed into its V^T
    // stage by both warps (alternate column groups); each warp's lane 0
    // arrives on the stage's full barrier.
    if (j0 < j1) {
      uint8_t* ring = smem_raw + (base - smem_addr(smem_raw));
      const int nvb = min(BN / BK, (p.T - j0 * BN + BK - 1) / BK);
      bool conv = true;
      for (int vb = 0; vb < nvb; ++vb) {
        if (conv && !mbar_wait(smem_addr(&rbar[Cfg::NKB + vb]), 0, abort_p, p.status))
          conv = false;
        if (conv) fused_split_v_slice<DHP, SPLIT3>(ring, vb, lane, warp - 10, 2);
        __syncwarp();
        if (conv && lane == 0) mbar_arrive(smem_addr(&vfull[vb]));
      }
    }
    if (p.nsplit > 1) {
      cluster_wait_acquire();
      cluster_arrive_relaxed();
    }
  } else {
    // ------------------------------------------------ softmax / output (8 warps)
    // Two warpgroups share every query row (TMEM lane): group g (warps 2-5:
    // g = 0, warps 6-9: g = 1) takes key columns [64g, 64g + 64) of each S
    // tile and output chunks [c_lo, c_hi) of the head dimension.  The row max
    // is exchanged through shared memory once per tile; the row sums are kept
    // per group and added at the end.
    const int g = warp >= 6 ? 1 : 0;
    const int sw = warp - 2;       // softmax warp 0..7
    const int quarter = warp & 3;  // TMEM lanes [32 * quarter, +32)
    const int r = quarter * 32 + lane;
    const int qrow = qt * BM + r;
    const bool leader = sw == 0 && lane == 0;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    constexpr int NCH = DHP / 32;       // 32-column chunks of the output row
    constexpr int CH0 = (NCH + 1) / 2;  // chunks of group 0 (group 1: the rest)
    constexpr int SCOLS = BN / 2;       // S columns per group
    const int c_lo = g ? CH0 : 0, c_hi = g ? NCH : CH0;
    uint8_t* ring = smem_raw + (base - smem_addr(smem_raw));
    __shared__ float red[2][BM];        // per-group row values being exchanged
    __shared__ int fail_slot[2];        // failures, by the parity of the tile they stop
    if (threadIdx.x == 64) fail_slot[0] = fail_slot[1] = 0;
    named_bar_sync(1, 256);
    float m = -INFINITY, l = 0.f;
    float o[CH0 * 32];
#pragma unroll
    for (int d = 0; d < CH0 * 32; ++d) o[d] = 0.f;
    // Every thread runs the same number of loop iterations and passes the
    // same barriers: a failed wait is recorded (sticky) and acted on by all
    // threads together at the next per-tile exchange.
    auto record_fail = [&](int slot) {
      fail_slot[slot & 1] = 1;
      softmax_failed = 1;
    };
    if constexpr (FUSED) if (j0 < j1) {
      bool conv = fused_split_qk<DHP, SPLIT3>(ring, rbar, sfull, threadIdx.x - 64, p.qscale,
                                              abort_p, p.status);
      if (!conv) record_fail(0);
    }
    // TMEM accesses: every wait covers two W-column loads -- the big and
    // small halves of a 3xTF32 value, or two neighbouring 1xTF32 column
    // blocks -- so few load latencies are exposed per tile.  W = 16 where the
    // output row already takes 64 registers (head size > 64).
    constexpr int W = DHP > 64 ? 16 : 32;
    constexpr int SSTEP = SPLIT3 ? W : 2 * W;  // S columns per wait
    static_assert(SCOLS % SSTEP == 0, "S columns per group");
    // Scores kept in registers between the two passes: in the fused form,
    // whose single tile leaves the output row zero (no registers) until the
    // P.V product is folded in.  Elsewhere the registers would spill.
    constexpr bool KEEP = FUSED;
    // The P.V drain updates the output row in place: 16-column loads once
    // that row takes 64 registers.
    constexpr int WD = DHP > 64 ? 16 : 32;
    constexpr int DSTEP = SPLIT3 ? WD : 2 * WD;  // output columns per wait
    // Folds P.V of tile t (accumulator t % NBUF) into o with its rescale factor
    // (o <- o * a + PV); false when the wait gave up.
    auto drain_pv = [&](int t, float a) {
      if (!mbar_wait(smem_addr(&pv_bar[t % Cfg::NBUF]), (t / Cfg::NBUF) & 1, abort_p, p.status))
        return false;
      tc_fence_after();
      const uint32_t pvb = tmem + lane_off + Cfg::PV_BASE + (t % Cfg::NBUF) * Cfg::PV_BUF;
      const int ncols = (c_hi - c_lo) * 32;  // this group's output columns
#pragma unroll
      for (int c0 = 0; c0 < CH0 * 32; c0 += DSTEP) {
        if (c0 >= ncols) break;
        const uint32_t col = c_lo * 32 + c0;
        uint32_t va[WD], vb[WD];
        if (SPLIT3) {
          tmem_ld_pair<WD>(pvb + Cfg::PV_BIG + col, va, pvb + Cfg::PV_SMALL + col, vb);
#pragma unroll
          for (int i = 0; i < WD; ++i)
            o[c0 + i] = fmaf(o[c0 + i], a, __uint_as_float(va[i]) + __uint_as_float(vb[i]));
        } else if (c0 + 2 * WD <= ncols) {
          tmem_ld_pair<WD>(pvb + col, va, pvb + col + WD, vb);
#pragma unroll
          for (int i = 0; i < WD; ++i) {
            o[c0 + i] = fmaf(o[c0 + i], a, __uint_as_float(va[i]));
            o[c0 + WD + i] = fmaf(o[c0 + WD + i], a, __uint_as_float(vb[i]));
          }
        } else {
          tmem_ld_one<WD>(pvb + col, va);
#pragma unroll
          for (int i = 0; i < WD; ++i) o[c0 + i] = fmaf(o[c0 + i], a, __uint_as_float(va[i]));
        }
      }
      tc_fence_before();
      return true;
    };
    // With two accumulators, PV(t) is folded in during tile t + 1, after P(t + 1)
    // has been handed over, so it overlaps the tensor core's next products.
    constexpr bool DEFER = Cfg::NBUF == 2;
    float alpha_prev = 1.f;
    bool pending = false;  // a P.V tile not yet folded into o
    int it = 0;
    // The fused form holds a single key tile: one iteration, which the
    // compiler can see (the output row is then still zero during the softmax
    // and takes no registers there).
    const int j_end = FUSED ? j0 + 1 : j1;
    for (int j = j0; j < j_end; ++j, ++it) {
      const uint32_t sbuf = tmem + lane_off + (it % Cfg::NBUF) * Cfg::S_BUF;
      const bool got_s =
          mbar_wait(smem_addr(&s_bar[it % Cfg::NBUF]), (it / Cfg::NBUF) & 1, abort_p, p.status);
      const int kbase = j * BN + g * SCOLS;
      const int kmax = p.causal ? min(p.T - 1, qrow) : p.T - 1;  // last valid key
      // Scores of this thread's row and columns, key c0 + i of a step in
      // va[i] (+ vb[i] for 3xTF32) or, for 1xTF32, keys c0 + i and c0 + W + i.
      // Both passes read them from TMEM; the steps stay rolled so one step's
      // registers are free before the next step loads.
      auto load_s = [&](int c0, uint32_t (&va)[W], uint32_t (&vb)[W]) {
        const uint32_t col = g * SCOLS + c0;
        if (SPLIT3)
          tmem_ld_pair<W>(sbuf + Cfg::S_BIG + col, va, sbuf + Cfg::S_SMALL + col, vb);
        else
          tmem_ld_pair<W>(sbuf + Cfg::S_BIG + col, va, sbuf + Cfg::S_BIG + col + W, vb);
      };
      // Every key of this thread's columns is valid: no masking in this tile.
      const bool full = kbase + SCOLS - 1 <= kmax;
      // Head sizes up to 64: the thread's scores (sv[e] is key kbase + e) stay
      // in registers from the max pass to the exponent pass.
      float sv[KEEP ? SCOLS : 1];
      float tmax = -INFINITY;
      if (got_s) {
        tc_fence_after();
        if constexpr (KEEP) {
#pragma unroll
          for (int c0 = 0; c0 < SCOLS; c0 += SSTEP) {
            uint32_t va[W], vb[W];
            load_s(c0, va, vb);
#pragma unroll
            for (int i = 0; i < W; ++i) {
              if (SPLIT3) {
                sv[c0 + i] = __uint_as_float(va[i]) + __uint_as_float(vb[i]);
              } else {
                sv[c0 + i] = __uint_as_float(va[i]);
                sv[c0 + W + i] = __uint_as_float(vb[i]);
              }
            }
          }
          if (full) {
#pragma unroll
            for (int e = 0; e < SCOLS; ++e) tmax = fmaxf(tmax, sv[e]);
          } else {
#pragma unroll
            for (int e = 0; e < SCOLS; ++e)
              if (kbase + e <= kmax) tmax = fmaxf(tmax, sv[e]);
          }
        } else {
#pragma unroll 1
          for (int c0 = 0; c0 < SCOLS; c0 += SSTEP) {
            uint32_t va[W], vb[W];
            load_s(c0, va, vb);
#pragma unroll
            for (int i = 0; i < W; ++i) {
              if (SPLIT3) {
                const float v = __uint_as_float(va[i]) + __uint_as_float(vb[i]);
                if (kbase + c0 + i <= kmax) tmax = fmaxf(tmax, v);
              } else {
                const float v0 = __uint_as_float(va[i]), v1 = __uint_as_float(vb[i]);
                if (kbase + c0 + i <= kmax) tmax = fmaxf(tmax, v0);
                if (kbase + c0 + W + i <= kmax) tmax = fmaxf(tmax, v1);
              }
            }
          }
        }
      } else {
        record_fail(it);
      }
      red[g][r] = tmax;
      named_bar_sync(1, 256);
      if (fail_slot[it & 1]) break;  // the same decision in every thread
      tmax = fmaxf(tmax, red[g ^ 1][r]);
      const float m_new = fmaxf(m, tmax);
      float lsum = 0.f;
      // P = 2^(s - m_new) (0 past the last valid key), split into tf32 hi and
      // the fp32 remainder for 3xTF32.
      auto p_of = [&](float v, int key, float& lo) {
        const float pv = (full || key <= kmax) ? fast_exp2(v - m_new) : 0.f;
        lsum += pv;
        const float hi = tf32_round(pv);
        lo = pv - hi;
        return hi;
      };
      // One step: P of columns c0.. into TMEM, from the scores in va / vb
      // (or, KEEP, in sv).
      auto p_step = [&](int c0, uint32_t (&va)[W], uint32_t (&vb)[W]) {
        const uint32_t col = g * SCOLS + c0;
#pragma unroll
        for (int i = 0; i < W; ++i) {
          float lo;
          if (SPLIT3) {
            const float v =
                KEEP ? sv[KEEP ? c0 + i : 0] : __uint_as_float(va[i]) + __uint_as_float(vb[i]);
            va[i] = __float_as_uint(p_of(v, kbase + c0 + i, lo));
            vb[i] = __float_as_uint(lo);
          } else {
            const float v0 = KEEP ? sv[KEEP ? c0 + i : 0] : __uint_as_float(va[i]);
            const float v1 = KEEP ? sv[KEEP ? c0 + W + i : 0] : __uint_as_float(vb[i]);
            va[i] = __float_as_uint(p_of(v0, kbase + c0 + i, lo));
            vb[i] = __float_as_uint(p_of(v1, kbase + c0 + W + i, lo));
          }
        }
        if (SPLIT3) {
          tmem_st_w<W>(sbuf + Cfg::S_BIG + col, va);
          tmem_st_w<W>(sbuf + Cfg::S_SMALL + col, vb);
        } else {
          tmem_st_w<W>(sbuf + Cfg::S_BIG + col, va);
          tmem_st_w<W>(sbuf + Cfg::S_BIG + col + W, vb);
        }
      };
      if constexpr (KEEP) {
#pragma unroll
        for (int c0 = 0; c0 < SCOLS; c0 += SSTEP) {
          uint32_t va[W], vb[W];
          p_step(c0, va, vb);
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < SCOLS; c0 += SSTEP) {
          uint32_t va[W], vb[W];
          load_s(c0, va, vb);
          p_step(c0, va, vb);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&p_bar));
      const float alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
      l = l * alpha + lsum;
      m = m_new;
      // o holds the P.V tiles up to it - 2 (DEFER) or it - 1, relative to the
      // running max of that tile; alpha_prev / alpha bring it to the next.
      if (DEFER && pending && !drain_pv(it - 1, alpha_prev)) {
        record_fail(it + 1);  // acted on at the next exchange (or after the loop)
        pending = false;
        continue;
      }
      if (DEFER) {
        alpha_prev = alpha;
        pending = true;
      } else if (!drain_pv(it, alpha)) {
        record_fail(it + 1);
      }
    }
    // The last P.V tile of the deferred schedule (only on the normal exit).
    if (DEFER && pending && it == j1 - j0 && !drain_pv(it - 1, alpha_prev)) softmax_failed = 1;
    // Rows are owned one per thread pair, so the output tile is staged in the
    // (now idle) shared-memory rings and written with TMA stores (or row by
    // row when the output view does not allow TMA); split tiles are staged
    // there for the cluster merge instead.
    // Wait results can differ between threads after an abort; every branch
    // below that holds a barrier of the softmax warps is taken on a decision
    // they share.
    auto all_ok = [&](bool mine) {
      if (!mine) softmax_failed = 1;
      named_bar_sync(1, 256);
      return softmax_failed == 0;
    };
    bool ok = all_ok(true);
    // Row sum over both groups (m is already common).
    red[g][r] = l;
    named_bar_sync(1, 256);
    l += red[g ^ 1][r];
    if (p.nsplit > 1) {
      // ---------------------------------------------------- split merge
      // Row r of the tile is merged by cluster rank q = r / rows_per.  Each
      // split stages the rows other ranks merge (this group's columns; group
      // 0 adds m, l and its validity) at their row positions past the receive
      // area, and one thread bulk-copies each rank's block of rows into that
      // rank's receive area (bytes counted on its recv_bar) once every rank
      // has reported its Q / S region idle.  The threads of rank q holding
      // row r then combine it with the received rows -- the online-softmax
      // merge m* = max m_s, O = sum 2^(m_s - m*) O_s, l likewise -- and store
      // it.  Nothing is stored for a row when any split reported a failure.
      const int ns = p.nsplit;
      const int me = (int)cluster_ctarank();
      const int rows_per = (BM + ns - 1) / ns;
      const int q = r / rows_per;
      float* stage = reinterpret_cast<float*>(ring + Cfg::RECV_MAX);
      if (q != me) {
        float* srow = stage + r * Cfg::OP;
#pragma unroll
        for (int c = 0; c < CH0; ++c) {
          if (c_lo + c >= c_hi) break;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(srow + (c_lo + c) * 32 + i * 4) =
                make_float4(o[c * 32 + i * 4], o[c * 32 + i * 4 + 1], o[c * 32 + i * 4 + 2],
                            o[c * 32 + i * 4 + 3]);
        }
        if (g == 0)
          *reinterpret_cast<float4*>(srow + DHP) = make_float4(m, l, ok ? 1.f : 0.f, 0.f);
        fence_proxy_async_smem();  // the rows leave by bulk copies (async proxy)
      }
      cluster_wait_acquire();  // the peers' barriers are initialised
      // Every S product of this CTA has completed (the tile loop ran to its
      // end), so nothing reads the Q / S region any more.
      if (leader && it == j1 - j0)
        for (int t = 0; t < ns; ++t)
          if (t != me) mbar_arrive_remote(map_shared_rank(smem_addr(&ready_bar), t));
      named_bar_sync(1, 256);  // every staged row is written
      if (threadIdx.x == 64 && mbar_wait_cluster(smem_addr(&ready_bar), 0, abort_p, p.status)) {
        for (int t = 0; t < ns; ++t) {
          if (t == me) continue;
          const int k = me < t ? me : me - 1;  // this split's block in t's receive area
          const int trows = min(rows_per, BM - t * rows_per);
          bulk_copy_to_peer(map_shared_rank(base + k * rows_per * Cfg::OP * 4, t),
                            base + Cfg::RECV_MAX + t * rows_per * Cfg::OP * 4,
                            trows * Cfg::OP * 4, map_shared_rank(smem_addr(&recv_bar), t));
        }
      }
      // The rows this CTA merges have all landed (or, after a failure, every
      // copy that was issued has), so the other ranks' staging is free when
      // the second phase ends.
      bool got = true;
      if (q == me) {
        got = mbar_wait_cluster(smem_addr(&recv_bar), 0, abort_p, p.status);
        if (!got) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait_cluster(smem_addr(&recv_bar), 0) &&
                 globaltimer() - t0 < ATTNB_WAIT_LIMIT_NS) {
          }
        }
      }
      cluster_arrive_relaxed();
      if (q == me) {
        const int lr = r - me * rows_per;
        const float* recv = reinterpret_cast<const float*>(ring);
        // Compact loops: this code runs once per CTA, so its instruction
        // fetches are on the critical path.
        bool valid = got && ok;
        float mstar = m;
#pragma unroll 1
        for (int t = 0; t < ns - 1; ++t) {
          const float* row = recv + (t * rows_per + lr) * Cfg::OP;
          valid = valid && row[DHP + 2] != 0.f;
          mstar = fmaxf(mstar, row[DHP]);
        }
        const int qrow = qt * BM + r;
        if (valid && qrow < p.L) {
          // This row's merged values of this group's columns, written over o.
          const float wme = m == -INFINITY ? 0.f : fast_exp2(m - mstar);
          float lsum = wme * l;
#pragma unroll
          for (int e = 0; e < CH0 * 32; ++e) o[e] *= wme;
#pragma unroll 1
          for (int t = 0; t < ns - 1; ++t) {
            const float* row = recv + (t * rows_per + lr) * Cfg::OP;
            const float w = row[DHP] == -INFINITY ? 0.f : fast_exp2(row[DHP] - mstar);
            lsum = fmaf(w, row[DHP + 1], lsum);
#pragma unroll
            for (int c = 0; c < CH0; ++c) {
              if (c_lo + c >= c_hi) break;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float4 v = *reinterpret_cast<const float4*>(row + (c_lo + c) * 32 + i * 4);
                o[c * 32 + i * 4] = fmaf(w, v.x, o[c * 32 + i * 4]);
                o[c * 32 + i * 4 + 1] = fmaf(w, v.y, o[c * 32 + i * 4 + 1]);
                o[c * 32 + i * 4 + 2] = fmaf(w, v.z, o[c * 32 + i * 4 + 2]);
                o[c * 32 + i * 4 + 3] = fmaf(w, v.w, o[c * 32 + i * 4 + 3]);
              }
            }
          }
          const float inv = 1.f / lsum;
          const bool vec = p.osD == 1 && (p.osT & 3) == 0 && (p.osH & 3) == 0 &&
                           (reinterpret_cast<uintptr_t>(p.O) & 15u) == 0 &&
                           c_hi * 32 <= p.Dh;
          float* orow = p.O + h * p.osH + (int64_t)qrow * p.osT;
          if (vec) {
#pragma unroll
            for (int c = 0; c < CH0; ++c) {
              if (c_lo + c >= c_hi) break;
#pragma unroll
              for (int i = 0; i < 8; ++i)
                *reinterpret_cast<float4*>(orow + (c_lo + c) * 32 + i * 4) =
                    make_float4(o[c * 32 + i * 4] * inv, o[c * 32 + i * 4 + 1] * inv,
                                o[c * 32 + i * 4 + 2] * inv, o[c * 32 + i * 4 + 3] * inv);
            }
          } else {
#pragma unroll
            for (int c = 0; c < CH0; ++c) {
              if (c_lo + c >= c_hi) break;
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int d = (c_lo + c) * 32 + i;
                if (d < p.Dh) orow[(int64_t)d * p.osD] = o[c * 32 + i] * inv;
              }
            }
          }
        }
      }
    }
    const bool write_out = (p.nsplit == 1) && ok;
    if (write_out) {
      const float inv = 1.f / l;
      if (p.o_tma) {
        // DHP/32 boxes of [128 rows x 32 columns], 128-byte swizzled, each
        // thread writing its row of its group's boxes as 16-byte chunks.
#pragma unroll
        for (int c = 0; c < CH0; ++c) {
          if (c_lo + c >= c_hi) break;
          uint8_t* box = ring + (c_lo + c) * (BM * 128);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int d = c * 32 + q * 4;
            *reinterpret_cast<float4*>(box + r * 128 + ((q ^ (r & 7)) << 4)) =
                make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(1, 256);
        if (leader) {
#pragma unroll
          for (int bx = 0; bx < NCH; ++bx)
            tma_store_3d(&tmO, base + bx * (BM * 128), bx * 32, qt * BM, h);
          bulk_commit_group();
          bulk_wait_read_all();
        }
      } else {
        // Stage the normalised tile (row stride DHP + 1: conflict-free column
        // writes), then write each row with a warp's lanes along the row.
        float* stile = reinterpret_cast<float*>(ring);
#pragma unroll
        for (int c = 0; c < CH0; ++c) {
          if (c_lo + c >= c_hi) break;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            stile[r * (DHP + 1) + (c_lo + c) * 32 + i] = o[c * 32 + i] * inv;
        }
        named_bar_sync(1, 256);
        const int rows = min(BM, p.L - qt * BM);
        float* obase = p.O + h * p.osH + (int64_t)qt * BM * p.osT;
#pragma unroll 4
        for (int rr = sw; rr < rows; rr += 8) {
          float* orow = obase + (int64_t)rr * p.osT;
#pragma unroll
          for (int dd = 0; dd < DHP; dd += 32)
            if (dd + lane < p.Dh) orow[(dd + lane) * p.osD] = stile[rr * (DHP + 1) + dd + lane];
        }
      }
    }
  }

  // Second phase of the split cluster barrier: every CTA's incoming copies
  // have landed (or been waited for after a failure), so no copy still reads
  // this CTA's staging or writes its receive area when it exits.
  if (p.nsplit > 1) cluster_wait_acquire();

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int DHP, bool SPLIT3, bool FUSED>
void launch_attn(const CUtensorMap* maps, const AttnParams& prm, int qtiles, cudaStream_t s) {
  using Cfg = AttnCfg<DHP, SPLIT3, !SPLIT3 && !FUSED>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  ATTNB_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    ATTNB_CUDA(cudaFuncSetAttribute(attn_tc_kernel<DHP, SPLIT3, FUSED>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    FUSED ? Cfg::SMEM_FUSED : Cfg::SMEM));
    configured.fetch_or(bit);
  }
  constexpr int smem = FUSED ? Cfg::SMEM_FUSED : Cfg::SMEM;
  const dim3 grid(qtiles, prm.nsplit, prm.H);
  if (prm.nsplit > 1) {
    // The key splits of a (head, query tile) form one cluster (merge through
    // distributed shared memory).
    ATTNB_CUDA(launch_pdl_cluster(attn_tc_kernel<DHP, SPLIT3, FUSED>, grid,
                                  dim3(FUSED ? kThreadsFused : kThreads), smem,
                                  s, dim3(1, prm.nsplit, 1), maps[0], maps[1], maps[2], maps[3],
                                  maps[4], maps[5], maps[6], prm));
  } else {
    ATTNB_CUDA(launch_pdl(attn_tc_kernel<DHP, SPLIT3, FUSED>, grid,
                          dim3(FUSED ? kThreadsFused : kThreads), smem, s,
                          maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], maps[6], prm));
  }
}

template <bool SPLIT3>
void dispatch_dhp(int dhp, bool fused, const CUtensorMap* maps, const AttnParams& prm,
                  int qtiles, cudaStream_t s) {
  if (fused) {
    switch (dhp) {
      case 32: launch_attn<32, SPLIT3, true>(maps, prm, qtiles, s); break;
      case 64: launch_attn<64, SPLIT3, true>(maps, prm, qtiles, s); break;
      default: fail(ATTNB_ERR_RUNTIME, "internal: fused form needs dhp <= 64");
    }
    return;
  }
  switch (dhp) {
    case 32: launch_attn<32, SPLIT3, false>(maps, prm, qtiles, s); break;
    case 64: launch_attn<64, SPLIT3, false>(maps, prm, qtiles, s); break;
    case 96: launch_attn<96, SPLIT3, false>(maps, prm, qtiles, s); break;
    case 128: launch_attn<128, SPLIT3, false>(maps, prm, qtiles, s); break;
    default: fail(ATTNB_ERR_RUNTIME, "internal: unsupported padded head size");
  }
}

}  // namespace

bool attn_tc_supported(int Dh) { return Dh >= 1 && Dh <= 128; }

AttnTcPlan attn_tc_plan(int H, int L, int T, int Dh, bool causal, int precision, int num_sms) {
  AttnTcPlan p{};
  p.H = H;
  p.L = L;
  p.T = T;
  p.Dh = Dh;
  p.dhp = (Dh + 31) / 32 * 32;
  p.tp = (T + 3) / 4 * 4;
  p.split3 = precision != ATTNB_PREC_TF32;
  p.qtiles = (L + BM - 1) / BM;
  const int n_kv = (T + BN - 1) / BN;
  // Split the key range when (head, query tile) pairs cannot fill the GPU.
  const int pairs = H * p.qtiles;
  int ns = 1;
  if (!causal && pairs < num_sms) ns = std::min(n_kv, std::max(1, num_sms / pairs));
  // The splits of a tile form one thread-block cluster (at most 8 portable).
  ns = std::min(ns, kMaxSplits);
  p.tiles_per_split = (n_kv + ns - 1) / ns;
  p.nsplit = (n_kv + p.tiles_per_split - 1) / p.tiles_per_split;
  p.fusable = p.tiles_per_split == 1 && p.dhp <= 64;
  static const bool pairs_on = [] {
    const char* e = std::getenv("ATTNB_ATTN_PAIRS");
    return !(e && std::strcmp(e, "0") == 0);
  }();
  // K3p takes about 1.5x K3's time per key tile (it serves two query tiles),
  // measured at head sizes 32-128; both hold one CTA per SM.  It pays when it
  // needs fewer waves of CTAs by more than that: e.g. 160 (head, query tile)
  // pairs take two waves of K3 and one of K3p, 128 pairs one wave of either.
  const int waves_k3 = (pairs + num_sms - 1) / num_sms;
  const int waves_pp = (H * ((p.qtiles + 1) / 2) + num_sms - 1) / num_sms;
  p.pairs = pairs_on && !p.split3 && p.nsplit == 1 && p.qtiles >= 2 && n_kv >= 2 &&
            waves_pp * 1.45 < waves_k3;
  static const bool cta_pairs_on = [] {
    const char* e = std::getenv("ATTNB_ATTN_CTA_PAIRS");
    return !(e && std::strcmp(e, "0") == 0);
  }();
  // K3q runs a key tile per CTA in about 4.8 K cycles (one query tile per
  // CTA); K3p in 9.0 K (two), K3 in 7.0 K (one), measured at head size 128 on
  // full waves.  K3q is taken when its waves of CTAs, so weighted, beat the
  // other two by 10 % or more, it fills at least one wave, and the key range
  // is long (eight tiles or more): with fewer CTAs or fewer tiles it
  // measured slower than the per-tile figure says.
  if (!p.split3 && !causal && p.nsplit == 1 && p.qtiles >= 2 && n_kv >= 8 && p.dhp == 128) {
    const int ctas_q = H * ((p.qtiles + 1) / 2) * 2;
    const double t_q = 4.8 * ((ctas_q + num_sms - 1) / num_sms);
    const double t_pp = 9.0 * waves_pp, t_k3 = 7.0 * waves_k3;
    p.cta_pairs = cta_pairs_on && ctas_q >= num_sms && t_q <= 0.9 * std::min(t_pp, t_k3);
  } else {
    p.cta_pairs = false;
  }
  if (p.cta_pairs) p.pairs = false;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const int parts = p.split3 ? 2 : 1;
  const size_t q = (size_t)H * L * p.dhp * 4, k = (size_t)H * T * p.dhp * 4,
               v = (size_t)H * p.dhp * p.tp * 4;
  // Packed copies (unused when the call takes the fused form; small then).
  p.off_q = take(q * parts);
  p.off_k = take(k * parts);
  p.off_v = take(v * parts);
  p.ws_bytes = off;
  return p;
}

void attn_tc_run(const AttnTcPlan& p, const View3& Q, const View3& K, const View3& V,
                 const MView3& O, bool causal, void* ws, int* status, int num_sms,
                 cudaStream_t s) {
  char* w = static_cast<char*>(ws);
  const float qscale = kLog2e / std::sqrt(static_cast<float>(p.Dh));
  CUtensorMap maps[7] = {};
  // Fused form: the raw views are read by TMA, so each needs a unit column
  // stride and 16-byte aligned base, row and head pitches.
  auto tma_view = [](const View3& x) {
    return x.sD == 1 && (reinterpret_cast<uintptr_t>(x.data) & 15u) == 0 && x.sT > 0 &&
           x.sT % 4 == 0 && (x.H == 1 || (x.sH > 0 && x.sH % 4 == 0));
  };
  const bool fused = p.fusable && tma_view(Q) && tma_view(K) && tma_view(V);
  if (fused) {
    auto pitch = [](const View3& x, int rows) { return x.H == 1 ? (int64_t)rows * x.sT : x.sH; };
    maps[0] = make_tmap_3d(Q.data, p.H, p.L, p.Dh, Q.sT, pitch(Q, p.L), BM, BK);
    maps[2] = make_tmap_3d(K.data, p.H, p.T, p.Dh, K.sT, pitch(K, p.T), BN, BK);
    maps[4] = make_tmap_3d(V.data, p.H, p.T, p.Dh, V.sT, pitch(V, p.T), BK, 32);
    maps[1] = maps[0];
    maps[3] = maps[2];
    maps[5] = maps[4];
  } else {
    const size_t q = (size_t)p.H * p.L * p.dhp, k = (size_t)p.H * p.T * p.dhp,
                 v = (size_t)p.H * p.dhp * p.tp;
    float* qh = reinterpret_cast<float*>(w + p.off_q);
    float* kh = reinterpret_cast<float*>(w + p.off_k);
    float* vh = reinterpret_cast<float*>(w + p.off_v);
    float* ql = p.split3 ? qh + q : nullptr;
    float* kl = p.split3 ? kh + k : nullptr;
    float* vl = p.split3 ? vh + v : nullptr;
    // Q (scaled by log2(e)/sqrt(Dh)) and K as [H, rows, dhp]; V transposed to
    // [H, dhp, tp]; all in one launch.
    const PackJob jobs[3] = {
        {Q.data, Q.sH, Q.sT, Q.sD, p.H, p.L, p.Dh, p.L, p.dhp, false, qscale, qh, ql},
        {K.data, K.sH, K.sT, K.sD, p.H, p.T, p.Dh, p.T, p.dhp, false, 1.f, kh, kl},
        {V.data, V.sH, V.sT, V.sD, p.H, p.T, p.Dh, p.dhp, p.tp, true, 1.f, vh, vl}};
    pack_launch(jobs, 3, p.split3, num_sms, s);
    maps[0] = make_tmap_3d(qh, p.H, p.L, p.dhp, p.dhp, (uint64_t)p.L * p.dhp, BM, BK);
    maps[2] = make_tmap_3d(kh, p.H, p.T, p.dhp, p.dhp, (uint64_t)p.T * p.dhp, BN, BK);
    maps[4] = make_tmap_3d(vh, p.H, p.dhp, p.tp, p.tp, (uint64_t)p.dhp * p.tp, p.dhp, BK);
    if (p.split3) {
      maps[1] = make_tmap_3d(ql, p.H, p.L, p.dhp, p.dhp, (uint64_t)p.L * p.dhp, BM, BK);
      maps[3] = make_tmap_3d(kl, p.H, p.T, p.dhp, p.dhp, (uint64_t)p.T * p.dhp, BN, BK);
      maps[5] = make_tmap_3d(vl, p.H, p.dhp, p.tp, p.tp, (uint64_t)p.dhp * p.tp, p.dhp, BK);
    } else {
      maps[1] = maps[0];
      maps[3] = maps[2];
      maps[5] = maps[4];
    }
  }
  // The output leaves through TMA stores when its view allows a tensor map
  // (unit column stride, 16-byte aligned base and row / head pitches).
  const bool o_tma = O.sD == 1 && (reinterpret_cast<uintptr_t>(O.data) & 15u) == 0 &&
                     (O.sT % 4) == 0 && (O.sH % 4) == 0 && O.sT > 0 && O.sH > 0;
  if (o_tma) maps[6] = make_tmap_3d(O.data, p.H, p.L, p.Dh, O.sT, O.sH, BM, 32);
  if (p.pairs || p.cta_pairs) {
    const AttnPPArgs a{p.L, p.T, p.H, p.Dh, causal ? 1 : 0, p.qtiles, o_tma ? 1 : 0,
                       O.data, O.sH, O.sT, O.sD, status};
    if (p.cta_pairs) {
      // Each CTA of a pair loads 64 keys of every K tile and dhp/2 rows of V^T.
      const float* kh = reinterpret_cast<const float*>(w + p.off_k);
      const float* vh = reinterpret_cast<const float*>(w + p.off_v);
      const CUtensorMap k_half =
          make_tmap_3d(kh, p.H, p.T, p.dhp, p.dhp, (uint64_t)p.T * p.dhp, BN / 2, BK);
      const CUtensorMap v_half =
          make_tmap_3d(vh, p.H, p.dhp, p.tp, p.tp, (uint64_t)p.dhp * p.tp, p.dhp / 2, BK);
      ProfScope prof("attn_tc", s);
      attn_pair_launch(p.dhp, maps[0], k_half, v_half, maps[6], a, s);
      return;
    }
    ProfScope prof("attn_tc", s);
    attn_pp_launch(p.dhp, maps[0], maps[2], maps[4], maps[6], a, s);
    return;
  }
  AttnParams prm{};
  prm.L = p.L;
  prm.T = p.T;
  prm.H = p.H;
  prm.Dh = p.Dh;
  prm.causal = causal ? 1 : 0;
  prm.nsplit = p.nsplit;
  prm.tiles_per_split = p.tiles_per_split;
  prm.qtiles = p.qtiles;
  prm.o_tma = o_tma ? 1 : 0;
  prm.O = O.data;
  prm.osH = O.sH;
  prm.osT = O.sT;
  prm.osD = O.sD;
  prm.q = Q.data;
  prm.k = K.data;
  prm.v = V.data;
  prm.qsH = Q.sH;
  prm.qsT = Q.sT;
  prm.qsD = Q.sD;
  prm.ksH = K.sH;
  prm.ksT = K.sT;
  prm.ksD = K.sD;
  prm.vsH = V.sH;
  prm.vsT = V.sT;
  prm.vsD = V.sD;
  prm.qscale = qscale;
  prm.status = status;
  ProfScope prof("attn_tc", s);
  if (p.split3) dispatch_dhp<true>(p.dhp, fused, maps, prm, p.qtiles, s);
  else dispatch_dhp<false>(p.dhp, fused, maps, prm, p.qtiles, s);
}

}  // namespace attnb
