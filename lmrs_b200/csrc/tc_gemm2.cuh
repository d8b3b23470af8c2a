// tc_gemm2.cuh — AWQ W4A16 prefill GEMM on CTA pairs (tcgen05 cta_group::2).
//
// A cluster of two CTAs on two SMs computes one 256 x 256 output tile with
// 256 x 256 x 16 tcgen05.mma instructions issued by the pair's first CTA:
//   * CTA r holds rows 128r .. 128r+127 of the x tile (operand A) and columns
//     128r .. 128r+127 of the weight tile (operand B); its TMEM holds its 128
//     output rows x 256 columns (two buffers -> 512 columns).
//   * Each CTA dequantises only ITS half of the weight tile (16 KB of fp16 per
//     64-row K-block instead of 32 KB): the dequant work and its shared-memory
//     traffic per FLOP halve relative to a one-SM 128 x 256 tile, which is what
//     bounds the fused W4A16 GEMM.
// Hand-offs (all mbarrier waits bounded, lmrs_ptx.cuh):
//   x tiles       TMA (.cta_group::2) in both CTAs complete on CTA 0's xfull[s]
//   packed tiles  TMA in each CTA complete on that CTA's pfull[s]
//   dequant       CTA 0's warps arrive on its bfull[sb]; CTA 1's warps arrive on a
//                 local barrier that a relay warp of CTA 1 forwards to CTA 0 with
//                 one cluster-scope release per stage (a release per warp puts
//                 the cluster fence into every warp's chain)
//   MMA           CTA 0 issues; tcgen05.commit multicasts to both CTAs' empty[s],
//                 bempty[sb] and, per tile, accfull[a]
//   epilogue      both CTAs read their own TMEM, then arrive on CTA 0's accempty[a]
// No TMA multicast anywhere.
#pragma once
#include <cooperative_groups.h>
#include "tc_gemm.cuh"

namespace lmrs {

constexpr int kP2BM = 256;        // tile rows (both CTAs)
constexpr int kP2BN = 256;        // tile columns (both CTAs)
constexpr int kP2BK = 64;
constexpr int kP2SA = 4;          // TMA stages
constexpr int kP2SB = 4;          // dequantised B stages
constexpr int kP2DqWarp0 = 6;
constexpr int kP2DqWarps = 8;     // per group
constexpr int kP2DqGroups = 2;    // groups alternate K-blocks
constexpr int kP2RelayWarp0 = kP2DqWarp0 + kP2DqWarps * kP2DqGroups;
constexpr int kP2Relays = 4;      // relay warps (CTA 1), round-robin over K-blocks
constexpr int kP2Threads = 32 * (kP2RelayWarp0 + kP2Relays);  // 832
// Every mbarrier must be waited on by one agent, phase after phase: a waiter
// that skips a phase owned by someone else can be fooled by the parity of the
// phase before it.  With SB a multiple of both the relay count and the dequant
// group count, B stage sb belongs to exactly one relay and one dequant group.
static_assert(kP2SB % kP2Relays == 0 && kP2SB % kP2DqGroups == 0, "stage ownership");
constexpr int kP2ABytes = 128 * kP2BK * 2;       // this CTA's x rows: 16 KB
constexpr int kP2PBytes = kP2BK * 16 * 4;        // packed half-tile: 64 rows x 16 words = 4 KB
constexpr int kP2SBytes = 128 * 2;               // scales of the 128 columns
constexpr int kP2ZBytes = 16 * 4;                // zeros of the 128 columns
constexpr int kP2Stage = kP2ABytes + kP2PBytes + kP2SBytes + kP2ZBytes;  // 20,800 B
constexpr int kP2StageAl = (kP2Stage + 1023) / 1024 * 1024;
constexpr int kP2BBytes = 128 * kP2BK * 2;       // dequantised half-tile: 16 KB
constexpr int kP2SmemBytes = 1024 + kP2SA * kP2StageAl + kP2SB * kP2BBytes + 512;

template <typename T>
__global__ void __launch_bounds__(kP2Threads, 1)
    awq_gemm_tc2_kernel(const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_s,
                        const __grid_constant__ CUtensorMap tm_z, T* __restrict__ y,
                        const T* __restrict__ bias, int M, int K, int N, int group) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sT = smem;                        // [x rows | packed | scales | zeros] per stage
  uint8_t* sB = sT + kP2SA * kP2StageAl;     // dequantised B half-tiles
  uint64_t* xfull = reinterpret_cast<uint64_t*>(sB + kP2SB * kP2BBytes);  // used in CTA 0
  uint64_t* pfull = xfull + kP2SA;           // local
  uint64_t* empty = pfull + kP2SA;           // local, multicast commit
  uint64_t* bfull = empty + kP2SA;           // used in CTA 0
  uint64_t* bempty = bfull + kP2SB;          // local, multicast commit
  uint64_t* accfull = bempty + kP2SB;        // [2] local, multicast commit
  uint64_t* accempty = accfull + 2;          // [2] used in CTA 0
  uint64_t* blocal = accempty + 2;           // [SB] CTA 1: its dequant warps -> relay
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(blocal + kP2SB);

  const uint32_t rank = cooperative_groups::this_cluster().block_rank();  // 0 or 1
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = K / kP2BK;
  const int n_tiles = (N + kP2BN - 1) / kP2BN;
  const int m_tiles = (M + kP2BM - 1) / kP2BM;
  const int tiles = n_tiles * m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kP2SA; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&pfull[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kP2SB; ++s) {
      mbar_init(&bfull[s], kP2DqWarps + 1);  // CTA 0's dequant warps + CTA 1's relay
      mbar_init(&bempty[s], 1);
      mbar_init(&blocal[s], kP2DqWarps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accfull[a], 1);
      mbar_init(&accempty[a], 2 * kTcEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_s);
    tma_prefetch_desc(&tm_z);
  }
  if (warp == 1) {
    tmem_alloc_cg2(tmem_slot, kTcTmemCols);
    tmem_relinquish_cg2();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // tile coordinates of the pair: groups of kTcGroupM 256-row bands (tile_coords
  // works on 128-row units, so feed it the pair geometry)
  auto coords = [&](int t, int& m0, int& n0) {
    const int per_group = kTcGroupM * n_tiles;
    const int grp = t / per_group;
    const int first_m = grp * kTcGroupM;
    const int gm = min(m_tiles - first_m, kTcGroupM);
    const int local = t - grp * per_group;
    m0 = (first_m + local % gm) * kP2BM;
    n0 = (local / gm) * kP2BN;
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t xfull0 = mapa_shared(smem_u32(xfull), 0);
      const uint64_t keep = policy_evict_last();
      uint32_t kg = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        int m0, n0;
        coords(t, m0, n0);
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % kP2SA;
          if (!(ok = mbar_wait(&empty[s], ((kg / kP2SA) & 1) ^ 1, kErrWaitEmpty))) break;
          const int k = kb * kP2BK;
          const int gi = k / group;
          uint8_t* st = sT + s * kP2StageAl;
          // x rows of both CTAs land on CTA 0's xfull[s]; CTA 0 announces both
          if (rank == 0) mbar_arrive_expect_tx(&xfull[s], 2 * kP2ABytes);
          tma_load_2d_cg2(&tm_x, xfull0 + s * 8, st, k, m0 + 128 * static_cast<int>(rank));
          (void)keep;
          mbar_arrive_expect_tx(&pfull[s], kP2PBytes + kP2SBytes + kP2ZBytes);
          const int wcol = n0 / 8 + 16 * static_cast<int>(rank);
          tma_load_2d(&tm_q, &pfull[s], st + kP2ABytes, wcol, k);
          tma_load_2d(&tm_s, &pfull[s], st + kP2ABytes + kP2PBytes, n0 + 128 * static_cast<int>(rank), gi);
          tma_load_2d(&tm_z, &pfull[s], st + kP2ABytes + kP2PBytes + kP2SBytes, wcol, gi);
        }
      }
    }
  } else if (warp >= kP2RelayWarp0) {
    // ---------------- relays (CTA 1 only): once this CTA's dequant warps finished
    // a B stage (CTA-scope arrivals), publish it to CTA 0 with ONE cluster-scope
    // release.  The fence takes longer than a K-block's MMAs, so kP2Relays
    // relays take K-blocks round-robin and keep that many fences in flight; a
    // release per dequant warp would put the fence into every warp's chain.
    const int g = warp - kP2RelayWarp0;
    if (rank == 1 && lane == 0) {
      const uint32_t bfull0 = mapa_shared(smem_u32(bfull), 0);
      uint32_t kg = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          if (static_cast<int>(kg % kP2Relays) != g) continue;
          const int sb = kg % kP2SB;
          if (!(ok = mbar_wait(&blocal[sb], (kg / kP2SB) & 1, kErrWaitDequant))) break;
          mbar_arrive_cluster(bfull0 + sb * 8);
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      // M = 256 across the pair, N = 256; A K-major, B MN-major
      constexpr uint32_t fmt = Act<T>::kUmmaFmt;  // both operands f16, or both bf16
      constexpr uint32_t idesc = make_idesc(fmt, fmt, 0, 1, kP2BM, kP2BN);
      uint32_t kg = 0, it = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs, ++it) {
        const uint32_t a = it & 1;
        if (!(ok = mbar_wait(&accempty[a], ((it >> 1) & 1) ^ 1, kErrWaitAccum))) break;
        tc_fence_after();
        const uint32_t d = tmem + a * kP2BN;
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % kP2SA, sb = kg % kP2SB;
          ok = mbar_wait(&bfull[sb], (kg / kP2SB) & 1, kErrWaitDequant) &&
               mbar_wait(&xfull[s], (kg / kP2SA) & 1, kErrWaitFull);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sT + s * kP2StageAl);
          const uint32_t b0 = smem_u32(sB + sb * kP2BBytes);
#pragma unroll
          for (int kk = 0; kk < kP2BK / 16; ++kk) {
            const uint64_t ad = make_sdesc(a0 + kk * 32, 16, 1024);
            const uint64_t bd = make_sdesc(b0 + kk * 2048, 8192, 1024);
            umma_f16_cg2(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit_cg2_mc(&empty[s], 0x3);
          umma_commit_cg2_mc(&bempty[sb], 0x3);
        }
        if (ok) umma_commit_cg2_mc(&accfull[a], 0x3);
      }
    }
  } else if (warp < kTcEpiWarp0 + kTcEpiWarps) {
    // ---------------- epilogue: this CTA's 128 rows of the tile
    const uint32_t accempty0 = mapa_shared(smem_u32(accempty), 0);
    const int quarter = warp & 3;
    uint32_t it = 0;
    for (int t = pair; t < tiles; t += npairs, ++it) {
      const uint32_t a = it & 1;
      if (!mbar_wait(&accfull[a], (it >> 1) & 1, kErrWaitAccum)) break;
      tc_fence_after();
      int m0, n0;
      coords(t, m0, n0);
      const int row = m0 + 128 * static_cast<int>(rank) + quarter * 32 + lane;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + a * kP2BN;
      for (int ch = 0; ch < kP2BN / 16; ++ch) {
        uint32_t r[16];
        tmem_ld16(tbase + ch * 16, r);
        tmem_ld_wait();
        const int n = n0 + ch * 16;
        if (row < M && n < N) {
          uint32_t packed[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float v0 = __uint_as_float(r[2 * e]), v1 = __uint_as_float(r[2 * e + 1]);
            if (bias != nullptr) {
              v0 += Act<T>::to_float(bias[n + 2 * e]);
              v1 += Act<T>::to_float(bias[n + 2 * e + 1]);
            }
            packed[e] = Act<T>::pack2(v0, v1);
          }
          uint4* dst = reinterpret_cast<uint4*>(y + static_cast<int64_t>(row) * N + n);
          dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(accempty0 + a * 8);
    }
  } else if (warp >= kP2DqWarp0) {
    // ---------------- dequant: this CTA's 128 columns; lane -> word j = lane % 16,
    // rows 2*it + lane/16 of the warp's 8; two groups alternate K-blocks
    const int dwa = warp - kP2DqWarp0;
    const int dgrp = dwa / kP2DqWarps, dw = dwa % kP2DqWarps;
    const int j = lane & 15, half = lane >> 4;
    const int blk = j >> 3, chunk = j & 7;
    uint32_t kg = 0;
    bool ok = true;
    for (int t = pair; t < tiles && ok; t += npairs) {
      for (int kb = 0; kb < KB; ++kb, ++kg) {
        if (static_cast<int>(kg % kP2DqGroups) != dgrp) continue;
        const int s = kg % kP2SA, sb = kg % kP2SB;
        ok = mbar_wait(&pfull[s], (kg / kP2SA) & 1, kErrWaitFull) &&
             mbar_wait(&bempty[sb], ((kg / kP2SB) & 1) ^ 1, kErrWaitEmpty);
        if (!ok) break;
        const uint8_t* st = sT + s * kP2StageAl;
        const uint32_t* pk = reinterpret_cast<const uint32_t*>(st + kP2ABytes);
        const uint4 sv = reinterpret_cast<const uint4*>(st + kP2ABytes + kP2PBytes)[j];
        const uint32_t zw =
            reinterpret_cast<const uint32_t*>(st + kP2ABytes + kP2PBytes + kP2SBytes)[j];
        uint32_t zb[4];
        awq_word_biased<T>(zw, zb);
        const AwqScale2 sp[4] = {awq_scale2<T>(sv.x), awq_scale2<T>(sv.y), awq_scale2<T>(sv.z),
                                 awq_scale2<T>(sv.w)};
        const uint32_t bbase = smem_u32(sB + sb * kP2BBytes) + blk * 8192;
        uint32_t w[4];
#pragma unroll
        for (int i2 = 0; i2 < 4; ++i2) w[i2] = pk[(dw * 8 + 2 * i2 + half) * 16 + j];
#pragma unroll
        for (int i2 = 0; i2 < 4; ++i2) {
          const int r = dw * 8 + 2 * i2 + half;
          uint32_t qb[4];
          awq_word_biased<T>(w[i2], qb);
          uint4 o;
          o.x = awq_dq<T>(qb[0], zb[0], sp[0]);
          o.y = awq_dq<T>(qb[1], zb[1], sp[1]);
          o.z = awq_dq<T>(qb[2], zb[2], sp[2]);
          o.w = awq_dq<T>(qb[3], zb[3], sp[3]);
          st_shared_v4(bbase + (r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4), o);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(rank == 0 ? &bfull[sb] : &blocal[sb]);
      }
    }
  }
  tc_fence_before();
  cluster_sync_all();  // no remote arrival may target a CTA that has left
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_cg2(tmem, kTcTmemCols);
  }
}

}  // namespace lmrs
