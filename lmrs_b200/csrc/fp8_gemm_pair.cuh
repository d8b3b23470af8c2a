// fp8_gemm_pair.cuh — FP8 W8A8 prefill GEMM on CTA pairs (tcgen05 cta_group::2).
//
// y[m, n] = bf16(s_x[m] * s_w[n] * sum_k xq[m, k] * wq[n, k]) (+ bias[n])
//
// A cluster of two CTAs on two SMs computes one 256 x 256 output tile; the
// pair's first CTA issues 256 x 256 x 32 e4m3 UMMAs:
//   * CTA r holds token rows 128r .. 128r+127 of the tile (operand A) and weight
//     rows 128r .. 128r+127 (its half of operand B), both K-major in 128-byte
//     swizzled stages at the same shared-memory offsets in both CTAs; its TMEM
//     holds its 128 output rows x 256 columns (two buffers: 512 columns).
//   * Why: a one-SM 128 x 256 tile streams 384 operand bytes per K byte into
//     its SM for 2 x 128 x 256 FLOP; at the FP8 tensor rate that is ~126 GB/s
//     per SM from L2, about what one SM can pull, so those tiles run at
//     ~65-70 % of the tensor peak.  The pair tile streams 256 bytes per K byte
//     per SM for the same FLOP.
// Hand-offs (mbarrier waits bounded): both CTAs' TMA loads of a stage complete
// on CTA 0's full[s] (CTA 0 announces both CTAs' bytes); CTA 0's
// tcgen05.commit multicasts to both CTAs' empty[s] and, per tile, accfull[a];
// both CTAs' epilogue warps arrive on CTA 0's accempty[a].  Persistent pairs
// walk 256 x 256 tiles in groups of group_m 256-row bands.  No TMA multicast.
#pragma once
#include <cooperative_groups.h>
#include "tc_gemm.cuh"

namespace lmrs {

constexpr int kF8PBM = 256, kF8PBN = 256;

template <int KSUB> struct F8Pair {
  static constexpr int kBK = kF8BK * KSUB;          // K bytes per stage
  static constexpr int kA = 128 * kBK;              // this CTA's token rows
  static constexpr int kB = 128 * kBK;              // this CTA's weight rows
  static constexpr int kStages = KSUB == 2 ? 3 : 6;
  static constexpr int kSmem = 1024 + kStages * (kA + kB) + 256;
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

template <int KSUB>
__global__ void __launch_bounds__(kF8Threads, 1)
    fp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a,
                         const __grid_constant__ CUtensorMap tm_b, __nv_bfloat16* __restrict__ y,
                         const float* __restrict__ sx, const float* __restrict__ sw,
                         const __nv_bfloat16* __restrict__ bias, int M, int K, int N,
                         int group_m) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  using TL = F8Pair<KSUB>;
  constexpr int kS = TL::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = sA + kS * TL::kA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kS * TL::kB);  // used in CTA 0
  uint64_t* empty = full + kS;                                      // local, multicast commit
  uint64_t* accfull = empty + kS;                                   // [2] local, multicast commit
  uint64_t* accempty = accfull + 2;                                 // [2] used in CTA 0
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 2);

  const uint32_t rank = cooperative_groups::this_cluster().block_rank();  // 0 or 1
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (K + TL::kBK - 1) / TL::kBK;  // a box past K is zero-filled
  const int n_tiles = (N + kF8PBN - 1) / kF8PBN;
  const int m_tiles = (M + kF8PBM - 1) / kF8PBM;
  const int tiles = n_tiles * m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accfull[a], 1);
      mbar_init(&accempty[a], 2 * kTcEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc_cg2(tmem_slot, kTcTmemCols);
    tmem_relinquish_cg2();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto coords = [&](int t, int& m0, int& n0) {
    const int per_group = group_m * n_tiles;
    const int grp = t / per_group;
    const int first_m = grp * group_m;
    const int gm = min(m_tiles - first_m, group_m);
    const int local = t - grp * per_group;
    m0 = (first_m + local % gm) * kF8PBM;
    n0 = (local / gm) * kF8PBN;
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);
      uint32_t kg = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        int m0, n0;
        coords(t, m0, n0);
        const int mr = m0 + 128 * static_cast<int>(rank), nr = n0 + 128 * static_cast<int>(rank);
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % kS;
          if (!(ok = mbar_wait(&empty[s], ((kg / kS) & 1) ^ 1, kErrWaitEmpty))) break;
          // both CTAs' bytes land on CTA 0's full[s]; CTA 0 announces them
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (TL::kA + TL::kB));
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            const int kx = kb * TL::kBK + sub * kF8BK;
            tma_load_2d_cg2(&tm_a, full0 + s * 8, sA + s * TL::kA + sub * (128 * kF8BK), kx, mr);
            tma_load_2d_cg2(&tm_b, full0 + s * 8, sB + s * TL::kB + sub * (128 * kF8BK), kx, nr);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = make_idesc(0, 0, 0, 0, kF8PBM, kF8PBN);  // e4m3 x e4m3, K-major
      uint32_t kg = 0, it = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs, ++it) {
        const uint32_t a = it & 1;
        if (!(ok = mbar_wait(&accempty[a], ((it >> 1) & 1) ^ 1, kErrWaitAccum))) break;
        tc_fence_after();
        const uint32_t d = tmem + a * kF8PBN;
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % kS;
          if (!(ok = mbar_wait(&full[s], (kg / kS) & 1, kErrWaitFull))) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * TL::kA);
          const uint32_t b0 = smem_u32(sB + s * TL::kB);
#pragma unroll
          for (int kk = 0; kk < TL::kBK / 32; ++kk) {  // box kk / 4, 32-byte K step kk % 4
            const uint64_t ad = make_sdesc(a0 + (kk >> 2) * (128 * kF8BK) + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = make_sdesc(b0 + (kk >> 2) * (128 * kF8BK) + (kk & 3) * 32, 16, 1024);
            umma_f8_cg2(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit_cg2_mc(&empty[s], 0x3);
        }
        if (ok) umma_commit_cg2_mc(&accfull[a], 0x3);
      }
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quarters 2,3,0,1 of this CTA's 128 rows
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
      const float rs = row < M ? sx[row] : 0.f;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + a * kF8PBN;
      for (int ch = 0; ch < kF8PBN / 16; ++ch) {
        uint32_t r[16];
        tmem_ld16(tbase + ch * 16, r);
        tmem_ld_wait();
        const int n = n0 + ch * 16;
        if (row < M && n < N) {
          uint32_t packed[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int na = n + 2 * e, nb = na + 1;
            float v0 = 0.f, v1 = 0.f;
            if (na < N) {
              v0 = __fmul_rn(__fmul_rn(__uint_as_float(r[2 * e]), rs), sw[na]);
              if (bias != nullptr) v0 = __fadd_rn(v0, __bfloat162float(bias[na]));
            }
            if (nb < N) {
              v1 = __fmul_rn(__fmul_rn(__uint_as_float(r[2 * e + 1]), rs), sw[nb]);
              if (bias != nullptr) v1 = __fadd_rn(v1, __bfloat162float(bias[nb]));
            }
            __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
            packed[e] = *reinterpret_cast<uint32_t*>(&h);
          }
          __nv_bfloat16* dst = y + static_cast<int64_t>(row) * N + n;
          if (n + 16 <= N && (N % 8) == 0) {
            reinterpret_cast<uint4*>(dst)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            reinterpret_cast<uint4*>(dst)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
          } else {
            for (int e = 0; e < 16 && n + e < N; ++e) {
              const uint32_t pv = packed[e >> 1];
              reinterpret_cast<uint16_t*>(dst)[e] =
                  static_cast<uint16_t>((e & 1) ? (pv >> 16) : (pv & 0xFFFFu));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(accempty0 + a * 8);
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
