// awq_gemm_pair.cuh — AWQ W4A16 prefill GEMM on CTA pairs with the dequantised
// weights as the tcgen05 A operand in tensor memory (cta_group::2).
//
// Same roles as awq_gemm_tmem.cuh (D[channel][token], weights dequantised by
// CUDA cores straight into TMEM, tokens from TMA as the B operand), but a
// cluster of two CTAs on two SMs computes a 256-channel x 256-token tile with
// M=256 UMMAs issued by CTA 0:
//   * CTA r dequantises channels n0 + 128 r .. + 127 into ITS TMEM (the A rows
//     of the pair MMA that live on its SM) and loads tokens m0 + 128 r .. + 127
//     of each 64-deep K-block (its half of B) into its shared memory; its TMEM
//     accumulator holds its 128 channels x all 256 tokens.
//   * So each SM streams 16 KB of tokens per K-block instead of 32 KB (the token
//     tile was re-read from L2 by every channel tile), and one MMA instruction
//     does 256 x 256 x 16: twice the work per issue of the one-SM kernel, whose
//     single issuer completed an M=128 UMMA only every ~175 cycles.
// Hand-offs (every wait bounded; no TMA multicast anywhere):
//   token halves   TMA .cta_group::2 in both CTAs, completing on CTA 0's xfull[s]
//                  (CTA 0 arms it for both halves)
//   packed weights TMA into each CTA, completing on that CTA's wfull[s] (a ring
//                  of its own, so the dequant never waits for a token tile); a
//                  weight slot is freed by the four dequant warps that read it
//   dequant        each CTA's four warps of a group write their TMEM stage and
//                  arrive on CTA 0's afull[ar] (CTA 1's with a cluster-scope
//                  release): 8 arrivals per K-block
//   MMA            CTA 0 issues; ONE tcgen05.commit per K-block (a commit costs
//                  the issuing thread about as much as an MMA), multicast to both
//                  CTAs' kfree[s], frees the token slot and, R K-blocks on, the
//                  TMEM A stage; per tile a commit multicast to both CTAs' accfull
//   epilogue       each CTA drains its own TMEM, then arrives on CTA 0's accempty
// The dequant and epilogue lane layouts are those of awq_gemm_tmem.cuh.
#pragma once
#include <cooperative_groups.h>
#include "awq_gemm_tmem.cuh"

namespace lmrs {

constexpr int kApCh = 256;             // output channels per pair tile (UMMA M)
constexpr int kApBT = 256;             // tokens per tile (UMMA N)
constexpr int kApThreads = kAgtThreads;

struct ApLayout {
  static constexpr int kXStages = 8;   // token half-tiles [128 tokens x 64 k], 16 KB
  static constexpr int kWStages = 12;  // packed weight rows [64 k x 16 words], 4 KB
  static constexpr int kAStages = 8;   // TMEM A stages (32 columns each) after the accumulator
  static constexpr int kX = 128 * kAgtBK * 2;
  static constexpr int kW = kAgtBK * kAgtWords * 4;
  static constexpr uint32_t kTmemA = kApBT;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kEpiPitch = 40;
  static constexpr int kEpi = 4 * 16 * kEpiPitch * 2;
  static constexpr int kBars = 512;
  static constexpr int kSmem = 1024 + kXStages * kX + kWStages * kW + kEpi + kBars;
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
  static_assert(kX % 1024 == 0 && kW % 128 == 0, "TMA destinations");
  static_assert(kTmemA + 32 * kAStages <= kTmemCols, "TMEM columns");
  // TMEM stage reuse waits on kfree[(kg - R) % SX]: R <= SX keeps that wait
  // from aliasing (awq_gemm_pair_kernel's dequant loop); R and SW multiples of
  // the four dequant groups give each A stage and weight slot one owning group
  static_assert(kAStages <= kXStages && kXStages >= kAgtDqGroups, "TMEM stage reuse");
  static_assert(kAStages % kAgtDqGroups == 0 && kWStages % kAgtDqGroups == 0, "stage ownership");
  static_assert((2 * kXStages + 2 * kWStages + kAStages + 2) * 8 + 4 <= kBars, "barrier area");
};

// Pair tile t -> (first token m0, first channel n0): groups of kTcGroupM token
// tiles walked channel tile by channel tile (x and weights stay in L2).
__device__ __forceinline__ void ap_coords(int t, int m_tiles, int n_tiles, int& m0, int& n0) {
  const int per_group = kTcGroupM * n_tiles;
  const int grp = t / per_group;
  const int first_m = grp * kTcGroupM;
  const int gm = min(m_tiles - first_m, kTcGroupM);
  const int local = t - grp * per_group;
  m0 = (first_m + local % gm) * kApBT;
  n0 = (local / gm) * kApCh;
}

// D (M = 256 across the pair) (+)= A[tmem, both CTAs] * B[smem desc, both CTAs].
__device__ __forceinline__ void umma_f16_tmem_a_cg2(uint32_t d_tmem, uint32_t a_tmem,
                                                    uint64_t b_desc, uint32_t idesc,
                                                    uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kApThreads, 1) awq_gemm_pair_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_q,
    const __half* __restrict__ scales, const uint32_t* __restrict__ qzeros,
    T* __restrict__ y, const T* __restrict__ bias, int M, int K, int N, int group) {
  using L = ApLayout;
  constexpr int SX = L::kXStages, SW = L::kWStages, R = L::kAStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sx = align1024(smem_raw);
  uint8_t* sw = sx + SX * L::kX;
  T* sepi = reinterpret_cast<T*>(sw + SW * L::kW);
  uint64_t* xfull = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sepi) + L::kEpi);
  uint64_t* kfree = xfull + SX;     // local; multicast commit: the K-block's MMAs are done
  uint64_t* wfull = kfree + SX;     // local
  uint64_t* wempty = wfull + SW;    // local; the dequant warps have read the slot
  uint64_t* afull = wempty + SW;    // used in CTA 0
  uint64_t* accfull = afull + R;    // local; multicast commit
  uint64_t* accempty = accfull + 1; // used in CTA 0
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 1);

  const uint32_t rank = cooperative_groups::this_cluster().block_rank();  // 0 or 1
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = K / kAgtBK;
  const int n_tiles = (N + kApCh - 1) / kApCh;
  const int m_tiles = (M + kApBT - 1) / kApBT;
  const int tiles = n_tiles * m_tiles;
  const int my_tiles = pair < tiles ? (tiles - 1 - pair) / npairs + 1 : 0;
  const int total = my_tiles * KB;  // K-blocks this pair streams

  if (threadIdx.x == 0) {
    for (int s = 0; s < SX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&kfree[s], 1);
    }
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 4);  // the group's four dequant warps
    }
    for (int a = 0; a < R; ++a) mbar_init(&afull[a], 8);  // 4 dequant warps x 2 CTAs
    mbar_init(accfull, 1);
    mbar_init(accempty, 8);                                // 4 epilogue warps x 2 CTAs
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_cg2(tmem_slot, L::kTmemCols);
    tmem_relinquish_cg2();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote signal
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA rings
    if (lane == 0) {
      // this CTA's token half of each K-block, completing on CTA 0's xfull
      tma_prefetch_desc(&tm_x);
      const uint32_t xfull0 = mapa_shared(smem_u32(xfull), 0);
      pdl_wait();  // the tokens are the previous kernel's output
      int m0 = 0, n0 = 0;
      for (int kg = 0; kg < total; ++kg) {
        const int kb = kg % KB;
        if (kb == 0) ap_coords(pair + (kg / KB) * npairs, m_tiles, n_tiles, m0, n0);
        const int s = kg % SX;
        if (kg >= SX && !mbar_wait(&kfree[s], ((kg / SX) - 1) & 1, kErrWaitEmpty)) break;
        if (rank == 0) mbar_arrive_expect_tx(&xfull[s], 2 * L::kX);
        tma_load_2d_cg2(&tm_x, xfull0 + s * 8, sx + s * L::kX, kb * kAgtBK,
                        m0 + 128 * static_cast<int>(rank));
      }
    } else if (lane == 1) {
      // this CTA's 128 channels of packed weight rows (weights: no PDL dependence)
      tma_prefetch_desc(&tm_q);
      int m0 = 0, n0 = 0;
      for (int kg = 0; kg < total; ++kg) {
        const int kb = kg % KB;
        if (kb == 0) ap_coords(pair + (kg / KB) * npairs, m_tiles, n_tiles, m0, n0);
        const int s = kg % SW;
        if (kg >= SW && !mbar_wait(&wempty[s], ((kg / SW) - 1) & 1, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&wfull[s], L::kW);
        tma_load_2d(&tm_q, &wfull[s], sw + s * L::kW, (n0 + 128 * static_cast<int>(rank)) / 8,
                    kb * kAgtBK);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA (CTA 0)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t fmt = Act<T>::kUmmaFmt;  // both operands f16, or both bf16
      constexpr uint32_t idesc = make_idesc(fmt, fmt, 0, 0, kApCh, kApBT);  // K-major
      int kg = 0;
      uint32_t it = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs, ++it) {
        if (!(ok = mbar_wait_cluster(accempty, (it & 1) ^ 1, kErrWaitAccum))) break;
        tc_fence_after();
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % SX, ar = kg % R;
          ok = mbar_wait(&xfull[s], (kg / SX) & 1, kErrWaitFull) &&
               mbar_wait_cluster(&afull[ar], (kg / R) & 1, kErrWaitDequant);
          if (!ok) break;
          tc_fence_after();
          const uint32_t xs = smem_u32(sx + s * L::kX);
          const uint32_t acol = tmem + L::kTmemA + ar * 32;
#pragma unroll
          for (int kk = 0; kk < kAgtBK / 16; ++kk)
            umma_f16_tmem_a_cg2(tmem, acol + kk * 8, make_sdesc(xs + kk * 32, 16, 1024), idesc,
                                (kb | kk) != 0 ? 1u : 0u);
          umma_commit_cg2_mc(&kfree[s], 0x3);  // token slot s; TMEM stage ar (R K-blocks on)
        }
        if (ok) umma_commit_cg2_mc(accfull, 0x3);
      }
    }
  } else if (warp < kAgtDqWarp0) {
    // ---------------------------------------- epilogue: this CTA's 128 channels
    const uint32_t accempty0 = mapa_shared(smem_u32(accempty), 0);
    const int quarter = warp & 3;
    // TMEM lane L of a quarter holds channel 8 ((L & 7) >> 1) + 2 (L >> 3) + (L & 1)
    // of the quarter's 32 (the dequant's ldmatrix / 16x128b layout)
    const int cq = 8 * ((lane & 7) >> 1) + 2 * (lane >> 3) + (lane & 1);
    const int c = 128 * static_cast<int>(rank) + quarter * 32 + cq;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    pdl_wait();  // y may still be read by the previous kernel
    uint32_t it = 0;
    for (int t = pair; t < tiles; t += npairs, ++it) {
      if (!mbar_wait(accfull, it & 1, kErrWaitAccum)) break;
      tc_fence_after();
      int m0, n0;
      ap_coords(t, m_tiles, n_tiles, m0, n0);
      const int n = n0 + c;
      const float bn = (bias != nullptr && n < N) ? Act<T>::to_float(bias[n]) : 0.f;
      T* tw = sepi + quarter * 16 * L::kEpiPitch;
      const int te = lane >> 1, th = lane & 1;   // read side: token, 16-channel half
      const int nw = n0 + 128 * static_cast<int>(rank) + quarter * 32 + 16 * th;
      for (int ch = 0; ch < kApBT / 16; ++ch) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_addr + ch * 16, r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          tw[e * L::kEpiPitch + cq] = Act<T>::from_float(__uint_as_float(r[e]) + bn);
        __syncwarp();
        const int m = m0 + ch * 16 + te;
        if (m < M && nw < N) {  // N % 32 == 0: whole 16-channel runs
          const uint4* src = reinterpret_cast<const uint4*>(tw + te * L::kEpiPitch + 16 * th);
          uint4* dst = reinterpret_cast<uint4*>(y + static_cast<int64_t>(m) * N + nw);
          dst[0] = src[0];
          dst[1] = src[1];
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(accempty0);
    }
  } else {
    // ----------------------------------------------- dequant: this CTA's channels
    // As in awq_gemm_tmem.cuh: quarter q takes the 16-byte chunk q of each
    // 64-byte packed row with ldmatrix.trans, one lop3 per nibble pair, the
    // exact T_rne((q - z) * s), tcgen05.st 16x128b.
    const uint32_t afull0 = mapa_shared(smem_u32(afull), 0);
    const int quarter = warp & 3;
    const int dgrp = (warp - kAgtDqWarp0) >> 2;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int hc = lane >> 2;
    const int wt = 4 * quarter + (hc >> 1);
    const int codd = hc & 1;
    const uint32_t sdup = codd ? 0x3232u : 0x1010u;
    const int words = N / 8;
    int ftile = -1, fm0 = 0, n0 = 0;
    auto fetch = [&](int kg, uint4& sv, uint32_t& zv) {
      sv = make_uint4(0u, 0u, 0u, 0u);
      zv = 0u;
      if (kg >= total) return;
      const int tt = kg / KB;
      if (tt != ftile) {
        ftile = tt;
        ap_coords(pair + tt * npairs, m_tiles, n_tiles, fm0, n0);
      }
      const int gi = (kg % KB) * kAgtBK / group;
      const int n = n0 + 128 * static_cast<int>(rank) + 8 * wt;
      if (n < N) {  // N % 8 == 0: the whole word is in range
        sv = *reinterpret_cast<const uint4*>(scales + static_cast<int64_t>(gi) * N + n);
        zv = qzeros[static_cast<int64_t>(gi) * words + (n >> 3)];
      }
    };
    uint4 s_nxt;
    uint32_t z_nxt;
    fetch(dgrp, s_nxt, z_nxt);
    bool ok = true;
    for (int kg = dgrp; kg < total && ok; kg += kAgtDqGroups) {
      const uint4 s_cur = s_nxt;
      const uint32_t z_cur = z_nxt >> (16 * codd);
      fetch(kg + kAgtDqGroups, s_nxt, z_nxt);
      const int s = kg % SW, ar = kg % R;
      if (!(ok = mbar_wait(&wfull[s], (kg / SW) & 1, kErrWaitFull))) break;
      // TMEM stage ar was last read by the MMAs of K-block j = kg - R, whose
      // commit completes phase j / SX of kfree[j % SX].  Its phase before that
      // (K-block j - SX <= kg - 4 - R) completed before this group's previous
      // wait returned, and the phase after it (K-block j + SX >= kg) needs this
      // stage's MMAs: the parity wait cannot alias.
      if (kg >= R) {
        const int j = kg - R;
        if (!(ok = mbar_wait(&kfree[j % SX], (j / SX) & 1, kErrWaitAccum))) break;
      }
      const uint32_t s4[4] = {s_cur.x, s_cur.y, s_cur.z, s_cur.w};
      uint32_t zz[4];
      AwqScale2 ss[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        zz[n] = awq_zero_pair<T>((z_cur >> (4 * n)) & 0xFu, n);
        ss[n] = awq_scale2<T>(prmt(s4[n], s4[n], sdup));  // channel 8 wt + 2n + codd
      }
      const uint8_t* sm = sw + s * L::kW;
      const uint32_t acol = tmem + lane_addr + L::kTmemA + ar * 32;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = 32 * h + lane;
        uint32_t d[4];
        ldsm_x4_t(d, smem_u32(sm + r * (kAgtWords * 4) + ((quarter ^ ((r >> 1) & 3)) << 4)));
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          lo[2 * i] = awq_dq<T>(awq_nib_pair<T>(d[i], 0), zz[0], ss[0]);
          lo[2 * i + 1] = awq_dq<T>(awq_nib_pair<T>(d[i], 1), zz[1], ss[1]);
          hi[2 * i] = awq_dq<T>(awq_nib_pair<T>(d[i], 2), zz[2], ss[2]);
          hi[2 * i + 1] = awq_dq<T>(awq_nib_pair<T>(d[i], 3), zz[3], ss[3]);
        }
        if (h == 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&wempty[s]);  // both halves of the slot are in registers
        }
        tmem_st16x128b_x4(acol + 16 * h, lo);
        tmem_st16x128b_x4(acol + (16u << 16) + 16 * h, hi);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&afull[ar]);
        else mbar_arrive_cluster(afull0 + ar * 8);
      }
    }
  }
  tc_fence_before();
  cluster_sync_all();  // no remote arrival may target a CTA that has left
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_cg2(tmem, L::kTmemCols);
  }
}

}  // namespace lmrs
