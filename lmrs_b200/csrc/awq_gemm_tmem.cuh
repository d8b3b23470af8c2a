// awq_gemm_tmem.cuh — AWQ W4A16 prefill GEMM with the dequantised weights as the
// tcgen05 A operand in tensor memory (roles swapped: D[channel][token]).
//
// Why: the shared-memory-staged GEMM (awq_gemm_tc_kernel) moves per 64-deep
// K-block the token tile (TMA write + UMMA read) and the dequantised fp16
// weight tile (st.shared + UMMA read) through shared memory, ~137 B/cycle at
// the tensor rate against ~128 available; it stalls at ~0.62 of the bf16 peak.
// Here the weights go CUDA cores -> TMEM (tcgen05.st) and are read by the MMA
// from TMEM; only the token tile crosses shared memory, and each dequantised
// weight serves BT tokens.
//
// One persistent CTA per SM walks tiles of 128 output channels (UMMA M, TMEM
// lanes) x BT tokens (UMMA N), K in blocks of 64:
//   * warp 0: TMA ring — lane 0 the token tile [BT rows x 64 k] (128 B
//     swizzle, K-major: x as stored), lane 1 the packed weight rows [64 k x 16
//     words]; tile coordinates once per tile.  (One thread issuing four copies
//     plus the index arithmetic per K-block was the bottleneck: ~900 cycles per
//     K-block for the bare pipeline.)
//   * warp 1: TMEM owner and MMA issuer — per K-block four UMMAs M=128, N=BT,
//     K=16, A from the TMEM stage, B from the token stage, then one commit
//     that frees the stage; accumulators double-buffered (2 x BT columns) up
//     to BT = 192, single at BT = 256.
//   * warps 2-5: epilogue — TMEM lane = channel (in the dequant's lane order), 16 token columns per
//     tcgen05.ld, + bias, transposed through shared memory so each lane stores
//     16 contiguous channels of one token (two 16-byte stores): one-channel
//     2-byte stores stalled the single-buffered accumulator at BT = 256.
//   * warps 6-21: dequant, four groups of four taking alternate K-blocks (one
//     warp per TMEM lane quarter and group) — quarter q takes the 16-byte
//     chunk q of each packed row with ldmatrix.trans (64-byte swizzled box),
//     whose registers pair rows r, r+1 of a half-word: one lop3 per nibble
//     makes the biased pair (fp16: 1024 + q or 64 + q; bf16: 128 + q after a
//     shift); each thread loads its word's 8 scales (16 bytes) and zero word
//     one K-block ahead; subtracting the same-biased zero is exact and the
//     scale product rounds once, so A holds exactly T_rne((q - z) * s) in the
//     activation type T (fp16 or bf16, lmrs_ptx.cuh Act<T>); tcgen05.st 16x128b lays each
//     channel along one TMEM lane (lane L of a quarter: channel
//     8 ((L & 7) >> 1) + 2 (L >> 3) + (L & 1)).
// Every mbarrier wait is bounded; on expiry the kernel records the site in the
// device error word and unwinds; TMEM is always released.
#pragma once
#include "awq_gemv.cuh"
#include "lmrs_ptx.cuh"
#include "tc_gemm.cuh"

namespace lmrs {

constexpr int kAgtCh = 128;          // output channels per tile (UMMA M)
constexpr int kAgtWords = kAgtCh / 8;
constexpr int kAgtBK = 64;           // k rows of one TMA box / UMMA sub-tile
constexpr int kAgtEpiWarp0 = 2;
constexpr int kAgtDqWarp0 = 6;
constexpr int kAgtDqGroups = 4;      // dequant warp groups, alternating K-blocks
constexpr int kAgtThreads = 32 * (kAgtDqWarp0 + 4 * kAgtDqGroups);  // 704

// Shared-memory ring of S stages (token tile + packed weights of one BK-deep
// K-block) and a TMEM ring of R stages (dequantised weights, BK / 2 columns
// each), R <= S.  One tcgen05.commit per K-block (on the shared-memory slot's
// barrier) frees both: the dequant warps reuse TMEM stage kg % R after the
// commit of K-block kg - R.  The MMA thread's own work per K-block bounds the
// kernel: measured with a clock64 trace of a copy of the kernel (config 1,
// M = 4096), four UMMA issues take ~330 cycles, a commit ~200 and a check of an
// mbarrier that completed long before ~130, against ~660 cycles of tensor work
// per 64-deep K-block; so BK = 128 (eight UMMAs per commit and per wait) where
// K and the quantisation group allow it.
// Accumulators: two BT-column buffers when they leave room for two A stages, one
// for BT = 256 (the A ring then keeps filling while the epilogue drains).
template <int BT, int BK = 64>
struct AgtLayout {
  static constexpr int kSub = BK / kAgtBK;           // 64-deep token boxes per K-block
  static constexpr int kAccBufs = 2 * BT + 64 <= 512 ? 2 : 1;
  static constexpr int kStages = (BT == 128 ? 10 : (BT == 192 ? 7 : 6)) / kSub;  // as deep as smem allows
  static constexpr int kACols = BK / 2;              // TMEM columns of one A stage
  static constexpr int kATmem = (512 - kAccBufs * BT) / kACols;  // A stages TMEM has room for
  static constexpr int kAStages = kATmem < kStages ? (kATmem < 8 ? kATmem : 8) : (kStages < 8 ? kStages : 8);
  // Dequant warp groups (four warps each, one per TMEM lane quarter) taking
  // K-blocks round robin: no more groups than ring stages (see the dequant
  // loop for why), and enough that each has several K-blocks of time.
  static constexpr int kGroups = kStages < kAgtDqGroups ? kStages : kAgtDqGroups;
  static constexpr int kThreads = 32 * (kAgtDqWarp0 + 4 * kGroups);
  static constexpr int kXSub = BT * kAgtBK * 2;      // one 64-deep token box
  static constexpr int kX = kSub * kXSub;            // token stage (1024-aligned)
  static constexpr int kW = BK * kAgtWords * 4;      // packed weight rows, 4 / 8 KB
  static constexpr int kSmall = kW;
  static constexpr uint32_t kTx = kX + kW;
  static constexpr uint32_t kTmemA = kAccBufs * BT; // A stages after the accumulators
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kEpiPitch = 40;               // halves per token row of a warp's chunk
  static constexpr int kEpi = 4 * 16 * kEpiPitch * 2; // epilogue transpose, 16 tokens x 32 channels per warp
  static constexpr int kSmem = 1024 + kStages * (kX + kSmall) + kEpi + 256;
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
  static_assert(kX % 1024 == 0, "128B-swizzled token stages are 1024-byte aligned");
  static_assert(kSmall % 128 == 0, "TMA destinations are 128-byte aligned");
  static_assert(kAccBufs * BT + kACols * kAStages <= 512 && kAStages >= 2 && kAStages <= kStages,
                "TMEM columns");
  static_assert(BT % 16 == 0 && BT <= 256, "UMMA N");
  static_assert(BK == 64 || BK == 128, "K-block depth");
  static_assert(kGroups >= 3 && kGroups <= kStages && kAStages <= kStages, "wait ordering");
};

// Tile t -> (first token m0, first channel n0): groups of kTcGroupM token tiles
// walked channel tile by channel tile, tokens fastest (x and weights stay in L2).
template <int BT>
__device__ __forceinline__ void agt_coords(int t, int m_tiles, int n_tiles, int& m0, int& n0) {
  const int per_group = kTcGroupM * n_tiles;
  const int grp = t / per_group;
  const int first_m = grp * kTcGroupM;
  const int gm = min(m_tiles - first_m, kTcGroupM);
  const int local = t - grp * per_group;
  m0 = (first_m + local % gm) * BT;
  n0 = (local / gm) * kAgtCh;
}

template <int BT, int BK, typename T>
__global__ void __launch_bounds__(AgtLayout<BT, BK>::kThreads, 1) awq_gemm_tmem_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_q,
    const __half* __restrict__ scales, const uint32_t* __restrict__ qzeros,
    T* __restrict__ y, const T* __restrict__ bias, int M, int K, int N, int group) {
  using L = AgtLayout<BT, BK>;
  constexpr int S = L::kStages, R = L::kAStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sx = align1024(smem_raw);
  uint8_t* ssm = sx + S * L::kX;
  T* sepi = reinterpret_cast<T*>(ssm + S * L::kSmall);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sepi) + L::kEpi);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;  // TMEM stage's dequantised weights are written
  AccBars* acc = reinterpret_cast<AccBars*>(afull + R);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = K / BK;   // K % BK == 0 (BK = 128 only when K and the group allow it)
  const int n_tiles = (N + kAgtCh - 1) / kAgtCh;
  const int m_tiles = (M + BT - 1) / BT;
  const int tiles = n_tiles * m_tiles;
  const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int total = my_tiles * KB;  // K-blocks this CTA streams

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < R; ++a) mbar_init(&afull[a], 4);  // one arrive per dequant warp
    acc_bars_init(acc);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA ring
    // lane 0 owns the stage's transaction count and the token tile, lane 1 the
    // packed weights (which may land first: the count then dips below zero)
    if (lane < 2) {
      if (lane == 0) tma_prefetch_desc(&tm_x); else tma_prefetch_desc(&tm_q);
      const uint64_t keep = policy_evict_last();  // token tiles are re-read by every channel tile
      if (lane == 0) pdl_wait();  // the tokens are the previous kernel's output
      int m0 = 0, n0 = 0;
      for (uint32_t kg = 0; kg < static_cast<uint32_t>(total); ++kg) {
        const int kb = static_cast<int>(kg % KB);
        if (kb == 0)
          agt_coords<BT>(blockIdx.x + static_cast<int>(kg / KB) * gridDim.x, m_tiles, n_tiles, m0, n0);
        const int s = kg % S;
        if (kg >= static_cast<uint32_t>(S) && !mbar_wait(&empty[s], ((kg / S) - 1) & 1, kErrWaitEmpty))
          break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], L::kTx);
#pragma unroll
          for (int sub = 0; sub < L::kSub; ++sub)
            tma_load_2d_hint(&tm_x, &full[s], sx + s * L::kX + sub * L::kXSub,
                             kb * BK + sub * kAgtBK, m0, keep);
        } else {
          tma_load_2d(&tm_q, &full[s], ssm + s * L::kSmall, n0 / 8, kb * BK);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t fmt = Act<T>::kUmmaFmt;  // both operands f16, or both bf16
      constexpr uint32_t idesc = make_idesc(fmt, fmt, 0, 0, kAgtCh, BT);  // K-major
      uint32_t kg = 0, it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
        const uint32_t a = it % L::kAccBufs, use = it / L::kAccBufs;
        if (!(ok = mbar_wait(&acc->empty[a], (use & 1) ^ 1, kErrWaitAccum))) break;
        tc_fence_after();
        const uint32_t d = tmem + a * BT;
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % S, ar = kg % R;
          // The MMA reads the token tile through the async proxy: this thread
          // observes full[s] itself rather than relying on the dequant warps'
          // afull arrival to order the TMA writes for the tensor core.
          ok = mbar_wait_fast(&full[s], (kg / S) & 1, kErrWaitFull) &&
               mbar_wait_fast(&afull[ar], (kg / R) & 1, kErrWaitDequant);
          if (!ok) break;
          tc_fence_after();
          const uint32_t xs = smem_u32(sx + s * L::kX);
          const uint32_t acol = tmem + L::kTmemA + ar * L::kACols;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16_tmem_a(d, acol + kk * 8,
                            make_sdesc(xs + (kk >> 2) * L::kXSub + (kk & 3) * 32, 16, 1024),
                            idesc, (kb | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);  // slot s and TMEM stage ar are free
        }
        if (ok) umma_commit(&acc->full[a]);
      }
    }
  } else if (warp < kAgtDqWarp0) {
    // ------------------------------------------- epilogue: lane = output channel
    const int quarter = warp & 3;
    // TMEM lane L of a quarter holds channel 8 ((L & 7) >> 1) + 2 (L >> 3) + (L & 1)
    // of the quarter's 32 (the dequant's ldmatrix / 16x128b layout)
    const int cq = 8 * ((lane & 7) >> 1) + 2 * (lane >> 3) + (lane & 1);
    const int c = quarter * 32 + cq;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    pdl_wait();  // y may still be read by the previous kernel
    uint32_t it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const uint32_t a = it % L::kAccBufs;
      if (!mbar_wait(&acc->full[a], (it / L::kAccBufs) & 1, kErrWaitAccum)) break;
      tc_fence_after();
      int m0, n0;
      agt_coords<BT>(t, m_tiles, n_tiles, m0, n0);
      const int n = n0 + c;
      const float bn = (bias != nullptr && n < N) ? Act<T>::to_float(bias[n]) : 0.f;
      T* tw = sepi + quarter * 16 * L::kEpiPitch;
      const int te = lane >> 1, th = lane & 1;          // read side: token, 16-channel half
      const int nw = n0 + quarter * 32 + 16 * th;       // N % 32 == 0: whole 16-channel runs
      for (int ch = 0; ch < BT / 16; ++ch) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_addr + a * BT + ch * 16, r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) tw[e * L::kEpiPitch + cq] = Act<T>::from_float(__uint_as_float(r[e]) + bn);
        __syncwarp();
        const int m = m0 + ch * 16 + te;
        if (m < M && nw < N) {
          const uint4* src = reinterpret_cast<const uint4*>(tw + te * L::kEpiPitch + 16 * th);
          uint4* dst = reinterpret_cast<uint4*>(y + static_cast<int64_t>(m) * N + nw);
          dst[0] = src[0];
          dst[1] = src[1];
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc->empty[a]);
    }
  } else {
    // ------------------------------------------- dequant
    // Quarter q's 32 TMEM lanes take the 16-byte chunk q (words 4q .. 4q+3, 32
    // channels) of every 64-byte packed row.  ldmatrix.trans of 32 rows gives
    // thread t = 4hc + pp, register i, half-word hc of the chunk for rows
    // 8i + 2pp (low half) and 8i + 2pp + 1 (high half): each of its four
    // nibbles already has its row pair in the two halves, so one lop3 (after
    // one shift for the upper byte) makes the biased half2.  tcgen05.st
    // 16x128b puts register 2j at lane hc, column 4j + pp, and 2j + 1 at lane
    // hc + 8: nibbles 0, 1 go to lanes hc, hc + 8, nibbles 2, 3 to 16 + hc,
    // 24 + hc, each lane one channel with k-pair kp in column kp.  The weight
    // box arrives with the 64-byte swizzle, so the 8-row reads are
    // conflict-free: 8 wavefronts per warp and K-block.
    constexpr int G = L::kGroups;
    const int quarter = warp & 3;
    const int dgrp = (warp - kAgtDqWarp0) >> 2;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int hc = lane >> 2;                 // half-word of the chunk
    const int wt = 4 * quarter + (hc >> 1);   // word of the tile
    const int codd = hc & 1;                  // nibbles 4 codd .. 4 codd + 3 of the word
    const uint32_t sdup = codd ? 0x3232u : 0x1010u;  // prmt: duplicate the high / low half
    const int words = N / 8;
    // scales of the word's 8 channels and its zero word for K-block kg
    int ftile = -1, fm0 = 0, n0 = 0;
    auto fetch = [&](uint32_t kg, uint4& sv, uint32_t& zv) {
      sv = make_uint4(0u, 0u, 0u, 0u);
      zv = 0u;
      if (kg >= static_cast<uint32_t>(total)) return;
      const int tt = static_cast<int>(kg / KB);
      if (tt != ftile) {
        ftile = tt;
        agt_coords<BT>(blockIdx.x + tt * gridDim.x, m_tiles, n_tiles, fm0, n0);
      }
      const int gi = static_cast<int>(kg % KB) * BK / group;  // BK <= group or BK == 64
      const int n = n0 + 8 * wt;
      if (n < N) {  // N % 8 == 0: the whole word is in range
        sv = *reinterpret_cast<const uint4*>(scales + static_cast<int64_t>(gi) * N + n);
        zv = qzeros[static_cast<int64_t>(gi) * words + (n >> 3)];
      }
    };
    uint4 s_nxt;
    uint32_t z_nxt;
    fetch(dgrp, s_nxt, z_nxt);
    bool ok = true;
    for (uint32_t kg = dgrp; kg < static_cast<uint32_t>(total) && ok; kg += G) {
      const uint4 s_cur = s_nxt;
      const uint32_t z_cur = z_nxt >> (16 * codd);
      fetch(kg + G, s_nxt, z_nxt);
      const int s = kg % S, ar = kg % R;
      // A parity wait for phase P of a barrier is only sound once phase P - 1
      // has completed (in phase P - 1 the parity test reads "done").  Several
      // groups share these barriers, so the order of the two waits carries it:
      //  1. TMEM stage ar was last read by the MMAs of K-block j = kg - R: wait
      //     for their commit (phase j / S of empty[j % S]).  Its phase before,
      //     the commit of j - S, is covered by this group's previous wait here
      //     (the commit of kg - G - R >= j - S since G <= S; commits complete
      //     in order); the phase after needs K-block j + S >= kg.
      //  2. Then slot s (phase kg / S of full[s]): its phase before belongs to
      //     K-block kg - S <= j, whose tokens the MMAs of step 1 consumed.
      if (kg >= static_cast<uint32_t>(R)) {
        const uint32_t j = kg - R;
        if (!(ok = mbar_wait(&empty[j % S], (j / S) & 1, kErrWaitAccum))) break;
      }
      if (!(ok = mbar_wait(&full[s], (kg / S) & 1, kErrWaitFull))) break;
      const uint32_t s4[4] = {s_cur.x, s_cur.y, s_cur.z, s_cur.w};
      uint32_t zz[4];
      AwqScale2 ss[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        zz[n] = awq_zero_pair<T>((z_cur >> (4 * n)) & 0xFu, n);
        ss[n] = awq_scale2<T>(prmt(s4[n], s4[n], sdup));  // channel 8 wt + 2n + codd
      }
      const uint8_t* sm = ssm + s * L::kSmall;
      const uint32_t acol = tmem + lane_addr + L::kTmemA + ar * L::kACols;
#pragma unroll
      for (int h = 0; h < BK / 32; ++h) {
        const int r = 32 * h + lane;  // row this lane addresses for ldmatrix
        uint32_t d[4];
        ldsm_x4_t(d, smem_u32(sm + r * (kAgtWords * 4) + ((quarter ^ ((r >> 1) & 3)) << 4)));
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // nibble j of each half: j = 0, 1 -> lanes hc, hc + 8; j = 2, 3 -> 16 + hc, 24 + hc
          lo[2 * i] = awq_dq<T>(awq_nib_pair<T>(d[i], 0), zz[0], ss[0]);
          lo[2 * i + 1] = awq_dq<T>(awq_nib_pair<T>(d[i], 1), zz[1], ss[1]);
          hi[2 * i] = awq_dq<T>(awq_nib_pair<T>(d[i], 2), zz[2], ss[2]);
          hi[2 * i + 1] = awq_dq<T>(awq_nib_pair<T>(d[i], 3), zz[3], ss[3]);
        }
        tmem_st16x128b_x4(acol + 16 * h, lo);
        tmem_st16x128b_x4(acol + (16u << 16) + 16 * h, hi);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[ar]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace lmrs
