// tc_gemm.cuh — tcgen05 (5th-gen tensor core) GEMMs for the prefill regime.
//
//   awq_gemm_tc_kernel : y fp16 [M,N] = x fp16 [M,K] @ dequant(AWQ int4) (+bias)
//   fp8_gemm_tc_kernel : y bf16 [M,N] = (xq e4m3 [M,K] @ wq e4m3 [N,K]^T) * sx[m] * sw[n] (+bias)
//
// Both are persistent, warp-specialised kernels: one CTA per SM walks output
// tiles (128 x 256) tile = blockIdx.x, blockIdx.x + gridDim.x, ... in grouped
// order (tile_coords) so the tiles in flight share x and weight tiles in L2.
//
//   warp 0        TMA producer: one thread streams K-blocks into a ring of
//                 shared-memory stages (cp.async.bulk.tensor, 128B swizzle,
//                 per-stage mbarrier with transaction count).
//   warp 1        TMEM owner (512 columns = two 128x256 fp32 accumulators) and
//                 MMA issuer: one thread issues tcgen05.mma from shared-memory
//                 descriptors; tcgen05.commit frees each stage and, at the end
//                 of a tile, hands the accumulator to the epilogue.
//   warps 2..5    epilogue: tcgen05.ld (32 lanes x 32 bit) -> scale/bias/round ->
//                 global, then release the accumulator buffer.  Double
//                 buffering lets tile i's epilogue overlap tile i+1's mainloop.
//   warps 6..21   AWQ only: dequant warps turn the TMA-staged packed int4 tile
//                 into fp16 directly in the UMMA MN-major 128B-swizzled layout
//                 (operand B): the dequant is fused into the shared-memory
//                 stage and weights cross HBM once, as int4.  Two groups of
//                 8 warps alternate K-blocks to hide the dequant latency.
// Every mbarrier wait is bounded (lmrs_ptx.cuh): on expiry the kernel records
// the site in the device error word and unwinds; TMEM is always released.
#pragma once
#include "lmrs_ptx.cuh"

namespace lmrs {

constexpr int kTcBM = 128;
constexpr int kTcBN = 256;
constexpr uint32_t kTcTmemCols = 512;  // two accumulators of kTcBN fp32 columns
constexpr int kTcEpiWarp0 = 2;         // epilogue warps 2..5
constexpr int kTcEpiWarps = 4;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Tile order: groups of kTcGroupM M-tiles walked N-tile by N-tile, M fastest,
// so the ~148 tiles in flight touch about 8 x-tiles and 19 weight tiles — both
// stay resident in L2 and each is fetched from HBM about once.
constexpr int kTcGroupM = 8;

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int bn, int& m0, int& n0,
                                            int group_m = kTcGroupM) {
  const int per_group = group_m * n_tiles;
  const int grp = t / per_group;
  const int first_m = grp * group_m;
  const int gm = min(m_tiles - first_m, group_m);
  const int local = t - grp * per_group;
  m0 = (first_m + local % gm) * kTcBM;
  n0 = (local / gm) * bn;
}

// Accumulator hand-off barriers (MMA -> epilogue -> MMA), two buffers.
struct AccBars {
  uint64_t full[2];
  uint64_t empty[2];
};

__device__ __forceinline__ void acc_bars_init(AccBars* b) {
  for (int i = 0; i < 2; ++i) {
    mbar_init(&b->full[i], 1);
    mbar_init(&b->empty[i], kTcEpiWarps);
  }
}

// ============================================================ AWQ W4A16 GEMM
constexpr int kAwqBK = 64;        // k rows per stage (one 128-byte fp16 row of A)
constexpr int kAwqSA = 4;         // TMA stages: A tile + packed tile + scales + zeros
constexpr int kAwqSB = 3;         // dequantised B stages
constexpr int kAwqDqGroups = 2;   // dequant warp groups, alternating K-blocks
constexpr int kAwqDqWarp0 = 6;
constexpr int kAwqDqWarps = 8;    // per group, 8 rows of the 64-row K-block each
constexpr int kAwqGemmThreads = 32 * (kAwqDqWarp0 + kAwqDqWarps * kAwqDqGroups);  // 704
constexpr int kAwqABytes = kTcBM * kAwqBK * 2;        // 16 KB
constexpr int kAwqBBytes = 256 * kAwqBK * 2;          // 32 KB: B stage sized for 4 blocks of 64 columns
// BN = 256 or 224 output columns per tile (224 evens out the waves of N = 14336);
// the B stage keeps four 64-column blocks, a 224-wide tile leaves half of the last unused.
// Every TMA destination in shared memory starts on a 128-byte boundary, so each
// per-stage region is padded to a multiple of 128 bytes (the transaction count
// stays the true box size).
constexpr int align128(int b) { return (b + 127) / 128 * 128; }
template <int BN> struct AwqTile {
  static constexpr int kWords = BN / 8;                       // packed words per k row
  static constexpr int kP = align128(kAwqBK * kWords * 4);    // packed stage
  static constexpr int kS = align128(BN * 2);                 // scales of one group
  static constexpr int kZ = align128(kWords * 4);             // zeros of one group
  static constexpr int kTx = kAwqABytes + kAwqBK * kWords * 4 + BN * 2 + kWords * 4;
  static constexpr int kSmem = 1024 + kAwqSA * (kAwqABytes + kP + kS + kZ) + kAwqSB * kAwqBBytes + 256;
  static_assert(kAwqABytes % 1024 == 0 && kAwqBBytes % 1024 == 0 && (kAwqSA * kP) % 128 == 0,
                "TMA destinations must stay 128-byte aligned");
};
constexpr int kAwqSmemBytes = AwqTile<256>::kSmem;

template <int BN, typename T>
__global__ void __launch_bounds__(kAwqGemmThreads, 1)
    awq_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_s,
                       const __grid_constant__ CUtensorMap tm_z, T* __restrict__ y,
                       const T* __restrict__ bias, int M, int K, int N, int group) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = sA + kAwqSA * kAwqABytes;
  using TL = AwqTile<BN>;
  uint8_t* sP = sB + kAwqSB * kAwqBBytes;
  uint8_t* sS = sP + kAwqSA * TL::kP;
  uint8_t* sZ = sS + kAwqSA * TL::kS;
  uint64_t* full = reinterpret_cast<uint64_t*>(sZ + kAwqSA * TL::kZ);
  uint64_t* empty = full + kAwqSA;
  uint64_t* bfull = empty + kAwqSA;
  uint64_t* bempty = bfull + kAwqSB;
  AccBars* acc = reinterpret_cast<AccBars*>(bempty + kAwqSB);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = K / kAwqBK;
  const int n_tiles = (N + BN - 1) / BN;
  const int m_tiles = (M + kTcBM - 1) / kTcBM;
  const int tiles = n_tiles * m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAwqSA; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kAwqSB; ++s) {
      mbar_init(&bfull[s], kAwqDqWarps);
      mbar_init(&bempty[s], 1);
    }
    acc_bars_init(acc);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_s);
    tma_prefetch_desc(&tm_z);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();  // x tile is re-read by every N tile
      uint32_t kg = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int m0, n0;
        tile_coords(t, m_tiles, n_tiles, BN, m0, n0);
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % kAwqSA;
          if (!(ok = mbar_wait(&empty[s], ((kg / kAwqSA) & 1) ^ 1, kErrWaitEmpty))) break;
          mbar_arrive_expect_tx(&full[s], TL::kTx);
          const int k = kb * kAwqBK;
          const int gi = k / group;
          tma_load_2d_hint(&tm_x, &full[s], sA + s * kAwqABytes, k, m0, keep);
          tma_load_2d(&tm_q, &full[s], sP + s * TL::kP, n0 / 8, k);
          tma_load_2d(&tm_s, &full[s], sS + s * TL::kS, n0, gi);
          tma_load_2d(&tm_z, &full[s], sZ + s * TL::kZ, n0 / 8, gi);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t fmt = Act<T>::kUmmaFmt;  // both operands f16, or both bf16
      constexpr uint32_t idesc = make_idesc(fmt, fmt, /*a K-major*/ 0, /*b MN-major*/ 1, kTcBM, BN);
      uint32_t kg = 0, it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
        const uint32_t a = it & 1;
        if (!(ok = mbar_wait(&acc->empty[a], ((it >> 1) & 1) ^ 1, kErrWaitAccum))) break;
        tc_fence_after();
        const uint32_t d = tmem + a * BN;
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % kAwqSA, sb = kg % kAwqSB;
          ok = mbar_wait(&bfull[sb], (kg / kAwqSB) & 1, kErrWaitDequant) &&
               mbar_wait(&full[s], (kg / kAwqSA) & 1, kErrWaitFull);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * kAwqABytes);
          const uint32_t b0 = smem_u32(sB + sb * kAwqBBytes);
#pragma unroll
          for (int kk = 0; kk < kAwqBK / 16; ++kk) {
            const uint64_t ad = make_sdesc(a0 + kk * 32, 16, 1024);
            const uint64_t bd = make_sdesc(b0 + kk * 2048, 8192, 1024);
            umma_f16(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
          umma_commit(&bempty[sb]);
        }
        if (ok) umma_commit(&acc->full[a]);
      }
    }
  } else if (warp < kTcEpiWarp0 + kTcEpiWarps) {
    // ---------------- epilogue: warp w reads TMEM lanes 32*(w%4) .. +31
    const int quarter = warp & 3;
    uint32_t it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const uint32_t a = it & 1;
      if (!mbar_wait(&acc->full[a], (it >> 1) & 1, kErrWaitAccum)) break;
      tc_fence_after();
      int m0, n0;
        tile_coords(t, m_tiles, n_tiles, BN, m0, n0);
      const int row = m0 + quarter * 32 + lane;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
      for (int ch = 0; ch < BN / 16; ++ch) {
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
      if (lane == 0) mbar_arrive(&acc->empty[a]);
    }
  } else {
    // ---------------- dequant warps: packed int4 stage -> MN-major SW128 B stage (fp16 or bf16)
    // two groups of 8 warps take alternate K-blocks, so two K-blocks are being
    // dequantised while the tensor core consumes a third
    const int dwa = warp - kAwqDqWarp0;
    const int dgrp = dwa / kAwqDqWarps, dw = dwa % kAwqDqWarps;
    const int bblk = lane >> 3, chunk = lane & 7;
    uint32_t kg = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++kg) {
        if (static_cast<int>(kg % kAwqDqGroups) != dgrp) continue;
        const int s = kg % kAwqSA, sb = kg % kAwqSB;
        ok = mbar_wait(&full[s], (kg / kAwqSA) & 1, kErrWaitFull) &&
             mbar_wait(&bempty[sb], ((kg / kAwqSB) & 1) ^ 1, kErrWaitEmpty);
        if (!ok) break;
        // lane = word column of the tile (BN/8 words; a 224-wide tile idles lanes 28..31)
        const bool live = lane < TL::kWords;
        const uint32_t zw = live ? reinterpret_cast<const uint32_t*>(sZ + s * TL::kZ)[lane] : 0u;
        const uint4 sv = live ? reinterpret_cast<const uint4*>(sS + s * TL::kS)[lane] : make_uint4(0u, 0u, 0u, 0u);
        uint32_t zb[4];
        awq_word_biased<T>(zw, zb);
        const AwqScale2 sp[4] = {awq_scale2<T>(sv.x), awq_scale2<T>(sv.y), awq_scale2<T>(sv.z),
                                 awq_scale2<T>(sv.w)};
        const uint32_t* prow = reinterpret_cast<const uint32_t*>(sP + s * TL::kP);
        const uint32_t bbase = smem_u32(sB + sb * kAwqBBytes) + bblk * 8192;
        uint32_t w[kAwqBK / kAwqDqWarps];
#pragma unroll
        for (int rr = 0; rr < kAwqBK / kAwqDqWarps; ++rr)
          w[rr] = live ? prow[(dw * (kAwqBK / kAwqDqWarps) + rr) * TL::kWords + lane] : 0u;
#pragma unroll
        for (int rr = 0; rr < kAwqBK / kAwqDqWarps; ++rr) {
          const int r = dw * (kAwqBK / kAwqDqWarps) + rr;
          uint32_t qb[4];
          awq_word_biased<T>(w[rr], qb);
          uint4 o;
          o.x = awq_dq<T>(qb[0], zb[0], sp[0]);
          o.y = awq_dq<T>(qb[1], zb[1], sp[1]);
          o.z = awq_dq<T>(qb[2], zb[2], sp[2]);
          o.w = awq_dq<T>(qb[3], zb[3], sp[3]);
          const uint32_t addr = bbase + (r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4);
          if (live) st_shared_v4(addr, o);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[sb]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

// ============================================================ FP8 W8A8 GEMM
constexpr int kF8BK = 128;  // bytes (= e4m3 elements) of K per stage
constexpr int kF8Stages = 4;
constexpr int kF8Threads = 32 * (kTcEpiWarp0 + kTcEpiWarps);  // 192
constexpr int kF8ABytes = kTcBM * kF8BK;  // 16 KB
// KSUB 128-byte TMA boxes of K per stage (one wait and one commit of the MMA
// thread per stage).  128-wide tiles run mid-size M: few tiles, each CTA walking
// all of K, where the MMA thread's fixed work per stage (a wait, a commit; ~0.39
// us per 128-byte stage at 14336 x 4096, M = 512) sets the pace, so they take
// 256-byte stages (eight UMMAs per wait and commit) in a 3-deep ring.
template <int BN, int KSUB = 1> struct F8Tile {
  static constexpr int kA = kTcBM * kF8BK * KSUB;  // token rows x KSUB x 128 bytes of K
  static constexpr int kB = BN * kF8BK * KSUB;     // weight rows of the tile x the same
  static constexpr int kStages = KSUB == 2 ? 3 : kF8Stages;
  static constexpr int kSmem = 1024 + kStages * (kA + kB) + 256;
  static_assert(kB % 1024 == 0 && kA % 1024 == 0, "128B-swizzled stages are 1024-byte aligned");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};
constexpr int kF8SmemBytes = F8Tile<256>::kSmem;

template <int BN, int KSUB>
__global__ void __launch_bounds__(kF8Threads, 1)
    fp8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a,
                       const __grid_constant__ CUtensorMap tm_b, __nv_bfloat16* __restrict__ y,
                       const float* __restrict__ sx, const float* __restrict__ sw,
                       const __nv_bfloat16* __restrict__ bias, int M, int K, int N, int group_m) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  using TL = F8Tile<BN, KSUB>;
  constexpr int kS = TL::kStages;
  constexpr int kF8ABytes = TL::kA;
  constexpr int kF8BBytes = TL::kB;
  constexpr int kBK = kF8BK * KSUB;  // bytes of K per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = sA + kS * kF8ABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kS * kF8BBytes);
  uint64_t* empty = full + kS;
  AccBars* acc = reinterpret_cast<AccBars*>(empty + kS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (K + kBK - 1) / kBK;  // a box past K is zero-filled
  const int n_tiles = (N + BN - 1) / BN;
  const int m_tiles = (M + kTcBM - 1) / kTcBM;
  const int tiles = n_tiles * m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    acc_bars_init(acc);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      uint32_t kg = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int m0, n0;
        tile_coords(t, m_tiles, n_tiles, BN, m0, n0, group_m);
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % kS;
          if (!(ok = mbar_wait(&empty[s], ((kg / kS) & 1) ^ 1, kErrWaitEmpty))) break;
          mbar_arrive_expect_tx(&full[s], kF8ABytes + kF8BBytes);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            tma_load_2d_hint(&tm_a, &full[s], sA + s * kF8ABytes + sub * (kTcBM * kF8BK),
                             kb * kBK + sub * kF8BK, m0, keep);
            tma_load_2d(&tm_b, &full[s], sB + s * kF8BBytes + sub * (BN * kF8BK),
                        kb * kBK + sub * kF8BK, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(0, 0, 0, 0, kTcBM, BN);  // e4m3 x e4m3, K-major
      uint32_t kg = 0, it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
        const uint32_t a = it & 1;
        if (!(ok = mbar_wait(&acc->empty[a], ((it >> 1) & 1) ^ 1, kErrWaitAccum))) break;
        tc_fence_after();
        const uint32_t d = tmem + a * BN;
        for (int kb = 0; kb < KB; ++kb, ++kg) {
          const int s = kg % kS;
          if (!(ok = mbar_wait(&full[s], (kg / kS) & 1, kErrWaitFull))) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * kF8ABytes);
          const uint32_t b0 = smem_u32(sB + s * kF8BBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {  // box kk / 4, 32-byte K step kk % 4
            const uint64_t ad = make_sdesc(a0 + (kk >> 2) * (kTcBM * kF8BK) + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = make_sdesc(b0 + (kk >> 2) * (BN * kF8BK) + (kk & 3) * 32, 16, 1024);
            umma_f8(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc->full[a]);
      }
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quarters 2,3,0,1
    const int quarter = warp & 3;
    uint32_t it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const uint32_t a = it & 1;
      if (!mbar_wait(&acc->full[a], (it >> 1) & 1, kErrWaitAccum)) break;
      tc_fence_after();
      int m0, n0;
      tile_coords(t, m_tiles, n_tiles, BN, m0, n0, group_m);
      const int row = m0 + quarter * 32 + lane;
      const float rs = row < M ? sx[row] : 0.f;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
      for (int ch = 0; ch < BN / 16; ++ch) {
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
              const uint32_t p = packed[e >> 1];
              reinterpret_cast<uint16_t*>(dst)[e] = static_cast<uint16_t>((e & 1) ? (p >> 16) : (p & 0xFFFFu));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc->empty[a]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

}  // namespace lmrs
