// awq_gemm_swap.cuh — AWQ W4A16 linear for small and medium batches (M <= 128),
// tcgen05 with the operands swapped and split-K over a thread-block cluster.
//
// For M up to ~128 the weight stream (K*N/2 bytes) still dominates, but a
// 128-token tile GEMM has only N/256 tiles to spread over 148 SMs and walks all
// of K serially per tile.  Here:
//   * the MMA "M" side is 128 output features (the dequantised weight tile W^T,
//     operand A, MN-major: n is contiguous, exactly the AWQ word order), the
//     "N" side is the padded token count NT in {16, 32, 64, 128} (operand B =
//     the x tile, K-major, TMA with 128-byte swizzle);
//   * dequant warps turn TMA-staged packed int4 (16 words x 64 k rows) plus the
//     group's zeros/scales into A stages of the activation type (fp16 or
//     bf16) in the UMMA MN-major SW128 layout (canonical T_rne((q - z) * s),
//     bit-identical to lmrs_awq_dequant_dtype);
//   * K is split over a cluster of C CTAs (grid = N/128 tiles x C, about two CTAs
//     per SM); each CTA's 128 x NT fp32 accumulator goes TMEM -> shared memory
//     and the cluster sums the C partials through distributed shared memory.
//     No global scratch, one launch.
//   warp 0: TMA producer; warp 1: TMEM owner + MMA issuer; warps 2..9: dequant,
//   then epilogue.  All mbarrier waits are bounded (lmrs_ptx.cuh).
#pragma once
#include <cooperative_groups.h>
#include "tc_gemm.cuh"

namespace lmrs {

constexpr int kSwBN = 128;       // output features per CTA (MMA M)
constexpr int kSwBK = 64;        // k rows per stage
constexpr int kSwSA = 4;         // TMA stages
constexpr int kSwSB = 2;         // dequantised A stages
constexpr int kSwDqWarps = 8;
constexpr int kSwThreads = 32 * (2 + kSwDqWarps);  // 320
constexpr int kSwPBytes = kSwBK * (kSwBN / 8) * 4;  // 4 KB packed
constexpr int kSwABytes = kSwBN * kSwBK * 2;        // 16 KB 16-bit A stage
constexpr int kSwSBytes = kSwBN * 2;                // 256 B scales
constexpr int kSwZBytes = (kSwBN / 8) * 4;          // 64 B zeros

__host__ __device__ constexpr int sw_xbytes(int nt) { return nt * kSwBK * 2; }
__host__ __device__ constexpr int sw_stage_bytes(int nt) {
  return sw_xbytes(nt) + kSwPBytes + kSwSBytes + kSwZBytes;
}
__host__ __device__ constexpr int sw_smem_bytes(int nt) {
  return 1024 + kSwSA * ((sw_stage_bytes(nt) + 1023) / 1024 * 1024) + kSwSB * kSwABytes + 256;
}

template <int NT, typename T>
__global__ void __launch_bounds__(kSwThreads, 2)
    awq_gemm_swap_kernel(const __grid_constant__ CUtensorMap tm_x,
                         const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_s,
                         const __grid_constant__ CUtensorMap tm_z, T* __restrict__ y,
                         const T* __restrict__ bias, int M, int K, int N, int group) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  namespace cg = cooperative_groups;
  constexpr int kStage = (sw_stage_bytes(NT) + 1023) / 1024 * 1024;
  constexpr int kX = sw_xbytes(NT);
  constexpr uint32_t kTmemCols = NT < 32 ? 32 : NT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sT = smem;                       // TMA stages: [x tile | packed | scales | zeros]
  uint8_t* sA = sT + kSwSA * kStage;        // dequantised A stages
  uint64_t* full = reinterpret_cast<uint64_t*>(sA + kSwSB * kSwABytes);
  uint64_t* empty = full + kSwSA;
  uint64_t* afull = empty + kSwSA;
  uint64_t* aempty = afull + kSwSB;
  uint64_t* accb = aempty + kSwSB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int tile = blockIdx.x / C;
  const int n0 = tile * kSwBN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = K / kSwBK;
  const int kb_lo = static_cast<int>((static_cast<long long>(rank) * KB) / C);
  const int kb_hi = static_cast<int>((static_cast<long long>(rank + 1) * KB) / C);
  const int nkb = kb_hi - kb_lo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSwSA; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kSwSB; ++s) {
      mbar_init(&afull[s], kSwDqWarps);
      mbar_init(&aempty[s], 1);
    }
    mbar_init(accb, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_s);
    tma_prefetch_desc(&tm_z);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool acc_ok = false;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % kSwSA;
        if (!mbar_wait(&empty[s], ((i / kSwSA) & 1) ^ 1, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&full[s], sw_stage_bytes(NT));
        const int k = (kb_lo + i) * kSwBK;
        const int gi = k / group;
        uint8_t* st = sT + s * kStage;
        tma_load_2d(&tm_x, &full[s], st, k, 0);
        tma_load_2d(&tm_q, &full[s], st + kX, n0 / 8, k);
        tma_load_2d(&tm_s, &full[s], st + kX + kSwPBytes, n0, gi);
        tma_load_2d(&tm_z, &full[s], st + kX + kSwPBytes + kSwSBytes, n0 / 8, gi);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // A = W^T tile (MN-major), B = x tile (K-major), D[n][m] in TMEM
      constexpr uint32_t fmt = Act<T>::kUmmaFmt;  // both operands f16, or both bf16
      constexpr uint32_t idesc = make_idesc(fmt, fmt, /*a MN-major*/ 1, /*b K-major*/ 0, kSwBN, NT);
      bool ok = true;
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % kSwSA, sa = i % kSwSB;
        ok = mbar_wait(&afull[sa], (i / kSwSB) & 1, kErrWaitDequant) &&
             mbar_wait(&full[s], (i / kSwSA) & 1, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + sa * kSwABytes);
        const uint32_t b0 = smem_u32(sT + s * kStage);
#pragma unroll
        for (int kk = 0; kk < kSwBK / 16; ++kk) {
          const uint64_t ad = make_sdesc(a0 + kk * 2048, 8192, 1024);
          const uint64_t bd = make_sdesc(b0 + kk * 32, 16, 1024);
          umma_f16(tmem, ad, bd, idesc, (i | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        umma_commit(&aempty[sa]);
      }
      if (ok && nkb > 0) umma_commit(accb);
    }
  } else {
    // ---------------- dequant: lane -> word column j = lane % 16, rows 2*it + lane/16
    const int dw = warp - 2;
    const int j = lane & 15, half = lane >> 4;
    const int blk = j >> 3, chunk = j & 7;
    bool ok = true;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kSwSA, sa = i % kSwSB;
      ok = mbar_wait(&full[s], (i / kSwSA) & 1, kErrWaitFull) &&
           mbar_wait(&aempty[sa], ((i / kSwSB) & 1) ^ 1, kErrWaitEmpty);
      if (!ok) break;
      const uint8_t* st = sT + s * kStage;
      const uint32_t* pk = reinterpret_cast<const uint32_t*>(st + kX);
      const uint4 sv = reinterpret_cast<const uint4*>(st + kX + kSwPBytes)[j];
      const uint32_t zw = reinterpret_cast<const uint32_t*>(st + kX + kSwPBytes + kSwSBytes)[j];
      uint32_t zb[4];
      awq_word_biased<T>(zw, zb);
      const AwqScale2 sp[4] = {awq_scale2<T>(sv.x), awq_scale2<T>(sv.y), awq_scale2<T>(sv.z),
                               awq_scale2<T>(sv.w)};
      const uint32_t abase = smem_u32(sA + sa * kSwABytes) + blk * 8192;
      uint32_t w[4];
#pragma unroll
      for (int it = 0; it < 4; ++it) w[it] = pk[(dw * 8 + 2 * it + half) * 16 + j];
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int r = dw * 8 + 2 * it + half;
        uint32_t qb[4];
        awq_word_biased<T>(w[it], qb);
        uint4 o;
        o.x = awq_dq<T>(qb[0], zb[0], sp[0]);
        o.y = awq_dq<T>(qb[1], zb[1], sp[1]);
        o.z = awq_dq<T>(qb[2], zb[2], sp[2]);
        o.w = awq_dq<T>(qb[3], zb[3], sp[3]);
        st_shared_v4(abase + (r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4), o);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[sa]);
    }
    // ---------------- epilogue part 1: TMEM -> registers (after the last MMA)
    acc_ok = ok && nkb > 0 && mbar_wait(accb, 0, kErrWaitAccum);
    acc_ok = __all_sync(0xffffffffu, acc_ok);  // tcgen05.ld below is warp-collective
  }

  // Partial sums to shared memory (the stages are drained once every role is done).
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem);  // [NT][kSwBN]
  if (warp >= 2) {
    const int q = warp & 3;            // TMEM lane quarter: features 32q .. 32q+31
    const int hsel = (warp - 2) >> 2;  // two warps per quarter split the token columns
    const int n_l = q * 32 + lane;
    tc_fence_after();
    for (int c0 = hsel * 16; c0 < NT; c0 += 32) {
      uint32_t r[16];
      if (acc_ok) {
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) r[e] = 0u;  // no K rows here (or a wait expired)
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) red[(c0 + e) * kSwBN + n_l] = __uint_as_float(r[e]);
    }
    tc_fence_before();
  }
  cluster.sync();
  const int f0 = (rank * kSwBN) / C, f1 = ((rank + 1) * kSwBN) / C;
  const int nf = f1 - f0;
  for (int e = threadIdx.x; e < M * nf; e += blockDim.x) {
    const int m = e / nf;
    const int f = f0 + (e - m * nf);
    const int n = n0 + f;
    float v = 0.f;
    for (int r = 0; r < C; ++r) v += cluster.map_shared_rank(red, r)[m * kSwBN + f];
    if (n < N) {
      if (bias != nullptr) v += Act<T>::to_float(bias[n]);
      y[static_cast<int64_t>(m) * N + n] = Act<T>::from_float(v);
    }
  }
  cluster.sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace lmrs
