// awq_tmem.cuh — AWQ W4A16 linear for 9..32 tokens with the dequantised weights
// staged in tensor memory (tcgen05.mma with the A operand in TMEM).
//
// Why: on sm_100 the register-fed mma.sync GEMV spends as many issue cycles
// on the nibble unpack (half-rate integer ops) as on the MMAs, the two do not
// overlap, and its MMA count grows with the token count.  Here the CUDA cores
// only unpack and dequantise (one prmt and two lop3 per 4 weights, then an
// exact fp16 (q - z) * s) and write the fp16 weights into TMEM with
// tcgen05.st; the MMAs run asynchronously at a cost that does not depend on
// the token count (16 or 32 columns).
//
// Measured on the B200 (one CTA, clock64 around back-to-back UMMAs): the MMAs
// one thread issues complete one after another, ~171 SM cycles each for any
// N <= 256 (TMEM or shared-memory A, one or several accumulators), while
// UMMAs from different warps overlap (eight issuing warps: ~22 cycles per
// M=128, N=16, K=16 UMMA).  A single issuer held this kernel to ~1370 cycles
// per 64-row box, so four warps issue here, each into its own accumulator.
//
// Layout of one CTA: a strip of 32 packed words (256 output channels) and a
// K range (clusters of C CTAs split K; C a power of two).
//   * Weight ring (warp 0, SW slots): boxes of 64 rows x 32 words
//     (8 KB) with the group's scale and zero rows.  A slot is free again as
//     soon as the four dequant warps have read it (one arrive each), so the
//     ring runs ahead of the MMAs.  None of it depends on the previous kernel:
//     it is issued before griddepcontrol.wait.
//   * Token ring (warp 9, SX slots): the 64-k token tile of a box
//     [NT rows x 128 B, 128-byte swizzle; rows >= M are the zero fill].  TMEM
//     A stage b % R is released by the box's MMAs (one tcgen05.commit per
//     issuer per box on mempty[b % R], count 4); the token slot of box b is
//     released by the dequant warps once they have seen that commit (at box
//     b + R), so the token ring runs SX - R boxes ahead of the MMAs without a
//     second commit (a commit costs the issuing thread about as much as an
//     MMA).
//   * Dequant (warps 1-4, one per TMEM lane quarter): the 128-row MMA group g
//     is the word half 16g .. 16g+15 of the strip; warp qv takes the 16-byte
//     chunk 4g + qv of each row with ldmatrix.trans (the weight box arrives
//     with the 128-byte swizzle, so its 8-row reads are conflict-free) and
//     finds rows r, r+1 of each nibble in the two halves of one register: one
//     lop3 per nibble makes the half2 (1024 + q_r, 1024 + q_r+1) (nibbles 0,
//     2) or (64 + q_r, 64 + q_r+1) (nibbles 1, 3: magic 64, ulp 1/16); with
//     bf16 activations each nibble is shifted to bits 0-3 first (128 + q).
//     Subtracting the same-biased zero is exact and the scale product rounds
//     once: bit for bit the dequant T_rne((q - z) * s) of the activation type.
//     tcgen05.st 16x128b lays each channel along one TMEM lane.  A TMEM stage
//     holds a whole 64-row box (64 columns: group g, k-pair kp at column
//     32g + kp) and is handed over with one arrive per warp.
//   * MMA (warps 5-8, lane 0 each): issuer p takes word half jj = p & 1 and
//     the 16-row steps 2 (p >> 1) and 2 (p >> 1) + 1 of every box: two UMMAs
//     M=128, N=NT, K=16, B = the token tile (x is already K-major), into its
//     own accumulator D[p] (NT columns) over the CTA's whole K range.
//   * Epilogue: lane L of quarter qv, group jj -> channel
//     8 (16 jj + 4 qv + (L & 7) / 2) + 2 (L >> 3) + (L & 1) (the AWQ nibble
//     order {0,2,4,6,1,3,5,7}) holds D[jj] + D[jj + 2]; partial sums go to
//     the owner CTA of each channel slice with 16-byte st.async; the owner adds
//     the C slices in rank order plus the bias and stores fp16.
// Every mbarrier wait is bounded; on expiry the kernel records the site in the
// device error word and unwinds; TMEM is always released.
#pragma once
#include <cooperative_groups.h>
#include "awq_gemv.cuh"
#include "lmrs_ptx.cuh"

namespace lmrs {

constexpr int kAtWords = 32;      // packed words per strip
constexpr int kAtCols = 256;      // output channels per strip
constexpr int kAtRows = 64;       // rows per TMA box (4 MMA steps of 16)
constexpr int kAtDqWarp0 = 1;
constexpr int kAtDqWarps = 4;     // one per TMEM lane quarter
constexpr int kAtMmaWarp0 = kAtDqWarp0 + kAtDqWarps;
constexpr int kAtIssuers = 4;     // MMA warps, one accumulator each
constexpr int kAtXWarp = kAtMmaWarp0 + kAtIssuers;  // token-tile producer
constexpr int kAtThreads = 32 * (kAtXWarp + 1);     // 320: the two producers wait on
                                                    // different barriers, so each has a warp
constexpr int kAtMaxCluster = 8;

template <int NT>
struct AtLayout {
  static constexpr int kWStages = NT == 16 ? 8 : 5;  // weight ring depth
  static constexpr int kXStages = NT == 16 ? 8 : 6;  // token ring depth
  static constexpr int kAStages = NT == 16 ? 3 : 2;  // TMEM A stages
  static constexpr int kW = kAtRows * kAtWords * 4;  // 8 KB
  static constexpr int kX = NT * 128;                // 64 k x NT tokens, fp16, swizzled
  static constexpr int kS = kAtCols * 2;
  static constexpr int kZ = kAtWords * 4;
  static constexpr int kSZ = kS + kZ;                // 640: 128-byte aligned rows
  static constexpr uint32_t kWTx = kW + kS + kZ;
  static constexpr int kPitch = NT + 4;              // recv row pitch (floats)
  static constexpr int kRecv = kAtCols * kPitch * 4;
  static constexpr uint32_t kTmemA = kAtIssuers * NT;  // A stages after the accumulators
  static constexpr uint32_t kTmemCols = 256;
  static_assert(kAtIssuers * NT + 64 * kAStages <= 256, "TMEM columns");
  static constexpr int kBars = 512;
  static constexpr int kSmem =
      1024 + kWStages * kW + kXStages * kX + kWStages * kSZ + kRecv + kBars;
  static_assert(kW % 1024 == 0 && kX % 1024 == 0, "swizzled token tiles are 1024-byte aligned");
  static_assert(kSZ % 128 == 0, "TMA destinations are 128-byte aligned");
  static_assert(kXStages >= kAStages, "token slots are released R boxes after their MMAs");
  static_assert((2 * kWStages + 2 * kXStages + 2 * kAStages + 2) * 8 + 4 <= kBars, "barrier area");
  static_assert(2 * (kSmem + 1024) <= 228 * 1024, "two CTAs per SM");
};

template <int NT, typename T>
__global__ void __launch_bounds__(kAtThreads, 2) awq_tmem_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_x,
    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
    T* __restrict__ y, const T* __restrict__ bias, int M, int K, int N, int group) {
  using L = AtLayout<NT>;
  constexpr int SW = L::kWStages;
  constexpr int R = L::kAStages;
  constexpr int SX = L::kXStages;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned by byte offset, so every access stays a shared-memory one
  uint8_t* wring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* xring = wring + SW * L::kW;
  uint8_t* sz = xring + SX * L::kX;
  float* recv = reinterpret_cast<float*>(sz + SW * L::kSZ);
  uint64_t* wfull = reinterpret_cast<uint64_t*>(recv + kAtCols * L::kPitch);
  uint64_t* wempty = wfull + SW;
  uint64_t* xfull = wempty + SW;
  uint64_t* xempty = xfull + SX;
  uint64_t* afull = xempty + SX;
  uint64_t* mempty = afull + R;
  uint64_t* dfull = mempty + R;
  uint64_t* recv_bar = dfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int strip = blockIdx.x / C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb_all = K / kAtRows;
  const int b_lo = static_cast<int>((static_cast<long long>(rank) * nb_all) / C);
  const int b_hi = static_cast<int>((static_cast<long long>(rank + 1) * nb_all) / C);
  const int nbox = b_hi - b_lo;
  const int M4 = (M + 3) >> 2;  // 16-byte partial chunks per channel

  if (threadIdx.x == 0) {
    for (int i = 0; i < SW; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], kAtDqWarps);  // one arrive per dequant warp once read
    }
    for (int i = 0; i < SX; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], kAtDqWarps);  // the box's MMAs are known to be done
    }
    for (int i = 0; i < R; ++i) {
      mbar_init(&afull[i], kAtDqWarps);   // TMEM stage written
      mbar_init(&mempty[i], kAtIssuers);  // one commit per issuer: MMAs of the box done
    }
    mbar_init(dfull, kAtIssuers);
    mbar_init(recv_bar, 1);
    mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(kAtCols * M4 * 16));
    fence_mbar_init();
  }
  if (warp == kAtMmaWarp0) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_arrive_relaxed();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ weight TMA ring
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_z);
      const int c0 = strip * kAtWords;
      for (int b = 0; b < nbox; ++b) {
        const int s = b % SW;
        if (b >= SW && !mbar_wait(&wempty[s], ((b / SW) - 1) & 1, kErrWaitEmpty)) break;
        const int krow = (b_lo + b) * kAtRows;
        const int gi = krow / group;
        mbar_arrive_expect_tx(&wfull[s], L::kWTx);
        tma_load_2d(&tm_q, &wfull[s], wring + s * L::kW, c0, krow);
        tma_load_2d(&tm_s, &wfull[s], sz + s * L::kSZ, strip * kAtCols, gi);
        tma_load_2d(&tm_z, &wfull[s], sz + s * L::kSZ + L::kS, c0, gi);
      }
    }
  } else if (warp == kAtXWarp) {
    // ------------------------------------------------------- token TMA ring
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      pdl_wait();  // the tokens are the previous kernel's output
      for (int b = 0; b < nbox; ++b) {
        const int sx = b % SX;
        if (b >= SX && !mbar_wait(&xempty[sx], ((b / SX) - 1) & 1, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&xfull[sx], static_cast<uint32_t>(L::kX));
        tma_load_2d(&tm_x, &xfull[sx], xring + sx * L::kX, (b_lo + b) * kAtRows, 0);
      }
    }
  } else if (warp >= kAtMmaWarp0) {
    // ---------------------------------------------------------- MMA (warps 5-8)
    if (lane == 0) {
      constexpr uint32_t fmt = Act<T>::kUmmaFmt;  // both operands f16, or both bf16
      constexpr uint32_t idesc = make_idesc(fmt, fmt, 0, 0, 128, NT);  // K-major
      const int p = warp - kAtMmaWarp0;
      const int jj = p & 1, st0 = 2 * (p >> 1);
      const uint32_t d = tmem + static_cast<uint32_t>(p * NT);
      for (int b = 0; b < nbox; ++b) {
        const int a = b % R, sx = b % SX;
        if (!mbar_wait(&xfull[sx], (b / SX) & 1, kErrWaitFull)) break;
        if (!mbar_wait(&afull[a], (b / R) & 1, kErrWaitDequant)) break;
        tc_fence_after();
        const uint32_t xs_addr = smem_u32(xring + sx * L::kX);
        const uint32_t acol = tmem + L::kTmemA + a * 64;
#pragma unroll
        for (int st = st0; st < st0 + 2; ++st)
          umma_f16_tmem_a(d, acol + 32 * jj + 8 * st, make_sdesc(xs_addr + st * 32, 16, 1024),
                          idesc, (b | (st - st0)) != 0 ? 1u : 0u);
        umma_commit(&mempty[a]);  // TMEM stage a (and, via the dequant, token slot sx) free
      }
      umma_commit(dfull);  // also fires (over no MMAs) if a wait gave up
    }
  } else {
    // ------------------------------------------------- dequant + epilogue
    // Warp qv owns TMEM lane quarter qv; for word half g (MMA group g, words
    // 16g .. 16g+15) it dequantises the 16-byte chunk 4g + qv of every row.
    // ldmatrix.trans of 32 rows x 16 bytes gives thread t = 4c + pp, register
    // i, half-word c of the chunk for rows 8i + 2pp (low) and 8i + 2pp + 1
    // (high): the row pair of each of its four nibbles already sits in the two
    // halves, so one lop3 per nibble (after one shift for the upper byte)
    // makes the biased half2.  tcgen05.st 16x128b puts register 2j at lane c,
    // column 4j + pp and 2j + 1 at lane c + 8: nibbles 0, 1 go to lanes c, c + 8,
    // nibbles 2, 3 to lanes 16 + c, 24 + c, and each lane holds one channel
    // with k-pair kp in column kp.  64 wavefronts per box against 256 for
    // per-row 4-byte loads (four lanes read each word).
    const int qv = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(qv * 32) << 16;
    const int c = lane >> 2;
    const int codd = c & 1;
    const uint32_t sdup = codd ? 0x3232u : 0x1010u;  // prmt: duplicate the high / low half
    bool ok = true;
    for (int b = 0; b < nbox && ok; ++b) {
      const int s = b % SW, a = b % R;
      if (!(ok = mbar_wait(&wfull[s], (b / SW) & 1, kErrWaitFull))) break;
      const uint8_t* wsl = wring + s * L::kW;
      const uint8_t* szb = sz + s * L::kSZ;
      uint32_t zz[2][4];
      AwqScale2 ss[2][4];
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int word = 16 * g + 4 * qv + (c >> 1);
        const uint32_t zw = ld_s32(szb + L::kS + 4 * word) >> (16 * codd);
        const uint4 sv = ld_s128(szb + 16 * word);  // scales of channels 8 word .. + 7
        const uint32_t s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          zz[g][n] = awq_zero_pair<T>((zw >> (4 * n)) & 0xFu, n);
          ss[g][n] = awq_scale2<T>(prmt(s4[n], s4[n], sdup));  // channel 8 word + 2n + codd
        }
      }
      // TMEM stage a was last read by the MMAs of box b - R (mempty[a] phase
      // (b - R) / R; the next phase needs this box's own afull arrive)
      if (b >= R) {
        if (!(ok = mbar_wait(&mempty[a], ((b / R) - 1) & 1, kErrWaitAccum))) break;
        if (lane == 0) mbar_arrive(&xempty[(b - R) % SX]);  // box b - R's token slot
      }
      const uint32_t acol = tmem + lane_addr + L::kTmemA + a * 64;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = 32 * h + lane;  // row this lane addresses for ldmatrix
          uint32_t d[4];
          ldsm_x4_t(d, smem_u32(wsl + r * 128 + (((4 * g + qv) ^ (r & 7)) << 4)));
          uint32_t lo[8], hi[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            lo[2 * i] = awq_dq<T>(awq_nib_pair<T>(d[i], 0), zz[g][0], ss[g][0]);
            lo[2 * i + 1] = awq_dq<T>(awq_nib_pair<T>(d[i], 1), zz[g][1], ss[g][1]);
            hi[2 * i] = awq_dq<T>(awq_nib_pair<T>(d[i], 2), zz[g][2], ss[g][2]);
            hi[2 * i + 1] = awq_dq<T>(awq_nib_pair<T>(d[i], 3), zz[g][3], ss[g][3]);
          }
          tmem_st16x128b_x4(acol + 32 * g + 16 * h, lo);
          tmem_st16x128b_x4(acol + (16u << 16) + 32 * g + 16 * h, hi);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[s]);  // every read of slot s is done
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[a]);
    }

    // TMEM lane L of quarter qv in group g: channel 8 (16g + 4qv + (L & 7) / 2)
    // + 2 (L >> 3) + (L & 1)
    const int ch0 = 8 * (4 * qv + ((lane & 7) >> 1)) + 2 * (lane >> 3) + (lane & 1);
    const int ch1 = ch0 + 128;
    // ---- epilogue: channel ch0 = D[0] + D[2], ch1 = D[1] + D[3], 16 tokens at
    // a time -> the owner CTA of each channel slice
    const bool have = mbar_wait(dfull, 0, kErrWaitAccum) && ok && nbox > 0;
    tc_fence_after();
    cluster_wait_acquire();
    const int cw = kAtCols / C;
    {
      const int r0 = ch0 / cw, l0 = ch0 - r0 * cw;
      const int r1 = ch1 / cw, l1 = ch1 - r1 * cw;
      const uint32_t d0 = mapa_shared(smem_u32(recv + (rank * cw + l0) * L::kPitch),
                                      static_cast<uint32_t>(r0));
      const uint32_t d1 = mapa_shared(smem_u32(recv + (rank * cw + l1) * L::kPitch),
                                      static_cast<uint32_t>(r1));
      const uint32_t b0 = mapa_shared(smem_u32(recv_bar), static_cast<uint32_t>(r0));
      const uint32_t b1 = mapa_shared(smem_u32(recv_bar), static_cast<uint32_t>(r1));
#pragma unroll
      for (int c = 0; c < NT / 16; ++c) {
        if (4 * c >= M4) break;
        float acc0[16], acc1[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) acc0[e] = acc1[e] = 0.f;
        if (have) {
#pragma unroll
          for (int p = 0; p < kAtIssuers; ++p) {
            uint32_t r[16];
            tmem_ld16(tmem + lane_addr + p * NT + c * 16, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              if (p & 1) acc1[e] += __uint_as_float(r[e]);
              else acc0[e] += __uint_as_float(r[e]);
            }
          }
        }
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int m4 = 4 * c + k4;
          if (m4 < M4) {
            st_async_v4(d0 + m4 * 16, make_float4(acc0[4 * k4], acc0[4 * k4 + 1],
                                                  acc0[4 * k4 + 2], acc0[4 * k4 + 3]), b0);
            st_async_v4(d1 + m4 * 16, make_float4(acc1[4 * k4], acc1[4 * k4 + 1],
                                                  acc1[4 * k4 + 2], acc1[4 * k4 + 3]), b1);
          }
        }
      }
    }
    tc_fence_before();
    // owner: thread = (channel c2, 4 tokens); C slices in rank order, + bias
    const bool rok = mbar_wait_cluster(recv_bar, 0, kErrWaitCluster);
    pdl_wait();
    if (rok) {
      for (int e = threadIdx.x - 32 * kAtDqWarp0; e < M4 * cw; e += 32 * kAtDqWarps) {
        const int m4 = e / cw, c2 = e - m4 * cw;
        const int n = strip * kAtCols + rank * cw + c2;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int src = 0; src < C; ++src) {
          const float4 p =
              *reinterpret_cast<const float4*>(recv + (src * cw + c2) * L::kPitch + 4 * m4);
          acc.x += p.x;
          acc.y += p.y;
          acc.z += p.z;
          acc.w += p.w;
        }
        if (n < N) {
          const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
          const float bn = bias != nullptr ? Act<T>::to_float(bias[n]) : 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int m = 4 * m4 + j;
            if (m < M) y[static_cast<int64_t>(m) * N + n] = Act<T>::from_float(a4[j] + bn);
          }
        }
      }
    }
  }
  if (warp == 0 || warp >= kAtMmaWarp0) {
    cluster_wait_acquire();  // every thread arrived at the start; match the wait
    pdl_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kAtMmaWarp0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace lmrs
