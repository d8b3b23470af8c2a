// awq_tmem.cuh — AWQ W4A16 linear for 9..32 tokens with the dequantised weights
// staged in tensor memory (tcgen05.mma with the A operand in TMEM).
//
// Why: on sm_100 the register-fed mma.sync GEMV spends as many issue cycles
// on the nibble unpack (half-rate integer ops) as on the MMAs, the two do not
// overlap, and its MMA count grows with the token count.  Here the CUDA cores
// only unpack and dequantise (one prmt and two lop3 per 4 weights, then an
// exact fp16 (q - z) * s), write the fp16 weights into TMEM with tcgen05.st,
// and one thread issues the MMAs, which run asynchronously at a cost that does
// not depend on the token count (16 or 32 columns).  The TMEM store bandwidth
// (about that of shared memory) bounds the unpack rate, so at 1..8 tokens the
// register-fed GEMV stays ahead; from 17 tokens (9 on wide N) this kernel is.
//
// Layout of one CTA: a strip of 32 packed words (256 output channels) and a
// K range (clusters of C CTAs split K; C a power of two).
//   * TMA ring (warp 0): boxes of 64 rows x 32 words (8 KB), the matching
//     64-k tile of the tokens [NT rows x 128 B, 128-byte swizzle; rows >= M
//     are the zero fill], and the group's scale and zero rows.  Weights of the
//     first stages go out before griddepcontrol.wait.
//   * Dequant (warps 1-4, 128 threads = 128 TMEM lanes): lane 4w + q owns byte
//     q of word w, i.e. nibbles 2q and 2q+1.  For rows r, r+1 (r even) one
//     prmt gathers byte q of both words and one lop3 per nibble makes the
//     half2 (1024 + q_r, 1024 + q_r+1) (low nibble) or (64 + q_r, 64 + q_r+1)
//     (high nibble: magic 64, ulp 1/16).  Subtracting the same-biased zero is
//     exact and the multiply by the scale rounds once: bit for bit the fp16
//     dequant fp16_rne((q - z) * s).  The two half2 are K elements (r, r+1) of
//     MMA jj = 0 (low) and jj = 1 (high).  A TMEM stage holds a whole 64-row
//     box (64 columns, two 32-column tcgen05.st per thread) and is handed over
//     with one arrive per warp: per-step stores, arrives and commits cost more
//     than the MMAs themselves.
//   * MMA (warp 5, one thread): per box eight UMMAs M=128, N=NT, K=16 (two per
//     16-row step), B = the token tile (x is already K-major: no transform),
//     D[jj] accumulated over the CTA's whole K range in TMEM; two commits per
//     box (TMEM stage free, TMA slot free).
//   * Epilogue: lane 4w + q, jj -> channel 8w + ORDER[2q + jj]
//     (ORDER = {0,2,4,6,1,3,5,7}); partial sums go to the owner CTA of each
//     channel slice with 16-byte st.async; the owner adds the C slices in rank
//     order plus the bias and stores fp16.
#pragma once
#include <cooperative_groups.h>
#include "awq_gemv.cuh"
#include "lmrs_ptx.cuh"

namespace lmrs {

constexpr int kAtWords = 32;      // packed words per strip
constexpr int kAtCols = 256;      // output channels per strip
constexpr int kAtRows = 64;       // rows per TMA box (4 MMA steps of 16)
constexpr int kAtThreads = 192;   // TMA, 4 dequant warps, MMA
constexpr int kAtAStages = 2;     // TMEM A ring (one 64-row box = 64 columns each)
constexpr int kAtMaxCluster = 8;

template <int NT>
struct AtLayout {
  static constexpr int kStages = NT == 16 ? 6 : 4;
  static constexpr int kW = kAtRows * kAtWords * 4;  // 8 KB
  static constexpr int kX = NT * 128;                // 64 k x NT tokens, fp16, swizzled
  static constexpr int kSlot = kW + kX;
  static constexpr int kS = kAtCols * 2;
  static constexpr int kZ = kAtWords * 4;
  static constexpr int kSZ = kS + kZ;                // 640: 128-byte aligned rows
  static constexpr uint32_t kTx = kW + kX + kS + kZ;
  static constexpr int kPitch = NT + 4;              // recv row pitch (floats)
  static constexpr int kRecv = kAtCols * kPitch * 4;
  static constexpr uint32_t kTmemA = 2 * NT;         // A stages after the two accumulators
  static constexpr uint32_t kTmemCols = 256;
  static_assert(2 * NT + 64 * kAtAStages <= 256, "TMEM columns");
  static constexpr int kSmem = 1024 + kStages * kSlot + kStages * kSZ + kRecv + 256;
  static_assert(kSlot % 1024 == 0, "swizzled token tiles need 1024-byte aligned slots");
  static_assert(kSZ % 128 == 0, "TMA destinations are 128-byte aligned");
  static_assert(2 * kSmem <= 228 * 1024, "two CTAs per SM");
};

template <int NT>
__global__ void __launch_bounds__(kAtThreads, 2) awq_tmem_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_x,
    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
    __half* __restrict__ y, const __half* __restrict__ bias, int M, int K, int N, int group) {
  using L = AtLayout<NT>;
  constexpr int S = L::kStages;
  constexpr int R = kAtAStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sz = ring + S * L::kSlot;
  float* recv = reinterpret_cast<float*>(sz + S * L::kSZ);
  uint64_t* full = reinterpret_cast<uint64_t*>(recv + kAtCols * L::kPitch);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;
  uint64_t* aempty = afull + R;
  uint64_t* dfull = aempty + R;
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
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < R; ++i) {
      mbar_init(&afull[i], 4);  // one arrive per dequant warp
      mbar_init(&aempty[i], 1);
    }
    mbar_init(dfull, 1);
    mbar_init(recv_bar, 1);
    mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(kAtCols * M4 * 16));
    fence_mbar_init();
  }
  if (warp == 5) {
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
    // ------------------------------------------------------------ TMA ring
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_z);
      const int c0 = strip * kAtWords;
      auto load_weights = [&](int b, int s) {
        const int krow = (b_lo + b) * kAtRows;
        const int gi = krow / group;
        mbar_arrive_expect_tx(&full[s], L::kTx);
        tma_load_2d(&tm_q, &full[s], ring + s * L::kSlot, c0, krow);
        tma_load_2d(&tm_s, &full[s], sz + s * L::kSZ, strip * kAtCols, gi);
        tma_load_2d(&tm_z, &full[s], sz + s * L::kSZ + L::kS, c0, gi);
      };
      auto load_tokens = [&](int b, int s) {
        tma_load_2d(&tm_x, &full[s], ring + s * L::kSlot + L::kW, (b_lo + b) * kAtRows, 0);
      };
      const int pre = nbox < S ? nbox : S;
      for (int b = 0; b < pre; ++b) load_weights(b, b);
      pdl_wait();  // the tokens are the previous kernel's output
      for (int b = 0; b < pre; ++b) load_tokens(b, b);
      for (int b = pre; b < nbox; ++b) {
        const int s = b % S;
        if (!mbar_wait(&empty[s], ((b / S) - 1) & 1, kErrWaitEmpty)) break;
        load_weights(b, s);
        load_tokens(b, s);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(0, 0, 0, 0, 128, NT);  // f16 x f16, K-major
      bool ok = true;
      for (int b = 0; b < nbox && ok; ++b) {
        const int s = b % S;
        if (!(ok = mbar_wait(&full[s], (b / S) & 1, kErrWaitFull))) break;
        const int a = b % R;
        if (!(ok = mbar_wait(&afull[a], (b / R) & 1, kErrWaitDequant))) break;
        tc_fence_after();
        const uint32_t xs_addr = smem_u32(ring + s * L::kSlot + L::kW);
        const uint32_t acol = tmem + L::kTmemA + a * 64;
#pragma unroll
        for (int st = 0; st < kAtRows / 16; ++st) {
          const uint64_t bd = make_sdesc(xs_addr + st * 32, 16, 1024);
          const uint32_t acc = (b | st) != 0 ? 1u : 0u;
          umma_f16_tmem_a(tmem, acol + st * 16, bd, idesc, acc);
          umma_f16_tmem_a(tmem + NT, acol + st * 16 + 8, bd, idesc, acc);
        }
        umma_commit(&aempty[a]);
        umma_commit(&empty[s]);
      }
      umma_commit(dfull);  // also fires (over no MMAs) if a wait gave up
    }
  } else {
    // ------------------------------------------------- dequant + epilogue
    const int qv = warp & 3;                  // TMEM lane quarter of this warp
    const int tl = qv * 32 + lane;            // TMEM lane = row of A
    const int w = tl >> 2, q = tl & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(qv * 32) << 16;
    const int o0 = (q >> 1) | ((q & 1) << 2);  // ORDER[2q]; ORDER[2q + 1] = o0 + 2
    const int ch0 = 8 * w + o0, ch1 = ch0 + 2;
    const uint32_t sel = static_cast<uint32_t>(q) | (static_cast<uint32_t>(4 + q) << 8);
    bool ok = true;
    for (int b = 0; b < nbox && ok; ++b) {
      const int s = b % S;
      if (!(ok = mbar_wait(&full[s], (b / S) & 1, kErrWaitFull))) break;
      const uint8_t* wb = ring + s * L::kSlot + 4 * w;
      const uint8_t* szb = sz + s * L::kSZ;
      const uint32_t zw = ld_s32(szb + L::kS + 4 * w);
      const uint32_t z0 = (zw >> (8 * q)) & 0xFu, z1 = (zw >> (8 * q + 4)) & 0xFu;
      const uint32_t zz0 = (0x6400u | z0) * 0x00010001u;          // 1024 + z, both halves
      const uint32_t zz1 = (0x5400u | (z1 << 4)) * 0x00010001u;   // 64 + z
      const uint32_t ss0 = h2_as_u32(__half2half2(*reinterpret_cast<const __half*>(szb + 2 * ch0)));
      const uint32_t ss1 = h2_as_u32(__half2half2(*reinterpret_cast<const __half*>(szb + 2 * ch1)));
      const int a = b % R;
      if (b >= R && !(ok = mbar_wait(&aempty[a], ((b / R) - 1) & 1, kErrWaitAccum))) break;
      const uint32_t acol = tmem + lane_addr + L::kTmemA + a * 64;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {  // two 16-row steps per 32-column store
        uint32_t r[32];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int st = 2 * h + j;
#pragma unroll
          for (int rr = 0; rr < 8; ++rr) {
            const uint32_t wa = ld_s32(wb + (16 * st + 2 * rr) * 128);
            const uint32_t wc = ld_s32(wb + (16 * st + 2 * rr + 1) * 128);
            const uint32_t t = prmt(wa, wc, sel);
            r[16 * j + rr] = dq_h2(lop3_and_or(t, 0x000F000Fu, 0x64006400u), zz0, ss0);
            r[16 * j + 8 + rr] = dq_h2(lop3_and_or(t, 0x00F000F0u, 0x54005400u), zz1, ss1);
          }
        }
        tmem_st32(acol + 32 * h, r);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[a]);
    }

    // accumulators -> registers
    float acc0[NT], acc1[NT];
#pragma unroll
    for (int m = 0; m < NT; ++m) acc0[m] = acc1[m] = 0.f;
    if (mbar_wait(dfull, 0, kErrWaitAccum) && ok && nbox > 0) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < NT / 16; ++c) {
        if (4 * c < M4) {
          uint32_t r0[16], r1[16];
          tmem_ld16(tmem + lane_addr + c * 16, r0);
          tmem_ld16(tmem + lane_addr + NT + c * 16, r1);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            acc0[c * 16 + e] = __uint_as_float(r0[e]);
            acc1[c * 16 + e] = __uint_as_float(r1[e]);
          }
        }
      }
    }
    tc_fence_before();

    // ---- epilogue: partial sums -> owner CTAs
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
      for (int m4 = 0; m4 < NT / 4; ++m4) {
        if (m4 < M4) {
          st_async_v4(d0 + m4 * 16, make_float4(acc0[4 * m4], acc0[4 * m4 + 1],
                                                acc0[4 * m4 + 2], acc0[4 * m4 + 3]), b0);
          st_async_v4(d1 + m4 * 16, make_float4(acc1[4 * m4], acc1[4 * m4 + 1],
                                                acc1[4 * m4 + 2], acc1[4 * m4 + 3]), b1);
        }
      }
    }
    // owner: thread = (channel c2, 4 tokens); C slices in rank order, + bias
    const bool rok = mbar_wait_cluster(recv_bar, 0, kErrWaitCluster);
    pdl_wait();
    if (rok) {
      for (int e = threadIdx.x - 32; e < M4 * cw; e += 128) {
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
          const float bn = bias != nullptr ? __half2float(bias[n]) : 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int m = 4 * m4 + j;
            if (m < M) y[static_cast<int64_t>(m) * N + n] = __float2half_rn(a4[j] + bn);
          }
        }
      }
    }
  }
  if (warp == 0 || warp == 5) {
    cluster_wait_acquire();  // every thread arrived at the start; match the wait
    pdl_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace lmrs
