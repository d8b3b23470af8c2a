// awq_gemv4.cuh — AWQ W4A16 decode GEMV for M <= 4 tokens (batch-1..4 decode).
//
// Same pipeline as awq_gemv.cuh (TMA ring of BR-row boxes of a 128-column
// strip plus the group's scale and zero rows, PDL weight prefetch, biased-nibble
// MMAs with a per-box zero/scale fix-up, cluster split-K reduced through
// distributed shared memory), but with an MMA operand encoding that needs no
// byte permutes, so a warp spends ~30 instructions per 128 packed words instead
// of ~47:
//   * MMA "K" runs over (row, column parity): k-slot 2j / 2j+1 is row R(j) of
//     the 8-row step with the even / odd column of a column pair.  A register of
//     the A fragment is then exactly what one lop3 makes of a packed word: the
//     half2 (B + q[row][2i], B + q[row][2i+1]) of nibble pair i.
//   * MMA "M" rows g and g+8 are words 2g and 2g+1 (nibble pair i in MMA i), so
//     a lane reads its two words of a row with one 64-bit LDS.
//   * MMA "N" column n carries token n/2 with parity n%2: lane (g, t)'s B
//     register holds x[g/2][R] in its low (g even) or high (g odd) half, zero
//     in the other, so each output column only meets its own parity.  One
//     8-wide tile serves 4 tokens.
//   * Rows R(t) alternate between 2t and 2t+1 by lane parity, which makes each
//     64-bit LDS conflict-free under the 64-byte swizzle; the B side follows
//     through per-lane byte selectors, at no cost.
// Lane (g, t) ends up owning token t and the 16 contiguous columns 16g..16g+15.
#pragma once
#include <cooperative_groups.h>
#include "awq_gemv.cuh"
#include "lmrs_ptx.cuh"

namespace lmrs {

constexpr int kAwqGemv4Threads = 160;  // 4 consumer warps (one box each in turn) + producer

// Ring slot: packed box + 64-k token sub-tiles of 8 rows (tokens >= M are zero).
template <int BR>
struct AwqGemv4Layout {
  static constexpr int kW = BR * kAwqGemvWords * 4;
  static constexpr int kXSub = 8 * 128;
  static constexpr int kX = (BR / 64) * kXSub;
  static constexpr int kSlot = kW + kX;
  static constexpr int kS = kAwqGemvStrip * 2;
  static constexpr int kZ = kAwqGemvWords * 4;
  static constexpr int kSZ = 384;
  static constexpr int kTx = kW + kX + kS + kZ;
  static constexpr int kRecv = 4 * kAwqGemvStrip * 4;  // 4 tokens x 128 columns fp32
  static constexpr int kRed = 4 * 4 * kAwqGemvStrip * 4;   // per-warp partials, after the loop
  static_assert(kSlot % 1024 == 0, "swizzled TMA destinations need 1024-byte slots");
  static_assert(BR == 64 || BR == 128, "box rows");
  static_assert(4 * kSlot >= kRed, "the drained ring (S >= 4) holds the partials");
  __host__ __device__ static constexpr int smem_bytes(int S) {
    return 1024 + S * kSlot + S * kSZ + kRecv + (2 * S + 1) * 8;
  }
};

template <int BR, typename T>
__global__ void __launch_bounds__(kAwqGemv4Threads, 4) awq_gemv4_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_x,
    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
    T* __restrict__ y, const T* __restrict__ bias, int M, int K, int N, int group,
    int S) {
  using L = AwqGemv4Layout<BR>;
  constexpr int kTok = 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sz = ring + S * L::kSlot;
  float* recv = reinterpret_cast<float*>(sz + S * L::kSZ);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(recv) + L::kRecv);
  uint64_t* empty = full + S;
  uint64_t* recv_bar = empty + S;

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int strip = blockIdx.x / C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int nb_all = K / BR;
  const int b_lo = static_cast<int>((static_cast<long long>(rank) * nb_all) / C);
  const int b_hi = static_cast<int>((static_cast<long long>(rank + 1) * nb_all) / C);
  const int nbox = b_hi - b_lo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);  // one consumer warp per box
    }
    // the owner's own arrive plus every peer's 16-byte st.async (C x 128 of them)
    mbar_init(recv_bar, 1);
    mbar_arrive_expect_tx(recv_bar, kTok * kAwqGemvStrip * 4);
    fence_mbar_init();
  }
  __syncthreads();
  cluster_arrive_relaxed();
  pdl_trigger();

  const int g = lane >> 2, t = lane & 3;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[i][c] = 0.f;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_z);
      const int c0 = strip * kAwqGemvWords;
      auto load_weights = [&](int b, int s) {
        const int krow = (b_lo + b) * BR;
        const int gi = krow / group;
        mbar_arrive_expect_tx(&full[s], L::kTx);
        tma_load_2d(&tm_q, &full[s], ring + s * L::kSlot, c0, krow);
        tma_load_2d(&tm_s, &full[s], sz + s * L::kSZ, strip * kAwqGemvStrip, gi);
        tma_load_2d(&tm_z, &full[s], sz + s * L::kSZ + L::kS, c0, gi);
      };
      auto load_tokens = [&](int b, int s) {
        const int krow = (b_lo + b) * BR;
#pragma unroll
        for (int j = 0; j < BR / 64; ++j)
          tma_load_2d(&tm_x, &full[s], ring + s * L::kSlot + L::kW + j * L::kXSub, krow + 64 * j,
                      0);
      };
      const int pre = nbox < S ? nbox : S;
      for (int b = 0; b < pre; ++b) load_weights(b, b);
      pdl_wait();
      for (int b = 0; b < pre; ++b) load_tokens(b, b);
      int s = 0;
      uint32_t ph = 0;
      for (int b = pre; b < nbox; ++b) {
        if (!mbar_wait(&empty[s], ph, kErrWaitEmpty)) break;
        load_weights(b, s);
        load_tokens(b, s);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else {
    // ---------------- consumers: warp p takes boxes p, p+4, p+8, ...
    const int p = warp;
    const int odd = t & 1;
    // A: words 2g, 2g+1 of rows R = 2t + odd and R' = 2t + 1 - odd of each 8-row
    // step (64-byte swizzle: chunk ^= (row / 2) % 4 = t for both rows)
    const uint32_t wa = static_cast<uint32_t>((2 * t + odd) * 64 + ((8 * g) ^ (16 * t)));
    const uint32_t wb = static_cast<uint32_t>((2 * t + 1 - odd) * 64 + ((8 * g) ^ (16 * t)));
    // B: half2 (x[tok][2t], x[tok][2t+1]) of token row g/2 (128-byte swizzle)
    const int tok = g >> 1;
    const uint32_t xo = static_cast<uint32_t>(tok * 128 + 4 * t);
    // byte selectors: value from the low (row 2t) or high (row 2t+1) half of the
    // loaded pair, placed in the low (g even) or high (g odd) half of b
    const uint32_t lo_v = 0x10u, hi_v = 0x32u;
    const uint32_t v0 = odd ? hi_v : lo_v, v1 = odd ? lo_v : hi_v;  // rows R, R'
    const uint32_t sel0 = (g & 1) ? (0x44u | (v0 << 8)) : (v0 | 0x4400u);
    const uint32_t sel1 = (g & 1) ? (0x44u | (v1 << 8)) : (v1 | 0x4400u);
    const uint32_t ones[4] = {Act<T>::kOne2, Act<T>::kOne2, Act<T>::kOne2, Act<T>::kOne2};
    int s = p;
    uint32_t ph = 0;
    for (int b = p; b < nbox; b += 4) {
      if (!mbar_wait(&full[s], ph, kErrWaitFull)) break;
      const uint8_t* sbase = ring + s * L::kSlot;
      float D[4][4], X0 = 0.f, X1 = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) D[i][c] = 0.f;
#pragma unroll 4
      for (int st = 0; st < BR / 8; ++st) {
        const uint2 pa = ld_s64(sbase + st * 512 + wa);   // row R:  words 2g, 2g+1
        const uint2 pb = ld_s64(sbase + st * 512 + wb);   // row R': words 2g, 2g+1
        const int sub = st >> 3, c16 = st & 7;             // 64-k sub-tile, 16-byte chunk
        const uint32_t xv = ld_s32(sbase + L::kW + sub * L::kXSub + xo + ((c16 ^ tok) << 4));
        const uint32_t b0 = prmt(xv, 0u, sel0), b1 = prmt(xv, 0u, sel1);
        const uint32_t ra[4] = {pa.x, pa.y, pb.x, pb.y};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t a[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) a[r] = awq_nib_pair<T>(ra[r], i);  // nibbles i, i + 4
          mma_16816<T>(D[i], a, b0, b1);
        }
        float xs[4] = {X0, X1, 0.f, 0.f};
        mma_16816<T>(xs, ones, b0, b1);
        X0 = xs[0];
        X1 = xs[1];
      }
      // fix-up: d0/d1 -> word 2g, columns 2i / 2i+1; d2/d3 -> word 2g+1
      const uint8_t* szb = sz + s * L::kSZ;
      const uint2 zw = ld_s64(szb + L::kS + 8 * g);
      const uint4 sa = ld_s128(szb + 32 * g);
      const uint4 sb = ld_s128(szb + 32 * g + 16);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      const uint32_t sva[4] = {sa.x, sa.y, sa.z, sa.w}, svb[4] = {sb.x, sb.y, sb.z, sb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float bias_i = awq_nib_bias<T>(i);
        const float za0 = bias_i + static_cast<float>((zw.x >> (4 * i)) & 0xFu);
        const float za1 = bias_i + static_cast<float>((zw.x >> (4 * i + 16)) & 0xFu);
        const float zb0 = bias_i + static_cast<float>((zw.y >> (4 * i)) & 0xFu);
        const float zb1 = bias_i + static_cast<float>((zw.y >> (4 * i + 16)) & 0xFu);
        const float2 s_a = __half22float2(u32_as_h2(sva[i]));
        const float2 s_b = __half22float2(u32_as_h2(svb[i]));
        acc[i][0] = fmaf(s_a.x, fmaf(-za0, X0, D[i][0]), acc[i][0]);
        acc[i][1] = fmaf(s_a.y, fmaf(-za1, X1, D[i][1]), acc[i][1]);
        acc[i][2] = fmaf(s_b.x, fmaf(-zb0, X0, D[i][2]), acc[i][2]);
        acc[i][3] = fmaf(s_b.y, fmaf(-zb1, X1, D[i][3]), acc[i][3]);
      }
      s += 4;
      if (s >= S) {
        s -= S;
        ph ^= 1;
      }
    }
  }

  // ---- reduction: the 4 warps' partials in the drained ring, then per owner
  cluster_wait_acquire();
  if (warp < 4) {
    const int ct = threadIdx.x;
    float* red = reinterpret_cast<float*>(ring);  // [4 warps][4 tokens][128 columns]
    named_bar_sync(1, 128);
    float* rp = red + warp * kTok * kAwqGemvStrip + t * kAwqGemvStrip + 16 * g;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      rp[2 * i] = acc[i][0];
      rp[2 * i + 1] = acc[i][1];
      rp[8 + 2 * i] = acc[i][2];
      rp[8 + 2 * i + 1] = acc[i][3];
    }
    named_bar_sync(1, 128);
    // thread ct sends column r * cw + li (all 4 tokens, one 16-byte st.async)
    // to owner r; recv is [source rank][column][token]
    const int cw = kAwqGemvStrip / C;
    const int r = ct / cw, li = ct - r * cw;
    const int col = r * cw + li;
    float v4[kTok];
#pragma unroll
    for (int m = 0; m < kTok; ++m) {
      const int e = m * kAwqGemvStrip + col;
      v4[m] = red[e] + red[kTok * kAwqGemvStrip + e] + red[2 * kTok * kAwqGemvStrip + e] +
              red[3 * kTok * kAwqGemvStrip + e];
    }
    st_async_v4(mapa_shared(smem_u32(recv + (rank * cw + li) * kTok), static_cast<uint32_t>(r)),
                make_float4(v4[0], v4[1], v4[2], v4[3]),
                mapa_shared(smem_u32(recv_bar), static_cast<uint32_t>(r)));

    const bool ok = mbar_wait_cluster(recv_bar, 0, kErrWaitCluster);
    pdl_wait();
    if (ok) {
      for (int e = ct; e < M * cw; e += 128) {
        const int m = e / cw, cl = e - m * cw;
        const int n = strip * kAwqGemvStrip + rank * cw + cl;
        float v = 0.f;
        for (int q = 0; q < C; ++q) v += recv[(q * cw + cl) * kTok + m];
        if (n < N) {
          if (bias != nullptr) v += Act<T>::to_float(bias[n]);
          y[static_cast<int64_t>(m) * N + n] = Act<T>::from_float(v);
        }
      }
    }
  } else {
    pdl_wait();
  }
}

}  // namespace lmrs
