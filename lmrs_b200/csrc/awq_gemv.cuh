// awq_gemv.cuh — AWQ W4A16 decode GEMV (M <= 16 tokens), HBM bound.
//
// y[m, n] = sum_k x[m, k] * w[k, n],  w = (q - z) * s  (AWQ int4, fp32 accumulate).
//
// Layout of the work:
//   * A CTA owns a 128-column strip (16 packed words per row) and a contiguous
//     range of K, cut into boxes of BR rows (BR = 128, or 64 for group 64; a
//     box never straddles a quantisation group).  Clusters of C CTAs (C a
//     power of two) split one strip's K; partial sums meet in distributed
//     shared memory.
//   * One producer thread streams each box into a ring slot with TMA: the
//     packed words (16 words x BR rows, 64-byte swizzle), the box's rows of
//     the token matrix (64-k sub-tiles, 128-byte swizzle, rows >= M zero
//     filled), and the group's scale row and zero-point row.  The consumers
//     issue no global loads at all.
//   * Programmatic dependent launch: the producer issues the weight, scale and
//     zero loads of the first ring slots before griddepcontrol.wait and only
//     the token loads after it, so a GEMV that follows another kernel streams
//     its weights while that kernel drains.
//   * Four consumer warps: warp (h, p) takes word columns 8h..8h+7 of the
//     boxes b = p, p+2, p+4, ...  Lane (g, t) reads word 8h+g of rows 2t, 2t+1,
//     2t+8, 2t+9 of each 16-row step (odd t in swapped row order, which with the
//     64-byte swizzle makes the 32-bit LDS conflict-free).  prmt pairs rows
//     (k, k+1); since AWQ stores columns (2i, 2i+1) in nibbles (i, i+4), one
//     lop3 turns a nibble pair into the half2 (B + q[k][c], B + q[k+1][c]),
//     B = 1024 (bits 0-3 of a half) or 64 (bits 4-7); with bf16 activations
//     (bf16 MMA operands) every nibble is shifted to bits 0-3, B = 128.  Output columns are the
//     MMA "M" (16 per m16n8k16 tile), tokens the "N" (8 per tile, MT tiles).
//   * Zero point and scale are applied once per box, not per weight: the MMAs
//     accumulate D = sum_k (B + q) x and, with an all-ones A tile, X = sum_k x;
//     at the end of the box y += s * (D - (B + z) X), exact in real arithmetic.
//   * Reduction without a trailing cluster barrier: each CTA writes its slice
//     of partials for owner CTA r straight into r's shared memory (st.shared::
//     cluster) and arrives on r's mbarrier with release semantics; r waits
//     (acquire), sums the C slices in rank order (deterministic) and stores
//     y.  A CTA leaves only after every peer has delivered to it, and no CTA
//     reads a peer's memory, so no CTA can leave while its memory is in use.
#pragma once
#include <cooperative_groups.h>
#include "lmrs_ptx.cuh"

namespace lmrs {
namespace cg = cooperative_groups;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Shared-memory loads as plain C++ (not asm volatile): the compiler may then
// hoist the next step's loads above this step's MMAs, while the "memory"
// clobber of the mbarrier wait still keeps them after the wait.
__device__ __forceinline__ uint32_t ld_s32(const uint8_t* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}
__device__ __forceinline__ uint2 ld_s64(const uint8_t* p) {
  return *reinterpret_cast<const uint2*>(p);
}
__device__ __forceinline__ uint4 ld_s128(const uint8_t* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// Not volatile: a pure function of its operands, free to be scheduled.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4],
                                              uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// m16n8k16 with both operands of the activation type T, fp32 accumulate.
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  if constexpr (Act<T>::kUmmaFmt == 0) mma_f16_16816(d, a, b0, b1);
  else mma_bf16_16816(d, a, b0, b1);
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

constexpr int kAwqGemvStrip = 128;                  // output columns per CTA
constexpr int kAwqGemvWords = kAwqGemvStrip / 8;    // packed words per box row
constexpr int kAwqGemvThreads = 160;                // 4 consumer warps + 1 producer warp
constexpr int kAwqGemvMaxCluster = 8;

// Shared-memory layout of one instantiation (ring of S slots chosen at launch).
template <int MT, int BR>
struct AwqGemvLayout {
  static constexpr int kW = BR * kAwqGemvWords * 4;   // packed words of a box
  static constexpr int kXSub = 8 * MT * 128;          // one 64-k token sub-tile
  static constexpr int kX = (BR / 64) * kXSub;
  static constexpr int kSlot = kW + kX;
  static constexpr int kS = kAwqGemvStrip * 2;        // scale row (fp16)
  static constexpr int kZ = kAwqGemvWords * 4;        // zero-point row (packed)
  static constexpr int kSZ = 384;                     // kS + kZ, padded to 128 B
  static constexpr int kTx = kW + kX + kS + kZ;       // TMA bytes per slot
  static constexpr int kRecv = 8 * MT * kAwqGemvStrip * 4;
  static constexpr int kRed = 2 * 8 * MT * kAwqGemvStrip * 4;  // per-p partials, after the loop
  static_assert(kSlot % 1024 == 0, "swizzled TMA destinations need 1024-byte slots");
  static_assert(kS + kZ <= kSZ && kSZ % 128 == 0, "scale/zero rows must stay 128-byte aligned");
  static_assert(BR == 64 || BR == 128, "box rows");
  // the ring area also holds the partials once drained: at least kRed bytes
  __host__ __device__ static constexpr int ring_bytes(int S) {
    return S * kSlot > kRed ? S * kSlot : (kRed + 1023) / 1024 * 1024;
  }
  __host__ __device__ static constexpr int smem_bytes(int S) {
    return 1024 + ring_bytes(S) + S * kSZ + kRecv + (2 * S + 1) * 8;
  }
};

// byte offset of (row r, word j) inside a 64-byte-swizzled box
__device__ __forceinline__ uint32_t sw64(int r, int j) {
  const uint32_t off = static_cast<uint32_t>(r * 64 + j * 4);
  return off ^ (((off >> 7) & 3u) << 4);
}

template <int MT, int BR, typename T>
__global__ void __launch_bounds__(kAwqGemvThreads, (MT == 1 ? 4 : 3)) awq_gemv_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_x,
    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
    T* __restrict__ y, const T* __restrict__ bias, int M, int K, int N, int group,
    int S) {
  using L = AwqGemvLayout<MT, BR>;
  constexpr int MP = 8 * MT;  // padded token count
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sz = ring + L::ring_bytes(S);
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
      mbar_init(&empty[i], 2);  // warps h = 0, 1 of one p read every box
    }
    // the owner's own arrive plus the peers' st.async bytes (MP floats per column)
    mbar_init(recv_bar, 1);
    mbar_arrive_expect_tx(recv_bar, MP * kAwqGemvStrip * 4);
    fence_mbar_init();
  }
  __syncthreads();
  cluster_arrive_relaxed();  // waited on just before the first remote store
  pdl_trigger();

  float acc[MT][4][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;
  const int g = lane >> 2, t = lane & 3;
  const int h = warp & 1, p = (warp >> 1) & 1;

  if (warp == 4) {
    // ---------------- producer (one thread)
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
      pdl_wait();  // the tokens are the previous kernel's output
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
    // ---------------- consumers
    const int odd = t & 1;
    const int jj = 8 * h + g;  // word column within the strip
    // per-lane smem offsets of the 4 rows of step 0 (a step adds 16 rows = 1024
    // bytes, which leaves the 64-byte swizzle bits unchanged); odd-t lanes swap
    // row pairs so each LDS hits 32 distinct banks
    const uint32_t o0 = sw64(2 * t + odd, jj), o1 = sw64(2 * t + 1 - odd, jj);
    const uint32_t o8 = sw64(2 * t + 8 + odd, jj), o9 = sw64(2 * t + 9 - odd, jj);
    const uint32_t ones[4] = {Act<T>::kOne2, Act<T>::kOne2, Act<T>::kOne2, Act<T>::kOne2};
    int s = p;
    uint32_t ph = 0;
    for (int b = p; b < nbox; b += 2) {
      if (!mbar_wait(&full[s], ph, kErrWaitFull)) break;
      const uint8_t* sbase = ring + s * L::kSlot;
      float D[MT][4][4], X[MT][2];
#pragma unroll
      for (int a = 0; a < MT; ++a) {
        X[a][0] = X[a][1] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 4; ++c) D[a][i][c] = 0.f;
      }
      // token tile (128-byte swizzle): row m holds x[m, 64j .. 64j+63] of sub-tile j;
      // chunk c of row m sits at chunk c ^ (m % 8), so the 8 rows g of a fragment
      // load hit 8 distinct chunks
      const uint8_t* xbase = sbase + L::kW + g * 128 + 4 * t;
#pragma unroll 4
      for (int s4 = 0; s4 < BR / 16; ++s4) {
        const uint8_t* rb = sbase + s4 * 1024;
        const uint32_t v0 = ld_s32(rb + o0), v1 = ld_s32(rb + o1);
        const uint32_t v8 = ld_s32(rb + o8), v9 = ld_s32(rb + o9);
        const uint32_t w0 = odd ? v1 : v0, w1 = odd ? v0 : v1;
        const uint32_t w8 = odd ? v9 : v8, w9 = odd ? v8 : v9;
        const uint8_t* xs = xbase + (s4 >> 2) * L::kXSub;
        const int c2 = 2 * (s4 & 3);
        uint32_t bx[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          bx[mt][0] = ld_s32(xs + mt * 1024 + ((c2 ^ g) << 4));
          bx[mt][1] = ld_s32(xs + mt * 1024 + (((c2 + 1) ^ g) << 4));
        }
        uint32_t pk[2][2];  // [row pair 01 / 89][lo 16 bits (nibbles 0-3), hi 16 bits (4-7)]
        pk[0][0] = prmt(w0, w1, 0x5410);
        pk[0][1] = prmt(w0, w1, 0x7632);
        pk[1][0] = prmt(w8, w9, 0x5410);
        pk[1][1] = prmt(w8, w9, 0x7632);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // nibble i of each half-word: column 2i (low half-word) and 2i+1 (high)
          uint32_t a[4];
          a[0] = awq_nib_pair<T>(pk[0][0], i);
          a[1] = awq_nib_pair<T>(pk[0][1], i);
          a[2] = awq_nib_pair<T>(pk[1][0], i);
          a[3] = awq_nib_pair<T>(pk[1][1], i);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma_16816<T>(D[mt][i], a, bx[mt][0], bx[mt][1]);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          float xsum[4] = {X[mt][0], X[mt][1], 0.f, 0.f};
          mma_16816<T>(xsum, ones, bx[mt][0], bx[mt][1]);
          X[mt][0] = xsum[0];
          X[mt][1] = xsum[1];
        }
      }
      // y += s * (D - (B + z) * X) for this box.  D fragment: d0, d1 = (row g ->
      // column 2i of word jj, tokens 2t, 2t+1); d2, d3 = (row g+8 -> column 2i+1).
      const uint8_t* szb = sz + s * L::kSZ;
      const uint32_t zw = ld_s32(szb + L::kS + 4 * jj);
      const uint4 sv4 = ld_s128(szb + 16 * jj);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      const uint32_t sv[4] = {sv4.x, sv4.y, sv4.z, sv4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // nibble pair i of the zero word holds columns (2i, 2i+1)
        const float bias_i = awq_nib_bias<T>(i);  // the magic each tile's A carries
        const float za = bias_i + static_cast<float>((zw >> (4 * i)) & 0xFu);
        const float zb = bias_i + static_cast<float>((zw >> (4 * i + 16)) & 0xFu);
        const float2 sp = __half22float2(u32_as_h2(sv[i]));
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[mt][i][0] = fmaf(sp.x, fmaf(-za, X[mt][0], D[mt][i][0]), acc[mt][i][0]);
          acc[mt][i][1] = fmaf(sp.x, fmaf(-za, X[mt][1], D[mt][i][1]), acc[mt][i][1]);
          acc[mt][i][2] = fmaf(sp.y, fmaf(-zb, X[mt][0], D[mt][i][2]), acc[mt][i][2]);
          acc[mt][i][3] = fmaf(sp.y, fmaf(-zb, X[mt][1], D[mt][i][3]), acc[mt][i][3]);
        }
      }
      s += 2;
      if (s >= S) {
        s -= S;
        ph ^= 1;
      }
    }
  }

  // ---- reduction: per-p partials in the drained ring, summed, then sent to the
  // owner CTA of each column slice
  cluster_wait_acquire();  // every peer has initialised its receive barrier
  if (warp < 4) {
    const int ct = threadIdx.x;   // 0..127
    float* red = reinterpret_cast<float*>(ring);
    named_bar_sync(1, 128);       // every consumer is done reading the ring
    float* rp = red + static_cast<size_t>(p) * MP * kAwqGemvStrip;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int col = 8 * (8 * h + g) + 2 * i;
        const int m0 = mt * 8 + 2 * t;
        rp[(m0 + 0) * kAwqGemvStrip + col] = acc[mt][i][0];
        rp[(m0 + 1) * kAwqGemvStrip + col] = acc[mt][i][1];
        rp[(m0 + 0) * kAwqGemvStrip + col + 1] = acc[mt][i][2];
        rp[(m0 + 1) * kAwqGemvStrip + col + 1] = acc[mt][i][3];
      }
    named_bar_sync(1, 128);
    // thread ct serves owner r = ct / cw, column r * cw + li of the strip: its MP
    // token sums go out as 16-byte st.async into recv[source rank][column][token]
    const int cw = kAwqGemvStrip / C;  // C is a power of two <= 8
    const int r = ct / cw, li = ct - r * cw;
    const int col = r * cw + li;
    const uint32_t dst = mapa_shared(smem_u32(recv + (rank * cw + li) * MP), static_cast<uint32_t>(r));
    const uint32_t rbar = mapa_shared(smem_u32(recv_bar), static_cast<uint32_t>(r));
#pragma unroll
    for (int m4 = 0; m4 < MP; m4 += 4) {
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = red[(m4 + j) * kAwqGemvStrip + col] + red[(MP + m4 + j) * kAwqGemvStrip + col];
      st_async_v4(dst + m4 * 4, make_float4(v[0], v[1], v[2], v[3]), rbar);
    }

    // ---- owner: sum the C slices in rank order, add bias, store
    const bool ok = mbar_wait_cluster(recv_bar, 0, kErrWaitCluster);
    pdl_wait();
    if (ok) {
      for (int e = ct; e < M * cw; e += 128) {
        const int m = e / cw, cl = e - m * cw;
        const int n = strip * kAwqGemvStrip + rank * cw + cl;
        float v = 0.f;
        for (int q = 0; q < C; ++q) v += recv[(q * cw + cl) * MP + m];
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
