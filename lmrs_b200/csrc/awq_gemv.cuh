// awq_gemv.cuh — AWQ W4A16 decode GEMV (small M), HBM bound.
//
// y[m, n] = sum_k x[m, k] * w[k, n],  w = fp16_rne((q - z) * s)  (AWQ int4).
//
// Design (swap-AB tensor-core GEMV, register dequant):
//   * Output columns play the MMA "M" role (16 per m16n8k16 tile), tokens play
//     "N" (8 per tile, MT tiles), k is the reduction.  No shared-memory staging
//     of weights: packed words go HBM -> registers with 64-bit streaming loads
//     (ld.global.nc.L1::no_allocate), are dequantised in registers and fed to
//     mma.sync as the A fragment.
//   * A warp owns a 128-column strip (16 packed words per row).  Lane (g, t)
//     (g = lane/4, t = lane%4) loads words 2g, 2g+1 of rows k0+2t, k0+2t+1,
//     k0+2t+8, k0+2t+9 of each 16-row step: each load instruction touches four
//     64-byte row segments, all bytes used.
//   * prmt pairs rows (k, k+1) of the same word, and because AWQ puts columns
//     (2i, 2i+1) in nibbles (i, i+4), (P >> 4i) & 0x000F000F | 0x6400.. yields
//     the half2 (1024+q[k][c], 1024+q[k+1][c]) that the A fragment wants.
//     Dequant is the canonical fp16 (q - z) * s (hsub2 exact, hmul2 rounds
//     once), so the MMA sees the bit-exact dequantised weights.
//   * Split-K: a thread-block cluster of C CTAs x W warps shares one strip; each
//     warp takes a contiguous run of 64-row units (group % 64 == 0, so a unit
//     never straddles a quantisation group).  Warp partials are summed in
//     shared memory, CTA partials across the cluster through distributed
//     shared memory; no global scratch, one launch.
#pragma once
#include <cooperative_groups.h>
#include "lmrs_ptx.cuh"

namespace lmrs {
namespace cg = cooperative_groups;

__device__ __forceinline__ uint2 ldg_stream_u2(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4],
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int kAwqGemvStrip = 128;  // output columns per warp / per cluster

// MT: number of 8-token MMA tiles (M <= 8 * MT).  W warps per CTA (blockDim = 32W).
template <int MT>
__global__ void __launch_bounds__(256) awq_gemv_kernel(
    __half* __restrict__ y, const __half* __restrict__ x, const uint32_t* __restrict__ qweight,
    const uint32_t* __restrict__ qzeros, const __half* __restrict__ scales,
    const __half* __restrict__ bias, int M, int K, int N, int group) {
  constexpr int MP = 8 * MT;  // padded token count
  extern __shared__ __align__(16) float red[];  // [W][MP][128], then reused

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int strip = blockIdx.x / C;
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int words_n = N >> 3;
  const int wc = strip * (kAwqGemvStrip / 8) + 2 * g;  // thread's first word column
  const bool col_ok = wc < words_n;                     // N % 16 == 0: both words or none

  const int units = K >> 6;  // 64-row units
  const int KS = C * W;
  const int slice = rank * W + warp;
  const int u0 = static_cast<int>((static_cast<long long>(slice) * units) / KS);
  const int u1 = static_cast<int>((static_cast<long long>(slice + 1) * units) / KS);

  float acc[MT][8][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

  // per word column c (0/1) and nibble pair i (0..3): duplicated (1024+z) and s
  // for the A-fragment rows g (column 2i) and g+8 (column 2i+1).
  uint32_t zlo[2][4], zhi[2][4], slo[2][4], shi[2][4];
  int cur_group = -1;

  const uint32_t* qrow_base = qweight + wc;
  for (int u = u0; u < u1; ++u) {
    const int kb = u << 6;
    const int gi = kb / group;
    if (gi != cur_group) {
      cur_group = gi;
      uint2 zw = make_uint2(0u, 0u);
      uint4 s0 = make_uint4(0u, 0u, 0u, 0u), s1 = s0;
      if (col_ok) {
        zw = __ldg(reinterpret_cast<const uint2*>(qzeros + static_cast<int64_t>(gi) * words_n + wc));
        const uint4* sp = reinterpret_cast<const uint4*>(scales + static_cast<int64_t>(gi) * N + wc * 8);
        s0 = __ldg(sp);
        s1 = __ldg(sp + 1);
      }
      const uint32_t zwv[2] = {zw.x, zw.y};
      const uint32_t sv[2][4] = {{s0.x, s0.y, s0.z, s0.w}, {s1.x, s1.y, s1.z, s1.w}};
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t zp = lop3_and_or(zwv[c] >> (4 * i), 0x000F000Fu, 0x64006400u);
          zlo[c][i] = prmt(zp, zp, 0x1010);  // (lo, lo)
          zhi[c][i] = prmt(zp, zp, 0x3232);  // (hi, hi)
          slo[c][i] = prmt(sv[c][i], sv[c][i], 0x1010);
          shi[c][i] = prmt(sv[c][i], sv[c][i], 0x3232);
        }
    }

    // issue all loads of the 4 steps of this unit first
    uint2 wv[4][4];  // [step][row slot: 2t, 2t+1, 2t+8, 2t+9]
    uint32_t bx[4][MT][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k0 = kb + 16 * j;
      const int rows[4] = {k0 + 2 * t, k0 + 2 * t + 1, k0 + 2 * t + 8, k0 + 2 * t + 9};
#pragma unroll
      for (int r = 0; r < 4; ++r)
        wv[j][r] = col_ok ? ldg_stream_u2(qrow_base + static_cast<int64_t>(rows[r]) * words_n)
                          : make_uint2(0u, 0u);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int m = mt * 8 + g;
        if (m < M) {
          const uint32_t* xr = reinterpret_cast<const uint32_t*>(x + static_cast<int64_t>(m) * K + k0);
          bx[j][mt][0] = __ldg(xr + t);
          bx[j][mt][1] = __ldg(xr + 4 + t);
        } else {
          bx[j][mt][0] = 0u;
          bx[j][mt][1] = 0u;
        }
      }
    }

#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t w0 = c ? wv[j][0].y : wv[j][0].x;
        const uint32_t w1 = c ? wv[j][1].y : wv[j][1].x;
        const uint32_t w8 = c ? wv[j][2].y : wv[j][2].x;
        const uint32_t w9 = c ? wv[j][3].y : wv[j][3].x;
        const uint32_t plo01 = prmt(w0, w1, 0x5410), phi01 = prmt(w0, w1, 0x7632);
        const uint32_t plo89 = prmt(w8, w9, 0x5410), phi89 = prmt(w8, w9, 0x7632);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t a[4];
          a[0] = dq_h2(lop3_and_or(plo01 >> (4 * i), 0x000F000Fu, 0x64006400u), zlo[c][i], slo[c][i]);
          a[1] = dq_h2(lop3_and_or(phi01 >> (4 * i), 0x000F000Fu, 0x64006400u), zhi[c][i], shi[c][i]);
          a[2] = dq_h2(lop3_and_or(plo89 >> (4 * i), 0x000F000Fu, 0x64006400u), zlo[c][i], slo[c][i]);
          a[3] = dq_h2(lop3_and_or(phi89 >> (4 * i), 0x000F000Fu, 0x64006400u), zhi[c][i], shi[c][i]);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma_f16_16816(acc[mt][c * 4 + i], a, bx[j][mt][0], bx[j][mt][1]);
        }
      }
    }
  }

  // ---- warp partials -> shared memory: red[warp][m][col], col in [0,128)
  // D fragment: d0,d1 = (row g, tokens 2t, 2t+1); d2,d3 = (row g+8, same tokens).
  // tile (c, i): row g = column 16g + 8c + 2i, row g+8 = that column + 1.
  float* rw = red + static_cast<size_t>(warp) * MP * kAwqGemvStrip;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int col = 16 * g + 8 * c + 2 * i;
        const int m0 = mt * 8 + 2 * t;
        const float* d = acc[mt][c * 4 + i];
        rw[(m0 + 0) * kAwqGemvStrip + col] = d[0];
        rw[(m0 + 1) * kAwqGemvStrip + col] = d[1];
        rw[(m0 + 0) * kAwqGemvStrip + col + 1] = d[2];
        rw[(m0 + 1) * kAwqGemvStrip + col + 1] = d[3];
      }
  __syncthreads();
  // sum over warps into red[0]
  for (int e = threadIdx.x; e < MP * kAwqGemvStrip; e += blockDim.x) {
    float s = red[e];
    for (int w = 1; w < W; ++w) s += red[static_cast<size_t>(w) * MP * kAwqGemvStrip + e];
    red[e] = s;
  }
  // ---- cluster reduction: rank r finalises columns [r*128/C, (r+1)*128/C)
  cluster.sync();
  const int c0 = (rank * kAwqGemvStrip) / C, c1 = ((rank + 1) * kAwqGemvStrip) / C;
  const int ncol = c1 - c0;
  for (int e = threadIdx.x; e < M * ncol; e += blockDim.x) {
    const int m = e / ncol;
    const int col = c0 + (e - m * ncol);
    const int n = strip * kAwqGemvStrip + col;
    float s = 0.f;
    for (int r = 0; r < C; ++r) {
      const float* peer = cluster.map_shared_rank(red, r);
      s += peer[m * kAwqGemvStrip + col];
    }
    if (n < N) {
      if (bias != nullptr) s += __half2float(bias[n]);
      y[static_cast<int64_t>(m) * N + n] = __float2half_rn(s);
    }
  }
  cluster.sync();  // peers' shared memory must outlive every remote read
}

}  // namespace lmrs
