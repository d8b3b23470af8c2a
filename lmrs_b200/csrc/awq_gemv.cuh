// awq_gemv.cuh — AWQ W4A16 decode GEMV (small M), HBM bound.
//
// y[m, n] = sum_k x[m, k] * w[k, n],  w = fp16_rne((q - z) * s)  (AWQ int4).
//
// Design (TMA-fed, swap-AB tensor-core GEMV, register dequant):
//   * A CTA owns a 128-column strip (16 packed words per row) and a slice of K.
//     A producer warp streams the strip's packed rows into a ring of
//     shared-memory slots with 2-D TMA boxes (16 words x 64 rows, 64-byte
//     swizzle), together with the matching 64-column tile of the tokens
//     (128-byte swizzle, rows >= M zero-filled by TMA), so each SM keeps
//     ~200 KB of weights in flight with no register cost and the consumers
//     issue no global loads on their critical path.
//   * Four consumer warps: warp (h, p) takes columns 64h..64h+63 and alternate
//     pairs of boxes p.  Lane (g, t) (g = lane/4, t = lane%4) reads word 8h+g of
//     rows 2t, 2t+1, 2t+8, 2t+9 of each 16-row step; the 64-byte swizzle plus
//     loading odd-t lanes' rows in swapped order makes every 32-bit LDS
//     conflict-free.
//   * Output columns play the MMA "M" role (16 per m16n8k16 tile), tokens play
//     "N" (8 per tile, MT tiles).  prmt pairs rows (k, k+1) of the word, and
//     because AWQ puts columns (2i, 2i+1) in nibbles (i, i+4), the half2
//     (1024+q[k][c], 1024+q[k+1][c]) is one shift + one lop3.  Zero point and
//     scale are applied once per quantisation group, not per weight (see the
//     kernel), which keeps the kernel memory-bound instead of issue-bound.
//   * Split-K across a thread-block cluster: CTA partials are summed through
//     distributed shared memory by the cluster; no global scratch, one launch.
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

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4],
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

constexpr int kAwqGemvStrip = 128;      // output columns per CTA
constexpr int kAwqGemvBoxRows = 64;     // k rows per TMA box
constexpr int kAwqGemvBoxBytes = kAwqGemvBoxRows * (kAwqGemvStrip / 8) * 4;  // 4 KB
constexpr int kAwqGemvThreads = 160;    // 4 consumer warps + 1 producer warp
constexpr int kAwqGemvMaxRing = 8;

// byte offset of (row r, word j) inside a 64-byte-swizzled box
__device__ __forceinline__ uint32_t sw64(int r, int j) {
  const uint32_t off = static_cast<uint32_t>(r * 64 + j * 4);
  return off ^ (((off >> 7) & 3u) << 4);
}

// The MMA runs on *biased* nibbles a = B + q, B = 1024 for nibble pairs at bits
// 0-3 and B = 64 for bits 4-7 of a 16-bit half (fp16 1024 has ulp 1, 64 has ulp
// 1/16, so OR-ing the magic onto the masked bits is exact): one lop3 per half2,
// one shift per two, no per-weight dequant arithmetic.  Per quantisation group
// it accumulates D[n][m] = sum_k (B + q[k][n]) x[m][k], and one extra MMA with an
// all-ones A tile accumulates X[m] = sum_k x[m][k] in the same fragment layout.
// When the group ends, y[m][n] += s[n] * (D[n][m] - (B + z[n]) * X[m]), which is
// sum_k (q - z) s x exactly in real arithmetic (fp32 here).
template <int MT>
__global__ void __launch_bounds__(kAwqGemvThreads, (MT == 1 ? 4 : 3)) awq_gemv_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_x,
    __half* __restrict__ y, const uint32_t* __restrict__ qzeros, const __half* __restrict__ scales,
    const __half* __restrict__ bias, int M, int K, int N, int group, int ring) {
  constexpr int MP = 8 * MT;  // padded token count
  constexpr int kXBytes = kAwqGemvBoxRows * 2 * MP;      // token tile of a box: MP rows x 64 k
  constexpr int kSlot = kAwqGemvBoxBytes + kXBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* slots = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(slots + ring * kSlot);
  uint64_t* empty = full + ring;

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int strip = blockIdx.x / C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int words_n = N >> 3;

  const int nb_all = K / kAwqGemvBoxRows;
  const int b_lo = static_cast<int>((static_cast<long long>(rank) * nb_all) / C);
  const int b_hi = static_cast<int>((static_cast<long long>(rank + 1) * nb_all) / C);
  const int nbox = b_hi - b_lo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 2);  // two consumer warps (h = 0, 1) read every box
    }
    fence_mbar_init();
  }
  __syncthreads();

  float acc[MT][4][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;
  const int g = lane >> 2, t = lane & 3;
  const int h = warp & 1, p = (warp >> 1) & 1;
  const int wj = strip * (kAwqGemvStrip / 8) + 8 * h + g;  // this lane's word column
  const bool col_ok = wj < words_n;

  if (warp == 4) {
    // ---------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_x);
      for (int b = 0; b < nbox; ++b) {
        const int s = b % ring;
        if (!mbar_wait(&empty[s], ((b / ring) & 1) ^ 1, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&full[s], kSlot);
        const int krow = (b_lo + b) * kAwqGemvBoxRows;
        tma_load_2d(&tm_q, &full[s], slots + s * kSlot, strip * (kAwqGemvStrip / 8), krow);
        tma_load_2d(&tm_x, &full[s], slots + s * kSlot + kAwqGemvBoxBytes, krow, 0);
      }
    }
  } else {
    // ---------------- consumers: boxes 2p, 2p+1, 2p+4, 2p+5, ...
    const int odd = t & 1;
    // per-lane smem offsets of the 4 rows of step 0 (steps add 16 rows = 1024 bytes,
    // which leaves the 64-byte swizzle bits unchanged); odd-t lanes swap row pairs
    // so each LDS hits 32 distinct banks
    const int jj = 8 * h + g;
    const uint32_t o0 = sw64(2 * t + odd, jj), o1 = sw64(2 * t + 1 - odd, jj);
    const uint32_t o8 = sw64(2 * t + 8 + odd, jj), o9 = sw64(2 * t + 9 - odd, jj);
    float D[MT][4][4], X[MT][2];
    uint32_t zw_c = 0;                              // current group: zero word
    uint4 sv_c = make_uint4(0u, 0u, 0u, 0u);        //                scales of the 8 columns
#pragma unroll
    for (int a = 0; a < MT; ++a) {
      X[a][0] = X[a][1] = 0.f;
#pragma unroll
      for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) D[a][b][c] = 0.f;
    }
    int cur_group = -1;
    uint32_t zw_n = 0;
    uint4 sv_n = make_uint4(0u, 0u, 0u, 0u);
    int pre_group = -1;
    auto fetch = [&](int gi) {
      pre_group = gi;
      if (col_ok) {
        zw_n = __ldg(qzeros + static_cast<int64_t>(gi) * words_n + wj);
        sv_n = __ldg(reinterpret_cast<const uint4*>(scales + static_cast<int64_t>(gi) * N + wj * 8));
      }
    };
    // y += s * (D - (1024 + z) * X) for the finished group; D, X restart at zero.
    // D fragment: d0,d1 = (row g -> column 2i, tokens 2t, 2t+1); d2,d3 = (row g+8 -> column 2i+1).
    auto flush = [&]() {
      const uint32_t sv[4] = {sv_c.x, sv_c.y, sv_c.z, sv_c.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // nibble pair i of the zero word holds columns (2i, 2i+1)
        const float bias_i = (i & 1) ? 64.f : 1024.f;  // the magic each tile's A carries
        const float za = bias_i + static_cast<float>((zw_c >> (4 * i)) & 0xFu);
        const float zb = bias_i + static_cast<float>((zw_c >> (4 * i + 16)) & 0xFu);
        const float2 sp = __half22float2(u32_as_h2(sv[i]));
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[mt][i][0] = fmaf(sp.x, fmaf(-za, X[mt][0], D[mt][i][0]), acc[mt][i][0]);
          acc[mt][i][1] = fmaf(sp.x, fmaf(-za, X[mt][1], D[mt][i][1]), acc[mt][i][1]);
          acc[mt][i][2] = fmaf(sp.y, fmaf(-zb, X[mt][0], D[mt][i][2]), acc[mt][i][2]);
          acc[mt][i][3] = fmaf(sp.y, fmaf(-zb, X[mt][1], D[mt][i][3]), acc[mt][i][3]);
          D[mt][i][0] = D[mt][i][1] = D[mt][i][2] = D[mt][i][3] = 0.f;
        }
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) X[mt][0] = X[mt][1] = 0.f;
    };
    const uint32_t ones[4] = {0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u};  // fp16 1.0
    bool ok = true;
    const int first = 2 * p;
    if (first < nbox) fetch(((b_lo + first) * kAwqGemvBoxRows) / group);
    for (int b = first; b < nbox && ok; b += ((b & 1) ? 3 : 1)) {
      const int krow = (b_lo + b) * kAwqGemvBoxRows;
      const int gi = krow / group;
      if (gi != cur_group) {
        if (cur_group >= 0) flush();
        cur_group = gi;
        if (pre_group != gi) fetch(gi);
        zw_c = zw_n;
        sv_c = sv_n;
        const int bn = b + ((b & 1) ? 3 : 1);  // prefetch the next group this warp meets
        if (bn < nbox) {
          const int gn = ((b_lo + bn) * kAwqGemvBoxRows) / group;
          if (gn != gi) fetch(gn);
        }
      }
      const int slot = b % ring;
      if (!(ok = mbar_wait(&full[slot], (b / ring) & 1, kErrWaitFull))) break;
      const uint32_t sbase = smem_u32(slots + slot * kSlot);
      // token tile (TMA, 128-byte swizzle): row m holds x[m, krow .. krow+63];
      // chunk c of row m sits at chunk c ^ (m % 8): the 8 rows g of a fragment
      // load hit 8 distinct chunks
      const uint32_t xbase = sbase + kAwqGemvBoxBytes + g * 128 + 4 * t;
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        const uint32_t rb = sbase + s4 * 1024;
        const uint32_t v0 = lds_u32(rb + o0), v1 = lds_u32(rb + o1);
        const uint32_t v8 = lds_u32(rb + o8), v9 = lds_u32(rb + o9);
        const uint32_t w0 = odd ? v1 : v0, w1 = odd ? v0 : v1;
        const uint32_t w8 = odd ? v9 : v8, w9 = odd ? v8 : v9;
        uint32_t bx[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          bx[mt][0] = lds_u32(xbase + mt * 1024 + (((2 * s4) ^ g) << 4) - 0);
          bx[mt][1] = lds_u32(xbase + mt * 1024 + (((2 * s4 + 1) ^ g) << 4) - 0);
        }
        uint32_t pk[2][4];  // [row pair 01 / 89][lo 16 bits, hi 16 bits, and the same >> 8]
        pk[0][0] = prmt(w0, w1, 0x5410);
        pk[0][1] = prmt(w0, w1, 0x7632);
        pk[1][0] = prmt(w8, w9, 0x5410);
        pk[1][1] = prmt(w8, w9, 0x7632);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          pk[r][2] = pk[r][0] >> 8;
          pk[r][3] = pk[r][1] >> 8;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // nibble pair i sits at bits 0-3 (i even) or 4-7 (i odd) of pk[.][2*(i>>1)+..]:
          // OR-ing fp16 1024 (ulp 1) or 64 (ulp 1/16) makes each half bias + q exactly
          const uint32_t mask = (i & 1) ? 0x00F000F0u : 0x000F000Fu;
          const uint32_t magic = (i & 1) ? 0x54005400u : 0x64006400u;
          const int sh = (i >> 1) * 2;
          uint32_t a[4];
          a[0] = lop3_and_or(pk[0][sh + 0], mask, magic);
          a[1] = lop3_and_or(pk[0][sh + 1], mask, magic);
          a[2] = lop3_and_or(pk[1][sh + 0], mask, magic);
          a[3] = lop3_and_or(pk[1][sh + 1], mask, magic);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma_f16_16816(D[mt][i], a, bx[mt][0], bx[mt][1]);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          float xs[4] = {X[mt][0], X[mt][1], 0.f, 0.f};
          mma_f16_16816(xs, ones, bx[mt][0], bx[mt][1]);
          X[mt][0] = xs[0];
          X[mt][1] = xs[1];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (cur_group >= 0) flush();
  }

  // ---- reduction: red[p][m][col] in the (drained) ring, then over p, then the cluster
  float* red = reinterpret_cast<float*>(slots);
  if (warp < 4) {
    named_bar_sync(1, 128);  // every consumer is done reading the ring
    // tile i: row g = column 8*(8h+g) + 2i, row g+8 = that column + 1.
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
    for (int e = threadIdx.x; e < MP * kAwqGemvStrip; e += 128) red[e] += red[MP * kAwqGemvStrip + e];
  }
  cluster.sync();
  const int c0 = (rank * kAwqGemvStrip) / C, c1 = ((rank + 1) * kAwqGemvStrip) / C;
  const int ncol = c1 - c0;
  for (int e = threadIdx.x; e < M * ncol; e += blockDim.x) {
    const int m = e / ncol;
    const int col = c0 + (e - m * ncol);
    const int n = strip * kAwqGemvStrip + col;
    float s = 0.f;
    for (int r = 0; r < C; ++r) s += cluster.map_shared_rank(red, r)[m * kAwqGemvStrip + col];
    if (n < N) {
      if (bias != nullptr) s += __half2float(bias[n]);
      y[static_cast<int64_t>(m) * N + n] = __float2half_rn(s);
    }
  }
  cluster.sync();  // peers' shared memory must outlive every remote read
}

}  // namespace lmrs
