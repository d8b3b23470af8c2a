// fp8_kernels.cuh — FP8 e4m3 W8A8: per-row quantisation and the decode GEMV.
//
// Quantisation (per token for activations, per output channel for weights):
//   s[r] = absmax_k |x[r,k]| / 448 (fp32 IEEE division),
//   q[r,k] = e4m3 RNE satfinite (x[r,k] / s[r])   (IEEE division, then cvt),
//   rows with s == 0 quantise to 0.
// One CTA per row: pass 1 reduces the absmax with 16-byte loads, pass 2 re-reads
// the row (L1/L2 resident) and writes 8 e4m3 per thread per step.
//
// Decode GEMV (small M), swap-AB mma.sync m16n8k32 e4m3 x e4m3 -> fp32:
// output channels are the MMA "M" rows (W's K-contiguous rows are exactly the
// row-major A fragment), tokens are "N".  A producer warp streams weight tiles
// into a shared-memory ring with TMA, consumer warps read 16-byte chunks of two
// rows per 128-byte K unit.  The 32 k-slots of the four MMAs of a unit are a
// permutation of the unit's 128 bytes chosen so that every lane's A bytes are
// two contiguous 16-byte chunks; the token fragment is gathered with the same
// permutation.  Split-K across a thread-block cluster, reduced through
// distributed shared memory, scaled by s_x[m] * s_w[n] in the epilogue.
#pragma once
#include <cooperative_groups.h>
#include "lmrs_ptx.cuh"

namespace lmrs {
namespace cg = cooperative_groups;

template <int DT>
struct IoType;
template <>
struct IoType<0> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
};
template <>
struct IoType<1> {
  using T = __half;
  static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
};
template <>
struct IoType<2> {
  using T = float;
  static __device__ __forceinline__ float to_f(T v) { return v; }
};

constexpr int kQuantThreads = 256;

template <int DT>
__global__ void __launch_bounds__(kQuantThreads) fp8_quant_rows_kernel(
    uint8_t* __restrict__ q, float* __restrict__ scale, const typename IoType<DT>::T* __restrict__ x,
    int K) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  using T = typename IoType<DT>::T;
  constexpr int VEC = 16 / sizeof(T);  // elements per 16-byte load
  __shared__ float red[kQuantThreads / 32];
  const int row = blockIdx.x;
  const T* xr = x + static_cast<int64_t>(row) * K;
  uint8_t* qr = q + static_cast<int64_t>(row) * K;

  float amax = 0.f;
  for (int k = threadIdx.x * VEC; k < K; k += kQuantThreads * VEC) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + k));
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < VEC; ++i) amax = fmaxf(amax, fabsf(IoType<DT>::to_f(e[i])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < kQuantThreads / 32; ++w) m = fmaxf(m, red[w]);
  const float s = __fdiv_rn(m, 448.0f);
  if (threadIdx.x == 0) scale[row] = s;

  // 8 elements per step -> one 8-byte store
  for (int k = threadIdx.x * 8; k < K; k += kQuantThreads * 8) {
    float f[8];
    if (sizeof(T) == 2) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + k));
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = IoType<DT>::to_f(e[i]);
    } else {
      const uint4 v0 = __ldg(reinterpret_cast<const uint4*>(xr + k));
      const uint4 v1 = __ldg(reinterpret_cast<const uint4*>(xr + k) + 1);
      f[0] = __uint_as_float(v0.x); f[1] = __uint_as_float(v0.y);
      f[2] = __uint_as_float(v0.z); f[3] = __uint_as_float(v0.w);
      f[4] = __uint_as_float(v1.x); f[5] = __uint_as_float(v1.y);
      f[6] = __uint_as_float(v1.z); f[7] = __uint_as_float(v1.w);
    }
    uint32_t out[2] = {0u, 0u};
    if (s != 0.f) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 pr = make_float2(__fdiv_rn(f[2 * i], s), __fdiv_rn(f[2 * i + 1], s));
        const uint32_t b = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(pr, __NV_SATFINITE, __NV_E4M3));
        out[i >> 1] |= b << ((i & 1) * 16);
      }
    }
    *reinterpret_cast<uint2*>(qr + k) = make_uint2(out[0], out[1]);
  }
}

// ------------------------------------------------------------------ GEMV
__device__ __forceinline__ void mma_e4m3_16832(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

constexpr int kF8GemvRows = 64;          // output channels per CTA strip (4 MMA tiles)
constexpr int kF8GemvBoxBytes = kF8GemvRows * 128;  // 64 rows x 128 bytes of K = 8 KB
constexpr int kF8GemvThreads = 160;      // 4 consumer warps + 1 producer warp
constexpr int kF8GemvMaxRing = 4;  // 4 x (8 KB + token tile): 5 CTAs per SM

// MT: 8-token MMA tiles (M <= 8 * MT).  A producer warp streams the strip's
// weight rows (TMA boxes of 128 bytes of K x 64 rows, 128-byte swizzle) into a
// ring of shared-memory slots; consumer warp w owns MMA tile w (channels
// 16w..16w+15).  Within each 128-byte K unit, lane (g, t) takes the 16-byte
// chunks t and 4+t of its two rows: the 32 k-slots of the unit's four MMAs are
// a fixed permutation of the unit's bytes, and the token fragment (xq, read
// through L1) uses the same permutation.
template <int MT>
__global__ void __launch_bounds__(kF8GemvThreads, 4) fp8_gemv_kernel(
    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
    __nv_bfloat16* __restrict__ y, const float* __restrict__ sx, const float* __restrict__ sw,
    const __nv_bfloat16* __restrict__ bias, int M, int K, int N, int ring) {
  pdl_wait();     // activations are the previous kernel's output
  pdl_trigger();
  constexpr int MP = 8 * MT;
  constexpr int kSlot = kF8GemvBoxBytes + MP * 128;  // weights + token tile (MP rows x 128 B)
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
  const int g = lane >> 2, t = lane & 3;
  const int nbase = strip * kF8GemvRows;

  const int units = (K + 127) >> 7;
  const int u_lo = static_cast<int>((static_cast<long long>(rank) * units) / C);
  const int u_hi = static_cast<int>((static_cast<long long>(rank + 1) * units) / C);
  const int nbox = u_hi - u_lo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);  // every consumer warp reads every box
    }
    fence_mbar_init();
  }
  __syncthreads();

  float acc[MT][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_x);
      for (int b = 0; b < nbox; ++b) {
        const int s = b % ring;
        if (!mbar_wait(&empty[s], ((b / ring) & 1) ^ 1, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&full[s], kSlot);
        tma_load_2d(&tm_w, &full[s], slots + s * kSlot, (u_lo + b) * 128, nbase);
        tma_load_2d(&tm_x, &full[s], slots + s * kSlot + kF8GemvBoxBytes, (u_lo + b) * 128, 0);
      }
    }
  } else {
    const int r0 = 16 * warp + g;  // rows r0 and r0 + 8 of the box; (r0 % 8) == g
    for (int b = 0; b < nbox; ++b) {
      const int slot = b % ring;
      if (!mbar_wait(&full[slot], (b / ring) & 1, kErrWaitFull)) break;
      const uint32_t sb = smem_u32(slots + slot * kSlot);
      // 128-byte swizzle: chunk c of row r sits at chunk c ^ (r % 8)
      const uint4 ga = lds_u4(sb + r0 * 128 + ((t ^ g) << 4));
      const uint4 gc = lds_u4(sb + r0 * 128 + (((4 + t) ^ g) << 4));
      const uint4 ha = lds_u4(sb + (r0 + 8) * 128 + ((t ^ g) << 4));
      const uint4 hc = lds_u4(sb + (r0 + 8) * 128 + (((4 + t) ^ g) << 4));
      uint4 xb[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint32_t xr = sb + kF8GemvBoxBytes + (mt * 8 + g) * 128;  // token rows >= M are zero
        xb[mt][0] = lds_u4(xr + ((t ^ g) << 4));
        xb[mt][1] = lds_u4(xr + (((4 + t) ^ g) << 4));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 g0 = (j >> 1) ? gc : ga, g8 = (j >> 1) ? hc : ha;
        const bool hi = j & 1;
        const uint32_t a0 = hi ? g0.z : g0.x, a2 = hi ? g0.w : g0.y;
        const uint32_t a1 = hi ? g8.z : g8.x, a3 = hi ? g8.w : g8.y;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint4 xv = xb[mt][j >> 1];
          mma_e4m3_16832(acc[mt], a0, a1, a2, a3, hi ? xv.z : xv.x, hi ? xv.w : xv.y);
        }
      }
    }
  }

  // ---- partials in the drained ring: red[m][row], rows 0..63 of the strip
  float* red = reinterpret_cast<float*>(slots);
  if (warp < 4) {
    asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int ch = 16 * warp + g;
      const int m0 = mt * 8 + 2 * t;
      red[(m0 + 0) * kF8GemvRows + ch] = acc[mt][0];
      red[(m0 + 1) * kF8GemvRows + ch] = acc[mt][1];
      red[(m0 + 0) * kF8GemvRows + ch + 8] = acc[mt][2];
      red[(m0 + 1) * kF8GemvRows + ch + 8] = acc[mt][3];
    }
  }
  cluster.sync();
  const int c0 = (rank * kF8GemvRows) / C, c1 = ((rank + 1) * kF8GemvRows) / C;
  const int ncol = c1 - c0;
  for (int e = threadIdx.x; e < M * ncol; e += blockDim.x) {
    const int m = e / ncol;
    const int ch = c0 + (e - m * ncol);
    const int n = nbase + ch;
    float s = 0.f;
    for (int r = 0; r < C; ++r) s += cluster.map_shared_rank(red, r)[m * kF8GemvRows + ch];
    if (n < N) {
      float v = __fmul_rn(__fmul_rn(s, sx[m]), sw[n]);
      if (bias != nullptr) v = __fadd_rn(v, __bfloat162float(bias[n]));
      y[static_cast<int64_t>(m) * N + n] = __float2bfloat16_rn(v);
    }
  }
  cluster.sync();
  (void)MP;
}

}  // namespace lmrs
