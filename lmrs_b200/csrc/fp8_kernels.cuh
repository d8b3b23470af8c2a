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
  asm(
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

// The ring area also holds the per-CTA partials [64 channels][MP + 4] fp32
// once drained; then the receive area [64 channels][MP] fp32 and the barriers.
__host__ __device__ constexpr int f8_gemv_ring_bytes(int ring, int MT) {
  return ring * (kF8GemvBoxBytes + 8 * MT * 128) > (8 * MT + 4) * kF8GemvRows * 4
             ? ring * (kF8GemvBoxBytes + 8 * MT * 128)
             : (8 * MT + 4) * kF8GemvRows * 4;
}
__host__ __device__ constexpr int f8_gemv_smem_bytes(int ring, int MT) {
  return 1024 + f8_gemv_ring_bytes(ring, MT) + kF8GemvRows * 8 * MT * 4 + (2 * ring + 1) * 8;
}

// MT: 8-token MMA tiles (M <= 8 * MT).  A producer thread streams the strip's
// weight rows (TMA boxes of 128 bytes of K x 64 rows, 128-byte swizzle) into a
// ring of shared-memory slots, the weights of the first slots before
// griddepcontrol.wait (programmatic dependent launch) and the token tiles after
// it; consumer warp w owns MMA tile w (channels 16w..16w+15).  Within each
// 128-byte K unit, lane (g, t) takes the 16-byte chunks t and 4+t of its two
// rows: the 32 k-slots of the unit's four MMAs are a fixed permutation of the
// unit's bytes, and the token fragment uses the same permutation.  Clusters of
// C CTAs (a power of two) split K; each CTA sends the owner of every channel
// slice its partial sums with 16-byte st.async into the owner's shared memory
// (completion counted on the owner's mbarrier), and the owner applies the
// scales and bias and stores y.
template <int MT>
__global__ void __launch_bounds__(kF8GemvThreads, MT == 4 ? 3 : 4) fp8_gemv_kernel(
    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
    __nv_bfloat16* __restrict__ y, const float* __restrict__ sx, const float* __restrict__ sw,
    const __nv_bfloat16* __restrict__ bias, int M, int K, int N, int ring) {
  constexpr int MP = 8 * MT;
  constexpr int kSlot = kF8GemvBoxBytes + MP * 128;  // weights + token tile (MP rows x 128 B)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* slots = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const int ring_bytes = f8_gemv_ring_bytes(ring, MT);
  float* recv = reinterpret_cast<float*>(slots + ring_bytes);         // [C][cw][MP]
  uint64_t* full = reinterpret_cast<uint64_t*>(recv + kF8GemvRows * MP);
  uint64_t* empty = full + ring;
  uint64_t* recv_bar = empty + ring;

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int strip = blockIdx.x / C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nbase = strip * kF8GemvRows;
  const int cw = kF8GemvRows / C;  // channels per owner

  const int units = (K + 127) >> 7;
  const int u_lo = static_cast<int>((static_cast<long long>(rank) * units) / C);
  const int u_hi = static_cast<int>((static_cast<long long>(rank + 1) * units) / C);
  const int nbox = u_hi - u_lo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);  // every consumer warp reads every box
    }
    mbar_init(recv_bar, 1);
    mbar_arrive_expect_tx(recv_bar, C * cw * MP * 4);  // every peer's st.async bytes
    fence_mbar_init();
  }
  __syncthreads();
  cluster_arrive_relaxed();
  pdl_trigger();

  float acc[MT][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_x);
      const int pre = nbox < ring ? nbox : ring;
      for (int b = 0; b < pre; ++b) {
        mbar_arrive_expect_tx(&full[b], kSlot);
        tma_load_2d(&tm_w, &full[b], slots + b * kSlot, (u_lo + b) * 128, nbase);
      }
      pdl_wait();  // the quantised tokens are the previous kernel's output
      for (int b = 0; b < pre; ++b)
        tma_load_2d(&tm_x, &full[b], slots + b * kSlot + kF8GemvBoxBytes, (u_lo + b) * 128, 0);
      int s = 0;
      uint32_t ph = 0;
      for (int b = pre; b < nbox; ++b) {
        if (!mbar_wait(&empty[s], ph, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&full[s], kSlot);
        tma_load_2d(&tm_w, &full[s], slots + s * kSlot, (u_lo + b) * 128, nbase);
        tma_load_2d(&tm_x, &full[s], slots + s * kSlot + kF8GemvBoxBytes, (u_lo + b) * 128, 0);
        if (++s == ring) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else {
    const int r0 = 16 * warp + g;  // rows r0 and r0 + 8 of the box; (r0 % 8) == g
    int slot = 0;
    uint32_t ph = 0;
    for (int b = 0; b < nbox; ++b) {
      if (!mbar_wait(&full[slot], ph, kErrWaitFull)) break;
      const uint8_t* sb = slots + slot * kSlot;
      // 128-byte swizzle: chunk c of row r sits at chunk c ^ (r % 8)
      const uint4 ga = *reinterpret_cast<const uint4*>(sb + r0 * 128 + ((t ^ g) << 4));
      const uint4 gc = *reinterpret_cast<const uint4*>(sb + r0 * 128 + (((4 + t) ^ g) << 4));
      const uint4 ha = *reinterpret_cast<const uint4*>(sb + (r0 + 8) * 128 + ((t ^ g) << 4));
      const uint4 hc = *reinterpret_cast<const uint4*>(sb + (r0 + 8) * 128 + (((4 + t) ^ g) << 4));
      uint4 xb[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint8_t* xr = sb + kF8GemvBoxBytes + (mt * 8 + g) * 128;  // rows >= M are zero
        xb[mt][0] = *reinterpret_cast<const uint4*>(xr + ((t ^ g) << 4));
        xb[mt][1] = *reinterpret_cast<const uint4*>(xr + (((4 + t) ^ g) << 4));
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
      if (++slot == ring) {
        slot = 0;
        ph ^= 1;
      }
    }
  }

  // ---- partials in the drained ring: red[channel][token] (row pitch MP + 4
  // floats: 16-byte aligned, and the 8 channels g of a fragment store land in
  // distinct banks), then to the owners
  constexpr int kPitch = MP + 4;
  float* red = reinterpret_cast<float*>(slots);
  cluster_wait_acquire();  // peers have initialised their receive barriers
  if (warp < 4) {
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the ring is drained
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int ch = 16 * warp + g;
      const int m0 = mt * 8 + 2 * t;
      red[ch * kPitch + m0] = acc[mt][0];
      red[ch * kPitch + m0 + 1] = acc[mt][1];
      red[(ch + 8) * kPitch + m0] = acc[mt][2];
      red[(ch + 8) * kPitch + m0 + 1] = acc[mt][3];
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    // (channel, 4 tokens) -> owner r = channel / cw, recv[rank][channel - r*cw][tokens]
    for (int e = threadIdx.x; e < kF8GemvRows * (MP / 4); e += 128) {
      const int ch = e / (MP / 4), m4 = (e - ch * (MP / 4)) * 4;
      const int r = ch / cw, cl = ch - r * cw;
      const float4 v = *reinterpret_cast<const float4*>(red + ch * kPitch + m4);
      st_async_v4(mapa_shared(smem_u32(recv + (rank * cw + cl) * MP + m4), static_cast<uint32_t>(r)),
                  v, mapa_shared(smem_u32(recv_bar), static_cast<uint32_t>(r)));
    }
    // ---- owner: sum the C slices in rank order, scale, bias, store
    const bool ok = mbar_wait_cluster(recv_bar, 0, kErrWaitCluster);
    pdl_wait();
    if (ok) {
      for (int e = threadIdx.x; e < M * cw; e += 128) {
        const int m = e / cw, cl = e - m * cw;
        const int n = nbase + rank * cw + cl;
        float s = 0.f;
        for (int q = 0; q < C; ++q) s += recv[(q * cw + cl) * MP + m];
        if (n < N) {
          float v = __fmul_rn(__fmul_rn(s, sx[m]), sw[n]);
          if (bias != nullptr) v = __fadd_rn(v, __bfloat162float(bias[n]));
          y[static_cast<int64_t>(m) * N + n] = __float2bfloat16_rn(v);
        }
      }
    }
  } else {
    pdl_wait();
  }
}

}  // namespace lmrs
